// NVLink peer-memory collectives written as single kernels (no NCCL on these paths).
//
// allreduce (two-shot, one launch per rank, all ranks concurrent):
//   phase A  every chunk of the local input goes to its owner (chunk c is owned by rank c % S)
//            with P2P stores into land[src][owned slot], then a release-add on the owner's
//            arrival counter of that chunk;
//   phase B  the owner waits for all S arrivals, sums them in rank order in fp32, applies the
//            fused scale (e.g. 1/world for a gradient mean), rounds to the element type and stores
//            the result into every rank's `out` area, publishing one epoch flag per chunk;
//   phase C  after the work counter ran dry, each CTA waits for the flags of a share of the
//            chunks, so the whole result is in local memory when the kernel ends.
// Work items come from one counter (phase A items first), so no wait depends on a CTA that is
// not running.  NVLink bytes per rank: 2 (S-1)/S n elements, the bandwidth-optimal amount.
// Replaces the gradient / statistics all-reduces of the reference's DDP and TP paths
// (sae_lens/training/sae_trainer.py DDP wrapper, sae_lens/distributed.py:404-461).
//
// wait_flags: wait (bounded) until n epoch flags of the local slab reach `target`.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "common.cuh"
#include "p2p.cuh"

namespace sb {
namespace p2p {

constexpr int AR_THREADS = 256;
constexpr int AR_CHUNK = 4096;  // elements per chunk (multiple of 8 * AR_THREADS / 2)

template <class T>
struct Elt;
template <>
struct Elt<float> {
  static __device__ __forceinline__ float ld(const float* p) { return __ldcg(p); }
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <>
struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) {
    return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(p))));
  }
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

struct ArArgs {
  const void* x;  // local input [n]
  int64_t n;
  float scale;
  Peers P;
  int64_t land_off;  // T [S][owned_chunks * CHUNK]
  int64_t cnt_off;   // u32 [nch]
  int64_t out_off;   // T [nch * CHUNK]
  int64_t flag_off;  // u32 [nch]
  uint32_t epoch;
  int* ticket;
  int* status;
};

template <class T>
__global__ void __launch_bounds__(AR_THREADS) allreduce_kernel(const __grid_constant__ ArArgs a) {
  __shared__ int s_tk, s_ok;
  const int t = threadIdx.x;
  const int S = a.P.world, r = a.P.rank;
  const int64_t nch = (a.n + AR_CHUNK - 1) / AR_CHUNK;
  const int64_t per_owner = (nch + S - 1) / S;  // land slots per source
  const int64_t n_own = (nch - r + S - 1) / S;   // chunks r, r+S, ...
  const T* x = reinterpret_cast<const T*>(a.x);
  while (true) {
    __syncthreads();
    if (t == 0) s_tk = atomicAdd(a.ticket, 1);
    __syncthreads();
    const int64_t tk = s_tk;
    if (tk >= nch + n_own) break;
    if (tk < nch) {
      const int64_t c = (tk + int64_t(r) * per_owner) % nch;  // spread the receivers
      const int o = int(c % S);
      const int64_t e0 = c * AR_CHUNK;
      const int64_t len = min(int64_t(AR_CHUNK), a.n - e0);
      T* dst = at<T>(a.P, o, a.land_off) + (int64_t(r) * per_owner + c / S) * AR_CHUNK;
      if (len == AR_CHUNK && (reinterpret_cast<uintptr_t>(x + e0) & 15) == 0) {
        constexpr int V = 16 / sizeof(T);
        for (int v = t; v < AR_CHUNK / V; v += AR_THREADS)
          reinterpret_cast<uint4*>(dst)[v] = __ldg(reinterpret_cast<const uint4*>(x + e0) + v);
      } else {
        for (int64_t e = t; e < len; e += AR_THREADS) dst[e] = x[e0 + e];
      }
      __threadfence_system();
      __syncthreads();
      if (t == 0) red_release_sys_add_u32(at<uint32_t>(a.P, o, a.cnt_off) + c, 1u);
    } else {
      const int64_t c = r + (tk - nch) * S;
      if (t == 0)
        s_ok = wait_geq_sys(at<uint32_t>(a.P, r, a.cnt_off) + c, uint32_t(S) * a.epoch, a.status,
                            kTimeoutPeerFlag)
                   ? 1
                   : 0;
      __syncthreads();
      if (!s_ok) continue;
      const int64_t e0 = c * AR_CHUNK;
      const int64_t len = min(int64_t(AR_CHUNK), a.n - e0);
      const T* land = at<T>(a.P, r, a.land_off) + (c / S) * AR_CHUNK;
      for (int64_t e = t; e < len; e += AR_THREADS) {
        float acc = 0.f;
        for (int s = 0; s < S; ++s) acc += Elt<T>::ld(land + int64_t(s) * per_owner * AR_CHUNK + e);
        const T v = Elt<T>::from_f(acc * a.scale);
        for (int d = 0; d < S; ++d) at<T>(a.P, (r + d) % S, a.out_off)[e0 + e] = v;
      }
      __threadfence_system();
      __syncthreads();
      if (t < S) st_release_sys_u32(at<uint32_t>(a.P, t, a.flag_off) + c, a.epoch);
    }
  }
  // phase C: the result of every chunk is local before the kernel ends
  for (int64_t c = int64_t(blockIdx.x) * AR_THREADS + t; c < nch; c += int64_t(gridDim.x) * AR_THREADS)
    wait_geq_sys(at<uint32_t>(a.P, r, a.flag_off) + c, a.epoch, a.status, kTimeoutPeerFlag);
}

__global__ void wait_flags_kernel(const uint32_t* flags, int64_t n, uint32_t target, int* status) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    wait_geq_sys(flags + i, target, status, kTimeoutPeerFlag);
}

}  // namespace p2p

static int p2p_sm_count() {
  int dev = 0, n = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

// Slab bytes the all-reduce needs for n elements of `elem_bytes` on `world` ranks:
// returns (land, counters, out, flags) sizes; callers place them at 256-byte aligned offsets.
std::vector<int64_t> p2p_allreduce_sizes(int64_t n, int64_t elem_bytes, int64_t world) {
  const int64_t nch = (n + p2p::AR_CHUNK - 1) / p2p::AR_CHUNK;
  const int64_t per_owner = (nch + world - 1) / world;
  return {world * per_owner * p2p::AR_CHUNK * elem_bytes, nch * 4, nch * p2p::AR_CHUNK * elem_bytes, nch * 4};
}

// Sum `x` (fp32 or bf16, [n]) over the group, times `scale`; the result lands in the `out` area
// of every rank's slab (offset out_off, same dtype).  Offsets are those of p2p_allreduce_sizes.
void p2p_allreduce(const torch::Tensor& x, double scale, const std::vector<int64_t>& peer_bases, int64_t rank,
                   int64_t land_off, int64_t cnt_off, int64_t out_off, int64_t flag_off, int64_t epoch,
                   const torch::Tensor& ticket, const torch::Tensor& status) {
  const int64_t S = int64_t(peer_bases.size());
  TORCH_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "p2p_allreduce: bad group");
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && (x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16),
              "p2p_allreduce: contiguous fp32/bf16 CUDA tensor required");
  TORCH_CHECK(land_off % 16 == 0 && out_off % 16 == 0, "p2p_allreduce: offsets");
  const int64_t n = x.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  p2p::ArArgs a{};
  a.x = x.data_ptr();
  a.n = n;
  a.scale = float(scale);
  a.P = p2p::make_peers(peer_bases, rank);
  a.land_off = land_off;
  a.cnt_off = cnt_off;
  a.out_off = out_off;
  a.flag_off = flag_off;
  a.epoch = uint32_t(epoch);
  a.ticket = ticket.data_ptr<int>();
  a.status = status.data_ptr<int>();
  C10_CUDA_CHECK(cudaMemsetAsync(a.ticket, 0, sizeof(int), stream));
  const int64_t nch = (n + p2p::AR_CHUNK - 1) / p2p::AR_CHUNK;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(2 * nch, int64_t(p2p_sm_count()) * 8));
  if (x.scalar_type() == at::kFloat)
    p2p::allreduce_kernel<float><<<dim3(grid), dim3(p2p::AR_THREADS), 0, stream>>>(a);
  else
    p2p::allreduce_kernel<__nv_bfloat16><<<dim3(grid), dim3(p2p::AR_THREADS), 0, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Stream-ordered wait until `n` u32 epoch flags at `flags` (local memory) reach `target`.
void p2p_wait_flags(const torch::Tensor& flags, int64_t target, const torch::Tensor& status) {
  TORCH_CHECK(flags.is_cuda() && flags.scalar_type() == at::kInt && flags.is_contiguous(), "p2p_wait_flags");
  const int64_t n = flags.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(flags.device());
  const int64_t grid = std::min<int64_t>((n + 255) / 256, 64);
  p2p::wait_flags_kernel<<<dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(flags.data_ptr<int>()), n, uint32_t(target), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

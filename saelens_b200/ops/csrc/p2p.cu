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
//            chunks, so the whole result is in local memory when the kernel ends; with an
//            output tensor (`x_out`, may be `x` itself) each arrived chunk is also copied there.
//            In place is safe: a chunk's flag comes from its owner after all S arrivals, so this
//            rank's phase A has finished reading that chunk of `x`.
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
#include "check.h"
#include "bounds.cuh"

namespace sb {
namespace p2p {

constexpr int AR_THREADS = 256;

// Element traits: A = accumulator type, to_a/ld widen, fin scales and rounds, sqv is the value's
// square for the per-chunk sum of squares.  int32 sums are exact (scale and sums of squares do
// not apply; the host checks).
template <class T>
struct Elt;
template <>
struct Elt<float> {
  using A = float;
  static __device__ __forceinline__ float ld(const float* p) { return __ldcg(p); }
  static __device__ __forceinline__ float to_a(float v) { return v; }
  static __device__ __forceinline__ float fin(float v, float s) { return v * s; }
  static __device__ __forceinline__ float sqv(float v) { return v * v; }
};
template <>
struct Elt<__nv_bfloat16> {
  using A = float;
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) {
    return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(p))));
  }
  static __device__ __forceinline__ float to_a(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 fin(float v, float s) { return __float2bfloat16_rn(v * s); }
  static __device__ __forceinline__ float sqv(__nv_bfloat16 v) {
    const float f = __bfloat162float(v);
    return f * f;
  }
};
template <>
struct Elt<int> {
  using A = int;
  static __device__ __forceinline__ int ld(const int* p) { return __ldcg(p); }
  static __device__ __forceinline__ int to_a(int v) { return v; }
  static __device__ __forceinline__ int fin(int v, float) { return v; }
  static __device__ __forceinline__ float sqv(int) { return 0.f; }
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
  int64_t sq_off;    // fp32 [nch]: per-chunk sum of squares of the result, on every rank (< 0: none)
  int64_t chunk;     // elements per chunk
  void* x_out;       // optional local copy of the result [n] (may alias x)
  uint32_t epoch;
  int* ticket;
  int* status;
};

template <class T>
__global__ void __launch_bounds__(AR_THREADS) allreduce_kernel(const __grid_constant__ ArArgs a) {
  __shared__ int s_tk, s_ok;
  __shared__ float s_red[AR_THREADS / 32];
  const int t = threadIdx.x;
  const int S = a.P.world, r = a.P.rank;
  const int64_t CH = a.chunk;
  const int64_t nch = (a.n + CH - 1) / CH;
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
      const int64_t e0 = c * CH;
      const int64_t len = min(CH, a.n - e0);
      T* dst = at<T>(a.P, o, a.land_off) + (int64_t(r) * per_owner + c / S) * CH;
      if (len == CH && (reinterpret_cast<uintptr_t>(x + e0) & 15) == 0) {
        constexpr int V = 16 / sizeof(T);
        for (int v = t; v < CH / V; v += AR_THREADS)
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
      const int64_t e0 = c * CH;
      const int64_t len = min(CH, a.n - e0);
      const T* land = at<T>(a.P, r, a.land_off) + (c / S) * CH;
      float sq = 0.f;
      if (len == CH) {
        // 16-byte vectors: V elements per thread and step, S loads and S stores of 16 bytes
        constexpr int V = 16 / sizeof(T);
        for (int v = t; v < CH / V; v += AR_THREADS) {
          typename Elt<T>::A acc[V];
#pragma unroll
          for (int i = 0; i < V; ++i) acc[i] = 0;
          for (int s = 0; s < S; ++s) {
            const uint4 q = __ldcg(reinterpret_cast<const uint4*>(land + int64_t(s) * per_owner * CH) + v);
            const T* qe = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int i = 0; i < V; ++i) acc[i] += Elt<T>::to_a(qe[i]);
          }
          uint4 o;
          T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            oe[i] = Elt<T>::fin(acc[i], a.scale);
            sq += Elt<T>::sqv(oe[i]);
          }
          for (int d = 0; d < S; ++d)
            reinterpret_cast<uint4*>(at<T>(a.P, (r + d) % S, a.out_off) + e0)[v] = o;
        }
      } else {
        for (int64_t e = t; e < len; e += AR_THREADS) {
          typename Elt<T>::A acc = 0;
          for (int s = 0; s < S; ++s) acc += Elt<T>::ld(land + int64_t(s) * per_owner * CH + e);
          const T v = Elt<T>::fin(acc, a.scale);
          sq += Elt<T>::sqv(v);
          for (int d = 0; d < S; ++d) at<T>(a.P, (r + d) % S, a.out_off)[e0 + e] = v;
        }
      }
      if (a.sq_off >= 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if ((t & 31) == 0) s_red[t >> 5] = sq;
        __syncthreads();
        if (t == 0) {
          float tot = 0.f;
          for (int w = 0; w < AR_THREADS / 32; ++w) tot += s_red[w];
          for (int d = 0; d < S; ++d) at<float>(a.P, d, a.sq_off)[c] = tot;
        }
      }
      __threadfence_system();
      __syncthreads();
      if (t < S) st_release_sys_u32(at<uint32_t>(a.P, t, a.flag_off) + c, a.epoch);
    }
  }
  // phase C: the result of every chunk is local before the kernel ends
  if (a.x_out == nullptr) {
    for (int64_t c = int64_t(blockIdx.x) * AR_THREADS + t; c < nch; c += int64_t(gridDim.x) * AR_THREADS)
      wait_geq_sys(at<uint32_t>(a.P, r, a.flag_off) + c, a.epoch, a.status, kTimeoutPeerFlag);
    return;
  }
  const T* res = at<T>(a.P, r, a.out_off);
  T* xo = reinterpret_cast<T*>(a.x_out);
  for (int64_t c = blockIdx.x; c < nch; c += gridDim.x) {
    __syncthreads();
    if (t == 0)
      s_ok = wait_geq_sys(at<uint32_t>(a.P, r, a.flag_off) + c, a.epoch, a.status, kTimeoutPeerFlag) ? 1 : 0;
    __syncthreads();
    if (!s_ok) return;
    const int64_t e0 = c * CH;
    const int64_t len = min(CH, a.n - e0);
    if (len == CH && (reinterpret_cast<uintptr_t>(xo + e0) & 15) == 0) {
      constexpr int V = 16 / sizeof(T);
      for (int v = t; v < CH / V; v += AR_THREADS)
        reinterpret_cast<uint4*>(xo + e0)[v] = __ldcg(reinterpret_cast<const uint4*>(res + e0) + v);
    } else {
      for (int64_t e = t; e < len; e += AR_THREADS) xo[e0 + e] = res[e0 + e];
    }
  }
}

// Owner side of the gradient reduce-scatter of sharded data parallel: every rank stored its
// gradient rows of this rank's latents into slot [src] of land [S, n*D] (bf16); out = scale *
// sum over src (rank order, fp32), rounded to bf16, and sumsq += the rounded result's squares.
__global__ void slot_reduce_kernel(const __nv_bfloat16* __restrict__ land, int S, int64_t nvec, float scale,
                                   __nv_bfloat16* __restrict__ out, float* __restrict__ sumsq) {
  __shared__ float s_red[AR_THREADS / 32];
  float sq = 0.f;
  for (int64_t v = int64_t(blockIdx.x) * AR_THREADS + threadIdx.x; v < nvec; v += int64_t(gridDim.x) * AR_THREADS) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int src = 0; src < S; ++src) {
      const uint4 q = __ldcg(reinterpret_cast<const uint4*>(land) + int64_t(src) * nvec + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    uint4 o;
    uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 hb = __floats2bfloat162_rn(acc[2 * e] * scale, acc[2 * e + 1] * scale);
      w[e] = *reinterpret_cast<const uint32_t*>(&hb);
      const float2 f = __bfloat1622float2(hb);
      sq += f.x * f.x + f.y * f.y;
    }
    reinterpret_cast<uint4*>(out)[v] = o;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0 && sumsq) {
    float t = 0.f;
    for (int i = 0; i < AR_THREADS / 32; ++i) t += s_red[i];
    atomicAdd(sumsq, t);
  }
}

// ---------------------------------------------------------------------------------------
// Device activation ring (streaming between disjoint producer and consumer GPUs).  N chunk slots
// of [chunk_rows, D] bf16 live in the consumer's slab with one state word per slot (FREE ->
// WRITING -> READY -> CONSUMING -> FREE, the state machine of the reference's /dev/shm ring,
// sae_lens/training/shared_activation_buffer.py:36-41 and 151-296) and meta [N][4] (rows,
// producer, sequence, 0).  Claims are system-scope compare-and-swaps on the state words (over
// NVLink for producers); the rows travel as P2P stores from the producer GPU, normalised and
// cast to bf16 in the same kernel; READY / FREE are published with release stores.
// ---------------------------------------------------------------------------------------
__global__ void ring_claim_kernel(Peers P, int owner, int64_t state_off, int n_slots, uint32_t from, uint32_t to,
                                  int start, long long timeout_ns, int* out_slot) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  uint32_t* st = at<uint32_t>(P, owner, state_off);
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < n_slots; ++i) {
      const int sidx = (start + i) % n_slots;
      if (atomicCAS_system(st + sidx, from, to) == from) {
        __threadfence_system();  // later reads of the slot are ordered after the claim
        *out_slot = sidx;
        return;
      }
    }
    if ((long long)(globaltimer_ns() - t0) > timeout_ns) {
      *out_slot = -1;
      return;
    }
    __nanosleep(1000);
  }
}

// One warp per row: sum of squares (mode 2), then scale, bf16 cast and 16-byte P2P stores.
__global__ void ring_write_kernel(const void* __restrict__ src, int64_t ld_src, int src_f32, int rows, int D,
                                  int mode, float scale, Peers P, int owner, int64_t data_off, int chunk_rows,
                                  const int* __restrict__ slot_ptr) {
  const int slot = *slot_ptr;
  if (slot < 0) return;
  __nv_bfloat16* dst = at<__nv_bfloat16>(P, owner, data_off) + int64_t(slot) * chunk_rows * D;
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  auto load8 = [&](int64_t row, int v, float* f) {
    if (src_f32) {
      const float4* s4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + row * ld_src) + 2 * v;
      const float4 a = __ldg(s4), b = __ldg(s4 + 1);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src) + row * ld_src) + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 t = __bfloat1622float2(h[e]);
        f[2 * e] = t.x;
        f[2 * e + 1] = t.y;
      }
    }
  };
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    float mul = mode == 1 ? scale : 1.f;
    if (mode == 2) {
      float ss = 0.f;
      for (int v = lane; v < nvec; v += 32) {
        float f[8];
        load8(row, v, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      mul = ss > 0.f ? scale * rsqrtf(ss) : 0.f;
    }
    for (int v = lane; v < nvec; v += 32) {
      float f[8];
      load8(row, v, f);
      uint4 q;
      uint32_t* w = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * e] * mul, f[2 * e + 1] * mul);
        w[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      reinterpret_cast<uint4*>(dst + int64_t(row) * D)[v] = q;
    }
  }
  __threadfence_system();  // the publish launch that follows orders after these stores
}

// Thread 0: optional meta (rows >= 0), then a release store of `value` into the slot's state.
__global__ void ring_publish_kernel(Peers P, int owner, int64_t state_off, int64_t meta_off,
                                    const int* __restrict__ slot_ptr, int rows, int producer, int seq,
                                    uint32_t value) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int slot = *slot_ptr;
  if (slot < 0) return;
  if (rows >= 0) {
    int* meta = at<int>(P, owner, meta_off) + 4 * slot;
    meta[0] = rows;
    meta[1] = producer;
    meta[2] = seq;
  }
  __threadfence_system();
  st_release_sys_u32(at<uint32_t>(P, owner, state_off) + slot, value);
}

// out[i] = slot rows[perm ? perm[i] : i] (local ring data), one warp per output row.
__global__ void ring_gather_kernel(const __nv_bfloat16* __restrict__ data, int chunk_rows, int D,
                                   const int* __restrict__ slot_ptr, const int* __restrict__ perm, int rows,
                                   __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int slot = *slot_ptr;
  if (slot < 0) return;
  const __nv_bfloat16* base = data + int64_t(slot) * chunk_rows * D;
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rows; i += warps) {
    const int r = perm ? perm[i] : i;
    if (!SB_IN_RANGE(r, chunk_rows)) continue;  // debug builds: a permutation entry past the chunk
    const uint4* s4 = reinterpret_cast<const uint4*>(base + int64_t(r) * D);
    uint4* o4 = reinterpret_cast<uint4*>(out + int64_t(i) * ldo);
    for (int v = lane; v < nvec; v += 32) o4[v] = __ldcg(s4 + v);
  }
}

__global__ void wait_flags_kernel(const uint32_t* flags, int64_t n, uint32_t target, int* status) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    wait_geq_sys(flags + i, target, status, kTimeoutPeerFlag);
}


// ---------------------------------------------------------------------------------------
// Row routing: the producer-to-consumer all-to-all of activation rows (shard routing), with the
// activation normalisation and the bf16 cast fused into the NVLink stores.  Each route sends a
// contiguous run of the producer's rows to a row offset of one consumer's landing buffer (in
// that consumer's slab, slot `slot` of a double buffer).  CTAs take RR-row chunks; after a chunk
// a release-add on the consumer's arrival counter for this producer publishes it.  Before
// writing slot s for epoch e >= 3 the kernel waits (bounded) until every destination consumer
// released epoch e - 2, which used the same slot.
// Normalisation: mode 0 none, 1 multiply by `scale`, 2 rescale every row to L2 norm `scale`.
// Reference path replaced: NCCL batch_isend_irecv per route + cast/normalise passes
// (sae_lens/training/activations_store.py:1482-1606, 1063; activation_scaler.py:16-23).
// ---------------------------------------------------------------------------------------
constexpr int RT_RR = 8;                 // rows per published chunk
constexpr int RT_THREADS = 32 * RT_RR;   // one warp per row of a chunk
constexpr int RT_MAX_ROUTES = 16;

struct RouteArgs {
  const void* src;
  int src_f32;
  int64_t ld_src;
  int64_t src_rows;  // rows of `src` (source row bound)
  int D;
  int n_routes;
  int r_src[RT_MAX_ROUTES];    // first source row
  int r_rows[RT_MAX_ROUTES];   // rows
  int r_rank[RT_MAX_ROUTES];   // destination rank
  int r_dst[RT_MAX_ROUTES];    // first destination row in the consumer's landing slot
  int r_chunk0[RT_MAX_ROUTES + 1];
  Peers P;
  int64_t land_off;       // bf16 [2][rows_cap][D] on every consumer
  int64_t rows_cap;
  int slot;
  int64_t cnt_off;        // u32 [n_producer_slots] on every consumer
  int cnt_slot;           // this producer's counter index on the consumers
  int64_t free_off;       // u32 [n_consumer_slots] on every producer: last epoch each consumer released
  int free_slot[RT_MAX_ROUTES];
  int mode;
  float scale;
  uint32_t epoch;
  int* status;
};

// One warp per row: the CTA's RT_RR warps each own one row of the chunk.  Pass 1 reads the row
// (16-byte vectors) for its sum of squares, pass 2 re-reads it (from L1 / L2), scales, casts to
// bf16 and stores it into the destination's landing slot over NVLink.  Then one system-scope fence
// per thread, one barrier and one release per chunk.
__global__ void __launch_bounds__(RT_THREADS) route_rows_kernel(const __grid_constant__ RouteArgs a) {
  __shared__ int s_ok;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nvec = a.D >> 3;
  if (a.epoch >= 3) {
    if (t == 0) {
      bool ok = true;
      for (int i = 0; i < a.n_routes && ok; ++i)
        ok = wait_geq_sys(at<uint32_t>(a.P, a.P.rank, a.free_off) + a.free_slot[i], a.epoch - 2, a.status,
                          kTimeoutPeerFlag);
      s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok) return;
  }
  const int nchunks = a.r_chunk0[a.n_routes];
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    int ri = 0;
    while (c >= a.r_chunk0[ri + 1]) ++ri;
    const int row0 = (c - a.r_chunk0[ri]) * RT_RR;
    const int nr = min(RT_RR, a.r_rows[ri] - row0);
    const int dst_rank = a.r_rank[ri];
    __nv_bfloat16* land = at<__nv_bfloat16>(a.P, dst_rank, a.land_off) + (int64_t(a.slot) * a.rows_cap) * a.D;
    if (warp < nr && SB_IN_RANGE(a.r_src[ri] + row0 + warp, a.src_rows) &&
        SB_IN_RANGE(a.r_dst[ri] + row0 + warp, a.rows_cap)) {
      const int64_t srow = a.r_src[ri] + row0 + warp;
      const int64_t drow = a.r_dst[ri] + row0 + warp;
      const float* sf = reinterpret_cast<const float*>(a.src) + srow * a.ld_src;
      const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(a.src) + srow * a.ld_src;
      auto load8 = [&](int vi, float (&v)[8]) {
        if (a.src_f32) {
          const float4* s4 = reinterpret_cast<const float4*>(sf) + 2 * vi;
          const float4 x0 = __ldg(s4), x1 = __ldg(s4 + 1);
          v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
          v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
        } else {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(sb) + vi);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            v[2 * e] = f.x;
            v[2 * e + 1] = f.y;
          }
        }
      };
      float mul = a.mode == 1 ? a.scale : 1.f;
      if (a.mode == 2) {
        float ss = 0.f;
#pragma unroll 4
        for (int vi = lane; vi < nvec; vi += 32) {
          float v[8];
          load8(vi, v);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        mul = ss > 0.f ? a.scale * rsqrtf(ss) : 0.f;
      }
      uint4* dst = reinterpret_cast<uint4*>(land + drow * a.D);
#pragma unroll 4
      for (int vi = lane; vi < nvec; vi += 32) {
        float v[8];
        load8(vi, v);
        uint4 q;
        uint32_t* w = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e] * mul, v[2 * e + 1] * mul);
          w[e] = *reinterpret_cast<uint32_t*>(&h);
        }
        dst[vi] = q;
      }
    }
    __threadfence_system();
    __syncthreads();
    if (t == 0) red_release_sys_add_u32(at<uint32_t>(a.P, dst_rank, a.cnt_off) + a.cnt_slot, 1u);
  }
}

__global__ void wait_targets_kernel(const uint32_t* counters, const int64_t* targets, int n, int* status) {
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    wait_geq_sys(counters + i, uint32_t(targets[i]), status, kTimeoutPeerFlag);
}

__global__ void signal_kernel(Peers P, int64_t off, int index, int n_ranks_mask, uint32_t value) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < P.world; ++r)
      if (n_ranks_mask & (1 << r)) st_release_sys_u32(at<uint32_t>(P, r, off) + index, value);
  }
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
// Chunk size for n elements when the caller passes none: large chunks keep NVLink busy (measured
// on 2 B200s: 65536 elements reach ~586 GB/s bus bandwidth at 1 GB, 4096 only ~117 GB/s), small
// messages need enough chunks to spread over the SMs.  A power of two in [2048, 65536].
static int64_t auto_chunk(int64_t n) {
  int64_t c = 2048;
  while (c < 65536 && c * 2 * 512 <= n) c *= 2;
  return c;
}

std::vector<int64_t> p2p_allreduce_sizes(int64_t n, int64_t elem_bytes, int64_t world, int64_t chunk) {
  if (chunk <= 0) chunk = auto_chunk(n);
  const int64_t nch = (n + chunk - 1) / chunk;
  const int64_t per_owner = (nch + world - 1) / world;
  return {world * per_owner * chunk * elem_bytes, nch * 4, nch * chunk * elem_bytes, nch * 4};
}

// Sum `x` (fp32, bf16 or int32, [n]) over the group, times `scale`; the result lands in the `out` area
// of every rank's slab (offset out_off, same dtype).  Offsets are those of p2p_allreduce_sizes.
// With sq_off >= 0, every rank also receives the sum of squares of each result chunk (fp32
// [nch] at sq_off), e.g. for the norm of an averaged gradient.
void p2p_allreduce(const torch::Tensor& x, double scale, const std::vector<int64_t>& peer_bases, int64_t rank,
                   int64_t land_off, int64_t cnt_off, int64_t out_off, int64_t flag_off, int64_t epoch,
                   const torch::Tensor& ticket, const torch::Tensor& status, int64_t sq_off, int64_t chunk,
                   int64_t max_ctas, const c10::optional<torch::Tensor>& x_out) {
  const int64_t S = int64_t(peer_bases.size());
  SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "p2p_allreduce: bad group");
  SB_CHECK(x.is_cuda() && x.is_contiguous() &&
                  (x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kInt),
              "p2p_allreduce: contiguous fp32/bf16/int32 CUDA tensor required");
  SB_CHECK(x.scalar_type() != at::kInt || (scale == 1.0 && sq_off < 0),
              "p2p_allreduce: int32 sums take no scale and no sums of squares");
  SB_CHECK(land_off % 16 == 0 && out_off % 16 == 0, "p2p_allreduce: offsets must be 16-byte aligned");
  const int64_t n = x.numel();
  if (n == 0) return;
  if (chunk <= 0) chunk = auto_chunk(n);
  SB_CHECK(chunk % (8 * p2p::AR_THREADS) == 0, "p2p_allreduce: chunk must be a multiple of ", 8 * p2p::AR_THREADS);
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  p2p::ArArgs a{};
  a.chunk = chunk;
  a.x = x.data_ptr();
  a.n = n;
  a.scale = float(scale);
  a.P = p2p::make_peers(peer_bases, rank);
  a.land_off = land_off;
  a.cnt_off = cnt_off;
  a.out_off = out_off;
  a.flag_off = flag_off;
  a.sq_off = sq_off;
  a.epoch = uint32_t(epoch);
  a.ticket = ticket.data_ptr<int>();
  a.status = status.data_ptr<int>();
  if (x_out) {
    SB_CHECK(x_out->is_cuda() && x_out->is_contiguous() && x_out->scalar_type() == x.scalar_type() &&
                    x_out->numel() == n,
                "p2p_allreduce: x_out must be a contiguous tensor like x");
    a.x_out = x_out->data_ptr();
  }
  C10_CUDA_CHECK(cudaMemsetAsync(a.ticket, 0, sizeof(int), stream));
  const int64_t nch = (n + chunk - 1) / chunk;
  int64_t grid = std::max<int64_t>(1, std::min<int64_t>(2 * nch, int64_t(p2p_sm_count()) * 8));
  if (max_ctas > 0) grid = std::min(grid, max_ctas);  // leave SMs to overlapping compute
  if (x.scalar_type() == at::kFloat)
    p2p::allreduce_kernel<float><<<dim3(grid), dim3(p2p::AR_THREADS), 0, stream>>>(a);
  else if (x.scalar_type() == at::kInt)
    p2p::allreduce_kernel<int><<<dim3(grid), dim3(p2p::AR_THREADS), 0, stream>>>(a);
  else
    p2p::allreduce_kernel<__nv_bfloat16><<<dim3(grid), dim3(p2p::AR_THREADS), 0, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out [n, D] bf16 = scale * sum over the S slots of land [S, n, D] bf16 (see slot_reduce_kernel);
// sumsq (fp32 [1], optional) accumulates the squares of the result.
void p2p_slot_reduce(const torch::Tensor& land, double scale, const torch::Tensor& out,
                     const c10::optional<torch::Tensor>& sumsq) {
  SB_CHECK(land.is_cuda() && land.scalar_type() == at::kBFloat16 && land.is_contiguous() && land.dim() == 3,
              "p2p_slot_reduce: land must be contiguous bf16 [S, n, D]");
  SB_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == land.size(1) * land.size(2),
              "p2p_slot_reduce: out must be contiguous bf16 [n, D]");
  const int64_t n_el = out.numel();
  SB_CHECK(n_el % 8 == 0, "p2p_slot_reduce: n * D must be a multiple of 8");
  if (sumsq) SB_CHECK(sumsq->scalar_type() == at::kFloat && sumsq->is_cuda(), "p2p_slot_reduce: sumsq");
  if (n_el == 0) return;
  const at::cuda::CUDAGuard guard(land.device());
  const int64_t nvec = n_el / 8;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((nvec + p2p::AR_THREADS - 1) / p2p::AR_THREADS,
                                                              int64_t(p2p_sm_count()) * 8));
  p2p::slot_reduce_kernel<<<dim3(grid), dim3(p2p::AR_THREADS), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(land.data_ptr()), int(land.size(0)), nvec, float(scale),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), sumsq ? sumsq->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Device activation ring host entry points (see ring_claim_kernel).  `slot` is an int32 [1]
// device word: the claimed slot index, or -1 when the bounded claim timed out.
void ring_claim(const std::vector<int64_t>& peer_bases, int64_t rank, int64_t owner, int64_t state_off,
                int64_t n_slots, int64_t from, int64_t to, int64_t start, double timeout_ms, const torch::Tensor& slot) {
  SB_CHECK(slot.is_cuda() && slot.scalar_type() == at::kInt && slot.numel() >= 1, "ring_claim: slot");
  SB_CHECK(n_slots >= 1 && owner >= 0 && owner < int64_t(peer_bases.size()) && state_off % 4 == 0,
              "ring_claim: ring");
  const at::cuda::CUDAGuard guard(slot.device());
  p2p::Peers P = p2p::make_peers(peer_bases, rank);
  p2p::ring_claim_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, int(owner), state_off, int(n_slots), uint32_t(from), uint32_t(to), int(start % n_slots),
      (long long)(timeout_ms * 1e6), slot.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ring_write(const torch::Tensor& src, const std::vector<int64_t>& peer_bases, int64_t rank, int64_t owner,
                int64_t data_off, int64_t chunk_rows, const torch::Tensor& slot, int64_t mode, double scale) {
  SB_CHECK(src.is_cuda() && src.dim() == 2 && src.stride(1) == 1 &&
                  (src.scalar_type() == at::kFloat || src.scalar_type() == at::kBFloat16),
              "ring_write: src must be a CUDA fp32/bf16 matrix with contiguous rows");
  const int64_t rows = src.size(0), D = src.size(1);
  SB_CHECK(rows <= chunk_rows && D % 8 == 0 && data_off % 16 == 0, "ring_write: rows <= chunk_rows, D % 8");
  SB_CHECK(src.scalar_type() == at::kBFloat16 ? src.stride(0) % 8 == 0 : src.stride(0) % 4 == 0,
              "ring_write: row stride alignment");
  SB_CHECK(mode >= 0 && mode <= 2, "ring_write: mode");
  if (rows == 0) return;
  const at::cuda::CUDAGuard guard(src.device());
  p2p::Peers P = p2p::make_peers(peer_bases, rank);
  const int grid = int(std::min<int64_t>((rows + 7) / 8, int64_t(p2p_sm_count()) * 8));
  p2p::ring_write_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      src.data_ptr(), src.stride(0), src.scalar_type() == at::kFloat ? 1 : 0, int(rows), int(D), int(mode),
      float(scale), P, int(owner), data_off, int(chunk_rows), slot.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ring_publish(const std::vector<int64_t>& peer_bases, int64_t rank, int64_t owner, int64_t state_off,
                  int64_t meta_off, const torch::Tensor& slot, int64_t rows, int64_t producer, int64_t seq,
                  int64_t value) {
  const at::cuda::CUDAGuard guard(slot.device());
  p2p::Peers P = p2p::make_peers(peer_bases, rank);
  p2p::ring_publish_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, int(owner), state_off, meta_off, slot.data_ptr<int>(), int(rows), int(producer), int(seq), uint32_t(value));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ring_gather(const torch::Tensor& data, const torch::Tensor& slot, const c10::optional<torch::Tensor>& perm,
                 const torch::Tensor& out) {
  SB_CHECK(data.is_cuda() && data.scalar_type() == at::kBFloat16 && data.dim() == 3 && data.is_contiguous(),
              "ring_gather: data must be contiguous bf16 [N, chunk_rows, D]");
  SB_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(1) == data.size(2) &&
                  out.stride(1) == 1 && out.stride(0) % 8 == 0 && out.size(0) <= data.size(1),
              "ring_gather: out must be bf16 [rows <= chunk_rows, D] with contiguous rows");
  if (perm) SB_CHECK(perm->is_cuda() && perm->scalar_type() == at::kInt && perm->numel() >= out.size(0),
                        "ring_gather: perm must be CUDA int32 [rows]");
  const int64_t rows = out.size(0);
  if (rows == 0) return;
  const at::cuda::CUDAGuard guard(data.device());
  const int grid = int(std::min<int64_t>((rows + 7) / 8, int64_t(p2p_sm_count()) * 8));
  p2p::ring_gather_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(data.data_ptr()), int(data.size(1)), int(data.size(2)),
      slot.data_ptr<int>(), perm ? perm->data_ptr<int>() : nullptr, int(rows),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Stream-ordered wait until `n` u32 epoch flags at `flags` (local memory) reach `target`.
void p2p_wait_flags(const torch::Tensor& flags, int64_t target, const torch::Tensor& status) {
  SB_CHECK(flags.is_cuda() && flags.scalar_type() == at::kInt && flags.is_contiguous(), "p2p_wait_flags");
  const int64_t n = flags.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(flags.device());
  const int64_t grid = std::min<int64_t>((n + 255) / 256, 64);
  p2p::wait_flags_kernel<<<dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(flags.data_ptr<int>()), n, uint32_t(target), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Route rows of `src` ([rows, D] fp32 or bf16) to consumers: routes = int64 [n, 4] rows of
// (first source row, rows, destination rank, first destination row).  Writes bf16 rows into slot
// `slot` of each consumer's landing area (land_off, capacity rows_cap) and counts RR-row chunks
// on counter `cnt_slot` at cnt_off of the consumer.  free_slots[i] is the index, in this rank's
// free flags at free_off, of route i's consumer.
void p2p_route_rows(const torch::Tensor& src, const torch::Tensor& routes, const std::vector<int64_t>& peer_bases,
                    int64_t rank, int64_t land_off, int64_t rows_cap, int64_t slot, int64_t cnt_off,
                    int64_t cnt_slot, int64_t free_off, const std::vector<int64_t>& free_slots, int64_t mode,
                    double scale, int64_t epoch, const torch::Tensor& status) {
  SB_CHECK(src.is_cuda() && src.dim() == 2 && src.stride(1) == 1 &&
                  (src.scalar_type() == at::kFloat || src.scalar_type() == at::kBFloat16),
              "p2p_route_rows: src must be a CUDA fp32/bf16 matrix with contiguous rows");
  SB_CHECK(routes.device().is_cpu() && routes.scalar_type() == at::kLong && routes.dim() == 2 &&
                  routes.size(1) == 4 && routes.size(0) <= p2p::RT_MAX_ROUTES,
              "p2p_route_rows: routes must be a CPU int64 [n <= 16, 4] table");
  const int64_t D = src.size(1);
  SB_CHECK(D % 8 == 0, "p2p_route_rows: d must be a multiple of 8");
  SB_CHECK(mode >= 0 && mode <= 2, "p2p_route_rows: mode");
  SB_CHECK(int64_t(free_slots.size()) == routes.size(0), "p2p_route_rows: free_slots");
  const at::cuda::CUDAGuard guard(src.device());
  p2p::RouteArgs a{};
  a.src = src.data_ptr();
  a.src_f32 = src.scalar_type() == at::kFloat ? 1 : 0;
  a.ld_src = src.stride(0);
  a.src_rows = src.size(0);
  a.D = int(D);
  a.n_routes = int(routes.size(0));
  auto R = routes.accessor<int64_t, 2>();
  int chunks = 0;
  for (int i = 0; i < a.n_routes; ++i) {
    a.r_src[i] = int(R[i][0]);
    a.r_rows[i] = int(R[i][1]);
    a.r_rank[i] = int(R[i][2]);
    a.r_dst[i] = int(R[i][3]);
    SB_CHECK(R[i][0] >= 0 && R[i][0] + R[i][1] <= src.size(0) && R[i][3] >= 0 && R[i][3] + R[i][1] <= rows_cap &&
                    R[i][2] >= 0 && R[i][2] < int64_t(peer_bases.size()),
                "p2p_route_rows: route ", i, " out of range");
    a.r_chunk0[i] = chunks;
    chunks += int((R[i][1] + p2p::RT_RR - 1) / p2p::RT_RR);
    a.free_slot[i] = int(free_slots[i]);
  }
  a.r_chunk0[a.n_routes] = chunks;
  a.P = p2p::make_peers(peer_bases, rank);
  a.land_off = land_off;
  a.rows_cap = rows_cap;
  a.slot = int(slot);
  a.cnt_off = cnt_off;
  a.cnt_slot = int(cnt_slot);
  a.free_off = free_off;
  a.mode = int(mode);
  a.scale = float(scale);
  a.epoch = uint32_t(epoch);
  a.status = status.data_ptr<int>();
  if (chunks == 0) return;
  const int grid = std::min(chunks, p2p_sm_count() * 8);
  p2p::route_rows_kernel<<<dim3(grid), dim3(p2p::RT_THREADS), 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Wait (bounded, stream-ordered) until counters[i] >= targets[i] (targets: CUDA int64).
void p2p_wait_targets(const torch::Tensor& counters, const torch::Tensor& targets, const torch::Tensor& status) {
  SB_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && targets.is_cuda() &&
                  targets.scalar_type() == at::kLong && targets.numel() <= counters.numel(),
              "p2p_wait_targets");
  const at::cuda::CUDAGuard guard(counters.device());
  p2p::wait_targets_kernel<<<1, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(counters.data_ptr<int>()), targets.data_ptr<int64_t>(),
      int(targets.numel()), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Stream-ordered release store of `value` into flag `index` at `off` of every rank in rank_mask.
void p2p_signal(const std::vector<int64_t>& peer_bases, int64_t rank, int64_t off, int64_t index,
                int64_t rank_mask, int64_t value) {
  p2p::Peers P = p2p::make_peers(peer_bases, rank);
  p2p::signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(P, off, int(index), int(rank_mask),
                                                                       uint32_t(value));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

#if SB_DEBUG_BOUNDS
namespace sb {
// {line, value, bound, violations} of this file's first bounds violation (debug module only).
std::vector<int64_t> p2p_bounds_info(bool reset) { return bounds_read(reset); }
}  // namespace sb
#endif

// Matching-pursuit encode: the per-iteration update and its backward
// (sae_lens/saes/matching_pursuit_sae.py:258-335, `_encode_matching_pursuit`).
//
// One encode iteration is two launches:
//   1. the score GEMM on the tcgen05 tensor cores (gemm_tc.cu, `gemm_tn_bf16` with `amax`):
//      relu(bf16(residual) @ bf16(W_dec)^T) with each row's argmax folded into a 64-bit key by
//      atomicMax in the epilogue, so the [rows, d_sae] score matrix is never written;
//   2. `step_kernel` below, one warp per row: decode the key, value = relu(<residual, W_dec[i]>)
//      in fp32, add it to the dense codes, subtract value * W_dec[i] from the residual (also
//      refreshing the bf16 copy the next GEMM reads), and decide whether the row stops.
// A row stops once an iteration adds no new latent (stop_on_duplicate_support: the support only
// grows, because every added value is >= 0, so "support unchanged" is "no new latent") or once its
// residual norm is below the threshold; stopped rows are skipped by later iterations, exactly as
// the reference masks their values to zero.
//
// The backward walks the recorded iterations in reverse, one warp per row, rebuilding each
// iteration's residual from the final one (r_t = r_{t+1} + v_t w_t) instead of storing all of
// them.  With G the gradient of the residual after iteration t and g the gradient of the codes:
//   g_v  = g[i_t] - <G, w_t>                 (the value feeds the code and the next residual)
//   dW[i_t] += g_v * r_t - v_t * G           (only iterations with v_t > 0: relu' and the mask)
//   G    += g_v * w_t
// The latent selection itself carries no gradient (it is taken under no_grad in the reference).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "check.h"

namespace sb {
namespace mp {

constexpr int WARPS = 8;  // rows per CTA (one warp per row)

// Four consecutive decoder elements as fp32 (16-byte fp32 or 8-byte bf16 loads).
__device__ __forceinline__ float4 load4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int key_index(unsigned long long k, int N) {
  if (k == 0ull) return -1;  // the GEMM saw no column for this row
  const int i = int(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
  return (i >= 0 && i < N) ? i : -1;
}

struct StepArgs {
  float* resid;               // [B, D] fp32 residual, updated in place
  __nv_bfloat16* resid_bf;    // [B, D] bf16 copy of the residual (A operand of the score GEMM)
  unsigned long long* key;    // [B] argmax keys from the score GEMM; reset to 0 for the next one
  float* acts;                // [B, N] dense codes (row stride lda)
  int64_t lda;
  uint8_t* done;              // [B] 1 once the row has stopped
  int32_t* idx_out;           // [B] latent picked this iteration (-1 for stopped rows) or nullptr
  float* val_out;             // [B] value added this iteration (0 for stopped rows) or nullptr
  int32_t* n_active;          // += rows still running after this iteration
  const int32_t* rows;        // [B] row of `acts` / idx_out / val_out for each residual row, or nullptr
  int64_t n_out;              // rows of acts / idx_out / val_out (row-id bound)
  float thresh;               // residual-norm stop (<= 0: off)
  int stop_dup;               // stop when no new latent was added
  int B, D, N;
};

template <typename T>
__global__ void __launch_bounds__(32 * WARPS) step_kernel(StepArgs a, const T* __restrict__ W) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * WARPS + (threadIdx.x >> 5);
  bool running = false;
  // with `rows` the residual rows are a compacted subset: codes and the trace use the original row
  const int64_t orow = row < a.B ? (a.rows ? int64_t(a.rows[row]) : int64_t(row)) : -1;
  if (row < a.B && orow >= 0 && orow < a.n_out) {
    const unsigned long long k = a.key[row];
    __syncwarp();
    if (lane == 0) a.key[row] = 0ull;
    int i = -1;
    float v = 0.f;
    if (!a.done[row]) {
      i = key_index(k, a.N);
      float* r = a.resid + int64_t(row) * a.D;
      float rr = 0.f;
      if (i >= 0) {
        const T* w = W + int64_t(i) * a.D;
        float dot = 0.f;
        for (int d = 4 * lane; d < a.D; d += 128) {
          const float4 x = *reinterpret_cast<const float4*>(r + d);
          const float4 y = load4(w + d);
          dot += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
          rr += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        }
        dot = warp_sum(dot);
        v = dot > 0.f ? dot : 0.f;
        if (v > 0.f) {
          rr = 0.f;
          __nv_bfloat16* rb = a.resid_bf + int64_t(row) * a.D;
          for (int d = 4 * lane; d < a.D; d += 128) {
            float4 x = *reinterpret_cast<const float4*>(r + d);
            const float4 y = load4(w + d);
            x.x -= v * y.x;
            x.y -= v * y.y;
            x.z -= v * y.z;
            x.w -= v * y.w;
            *reinterpret_cast<float4*>(r + d) = x;
            rr += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
            const __nv_bfloat162 lo = __floats2bfloat162_rn(x.x, x.y);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(x.z, x.w);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&lo);
            u.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(rb + d) = u;
          }
        }
      } else {
        for (int d = 4 * lane; d < a.D; d += 128) {
          const float4 x = *reinterpret_cast<const float4*>(r + d);
          rr += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        }
      }
      rr = warp_sum(rr);
      if (lane == 0) {
        bool added = false;
        if (i >= 0) {
          float* c = a.acts + orow * a.lda + i;
          const float old = *c, now = old + v;
          *c = now;
          added = old == 0.f && now != 0.f;
        }
        const bool stop = (a.stop_dup && !added) || (a.thresh > 0.f && sqrtf(rr) < a.thresh);
        if (stop) a.done[row] = 1;
        running = !stop;
      }
    }
    if (lane == 0) {
      if (a.idx_out) a.idx_out[orow] = i;
      if (a.val_out) a.val_out[orow] = v;
    }
  }
  const int n = __syncthreads_count(running);
  if (threadIdx.x == 0 && n) atomicAdd(a.n_active, n);
}

struct BwdArgs {
  float* resid;               // [B, D] final residual on entry; walked back to the initial one
  float* g_resid;             // [B, D] zero on entry; gradient of the initial residual on exit
  const float* g_acts;        // [B, N] gradient of the dense codes (row stride ldg)
  int64_t ldg;
  const int32_t* idx;         // [T, B] recorded latents
  const float* val;           // [T, B] recorded values
  float* g_W;                 // [N, D] fp32 decoder gradient (atomic adds) or nullptr
  int T, B, D, N;
};

template <typename T>
__global__ void __launch_bounds__(32 * WARPS) bwd_kernel(BwdArgs a, const T* __restrict__ W) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= a.B) return;
  float* r = a.resid + int64_t(row) * a.D;
  float* G = a.g_resid + int64_t(row) * a.D;
  for (int t = a.T - 1; t >= 0; --t) {
    const float v = a.val[int64_t(t) * a.B + row];
    const int i = a.idx[int64_t(t) * a.B + row];
    if (!(v > 0.f) || i < 0 || i >= a.N) continue;  // nothing was added: no gradient flows here
    const T* w = W + int64_t(i) * a.D;
    float gd = 0.f;
    for (int d = 4 * lane; d < a.D; d += 128) {
      const float4 g = *reinterpret_cast<const float4*>(G + d);
      const float4 y = load4(w + d);
      gd += g.x * y.x + g.y * y.y + g.z * y.z + g.w * y.w;
    }
    gd = warp_sum(gd);
    const float gv = a.g_acts[int64_t(row) * a.ldg + i] - gd;
    float* gw = a.g_W ? a.g_W + int64_t(i) * a.D : nullptr;
    for (int d = 4 * lane; d < a.D; d += 128) {
      const float4 y = load4(w + d);
      float4 x = *reinterpret_cast<const float4*>(r + d);
      float4 g = *reinterpret_cast<const float4*>(G + d);
      x.x += v * y.x;
      x.y += v * y.y;
      x.z += v * y.z;
      x.w += v * y.w;
      if (gw)
        atomicAdd(reinterpret_cast<float4*>(gw + d),
                  make_float4(gv * x.x - v * g.x, gv * x.y - v * g.y, gv * x.z - v * g.z, gv * x.w - v * g.w));
      g.x += gv * y.x;
      g.y += gv * y.y;
      g.z += gv * y.z;
      g.w += gv * y.w;
      *reinterpret_cast<float4*>(r + d) = x;
      *reinterpret_cast<float4*>(G + d) = g;
    }
    __syncwarp();
  }
}

}  // namespace mp

static void check_rows(const torch::Tensor& t, at::ScalarType dt, int64_t B, int64_t D, const char* what) {
  SB_CHECK(t.is_cuda() && t.scalar_type() == dt && t.dim() == 2 && t.size(0) == B && t.size(1) == D &&
               t.is_contiguous() && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
           "mp: ", what, " must be a contiguous 16-byte aligned [", B, ", ", D, "] tensor of the expected dtype");
}

// One matching-pursuit update (after the score GEMM filled `key`).  W: [N, D] fp32 or bf16.
void mp_step(const torch::Tensor& resid, const torch::Tensor& resid_bf, const torch::Tensor& key,
             const torch::Tensor& acts, const torch::Tensor& done, const c10::optional<torch::Tensor>& idx_out,
             const c10::optional<torch::Tensor>& val_out, const torch::Tensor& n_active, const torch::Tensor& W,
             double thresh, bool stop_dup, const c10::optional<torch::Tensor>& rows) {
  const int64_t B = resid.size(0), D = resid.size(1), N = W.size(0);
  const int64_t n_out = acts.size(0);
  SB_CHECK(D % 8 == 0 && W.dim() == 2 && W.size(1) == D, "mp_step: D must be a multiple of 8 and W [N, D]");
  check_rows(resid, at::kFloat, B, D, "resid");
  check_rows(resid_bf, at::kBFloat16, B, D, "resid_bf");
  SB_CHECK(W.is_contiguous() && (W.scalar_type() == at::kFloat || W.scalar_type() == at::kBFloat16),
           "mp_step: W must be contiguous fp32 or bf16");
  SB_CHECK(key.scalar_type() == at::kLong && key.numel() == B && key.is_contiguous(), "mp_step: key int64 [B]");
  SB_CHECK(acts.scalar_type() == at::kFloat && acts.dim() == 2 && acts.size(1) == N && acts.stride(1) == 1 &&
               (rows ? n_out >= B : n_out == B),
           "mp_step: acts fp32 [rows, N] (as many rows as resid without `rows`)");
  if (rows) SB_CHECK(rows->is_cuda() && rows->scalar_type() == at::kInt && rows->numel() == B && rows->is_contiguous(),
                     "mp_step: rows int32 [B]");
  SB_CHECK(done.scalar_type() == at::kByte && done.numel() == B && done.is_contiguous(), "mp_step: done uint8 [B]");
  SB_CHECK(n_active.scalar_type() == at::kInt && n_active.numel() >= 1, "mp_step: n_active int32");
  if (idx_out) SB_CHECK(idx_out->scalar_type() == at::kInt && idx_out->numel() == n_out && idx_out->is_contiguous(),
                        "mp_step: idx_out int32 [acts rows]");
  if (val_out) SB_CHECK(val_out->scalar_type() == at::kFloat && val_out->numel() == n_out && val_out->is_contiguous(),
                        "mp_step: val_out fp32 [acts rows]");
  SB_CHECK(B < (1ll << 31) && N < (1ll << 31), "mp_step: size");
  const at::cuda::CUDAGuard guard(resid.device());
  mp::StepArgs a{};
  a.resid = resid.data_ptr<float>();
  a.resid_bf = reinterpret_cast<__nv_bfloat16*>(resid_bf.data_ptr());
  a.key = reinterpret_cast<unsigned long long*>(key.data_ptr());
  a.acts = acts.data_ptr<float>();
  a.lda = acts.stride(0);
  a.done = done.data_ptr<uint8_t>();
  a.idx_out = idx_out ? idx_out->data_ptr<int32_t>() : nullptr;
  a.val_out = val_out ? val_out->data_ptr<float>() : nullptr;
  a.n_active = n_active.data_ptr<int32_t>();
  a.rows = rows ? rows->data_ptr<int32_t>() : nullptr;
  a.n_out = n_out;
  a.thresh = float(thresh);
  a.stop_dup = stop_dup ? 1 : 0;
  a.B = int(B);
  a.D = int(D);
  a.N = int(N);
  if (B == 0) return;
  const dim3 grid(unsigned((B + mp::WARPS - 1) / mp::WARPS)), block(32 * mp::WARPS);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (W.scalar_type() == at::kFloat)
    mp::step_kernel<float><<<grid, block, 0, stream>>>(a, W.data_ptr<float>());
  else
    mp::step_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(
        a, reinterpret_cast<const __nv_bfloat16*>(W.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward of the recorded iterations (see the file comment).  `resid` (the final residual) and
// `g_resid` (zeros) are overwritten; `g_W` (fp32 [N, D], optional) is accumulated into.
void mp_backward(const torch::Tensor& resid, const torch::Tensor& g_resid, const torch::Tensor& g_acts,
                 const torch::Tensor& idx, const torch::Tensor& val, const c10::optional<torch::Tensor>& g_W,
                 const torch::Tensor& W) {
  const int64_t B = resid.size(0), D = resid.size(1), N = W.size(0);
  SB_CHECK(D % 8 == 0 && W.dim() == 2 && W.size(1) == D && W.is_contiguous() &&
               (W.scalar_type() == at::kFloat || W.scalar_type() == at::kBFloat16),
           "mp_backward: W must be contiguous fp32 or bf16 [N, D] with D % 8 == 0");
  check_rows(resid, at::kFloat, B, D, "resid");
  check_rows(g_resid, at::kFloat, B, D, "g_resid");
  SB_CHECK(g_acts.scalar_type() == at::kFloat && g_acts.dim() == 2 && g_acts.size(0) == B && g_acts.size(1) == N &&
               g_acts.stride(1) == 1,
           "mp_backward: g_acts fp32 [B, N]");
  SB_CHECK(idx.scalar_type() == at::kInt && val.scalar_type() == at::kFloat && idx.dim() == 2 && val.dim() == 2 &&
               idx.size(1) == B && val.size(1) == B && idx.size(0) == val.size(0) && idx.is_contiguous() &&
               val.is_contiguous(),
           "mp_backward: idx int32 / val fp32 [T, B]");
  if (g_W) check_rows(*g_W, at::kFloat, N, D, "g_W");
  const at::cuda::CUDAGuard guard(resid.device());
  mp::BwdArgs a{};
  a.resid = resid.data_ptr<float>();
  a.g_resid = g_resid.data_ptr<float>();
  a.g_acts = g_acts.data_ptr<float>();
  a.ldg = g_acts.stride(0);
  a.idx = idx.data_ptr<int32_t>();
  a.val = val.data_ptr<float>();
  a.g_W = g_W ? g_W->data_ptr<float>() : nullptr;
  a.T = int(idx.size(0));
  a.B = int(B);
  a.D = int(D);
  a.N = int(N);
  if (B == 0 || a.T == 0) return;
  const dim3 grid(unsigned((B + mp::WARPS - 1) / mp::WARPS)), block(32 * mp::WARPS);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (W.scalar_type() == at::kFloat)
    mp::bwd_kernel<float><<<grid, block, 0, stream>>>(a, W.data_ptr<float>());
  else
    mp::bwd_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(a,
                                                              reinterpret_cast<const __nv_bfloat16*>(W.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

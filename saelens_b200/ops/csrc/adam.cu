// Fused Adam for latent-major SAE parameters, with gradient clipping read from device memory.
//
// Replaces clip_grad_norm_(1.0) + torch.optim.Adam.step() over W_enc, W_dec, b_enc, b_dec
// (sae_lens/training/sae_trainer.py:743-755, sae_lens/saes/topk_sae.py:575-613).
//
// Layout: W_dec and W_enc^T are both [N, D] (one row per latent).  Each row keeps an fp32
// master copy plus fp32 exp_avg / exp_avg_sq, and a bf16 copy that the GEMMs read.  b_enc and
// b_dec are fp32 only.  Gradient rows exist only for latents that fired this step (colptr
// marks them); the others take a zero gradient, which still decays their moments exactly as
// torch.optim.Adam does.
//
// The row kernel also produces what the next forward needs, so no extra pass over the weights
// is made: scale[j] = ||bf16(W_dec[j])||, inv_scale[j] = 1/scale[j] and the folded bias
// bias_eff[j] = b_enc[j] - <bf16(W_enc[j]), b_dec>.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "check.h"

namespace sb {
namespace adam {

struct Hyper {
  float beta1, beta2, eps;
  float step_size;       // lr / (1 - beta1^t)
  float inv_sqrt_bc2;    // 1 / sqrt(1 - beta2^t)
  float max_norm;        // <= 0 disables clipping
};

__device__ __forceinline__ float clip_coef(const float* sumsq, float max_norm) {
  if (max_norm <= 0.f || sumsq == nullptr) return 1.f;
  const float norm = sqrtf(*sumsq);
  return fminf(max_norm / (norm + 1e-6f), 1.f);
}

// The quotient m / denom uses the fast division intrinsic (about 2 ulp; denom >= eps, far inside
// its range): under the power cap the row kernel runs at a low SM clock and becomes bound by its
// instruction issue, and the IEEE division is the longest sequence per element.
__device__ __forceinline__ float adam_update(float& p, float& m, float& v, float g, const Hyper& h) {
  m = m + (g - m) * (1.f - h.beta1);
  v = v * h.beta2 + (1.f - h.beta2) * g * g;
  const float denom = sqrtf(v) * h.inv_sqrt_bc2 + h.eps;
  p = p - h.step_size * __fdividef(m, denom);
  return p;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

// Single CTA: gb_dec = bsum - bterm; sumsq += |gb_dec|^2; clip; Adam on b_dec (fp32).
__global__ void bdec_kernel(const float* __restrict__ bsum, const float* __restrict__ bterm,
                            float* __restrict__ gb_dec, float* __restrict__ sumsq,
                            float* __restrict__ clip_out, float* __restrict__ p, float* __restrict__ m,
                            float* __restrict__ v, int D, Hyper h, int update) {
  __shared__ float red[32];
  float sq = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float g = (bsum ? bsum[d] : 0.f) - (bterm ? bterm[d] : 0.f);
    gb_dec[d] = g;
    sq += g * g;
  }
  const float tot = block_sum(sq, red);
  __shared__ float s_clip;
  if (threadIdx.x == 0) {
    if (sumsq) *sumsq += tot;
    s_clip = clip_coef(sumsq, h.max_norm);
    if (clip_out) *clip_out = s_clip;
  }
  __syncthreads();
  if (!update) return;
  const float c = s_clip;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float pp = p[d], mm = m[d], vv = v[d];
    adam_update(pp, mm, vv, gb_dec[d] * c, h);
    p[d] = pp;
    m[d] = mm;
    v[d] = vv;
  }
}

struct RowArgs {
  // per-row matrices [N, D]
  float *pd, *md, *vd;            // W_dec master / moments
  float *pe, *me, *ve;            // W_enc^T master / moments
  __nv_bfloat16 *wd, *we;         // bf16 copies (written)
  const __nv_bfloat16 *gd, *ge;   // gradients (valid only where the row fired)
  // per-row vectors [N]
  float *pb, *mb, *vb;            // b_enc master / moments
  const float* gb;                // b_enc gradient
  const int64_t* colptr;          // [N+1]: row j has a gradient iff colptr[j+1] > colptr[j]
  const float* clip;              // device scalar written by bdec_kernel (or nullptr)
  const float* b_dec;             // [D] updated b_dec (for bias_eff)
  float *scale, *inv_scale, *bias_eff;  // outputs for the next forward (nullable)
  int N, D;
  int update;                     // 0: only recompute scale / bias_eff
};

constexpr int ROW_THREADS = 256;  // 8 warps, one latent row per warp
constexpr int ROW_UNROLL = 2;

__device__ __forceinline__ void unpack_g(const uint2& gr, float c, float* g) {
  const __nv_bfloat162* g2p = reinterpret_cast<const __nv_bfloat162*>(&gr);
  const float2 x = __bfloat1622float2(g2p[0]), y = __bfloat1622float2(g2p[1]);
  g[0] = x.x * c;
  g[1] = x.y * c;
  g[2] = y.x * c;
  g[3] = y.y * c;
}

// One warp per latent row.  Each iteration first issues every load of ROW_UNROLL 16-byte groups of
// both matrices (master, m, v, gradient), then does the math and the stores, so a thread keeps
// 2 * ROW_UNROLL * 56 bytes in flight instead of one group's worth.
__global__ void __launch_bounds__(ROW_THREADS) rows_kernel(RowArgs a, Hyper h) {
  const float c = (a.update && a.clip) ? *a.clip : 1.f;
  const int nv4 = a.D >> 2;
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (ROW_THREADS / 32);
  float* const Pm[2] = {a.pd, a.pe};
  float* const Mm[2] = {a.md, a.me};
  float* const Vm[2] = {a.vd, a.ve};
  __nv_bfloat16* const Wm[2] = {a.wd, a.we};
  const __nv_bfloat16* const Gm[2] = {a.gd, a.ge};
  for (int j = blockIdx.x * (ROW_THREADS / 32) + (threadIdx.x >> 5); j < a.N; j += warps_total) {
    const bool has_g = a.update && a.colptr && (a.colptr[j + 1] > a.colptr[j]);
    const int64_t base = int64_t(j) * a.D;
    float nrm = 0.f, dot = 0.f;
    for (int s0 = lane; s0 < nv4; s0 += 32 * ROW_UNROLL) {
      float4 P[2][ROW_UNROLL], M[2][ROW_UNROLL], V[2][ROW_UNROLL];
      uint2 G[2][ROW_UNROLL];
#pragma unroll
      for (int u = 0; u < ROW_UNROLL; ++u) {
        const int s = s0 + 32 * u;
        if (s < nv4) {
          const int64_t off = base + 4 * int64_t(s);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            P[t][u] = __ldcs(reinterpret_cast<const float4*>(Pm[t] + off));
            if (a.update) {
              M[t][u] = __ldcs(reinterpret_cast<const float4*>(Mm[t] + off));
              V[t][u] = __ldcs(reinterpret_cast<const float4*>(Vm[t] + off));
            }
            G[t][u] = has_g ? __ldcs(reinterpret_cast<const uint2*>(Gm[t] + off)) : make_uint2(0, 0);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < ROW_UNROLL; ++u) {
        const int s = s0 + 32 * u;
        if (s >= nv4) continue;
        const int64_t off = base + 4 * int64_t(s);
        float4 bd = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.b_dec) bd = __ldg(reinterpret_cast<const float4*>(a.b_dec) + s);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          float4 p = P[t][u];
          if (a.update) {
            float4 m = M[t][u], v = V[t][u];
            float g[4];
            unpack_g(G[t][u], c, g);
            adam_update(p.x, m.x, v.x, g[0], h);
            adam_update(p.y, m.y, v.y, g[1], h);
            adam_update(p.z, m.z, v.z, g[2], h);
            adam_update(p.w, m.w, v.w, g[3], h);
            __stcs(reinterpret_cast<float4*>(Pm[t] + off), p);
            __stcs(reinterpret_cast<float4*>(Mm[t] + off), m);
            __stcs(reinterpret_cast<float4*>(Vm[t] + off), v);
          }
          const __nv_bfloat162 lo = __floats2bfloat162_rn(p.x, p.y), hi = __floats2bfloat162_rn(p.z, p.w);
          uint2 o;
          o.x = *reinterpret_cast<const uint32_t*>(&lo);
          o.y = *reinterpret_cast<const uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(Wm[t] + off) = o;  // read by the next GEMM: keep in L2
          const float2 x = __bfloat1622float2(lo), y = __bfloat1622float2(hi);
          if (t == 0) nrm += x.x * x.x + x.y * x.y + y.x * y.x + y.y * y.y;
          else dot += x.x * bd.x + x.y * bd.y + y.x * bd.z + y.y * bd.w;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      nrm += __shfl_xor_sync(0xffffffffu, nrm, o);
      dot += __shfl_xor_sync(0xffffffffu, dot, o);
    }
    if (lane == 0) {
      float pb = a.pb[j];
      if (a.update) {
        float mb = a.mb[j], vb = a.vb[j];
        const float g = has_g ? a.gb[j] * c : 0.f;
        adam_update(pb, mb, vb, g, h);
        a.pb[j] = pb;
        a.mb[j] = mb;
        a.vb[j] = vb;
      }
      const float nr = sqrtf(nrm);
      if (a.scale) a.scale[j] = nr;
      if (a.inv_scale) a.inv_scale[j] = 1.f / nr;
      if (a.bias_eff) a.bias_eff[j] = pb - dot;
    }
  }
}

}  // namespace adam

static int sm_count_adam() {
  int dev, n;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

static adam::Hyper make_hyper(double lr, double beta1, double beta2, double eps, int64_t step,
                              double max_norm) {
  adam::Hyper h;
  h.beta1 = float(beta1);
  h.beta2 = float(beta2);
  h.eps = float(eps);
  const double bc1 = 1.0 - std::pow(beta1, double(step));
  const double bc2 = 1.0 - std::pow(beta2, double(step));
  h.step_size = float(lr / bc1);
  h.inv_sqrt_bc2 = float(1.0 / std::sqrt(bc2));
  h.max_norm = float(max_norm);
  return h;
}

// b_dec gradient + clip coefficient (+ optional b_dec Adam step).
void adam_bdec(const c10::optional<torch::Tensor>& bsum, const c10::optional<torch::Tensor>& bterm,
               const torch::Tensor& gb_dec, const c10::optional<torch::Tensor>& sumsq,
               const c10::optional<torch::Tensor>& clip_out, const torch::Tensor& p, const torch::Tensor& m,
               const torch::Tensor& v, double lr, double beta1, double beta2, double eps, int64_t step,
               double max_norm, bool update) {
  const at::cuda::CUDAGuard guard(p.device());
  const int D = int(p.numel());
  adam::bdec_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      bsum ? bsum->data_ptr<float>() : nullptr, bterm ? bterm->data_ptr<float>() : nullptr,
      gb_dec.data_ptr<float>(), sumsq ? sumsq->data_ptr<float>() : nullptr,
      clip_out ? clip_out->data_ptr<float>() : nullptr, p.data_ptr<float>(), m.data_ptr<float>(),
      v.data_ptr<float>(), D, make_hyper(lr, beta1, beta2, eps, std::max<int64_t>(step, 1), max_norm),
      update ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Row-fused Adam over W_dec / W_enc^T / b_enc.  With update=false it only refreshes the bf16
// copies, scale, inv_scale and bias_eff from the fp32 masters (used after loading weights).
void adam_rows(const torch::Tensor& pd, const torch::Tensor& md, const torch::Tensor& vd,
               const torch::Tensor& pe, const torch::Tensor& me, const torch::Tensor& ve,
               const torch::Tensor& wd, const torch::Tensor& we,
               const c10::optional<torch::Tensor>& gd, const c10::optional<torch::Tensor>& ge,
               const torch::Tensor& pb, const torch::Tensor& mb, const torch::Tensor& vb,
               const c10::optional<torch::Tensor>& gb, const c10::optional<torch::Tensor>& colptr,
               const c10::optional<torch::Tensor>& clip, const c10::optional<torch::Tensor>& b_dec,
               const c10::optional<torch::Tensor>& scale, const c10::optional<torch::Tensor>& inv_scale,
               const c10::optional<torch::Tensor>& bias_eff, double lr, double beta1, double beta2,
               double eps, int64_t step, bool update) {
  const at::cuda::CUDAGuard guard(pd.device());
  SB_CHECK(pd.is_contiguous() && pe.is_contiguous() && wd.is_contiguous() && we.is_contiguous(),
              "adam_rows: contiguous params required");
  const int64_t N = pd.size(0), D = pd.size(1);
  SB_CHECK(D % 4 == 0, "adam_rows: d_in must be a multiple of 4");
  adam::RowArgs a{};
  a.pd = pd.data_ptr<float>(); a.md = md.data_ptr<float>(); a.vd = vd.data_ptr<float>();
  a.pe = pe.data_ptr<float>(); a.me = me.data_ptr<float>(); a.ve = ve.data_ptr<float>();
  a.wd = reinterpret_cast<__nv_bfloat16*>(wd.data_ptr());
  a.we = reinterpret_cast<__nv_bfloat16*>(we.data_ptr());
  a.gd = gd ? reinterpret_cast<const __nv_bfloat16*>(gd->data_ptr()) : nullptr;
  a.ge = ge ? reinterpret_cast<const __nv_bfloat16*>(ge->data_ptr()) : nullptr;
  a.pb = pb.data_ptr<float>(); a.mb = mb.data_ptr<float>(); a.vb = vb.data_ptr<float>();
  a.gb = gb ? gb->data_ptr<float>() : nullptr;
  a.colptr = colptr ? colptr->data_ptr<int64_t>() : nullptr;
  a.clip = clip ? clip->data_ptr<float>() : nullptr;
  a.b_dec = b_dec ? b_dec->data_ptr<float>() : nullptr;
  a.scale = scale ? scale->data_ptr<float>() : nullptr;
  a.inv_scale = inv_scale ? inv_scale->data_ptr<float>() : nullptr;
  a.bias_eff = bias_eff ? bias_eff->data_ptr<float>() : nullptr;
  a.N = int(N);
  a.D = int(D);
  a.update = update ? 1 : 0;
  SB_CHECK(!update || (a.gd && a.ge && a.gb && a.colptr), "adam_rows: gradients required for update");
  if (N == 0) return;
  const int64_t grid = std::min<int64_t>((N + 7) / 8, int64_t(sm_count_adam()) * 8);
  adam::rows_kernel<<<dim3(grid), dim3(adam::ROW_THREADS), 0, at::cuda::getCurrentCUDAStream()>>>(
      a, make_hyper(lr, beta1, beta2, eps, std::max<int64_t>(step, 1), 0.0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

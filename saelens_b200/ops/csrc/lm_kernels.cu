// Producer-LM elementwise kernels (the activation-capture forward runs on these plus the tcgen05
// GEMM): RMSNorm, rotary position embedding applied in place, and the gated-MLP activation.
//
//  rmsnorm:   y = x * rsqrt(mean(x^2) + eps) * (w or 1 + w), fp32 math, one CTA per row,
//             16-byte vectors; bf16 or fp32 rows.
//  rope:      rotate-half convention (pairs (i, i + d/2)), cos/sin tables [S, d/2] fp32,
//             x [B, S, H, d] bf16 with a contiguous last dimension, in place.
//  gated_act: h = act(gate) * up with act SiLU (x * sigmoid(x)) or tanh-GELU
//             (0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), Hendrycks & Gimpel).
//  layernorm: y = (x - mean) * rsqrt(var + eps) * w + b (biased variance, fp32 math), one CTA per
//             row; the row is summed once for the mean and once for the centred squares.
//  embed:     y[t] = table[tokens[t]] * scale (+ pos[t mod S] for learned positions), one CTA per
//             token row, 16-byte vectors; out-of-range token ids give a zero row and a flag.
// Reference sites: the producer LM forward (HookedTransformer / vLLM layers) that
// sae_lens/vllm_model.py and load_model.py drive.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>
#include "check.h"

namespace sb {
namespace lm {

constexpr int NORM_THREADS = 256;

template <class T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* f) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(h[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float* f) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float* f) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* f) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
};

template <class T>
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const T* __restrict__ x, int64_t ldx,
                                                               const T* __restrict__ w, T* __restrict__ y,
                                                               int64_t ldy, int D, float eps, int one_plus) {
  __shared__ float red[NORM_THREADS / 32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  const int nvec = D / 8;
  float ss = 0.f;
  for (int v = threadIdx.x; v < nvec; v += NORM_THREADS) {
    float f[8];
    Vec8<T>::load(xr + 8 * v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NORM_THREADS / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / float(D) + eps);
  for (int v = threadIdx.x; v < nvec; v += NORM_THREADS) {
    float f[8], g[8];
    Vec8<T>::load(xr + 8 * v, f);
    Vec8<T>::load(w + 8 * v, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = f[j] * inv * (one_plus ? 1.f + g[j] : g[j]);
    Vec8<T>::store(y + row * ldy + 8 * v, f);
  }
}

// One thread per (row position, head, pair i < d/2).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, int64_t sb, int64_t ss, int64_t sh, int B, int S, int H,
                            int d, const float* __restrict__ cosv, const float* __restrict__ sinv, int64_t pos0) {
  const int half = d / 2;
  const int64_t total = int64_t(B) * S * H * half;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int i = int(e % half);
    int64_t r = e / half;
    const int h = int(r % H);
    r /= H;
    const int s = int(r % S);
    const int b = int(r / S);
    __nv_bfloat16* p = x + b * sb + s * ss + h * sh;
    const float c = cosv[(pos0 + s) * half + i], sn = sinv[(pos0 + s) * half + i];
    const float x1 = __bfloat162float(p[i]), x2 = __bfloat162float(p[i + half]);
    p[i] = __float2bfloat16_rn(x1 * c - x2 * sn);
    p[i + half] = __float2bfloat16_rn(x2 * c + x1 * sn);
  }
}

__device__ __forceinline__ float act_fn(float x, int kind) {
  if (kind == 0) return x / (1.f + expf(-x));  // SiLU
  const float k0 = 0.7978845608028654f;        // sqrt(2 / pi)
  return 0.5f * x * (1.f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

// gate / up rows may be strided (views of one fused [rows, 2 * width] projection output).
__global__ void gated_act_kernel(const __nv_bfloat16* __restrict__ gate, int64_t ldg,
                                 const __nv_bfloat16* __restrict__ up, int64_t ldu, __nv_bfloat16* __restrict__ out,
                                 int64_t rows, int width8, int kind) {
  const int64_t n8 = rows * width8;
  for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < n8; v += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = v / width8, c = v - r * width8;
    float g[8], u[8];
    Vec8<__nv_bfloat16>::load(gate + r * ldg + 8 * c, g);
    Vec8<__nv_bfloat16>::load(up + r * ldu + 8 * c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = act_fn(g[j], kind) * u[j];
    Vec8<__nv_bfloat16>::store(out + 8 * v, g);
  }
}

template <class T>
__global__ void __launch_bounds__(NORM_THREADS) layernorm_kernel(const T* __restrict__ x, int64_t ldx,
                                                                 const T* __restrict__ w, const T* __restrict__ bias,
                                                                 T* __restrict__ y, int64_t ldy, int D, float eps) {
  __shared__ float red[NORM_THREADS / 32];
  __shared__ float bcast;
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  const int nvec = D / 8;
  auto block_sum = [&](float v) -> float {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < NORM_THREADS / 32; ++i) t += red[i];
      bcast = t;
    }
    __syncthreads();
    return bcast;
  };
  float s1 = 0.f;
  for (int v = threadIdx.x; v < nvec; v += NORM_THREADS) {
    float f[8];
    Vec8<T>::load(xr + 8 * v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s1 += f[j];
  }
  const float mean = block_sum(s1) / float(D);
  float s2 = 0.f;
  for (int v = threadIdx.x; v < nvec; v += NORM_THREADS) {
    float f[8];
    Vec8<T>::load(xr + 8 * v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s2 += (f[j] - mean) * (f[j] - mean);
  }
  const float inv = rsqrtf(block_sum(s2) / float(D) + eps);
  for (int v = threadIdx.x; v < nvec; v += NORM_THREADS) {
    float f[8], g[8], bb[8];
    Vec8<T>::load(xr + 8 * v, f);
    Vec8<T>::load(w + 8 * v, g);
    if (bias) Vec8<T>::load(bias + 8 * v, bb);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = (f[j] - mean) * inv * g[j] + (bias ? bb[j] : 0.f);
    Vec8<T>::store(y + row * ldy + 8 * v, f);
  }
}

template <class T>
__global__ void __launch_bounds__(NORM_THREADS) embed_kernel(const int64_t* __restrict__ tokens, int64_t n, int S,
                                                             const T* __restrict__ table, int64_t vocab,
                                                             const T* __restrict__ pos, float scale, int D,
                                                             T* __restrict__ y, int* __restrict__ bad) {
  const int64_t t = blockIdx.x;
  const int64_t tok = tokens[t];
  const bool ok = tok >= 0 && tok < vocab;
  if (!ok && threadIdx.x == 0) atomicExch(bad, 1);
  const int nvec = D / 8;
  for (int v = threadIdx.x; v < nvec; v += NORM_THREADS) {
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (ok) {
      Vec8<T>::load(table + tok * D + 8 * v, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] *= scale;
    }
    if (pos) {
      float pp[8];
      Vec8<T>::load(pos + int64_t(t % S) * D + 8 * v, pp);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] += pp[j];
    }
    Vec8<T>::store(y + t * D + 8 * v, f);
  }
}

}  // namespace lm

static int lm_sm_count() {
  int dev = 0, n = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

// y = rmsnorm(x) * (w or 1 + w); x [M, D] (bf16 or fp32, contiguous rows), returns a new tensor.
torch::Tensor rmsnorm(const torch::Tensor& x, const torch::Tensor& w, double eps, bool one_plus) {
  SB_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "rmsnorm: CUDA [M, D] with contiguous rows");
  SB_CHECK(x.scalar_type() == w.scalar_type() && (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat),
              "rmsnorm: x and w must both be bf16 or fp32");
  const int64_t M = x.size(0), D = x.size(1);
  SB_CHECK(D % 8 == 0 && w.numel() == D && w.is_contiguous(), "rmsnorm: D % 8 and w [D]");
  SB_CHECK(x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "rmsnorm: alignment");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({M, D}, x.options());
  if (M == 0) return y;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16)
    lm::rmsnorm_kernel<__nv_bfloat16><<<dim3(M), dim3(lm::NORM_THREADS), 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), D,
        int(D), float(eps), one_plus ? 1 : 0);
  else
    lm::rmsnorm_kernel<float><<<dim3(M), dim3(lm::NORM_THREADS), 0, stream>>>(
        x.data_ptr<float>(), x.stride(0), w.data_ptr<float>(), y.data_ptr<float>(), D, int(D), float(eps),
        one_plus ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// y = layernorm(x) * w + b; x [M, D] (bf16 or fp32, contiguous rows), w / b [D] of x's dtype.
torch::Tensor layernorm(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& b,
                        double eps) {
  SB_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "layernorm: CUDA [M, D] with contiguous rows");
  SB_CHECK(x.scalar_type() == w.scalar_type() && (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat),
              "layernorm: x and w must both be bf16 or fp32");
  const int64_t M = x.size(0), D = x.size(1);
  SB_CHECK(D % 8 == 0 && w.numel() == D && w.is_contiguous(), "layernorm: D % 8 and w [D]");
  if (b) SB_CHECK(b->scalar_type() == x.scalar_type() && b->numel() == D && b->is_contiguous(), "layernorm: b [D]");
  SB_CHECK(x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "layernorm: alignment");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({M, D}, x.options());
  if (M == 0) return y;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16)
    lm::layernorm_kernel<__nv_bfloat16><<<dim3(M), dim3(lm::NORM_THREADS), 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        b ? reinterpret_cast<const __nv_bfloat16*>(b->data_ptr()) : nullptr,
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), D, int(D), float(eps));
  else
    lm::layernorm_kernel<float><<<dim3(M), dim3(lm::NORM_THREADS), 0, stream>>>(
        x.data_ptr<float>(), x.stride(0), w.data_ptr<float>(), b ? b->data_ptr<float>() : nullptr,
        y.data_ptr<float>(), D, int(D), float(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// y[b, s] = table[tokens[b, s]] * scale (+ pos[s]); tokens int64 [B, S], table [vocab, D] and pos
// [>= S, D] of one dtype (bf16 or fp32).  An out-of-range token id gives a zero row and sets
// `bad` (int32 on the device) to 1.
torch::Tensor embed(const torch::Tensor& tokens, const torch::Tensor& table, double scale,
                    const c10::optional<torch::Tensor>& pos, const torch::Tensor& bad) {
  SB_CHECK(tokens.is_cuda() && tokens.scalar_type() == at::kLong && tokens.dim() == 2 && tokens.is_contiguous(),
              "embed: tokens must be contiguous CUDA int64 [B, S]");
  SB_CHECK(table.dim() == 2 && table.is_contiguous() && table.size(1) % 8 == 0 &&
                  (table.scalar_type() == at::kBFloat16 || table.scalar_type() == at::kFloat),
              "embed: table must be contiguous bf16/fp32 [vocab, D] with D % 8 == 0");
  const int64_t B = tokens.size(0), S = tokens.size(1), D = table.size(1);
  if (pos)
    SB_CHECK(pos->scalar_type() == table.scalar_type() && pos->is_contiguous() && pos->size(1) == D &&
                    pos->size(0) >= S,
                "embed: pos must be [>= S, D] like the table");
  SB_CHECK(bad.is_cuda() && bad.scalar_type() == at::kInt && bad.numel() >= 1, "embed: bad flag");
  const at::cuda::CUDAGuard guard(tokens.device());
  auto y = torch::empty({B, S, D}, table.options());
  if (B * S == 0) return y;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (table.scalar_type() == at::kBFloat16)
    lm::embed_kernel<__nv_bfloat16><<<dim3(B * S), dim3(lm::NORM_THREADS), 0, stream>>>(
        tokens.data_ptr<int64_t>(), B * S, int(S), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
        table.size(0), pos ? reinterpret_cast<const __nv_bfloat16*>(pos->data_ptr()) : nullptr, float(scale), int(D),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), bad.data_ptr<int>());
  else
    lm::embed_kernel<float><<<dim3(B * S), dim3(lm::NORM_THREADS), 0, stream>>>(
        tokens.data_ptr<int64_t>(), B * S, int(S), table.data_ptr<float>(), table.size(0),
        pos ? pos->data_ptr<float>() : nullptr, float(scale), int(D), y.data_ptr<float>(), bad.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// In-place rotary embedding on x [B, S, H, d] bf16 (last dim contiguous) with tables [>= pos0+S, d/2].
void rope_(const torch::Tensor& x, const torch::Tensor& cos, const torch::Tensor& sin, int64_t pos0) {
  SB_CHECK(x.is_cuda() && x.dim() == 4 && x.stride(3) == 1 && x.scalar_type() == at::kBFloat16,
              "rope_: x must be CUDA bf16 [B, S, H, d] with a contiguous last dim");
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2), d = x.size(3);
  SB_CHECK(d % 2 == 0 && cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat &&
                  cos.is_contiguous() && sin.is_contiguous() && cos.size(-1) == d / 2 && cos.size(0) >= pos0 + S &&
                  sin.sizes() == cos.sizes(),
              "rope_: tables must be fp32 [positions, d/2]");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t total = B * S * H * (d / 2);
  if (total == 0) return;
  const int64_t grid = std::min<int64_t>((total + 255) / 256, int64_t(lm_sm_count()) * 16);
  lm::rope_kernel<<<dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), x.stride(1), x.stride(2), int(B), int(S), int(H),
      int(d), cos.data_ptr<float>(), sin.data_ptr<float>(), pos0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// act(gate) * up for bf16 tensors of equal shape [..., width] whose rows are contiguous (the rows
// themselves may be strided, e.g. halves of a fused gate/up projection); kind 0 = SiLU,
// 1 = tanh-GELU.  Returns a contiguous tensor.
torch::Tensor gated_act(const torch::Tensor& gate, const torch::Tensor& up, int64_t kind) {
  SB_CHECK(gate.is_cuda() && gate.scalar_type() == at::kBFloat16 && up.scalar_type() == at::kBFloat16 &&
                  gate.sizes() == up.sizes() && gate.dim() >= 1,
              "gated_act: bf16 CUDA tensors of equal shape");
  SB_CHECK(kind == 0 || kind == 1, "gated_act: kind 0 (SiLU) or 1 (tanh-GELU)");
  const int64_t width = gate.size(-1);
  const int64_t rows = width ? gate.numel() / width : 0;
  auto g2 = gate.reshape({rows, width});
  auto u2 = up.reshape({rows, width});
  SB_CHECK(width % 8 == 0 && g2.stride(1) == 1 && u2.stride(1) == 1 && g2.stride(0) % 8 == 0 &&
                  u2.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(g2.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(u2.data_ptr()) % 16 == 0,
              "gated_act: rows must be contiguous, 16-byte aligned, width % 8 == 0");
  const at::cuda::CUDAGuard guard(gate.device());
  auto out = torch::empty(gate.sizes(), gate.options().memory_format(at::MemoryFormat::Contiguous));
  const int64_t n8 = rows * (width / 8);
  if (n8 == 0) return out;
  const int64_t grid = std::min<int64_t>((n8 + 255) / 256, int64_t(lm_sm_count()) * 16);
  lm::gated_act_kernel<<<dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g2.data_ptr()), g2.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(u2.data_ptr()), u2.stride(0),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, int(width / 8), int(kind));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace sb

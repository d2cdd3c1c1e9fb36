// Sparse (k-active) decode, MSE, latent-major (CSC) gradient assembly for TopK-family SAEs.
//
// Reference path being replaced (sae_lens/saes/topk_sae.py:645-674, sae.py:986-996):
//   feature_acts = scatter(relu(topk(hidden_pre)))            # dense [B, d_sae]
//   sae_out      = (feature_acts / ||W_dec||) @ W_dec + b_dec  # dense GEMM, B x d_sae x d_in
//   mse          = ((sae_out - x)^2).sum(-1).mean()
//   backward: dense GEMMs for dW_dec, dFeature, dW_enc and dSaeIn.
// Here every product touches only the k selected latents of each row:
//   decode:  x_hat[b] = sum_i a[b,i] W_dec[idx[b,i]] + b_dec,   a = relu(h) / ||W_dec||
//   grads:   for each latent j over the rows b that selected it (CSC lists)
//              gW_dec[j] = sum_b a[b,j] dXhat[b]
//              dz[b,j]   = <dXhat[b], W_dec[j]> * 1[a>0]
//              gW_enc[j] = sum_b dz[b,j] (x[b] - b_dec),   gb_enc[j] = sum_b dz[b,j]
//            (the ||W_dec|| factors cancel exactly between the top-k rescale and the decode)
//   b_dec:   gb_dec = sum_b dXhat[b] - sum_j gb_enc[j] W_enc[j]
// An auxiliary pair list (dead-latent aux-k loss) uses raw coefficients h/||W_dec|| (no ReLU)
// and its own residual-gradient rows; it is merged into the same CSC pass.
#include <ATen/cuda/CUDAContext.h>
#include <cstdlib>
#include <string>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "p2p.cuh"
#include "check.h"
#include "bounds.cuh"

namespace sb {
namespace sparse {

constexpr int DEC_THREADS = 128;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float* f) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    w[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
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

// ---------------------------------------------------------------------------------------
// decode + MSE.  One CTA per row (grid-stride).  VPT = 8-element vectors per thread.
//   coef mode: relu=1 -> a = relu(val) * inv_scale[idx]; relu=0 -> a = val * inv_scale[idx]
//   err = x_hat - target;  dxhat = err * grad_coef;  loss_row[b] = sum err^2
//   bsum (optional, fp32 [D]) += sum_b dxhat[b]   (for the b_dec gradient)
// ---------------------------------------------------------------------------------------
template <int VPT>
__global__ void __launch_bounds__(DEC_THREADS)
    decode_mse_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int k,
                      int64_t ldk, int relu, const float* __restrict__ inv_scale,
                      const __nv_bfloat16* __restrict__ W, int64_t ldw,
                      const float* __restrict__ bias, const __nv_bfloat16* __restrict__ target,
                      int64_t ldt, __nv_bfloat16* __restrict__ out, int64_t ldo,
                      __nv_bfloat16* __restrict__ resid, int64_t ldr,
                      __nv_bfloat16* __restrict__ dxhat, int64_t ldd, const float* grad_coef_dev,
                      float grad_coef, float* __restrict__ loss_row, float* __restrict__ bsum,
                      int M, int D, int n_lat) {
  extern __shared__ float dsm[];
  float* s_a = dsm;                                  // k
  int* s_i = reinterpret_cast<int*>(dsm + k);        // k
  float* red = dsm + 2 * k;                          // 32
  const int nvec = D >> 3;
  const int t = threadIdx.x;
  float bacc[VPT][8];
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int e = 0; e < 8; ++e) bacc[v][e] = 0.f;
  const float gcoef = grad_coef_dev ? grad_coef * __ldg(grad_coef_dev) : grad_coef;

  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    __syncthreads();
    for (int i = t; i < k; i += DEC_THREADS) {
      const int j = idx[int64_t(row) * ldk + i];
      float a = 0.f;
      if (j >= 0 && SB_IN_RANGE(j, n_lat)) {
        const float v = vals[int64_t(row) * ldk + i];
        a = (relu ? fmaxf(v, 0.f) : v) * (inv_scale ? __ldg(inv_scale + j) : 1.f);
      }
      s_a[i] = a;
      s_i[i] = (a != 0.f) ? j : -1;
    }
    __syncthreads();
    float acc[VPT][8];
#pragma unroll
    for (int v = 0; v < VPT; ++v)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[v][e] = 0.f;
    constexpr int U = 4;  // selected latents whose rows are in flight together
    int i = 0;
    for (; i + U <= k; i += U) {
      int jj[U];
      float aa[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        jj[u] = s_i[i + u];
        aa[u] = s_a[i + u];
      }
      uint4 w[U][VPT];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int vi = t + v * DEC_THREADS;
          w[u][v] = (jj[u] >= 0 && vi < nvec)
                        ? __ldg(reinterpret_cast<const uint4*>(W + int64_t(jj[u]) * ldw) + vi)
                        : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          float f[8];
          bf16x8_to_f32(w[u][v], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[v][e] += aa[u] * f[e];
        }
    }
    for (; i < k; ++i) {
      const int j0 = s_i[i];
      if (j0 < 0) continue;
      const float a0 = s_a[i];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int vi = t + v * DEC_THREADS;
        if (vi < nvec) {
          float f0[8];
          bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(W + int64_t(j0) * ldw) + vi), f0);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[v][e] += a0 * f0[e];
        }
      }
    }
    float lsum = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * DEC_THREADS;
      if (vi >= nvec) continue;
      float xh[8], tg[8];
      if (bias) {
        const float4* b4 = reinterpret_cast<const float4*>(bias) + 2 * vi;
        const float4 b0 = __ldg(b4), b1 = __ldg(b4 + 1);
        xh[0] = acc[v][0] + b0.x; xh[1] = acc[v][1] + b0.y; xh[2] = acc[v][2] + b0.z; xh[3] = acc[v][3] + b0.w;
        xh[4] = acc[v][4] + b1.x; xh[5] = acc[v][5] + b1.y; xh[6] = acc[v][6] + b1.z; xh[7] = acc[v][7] + b1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) xh[e] = acc[v][e];
      }
      if (out) reinterpret_cast<uint4*>(out + int64_t(row) * ldo)[vi] = f32_to_bf16x8(xh);
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(target + int64_t(row) * ldt) + vi), tg);
      float err[8], g[8], rs[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        err[e] = xh[e] - tg[e];
        lsum += err[e] * err[e];
        g[e] = err[e] * gcoef;
        rs[e] = -err[e];
      }
      if (resid) reinterpret_cast<uint4*>(resid + int64_t(row) * ldr)[vi] = f32_to_bf16x8(rs);
      if (dxhat) {
        const uint4 gq = f32_to_bf16x8(g);
        reinterpret_cast<uint4*>(dxhat + int64_t(row) * ldd)[vi] = gq;
        if (bsum) {
          float gr[8];
          bf16x8_to_f32(gq, gr);  // sum exactly what the latent gradients consume
#pragma unroll
          for (int e = 0; e < 8; ++e) bacc[v][e] += gr[e];
        }
      }
    }
    const float tot = block_sum(lsum, red);
    if (t == 0 && loss_row) loss_row[row] = tot;
  }
  if (bsum) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * DEC_THREADS;
      if (vi < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) atomicAdd(bsum + 8 * vi + e, bacc[v][e]);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Tensor-parallel pieces of the decode.  `decode_partial` writes this rank's partial
// reconstruction sum_i a_i W_dec[idx_i] (fp32, no bias) for every row; after the partials are
// reduce-scattered, `finish_mse` adds b_dec and produces the loss, dL/dx_hat, the residual and
// the column sum for the b_dec gradient on this rank's rows.
// ---------------------------------------------------------------------------------------
// acc = sum_i a_i W[idx_i] for one row (no bias): coefficients are staged in s_a / s_i
// (k floats + k ints of shared memory); the caller owns the barriers around reuse of s_a/s_i.
template <int VPT>
__device__ __forceinline__ void decode_row_partial(int row, const float* __restrict__ vals,
                                                   const int* __restrict__ idx, int k, int64_t ldk, int relu,
                                                   const float* __restrict__ inv_scale,
                                                   const __nv_bfloat16* __restrict__ W, int64_t ldw, int n_lat,
                                                   int nvec, float* s_a, int* s_i, float (&acc)[VPT][8]) {
  const int t = threadIdx.x;
  __syncthreads();
  for (int i = t; i < k; i += DEC_THREADS) {
    const int j = idx[int64_t(row) * ldk + i];
    float a = 0.f;
    if (j >= 0 && SB_IN_RANGE(j, n_lat)) {
      const float v = vals[int64_t(row) * ldk + i];
      a = (relu ? fmaxf(v, 0.f) : v) * (inv_scale ? __ldg(inv_scale + j) : 1.f);
    }
    s_a[i] = a;
    s_i[i] = (a != 0.f) ? j : -1;
  }
  __syncthreads();
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[v][e] = 0.f;
  constexpr int U = 4;
  int i = 0;
  for (; i + U <= k; i += U) {
    uint4 w[U][VPT];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int jj = s_i[i + u];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int vi = t + v * DEC_THREADS;
        w[u][v] = (jj >= 0 && vi < nvec) ? __ldg(reinterpret_cast<const uint4*>(W + int64_t(jj) * ldw) + vi)
                                         : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float aa = s_a[i + u];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        float f[8];
        bf16x8_to_f32(w[u][v], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[v][e] += aa * f[e];
      }
    }
  }
  for (; i < k; ++i) {
    const int jj = s_i[i];
    if (jj < 0) continue;
    const float aa = s_a[i];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * DEC_THREADS;
      if (vi < nvec) {
        float f[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(W + int64_t(jj) * ldw) + vi), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[v][e] += aa * f[e];
      }
    }
  }
}

template <int VPT>
__global__ void __launch_bounds__(DEC_THREADS)
    decode_partial_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int k, int64_t ldk,
                          int relu, const float* __restrict__ inv_scale, const __nv_bfloat16* __restrict__ W,
                          int64_t ldw, float* __restrict__ out, int64_t ldo, int M, int D, int n_lat) {
  extern __shared__ float dsm[];
  float* s_a = dsm;
  int* s_i = reinterpret_cast<int*>(dsm + k);
  const int nvec = D >> 3;
  const int t = threadIdx.x;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    float acc[VPT][8];
    decode_row_partial<VPT>(row, vals, idx, k, ldk, relu, inv_scale, W, ldw, n_lat, nvec, s_a, s_i, acc);
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * DEC_THREADS;
      if (vi < nvec) {
        float4* o = reinterpret_cast<float4*>(out + int64_t(row) * ldo) + 2 * vi;
        o[0] = make_float4(acc[v][0], acc[v][1], acc[v][2], acc[v][3]);
        o[1] = make_float4(acc[v][4], acc[v][5], acc[v][6], acc[v][7]);
      }
    }
  }
}

__global__ void __launch_bounds__(DEC_THREADS)
    finish_mse_kernel(const float* __restrict__ xsum, int64_t lds, const float* __restrict__ bias,
                      const __nv_bfloat16* __restrict__ target, int64_t ldt, __nv_bfloat16* __restrict__ out,
                      __nv_bfloat16* __restrict__ resid, __nv_bfloat16* __restrict__ dxhat,
                      const float* grad_coef_dev, float grad_coef, float* __restrict__ loss_row,
                      float* __restrict__ bsum, int M, int D) {
  __shared__ float red[32];
  const int nvec = D >> 3;
  const float gcoef = grad_coef_dev ? grad_coef * __ldg(grad_coef_dev) : grad_coef;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    float lsum = 0.f;
    for (int vi = threadIdx.x; vi < nvec; vi += DEC_THREADS) {
      const float4* xs = reinterpret_cast<const float4*>(xsum + int64_t(row) * lds) + 2 * vi;
      const float4 a0 = xs[0], a1 = xs[1];
      float xh[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      if (bias) {
#pragma unroll
        for (int e = 0; e < 8; ++e) xh[e] += __ldg(bias + 8 * vi + e);
      }
      float tg[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(target + int64_t(row) * ldt) + vi), tg);
      float err[8], g[8], rs[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        err[e] = xh[e] - tg[e];
        lsum += err[e] * err[e];
        g[e] = err[e] * gcoef;
        rs[e] = -err[e];
      }
      if (out) reinterpret_cast<uint4*>(out + int64_t(row) * D)[vi] = f32_to_bf16x8(xh);
      if (resid) reinterpret_cast<uint4*>(resid + int64_t(row) * D)[vi] = f32_to_bf16x8(rs);
      if (dxhat) {
        const uint4 gq = f32_to_bf16x8(g);
        reinterpret_cast<uint4*>(dxhat + int64_t(row) * D)[vi] = gq;
        if (bsum) {
          float gr[8];
          bf16x8_to_f32(gq, gr);
#pragma unroll
          for (int e = 0; e < 8; ++e) atomicAdd(bsum + 8 * vi + e, gr[e]);
        }
      }
    }
    const float tot = block_sum(lsum, red);
    if (threadIdx.x == 0 && loss_row) loss_row[row] = tot;
  }
}

// ---------------------------------------------------------------------------------------
// CSC build.  Pair p (= b * k + i for the main list, M*k + b*k_aux + i for the aux list) is
// kept when its coefficient is non-zero.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ bool pair_live(const float* vals, const int* idx, int64_t p, int relu,
                                          int n_lat, int& j) {
  j = idx[p];
  if (j < 0 || !SB_IN_RANGE(j, n_lat)) return false;
  const float v = vals[p];
  return relu ? (v > 0.f) : (v != 0.f);
}

__global__ void csc_count_kernel(const float* __restrict__ vals, const int* __restrict__ idx,
                                 int64_t n_main, const float* __restrict__ aux_vals,
                                 const int* __restrict__ aux_idx, int64_t n_aux,
                                 int* __restrict__ counts, int* __restrict__ fire_counts, int n_lat) {
  const int64_t total = n_main + n_aux;
  for (int64_t p = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; p < total;
       p += int64_t(gridDim.x) * blockDim.x) {
    int j;
    const bool main = p < n_main;
    const bool live = main ? pair_live(vals, idx, p, 1, n_lat, j)
                           : pair_live(aux_vals, aux_idx, p - n_main, 0, n_lat, j);
    if (live) {
      atomicAdd(counts + j, 1);
      if (main && fire_counts) atomicAdd(fire_counts + j, 1);
    }
  }
}

__global__ void csc_fill_kernel(const float* __restrict__ vals, const int* __restrict__ idx,
                                int64_t n_main, const float* __restrict__ aux_vals,
                                const int* __restrict__ aux_idx, int64_t n_aux,
                                const int64_t* __restrict__ colptr, int* __restrict__ cursor,
                                int64_t* __restrict__ pairs, int n_lat, int64_t pairs_cap) {
  const int64_t total = n_main + n_aux;
  for (int64_t p = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; p < total;
       p += int64_t(gridDim.x) * blockDim.x) {
    int j;
    const bool main = p < n_main;
    const bool live = main ? pair_live(vals, idx, p, 1, n_lat, j)
                           : pair_live(aux_vals, aux_idx, p - n_main, 0, n_lat, j);
    if (live) {
      const int pos = atomicAdd(cursor + j, 1);
      const int64_t dst = colptr[j] + pos;
      if (SB_IN_RANGE(dst, pairs_cap)) pairs[dst] = p;
    }
  }
}

// ---------------------------------------------------------------------------------------
// latent gradients.  One CTA (256 threads) per latent, grid-stride over latents.  Entries of a
// latent are processed in groups of LG_GROUP: every thread loads its slice of all the group's
// gradient rows at once (many loads in flight), accumulates gW_dec and its partial dot products,
// one block reduction yields the group's dz, then the group's input rows are loaded for gW_enc.
// ---------------------------------------------------------------------------------------
constexpr int LG_THREADS = 256;
constexpr int LG_GROUP = 4;

struct LatentGradArgs {
  const int64_t* colptr;
  const int64_t* pairs;
  int64_t P;  // entries of `pairs`
  int64_t n_main;
  int k, k_aux;
  const float* vals;       // [M, k]
  const float* aux_vals;   // [M, k_aux]
  const float* inv_scale;  // [N] or nullptr
  const __nv_bfloat16* dxhat;   // [M, D]  main-loss gradient rows
  const __nv_bfloat16* daux;    // [M, D]  aux-loss gradient rows (or nullptr)
  const __nv_bfloat16* x;       // [M, D]  raw input
  const float* b_dec;           // [D] (subtracted from x for the encoder input) or nullptr
  const __nv_bfloat16* W_dec;   // [N, D]
  const __nv_bfloat16* W_enc;   // [N, D] (latent-major)
  __nv_bfloat16* gW_dec;        // [N, D]
  __nv_bfloat16* gW_enc;        // [N, D]
  float* gb_enc;                // [N]
  float* bterm;                 // [D]  += sum_j gb_enc[j] W_enc[j]
  float* sumsq;                 // [1]  += squared norm of the three gradients
  const int* fire_counts;       // [N] live main pairs per latent (firing statistics)
  float* act_freq;              // [N] += fire count (or nullptr)
  float* since_fired;           // [N] = 0 if fired else +1 (or nullptr)
  int64_t ldx;
  int N, D;
};

template <int VPT>
__global__ void __launch_bounds__(LG_THREADS, 2) latent_grad_kernel(LatentGradArgs a) {
  __shared__ float s_coef[LG_GROUP];
  __shared__ int64_t s_row[LG_GROUP];
  __shared__ int s_aux[LG_GROUP];
  __shared__ float s_red[LG_THREADS / 32][LG_GROUP];
  __shared__ float red[32];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nvec = a.D >> 3;
  float bt[VPT][8];
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int e = 0; e < 8; ++e) bt[v][e] = 0.f;
  float sq = 0.f;

  const int64_t n_pair_ids = a.n_main + (a.aux_vals ? (a.n_main / a.k) * a.k_aux : 0);
  for (int j = blockIdx.x; j < a.N; j += gridDim.x) {
    int64_t beg = a.colptr[j], end = a.colptr[j + 1];
    if (!(SB_IN_RANGE(beg, a.P + 1) && SB_IN_RANGE(end, a.P + 1) && SB_IN_RANGE(end - beg, a.P + 1))) end = beg = 0;
    if (t == 0 && a.fire_counts) {
      const int fc = a.fire_counts[j];
      if (a.act_freq) a.act_freq[j] += float(fc);
      if (a.since_fired) a.since_fired[j] = fc > 0 ? 0.f : a.since_fired[j] + 1.f;
    }
    if (beg == end) {
      if (t == 0) a.gb_enc[j] = 0.f;
      continue;
    }
    const float isc = a.inv_scale ? a.inv_scale[j] : 1.f;
    uint4 wraw[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * LG_THREADS;
      wraw[v] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(a.W_dec + int64_t(j) * a.D) + vi)
                          : make_uint4(0, 0, 0, 0);
    }
    float gd[VPT][8], ge[VPT][8];
#pragma unroll
    for (int v = 0; v < VPT; ++v)
#pragma unroll
      for (int e = 0; e < 8; ++e) gd[v][e] = ge[v][e] = 0.f;
    float gbe = 0.f;

    for (int64_t c0 = beg; c0 < end; c0 += LG_GROUP) {
      const int cn = int((end - c0) < int64_t(LG_GROUP) ? (end - c0) : int64_t(LG_GROUP));
      __syncthreads();  // previous group's s_* reads are done
      if (t < cn) {
        int64_t p = a.pairs[c0 + t];
        const bool p_ok = SB_IN_RANGE(p, n_pair_ids);
        if (!p_ok) p = 0;  // debug builds: stand-in pair with a zero coefficient
        if (p < a.n_main) {
          s_row[t] = p / a.k;
          s_coef[t] = p_ok ? fmaxf(a.vals[p], 0.f) * isc : 0.f;
          s_aux[t] = 0;
        } else {
          const int64_t q = p - a.n_main;
          s_row[t] = q / a.k_aux;
          s_coef[t] = a.aux_vals[q] * isc;
          s_aux[t] = 1;
        }
      }
      __syncthreads();
      // gradient rows of the whole group in flight at once
      uint4 graw[LG_GROUP][VPT];
#pragma unroll
      for (int e = 0; e < LG_GROUP; ++e) {
        const __nv_bfloat16* grow = e < cn ? (s_aux[e] ? a.daux : a.dxhat) + s_row[e] * int64_t(a.D) : nullptr;
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int vi = t + v * LG_THREADS;
          graw[e][v] = (e < cn && vi < nvec) ? __ldg(reinterpret_cast<const uint4*>(grow) + vi)
                                             : make_uint4(0, 0, 0, 0);
        }
      }
      float pd[LG_GROUP];
#pragma unroll
      for (int e = 0; e < LG_GROUP; ++e) {
        const float coef = e < cn ? s_coef[e] : 0.f;
        float d = 0.f;
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          float g[8], w[8];
          bf16x8_to_f32(graw[e][v], g);
          bf16x8_to_f32(wraw[v], w);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            gd[v][q] += coef * g[q];
            d += g[q] * w[q];
          }
        }
        pd[e] = d;
      }
#pragma unroll
      for (int e = 0; e < LG_GROUP; ++e) {
        float d = pd[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) s_red[warp][e] = d;
      }
      __syncthreads();
      float dz[LG_GROUP];
#pragma unroll
      for (int e = 0; e < LG_GROUP; ++e) {
        float d = 0.f;
#pragma unroll
        for (int w = 0; w < LG_THREADS / 32; ++w) d += s_red[w][e];
        dz[e] = e < cn ? d : 0.f;  // main pairs are live only where a > 0: no extra mask needed
        gbe += dz[e];
      }
      // encoder gradient: input rows of the group in flight at once
      uint4 xraw[LG_GROUP][VPT];
#pragma unroll
      for (int e = 0; e < LG_GROUP; ++e) {
        const __nv_bfloat16* xrow = e < cn ? a.x + s_row[e] * a.ldx : nullptr;
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int vi = t + v * LG_THREADS;
          xraw[e][v] = (e < cn && vi < nvec) ? __ldg(reinterpret_cast<const uint4*>(xrow) + vi)
                                             : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int vi = t + v * LG_THREADS;
        float bd[8];
        if (a.b_dec && vi < nvec) {
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(a.b_dec) + 2 * vi);
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.b_dec) + 2 * vi + 1);
          bd[0] = b0.x; bd[1] = b0.y; bd[2] = b0.z; bd[3] = b0.w;
          bd[4] = b1.x; bd[5] = b1.y; bd[6] = b1.z; bd[7] = b1.w;
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) bd[q] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < LG_GROUP; ++e) {
          float xv[8];
          bf16x8_to_f32(xraw[e][v], xv);
#pragma unroll
          for (int q = 0; q < 8; ++q) ge[v][q] += dz[e] * (xv[q] - bd[q]);
        }
      }
    }
    // write gradient rows (bf16), squared norm of what Adam will read, b_dec term
    uint4 weraw[VPT];
    if (a.bterm) {
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int vi = t + v * LG_THREADS;
        weraw[v] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(a.W_enc + int64_t(j) * a.D) + vi)
                             : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * LG_THREADS;
      if (vi < nvec) {
        const uint4 qd = f32_to_bf16x8(gd[v]);
        const uint4 qe = f32_to_bf16x8(ge[v]);
        reinterpret_cast<uint4*>(a.gW_dec + int64_t(j) * a.D)[vi] = qd;
        reinterpret_cast<uint4*>(a.gW_enc + int64_t(j) * a.D)[vi] = qe;
        float rd[8], re[8];
        bf16x8_to_f32(qd, rd);
        bf16x8_to_f32(qe, re);
#pragma unroll
        for (int q = 0; q < 8; ++q) sq += rd[q] * rd[q] + re[q] * re[q];
        if (a.bterm) {
          float we[8];
          bf16x8_to_f32(weraw[v], we);
#pragma unroll
          for (int q = 0; q < 8; ++q) bt[v][q] += gbe * we[q];
        }
      }
    }
    if (t == 0) {
      a.gb_enc[j] = gbe;
      sq += gbe * gbe;
    }
  }
  if (a.bterm) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * LG_THREADS;
      if (vi < nvec)
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (bt[v][q] != 0.f) atomicAdd(a.bterm + 8 * vi + q, bt[v][q]);
    }
  }
  const float tot = block_sum(sq, red);
  if (t == 0 && a.sumsq) atomicAdd(a.sumsq, tot);
}


// ---------------------------------------------------------------------------------------
// Tensor-parallel decode -> reduce-scatter, two launches per rank, all ranks running concurrently.
//   phase A (its own launch, full occupancy, no waits): this rank's partial reconstruction of RB
//           consecutive rows (from its own winners), stored straight into the row owner's landing
//           area land[src = this rank][row - owner*Bo] with NVLink P2P stores, then one
//           release-add on the owner's arrival counter of that row block.
//   phase B (the next launch): for a row block this rank owns, wait until all S sources arrived,
//           reduce the S partials in rank order, add b_dec, and produce loss_row, sae_out, the
//           residual, dL/dx_hat and its column sum; dL/dx_hat rows are stored into EVERY rank's dx
//           buffer and published with one epoch flag per block.
// A phase-B wait depends only on the phase-A launches of the other GPUs (each GPU runs its own),
// never on a CTA of the same launch.  Phase A walks the owners starting at rank+1, so at any
// moment the ranks push to different receivers.  Replaces the reference's dense decode +
// reduce-scatter + loss (sae_lens/distributed.py:404-461, sae_lens/saes/topk_sae.py:645-674).
// ---------------------------------------------------------------------------------------
constexpr int RS_RB = 16;

struct DecodeRsArgs {
  const float* vals;
  const int* idx;
  int k;
  int64_t ldk;
  int relu;
  const float* inv_scale;
  const __nv_bfloat16* W;
  int64_t ldw;
  int B, Bo, D;
  int n_lat;  // rows of W (latent id bound)
  p2p::Peers P;
  int64_t land_off, lcnt_off, dx_off, dcnt_off;  // slab byte offsets; dx_off < 0: no broadcast
  uint32_t epoch;
  const float* bias;
  const __nv_bfloat16* target;
  int64_t ldt;
  __nv_bfloat16* out;
  __nv_bfloat16* resid;
  const float* grad_coef_dev;
  float grad_coef;
  float* loss_row;
  float* bsum;
  int* ticket;
  int* status;
};

// PHASE 0: one launch, both phases, work items from one ticket counter (phase-A tickets first, so a
//          phase-B item is claimed only after every phase-A item has been claimed by a resident CTA);
// PHASE 1: phase A only (static strided items); PHASE 2: phase B only (the following launch).
template <int VPT, int PHASE>
__global__ void __launch_bounds__(DEC_THREADS) decode_rs_kernel(const __grid_constant__ DecodeRsArgs a) {
  extern __shared__ float dsm[];
  float* s_a = dsm;
  int* s_i = reinterpret_cast<int*>(dsm + a.k);
  float* red = dsm + 2 * a.k;
  __shared__ int s_tk, s_ok;
  const int t = threadIdx.x;
  const int S = a.P.world, r = a.P.rank, D = a.D;
  const int nvec = D >> 3;
  const int nbo = a.Bo / RS_RB, nA = a.B / RS_RB, nT = nA + nbo;
  const float gcoef = a.grad_coef_dev ? a.grad_coef * __ldg(a.grad_coef_dev) : a.grad_coef;
  float bacc[VPT][8];
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int e = 0; e < 8; ++e) bacc[v][e] = 0.f;

  for (int it = blockIdx.x;; it += gridDim.x) {
    __syncthreads();
    int tk;
    if (PHASE == 0) {
      if (t == 0) s_tk = atomicAdd(a.ticket, 1);
      __syncthreads();
      tk = s_tk;
    } else {
      tk = PHASE == 1 ? it : nA + it;
    }
    if (tk >= (PHASE == 1 ? nA : nT)) break;
    if (PHASE == 1 || (PHASE == 0 && tk < nA)) {  // compile-time split for PHASE 1 / 2
      // ---------------- phase A: partial rows -> owner ----------------
      const int blk = (tk + (r + 1) * nbo) % nA;
      const int o = blk / nbo, lb = blk - o * nbo;
      float* land = p2p::at<float>(a.P, o, a.land_off) + (int64_t(r) * a.Bo + int64_t(lb) * RS_RB) * D;
      for (int rr = 0; rr < RS_RB; ++rr) {
        float acc[VPT][8];
        decode_row_partial<VPT>(blk * RS_RB + rr, a.vals, a.idx, a.k, a.ldk, a.relu, a.inv_scale, a.W, a.ldw,
                                a.n_lat, nvec, s_a, s_i, acc);
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int vi = t + v * DEC_THREADS;
          if (vi < nvec) {
            float4* o4 = reinterpret_cast<float4*>(land + int64_t(rr) * D) + 2 * vi;
            o4[0] = make_float4(acc[v][0], acc[v][1], acc[v][2], acc[v][3]);
            o4[1] = make_float4(acc[v][4], acc[v][5], acc[v][6], acc[v][7]);
          }
        }
      }
      __threadfence_system();
      __syncthreads();
      if (t == 0) red_release_sys_add_u32(p2p::at<uint32_t>(a.P, o, a.lcnt_off) + lb, 1u);
    } else {
      // ---------------- phase B: reduce owned rows, loss, dL/dx_hat -> everyone ----------------
      const int ob = tk - nA;
      if (t == 0)
        s_ok = wait_geq_sys(p2p::at<uint32_t>(a.P, r, a.lcnt_off) + ob, uint32_t(S) * a.epoch, a.status,
                            kTimeoutPeerFlag)
                   ? 1
                   : 0;
      __syncthreads();
      if (!s_ok) continue;
      const float* land = p2p::at<float>(a.P, r, a.land_off);
      for (int rr = 0; rr < RS_RB; ++rr) {
        const int row = ob * RS_RB + rr;  // local row
        float lsum = 0.f;
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int vi = t + v * DEC_THREADS;
          if (vi >= nvec) continue;
          float xh[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) xh[e] = 0.f;
          for (int src = 0; src < S; ++src) {
            const float4* p4 = reinterpret_cast<const float4*>(land + (int64_t(src) * a.Bo + row) * D) + 2 * vi;
            const float4 p0 = __ldcg(p4), p1 = __ldcg(p4 + 1);
            xh[0] += p0.x; xh[1] += p0.y; xh[2] += p0.z; xh[3] += p0.w;
            xh[4] += p1.x; xh[5] += p1.y; xh[6] += p1.z; xh[7] += p1.w;
          }
          if (a.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(a.bias) + 2 * vi;
            const float4 b0 = __ldg(b4), b1 = __ldg(b4 + 1);
            xh[0] += b0.x; xh[1] += b0.y; xh[2] += b0.z; xh[3] += b0.w;
            xh[4] += b1.x; xh[5] += b1.y; xh[6] += b1.z; xh[7] += b1.w;
          }
          float tg[8], err[8], g[8], rs[8];
          bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(a.target + int64_t(row) * a.ldt) + vi), tg);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            err[e] = xh[e] - tg[e];
            lsum += err[e] * err[e];
            g[e] = err[e] * gcoef;
            rs[e] = -err[e];
          }
          if (a.out) reinterpret_cast<uint4*>(a.out + int64_t(row) * D)[vi] = f32_to_bf16x8(xh);
          if (a.resid) reinterpret_cast<uint4*>(a.resid + int64_t(row) * D)[vi] = f32_to_bf16x8(rs);
          const uint4 gq = f32_to_bf16x8(g);
          if (a.dx_off >= 0) {
            const int64_t off = (int64_t(r) * a.Bo + row) * D;
            for (int d = 0; d < S; ++d)
              reinterpret_cast<uint4*>(p2p::at<__nv_bfloat16>(a.P, d, a.dx_off) + off)[vi] = gq;
          }
          if (a.bsum) {
            float gr[8];
            bf16x8_to_f32(gq, gr);
#pragma unroll
            for (int e = 0; e < 8; ++e) bacc[v][e] += gr[e];
          }
        }
        const float tot = block_sum(lsum, red);
        if (t == 0 && a.loss_row) a.loss_row[row] = tot;
      }
      if (a.dx_off >= 0) {
        __threadfence_system();
        __syncthreads();
        if (t == 0)
          for (int d = 0; d < S; ++d)
            st_release_sys_u32(p2p::at<uint32_t>(a.P, d, a.dcnt_off) + (r * nbo + ob), a.epoch);
      }
    }
  }
  if (PHASE != 1 && a.bsum) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int vi = t + v * DEC_THREADS;
      if (vi < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) atomicAdd(a.bsum + 8 * vi + e, bacc[v][e]);
    }
  }
}


// ---------------------------------------------------------------------------------------
// latent gradients, two passes over the CSC pair lists (the pairs of a latent are contiguous):
//  pass 1 (pair_dz_kernel, one warp per pair): row b, coefficient a and
//         dz = <dL/dx_hat[b], W_dec[j]> of every pair, stored in CSC order.  The dot product is
//         the only reduction over d_in; after it every column is independent.
//  pass 2 (latent_rows_kernel, one warp per (latent, d_in slice), slice fixed per warp):
//         gW_dec[j] = sum a dXhat[b], gW_enc[j] = sum dz (x[b] - b_dec), gb_enc[j] = sum dz, the
//         firing statistics, the squared gradient norm and per-warp partials of the b_dec term
//         sum_j gb_enc[j] W_enc[j]; col_reduce_kernel sums those partials into bterm.
// No block barrier sits on the per-latent path, so many latents' loads are in flight per SM.
// ---------------------------------------------------------------------------------------
constexpr int LR_THREADS = 256;
constexpr int LR_WARPS = LR_THREADS / 32;

struct PairDzArgs {
  const int64_t* pairs;
  const int64_t* pos_begin;  // colptr + j0: first pair position of the latent range
  const int64_t* pos_end;    // colptr + j1: end of the range (only live pairs are ever listed)
  int64_t P, n_main;
  int k, k_aux;
  const float* vals;
  const int* idx;
  const float* aux_vals;
  const int* aux_idx;
  const float* inv_scale;
  const __nv_bfloat16* dxhat;
  const __nv_bfloat16* daux;
  const __nv_bfloat16* W_dec;
  int D;
  int N;          // latent id bound
  int* prow;      // [P] row | (aux << 31)
  float* pcoef;   // [P]
  float* pdz;     // [P]
  // JumpReLU mode (jr_thr != nullptr): main pairs are candidate entries with pre-activation
  // jr_pre[p]; active = pre > threshold; coefficient and gradient flow only through active entries,
  // and every entry inside the rectangle window |pre - threshold| < bandwidth/2 adds
  // -(threshold / bandwidth) dz - jr_l0c to jr_gthr[j] (MSE and L0 straight-through terms).
  const float* jr_thr;
  const float* jr_pre;
  float jr_inv_bw;
  float jr_l0c;
  float* jr_gthr;
};

__global__ void __launch_bounds__(LR_THREADS) pair_dz_kernel(const __grid_constant__ PairDzArgs a) {
  constexpr int U = 8;  // 16-byte loads in flight per lane and operand
  const int lane = threadIdx.x & 31;
  const int nvec = a.D >> 3;
  const int64_t nw = int64_t(gridDim.x) * LR_WARPS;
  const int64_t pend = min(*a.pos_end, a.P);
  const int64_t n_pair_ids = a.n_main + (a.aux_vals ? (a.n_main / a.k) * a.k_aux : 0);
  for (int64_t pos = *a.pos_begin + ((int64_t(blockIdx.x) * LR_THREADS + threadIdx.x) >> 5); pos < pend;
       pos += nw) {
    if (!SB_IN_RANGE(pos, a.P)) break;  // debug builds: a negative range start
    const int64_t p = a.pairs[pos];
    if (!SB_IN_RANGE(p, n_pair_ids) ||
        !SB_IN_RANGE(p < a.n_main ? a.idx[p] : a.aux_idx[p - a.n_main], a.N)) {
      // debug builds: an entry that cannot be resolved contributes nothing (row 0, zero weights)
      if ((threadIdx.x & 31) == 0) {
        a.prow[pos] = 0;
        a.pcoef[pos] = 0.f;
        a.pdz[pos] = 0.f;
      }
      continue;
    }
    int64_t b;
    int j, aux;
    float coef;
    float jr_pre = 0.f, jr_th = 0.f;
    bool jr_active = true;
    if (p < a.n_main) {
      b = p / a.k;
      j = a.idx[p];
      if (a.jr_thr) {
        jr_pre = a.jr_pre[p];
        jr_th = __ldg(a.jr_thr + j);
        jr_active = jr_pre > jr_th;
        coef = jr_active ? jr_pre : 0.f;
      } else {
        coef = fmaxf(a.vals[p], 0.f);
      }
      aux = 0;
    } else {
      const int64_t q = p - a.n_main;
      b = q / a.k_aux;
      j = a.aux_idx[q];
      coef = a.aux_vals[q];
      aux = 1;
    }
    if (a.inv_scale) coef *= __ldg(a.inv_scale + j);
    const uint4* g4 = reinterpret_cast<const uint4*>((aux ? a.daux : a.dxhat) + b * int64_t(a.D));
    const uint4* w4 = reinterpret_cast<const uint4*>(a.W_dec + int64_t(j) * a.D);
    float d = 0.f;
    for (int v0 = lane; v0 < nvec; v0 += 32 * U) {
      uint4 g[U], w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int vi = v0 + 32 * u;
        g[u] = vi < nvec ? __ldg(g4 + vi) : make_uint4(0, 0, 0, 0);
        w[u] = vi < nvec ? __ldg(w4 + vi) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float gf[8], wf[8];
        bf16x8_to_f32(g[u], gf);
        bf16x8_to_f32(w[u], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) d += gf[e] * wf[e];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (lane == 0) {
      a.prow[pos] = int(b) | (aux << 31);
      a.pcoef[pos] = coef;
      a.pdz[pos] = jr_active ? d : 0.f;
      if (a.jr_thr && fabsf(jr_pre - jr_th) * a.jr_inv_bw < 0.5f)
        atomicAdd(a.jr_gthr + j, -(jr_th * a.jr_inv_bw) * d - a.jr_l0c);
    }
  }
}

struct LatentRowsArgs {
  const int64_t* colptr;
  const int* prow;
  const float* pcoef;
  const float* pdz;
  const __nv_bfloat16* dxhat;
  const __nv_bfloat16* daux;
  const __nv_bfloat16* x;
  int64_t ldx;
  const float* b_dec;
  const __nv_bfloat16* W_enc;
  __nv_bfloat16* gW_dec;
  __nv_bfloat16* gW_enc;
  float* gb_enc;
  float* bpart;   // [total warps, slice width] b_dec-term partials (or nullptr)
  float* sumsq;
  const int* fire_counts;
  float* act_freq;
  float* since_fired;
  int N, D, nslices;
  int M;           // rows of dxhat / daux / x (pair row bound)
  int64_t n_pairs; // pair-list length (CSC offset bound)
  int j0, j1;      // latent range of this launch
  int zero_empty;  // write zero gradient rows for latents without a live pair (dense consumers)
  // Reduce-scatter destination (sharded data parallel): with rs_n > 0 the gradient rows of
  // latent j go to the slab of its owner o = j / rs_n, into slot [this rank][j - o * rs_n] of the
  // [S, rs_n, D] areas at rs_dec_off / rs_enc_off, instead of gW_dec / gW_enc.
  p2p::Peers P;
  int64_t rs_dec_off, rs_enc_off;
  int rs_n;
};

__device__ __forceinline__ __nv_bfloat16* grad_row(const LatentRowsArgs& a, __nv_bfloat16* local, int64_t off,
                                                   int j) {
  if (a.rs_n == 0) return local + int64_t(j) * a.D;
  const int o = j / a.rs_n;
  return p2p::at<__nv_bfloat16>(a.P, o, off) + (int64_t(a.P.rank) * a.rs_n + (j - o * a.rs_n)) * a.D;
}

template <int VPL>
__global__ void __launch_bounds__(LR_THREADS, 2) latent_rows_kernel(const __grid_constant__ LatentRowsArgs a) {
  __shared__ float red[32];
  const int lane = threadIdx.x & 31;
  const int nvec = a.D >> 3;
  const int gw = (blockIdx.x * LR_THREADS + threadIdx.x) >> 5;
  const int tw = gridDim.x * LR_WARPS;
  const int sl = gw % a.nslices;
  const int vbase = sl * 32 * VPL + lane;
  float bt[VPL][8];
#pragma unroll
  for (int u = 0; u < VPL; ++u)
#pragma unroll
    for (int e = 0; e < 8; ++e) bt[u][e] = 0.f;
  float sq = 0.f;
  const int jstep = tw / a.nslices;
  int j = a.j0 + gw / a.nslices;
  int64_t nbeg = 0, nend = 0;
  if (j < a.j1) {
    nbeg = a.colptr[j];
    nend = a.colptr[j + 1];
  }
  for (; j < a.j1; j += jstep) {
    int64_t beg = nbeg, end = nend;
    if (j + jstep < a.j1) {  // the next item's offsets load while this item runs
      nbeg = __ldg(a.colptr + j + jstep);
      nend = __ldg(a.colptr + j + jstep + 1);
    }
    if (!(SB_IN_RANGE(beg, a.n_pairs + 1) && SB_IN_RANGE(end, a.n_pairs + 1) && SB_IN_RANGE(end - beg, a.n_pairs + 1))) end = beg = 0;
    if (sl == 0 && lane == 0 && a.fire_counts) {
      const int fc = a.fire_counts[j];
      if (a.act_freq) a.act_freq[j] += float(fc);
      if (a.since_fired) a.since_fired[j] = fc > 0 ? 0.f : a.since_fired[j] + 1.f;
    }
    if (beg == end) {
      if (sl == 0 && lane == 0) a.gb_enc[j] = 0.f;
      if (a.zero_empty) {
#pragma unroll
        for (int u = 0; u < VPL; ++u) {
          const int vi = vbase + 32 * u;
          if (vi < nvec) {
            reinterpret_cast<uint4*>(grad_row(a, a.gW_dec, a.rs_dec_off, j))[vi] = make_uint4(0, 0, 0, 0);
            reinterpret_cast<uint4*>(grad_row(a, a.gW_enc, a.rs_enc_off, j))[vi] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      continue;
    }
    // the W_enc slice of the b_dec term does not depend on the pairs: issue it first
    uint4 WE[VPL];
    if (a.bpart) {
#pragma unroll
      for (int u = 0; u < VPL; ++u) {
        const int vi = vbase + 32 * u;
        WE[u] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(a.W_enc + int64_t(j) * a.D) + vi)
                          : make_uint4(0, 0, 0, 0);
      }
    }
    float gd[VPL][8], ge[VPL][8];
#pragma unroll
    for (int u = 0; u < VPL; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e) gd[u][e] = ge[u][e] = 0.f;
    float gbe = 0.f;
    // pair entries 32 at a time: lane l loads entry cb + l in one round trip, and each pair's row,
    // coefficient and dz reach the warp by shuffles (the pairs of a latent are few, so one round
    // trip usually covers them all)
    for (int64_t cb = beg; cb < end; cb += 32) {
      const int nc = end - cb < 32 ? int(end - cb) : 32;
      int mr = 0;
      float mc = 0.f, mz = 0.f;
      if (lane < nc) {
        mr = a.prow[cb + lane];
        mc = a.pcoef[cb + lane];
        mz = a.pdz[cb + lane];
        if (!SB_IN_RANGE(mr & 0x7fffffff, a.M)) mr = 0, mc = mz = 0.f;  // debug builds: drop the entry
      }
      for (int q = 0; q < nc; q += 2) {
        const bool two = q + 1 < nc;
        const int r0 = __shfl_sync(0xffffffffu, mr, q);
        const float c0 = __shfl_sync(0xffffffffu, mc, q);
        const float z0 = __shfl_sync(0xffffffffu, mz, q);
        const int q1 = two ? q + 1 : q;
        const int r1 = __shfl_sync(0xffffffffu, mr, q1);
        const float c1 = two ? __shfl_sync(0xffffffffu, mc, q1) : 0.f;
        const float z1 = two ? __shfl_sync(0xffffffffu, mz, q1) : 0.f;
        const __nv_bfloat16* g0 = ((r0 < 0) ? a.daux : a.dxhat) + int64_t(r0 & 0x7fffffff) * a.D;
        const __nv_bfloat16* g1 = ((r1 < 0) ? a.daux : a.dxhat) + int64_t(r1 & 0x7fffffff) * a.D;
        const __nv_bfloat16* x0 = a.x + int64_t(r0 & 0x7fffffff) * a.ldx;
        const __nv_bfloat16* x1 = a.x + int64_t(r1 & 0x7fffffff) * a.ldx;
        uint4 G0[VPL], G1[VPL], X0[VPL], X1[VPL];
#pragma unroll
        for (int u = 0; u < VPL; ++u) {
          const int vi = vbase + 32 * u;
          const bool ok = vi < nvec;
          G0[u] = ok ? __ldg(reinterpret_cast<const uint4*>(g0) + vi) : make_uint4(0, 0, 0, 0);
          X0[u] = ok ? __ldg(reinterpret_cast<const uint4*>(x0) + vi) : make_uint4(0, 0, 0, 0);
          G1[u] = (ok && two) ? __ldg(reinterpret_cast<const uint4*>(g1) + vi) : make_uint4(0, 0, 0, 0);
          X1[u] = (ok && two) ? __ldg(reinterpret_cast<const uint4*>(x1) + vi) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < VPL; ++u) {
          float f0[8], f1[8], y0[8], y1[8];
          bf16x8_to_f32(G0[u], f0);
          bf16x8_to_f32(G1[u], f1);
          bf16x8_to_f32(X0[u], y0);
          bf16x8_to_f32(X1[u], y1);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            gd[u][e] += c0 * f0[e] + c1 * f1[e];
            ge[u][e] += z0 * y0[e] + z1 * y1[e];
          }
        }
        gbe += z0 + z1;
      }
    }
    // sum dz (x - b_dec) = sum dz x - (sum dz) b_dec
    if (a.b_dec) {
#pragma unroll
      for (int u = 0; u < VPL; ++u) {
        const int vi = vbase + 32 * u;
        if (vi < nvec) {
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(a.b_dec) + 2 * vi);
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.b_dec) + 2 * vi + 1);
          ge[u][0] -= gbe * b0.x;
          ge[u][1] -= gbe * b0.y;
          ge[u][2] -= gbe * b0.z;
          ge[u][3] -= gbe * b0.w;
          ge[u][4] -= gbe * b1.x;
          ge[u][5] -= gbe * b1.y;
          ge[u][6] -= gbe * b1.z;
          ge[u][7] -= gbe * b1.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      const int vi = vbase + 32 * u;
      if (vi < nvec) {
        const uint4 qd = f32_to_bf16x8(gd[u]);
        const uint4 qe = f32_to_bf16x8(ge[u]);
        reinterpret_cast<uint4*>(grad_row(a, a.gW_dec, a.rs_dec_off, j))[vi] = qd;
        reinterpret_cast<uint4*>(grad_row(a, a.gW_enc, a.rs_enc_off, j))[vi] = qe;
        float rd[8], re[8];
        bf16x8_to_f32(qd, rd);
        bf16x8_to_f32(qe, re);
#pragma unroll
        for (int e = 0; e < 8; ++e) sq += rd[e] * rd[e] + re[e] * re[e];
        if (a.bpart) {
          float we[8];
          bf16x8_to_f32(WE[u], we);
#pragma unroll
          for (int e = 0; e < 8; ++e) bt[u][e] += gbe * we[e];
        }
      }
    }
    if (sl == 0 && lane == 0) {
      a.gb_enc[j] = gbe;
      sq += gbe * gbe;
    }
  }
  if (a.bpart) {
    float* dst = a.bpart + int64_t(gw) * (32 * VPL * 8);
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      float4* d4 = reinterpret_cast<float4*>(dst + (u * 32 + lane) * 8);
      d4[0] = make_float4(bt[u][0], bt[u][1], bt[u][2], bt[u][3]);
      d4[1] = make_float4(bt[u][4], bt[u][5], bt[u][6], bt[u][7]);
    }
  }
  // peer rows: this thread's stores are performed system-wide before the kernel ends, so a
  // release published by a later launch on this stream orders after them
  if (a.rs_n) __threadfence_system();
  const float tot = block_sum(sq, red);
  if (threadIdx.x == 0 && a.sumsq) atomicAdd(a.sumsq, tot);
}

// bterm[d] += sum over the warps w with slice(d) of bpart[w][d - slice start].
// One block per 32 consecutive columns; its 32 warps split the warp range (w = s, s + ns, ...)
// round-robin, and the 32 partials of a column are summed in a fixed order (deterministic).
// With thousands of partials per column this keeps ~32x more loads in flight than a thread per
// column walking the whole range.
constexpr int CR_ROWS = 32;
__global__ void __launch_bounds__(32 * CR_ROWS) col_reduce_kernel(const float* __restrict__ bpart, int tw,
                                                                 int nslices, int sw, int D,
                                                                 float* __restrict__ bterm) {
  __shared__ float part[CR_ROWS][33];
  const int d = blockIdx.x * 32 + threadIdx.x;
  float acc = 0.f;
  if (d < D) {
    const int s = d / sw, c = d - s * sw;
    for (int w = s + threadIdx.y * nslices; w < tw; w += CR_ROWS * nslices) acc += bpart[int64_t(w) * sw + c];
  }
  part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && d < D) {
    float t = 0.f;
#pragma unroll 8
    for (int i = 0; i < CR_ROWS; ++i) t += part[i][threadIdx.x];
    bterm[d] += t;
  }
}
}  // namespace sparse

static inline int pick_vpt(int64_t D, int threads) {
  const int64_t need = (D / 8 + threads - 1) / threads;
  if (need <= 1) return 1;
  if (need <= 2) return 2;
  if (need <= 4) return 4;
  SB_CHECK(need <= 8, "d_in too large for the sparse kernels (max 8192)");
  return 8;
}

static int sm_count() {
  int dev, n;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

void decode_mse(const torch::Tensor& vals, const torch::Tensor& idx, bool relu,
                const c10::optional<torch::Tensor>& inv_scale, const torch::Tensor& W,
                const c10::optional<torch::Tensor>& bias, const torch::Tensor& target,
                const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& resid,
                const c10::optional<torch::Tensor>& dxhat, const c10::optional<torch::Tensor>& grad_coef_dev,
                double grad_coef, const c10::optional<torch::Tensor>& loss_row,
                const c10::optional<torch::Tensor>& bsum) {
  SB_CHECK(vals.scalar_type() == at::kFloat && idx.scalar_type() == at::kInt && vals.dim() == 2 &&
                  vals.sizes() == idx.sizes() && vals.is_contiguous() && idx.is_contiguous(),
              "decode_mse: vals fp32 / idx int32 [M, k]");
  SB_CHECK(W.scalar_type() == at::kBFloat16 && W.dim() == 2 && W.stride(1) == 1, "decode_mse: W");
  const int64_t M = vals.size(0), k = vals.size(1), D = W.size(1);
  SB_CHECK(D % 8 == 0 && W.stride(0) % 8 == 0, "decode_mse: d_in must be a multiple of 8");
  SB_CHECK(target.scalar_type() == at::kBFloat16 && target.size(0) == M && target.size(1) == D &&
                  target.stride(1) == 1 && target.stride(0) % 8 == 0,
              "decode_mse: target bf16 [M, D]");
  auto chk_out = [&](const c10::optional<torch::Tensor>& o, const char* name) -> __nv_bfloat16* {
    if (!o) return nullptr;
    SB_CHECK(o->scalar_type() == at::kBFloat16 && o->size(0) == M && o->size(1) == D &&
                    o->stride(1) == 1 && o->stride(0) % 8 == 0,
                "decode_mse: bad ", name);
    return reinterpret_cast<__nv_bfloat16*>(o->data_ptr());
  };
  __nv_bfloat16* po = chk_out(out, "out");
  __nv_bfloat16* pr = chk_out(resid, "resid");
  __nv_bfloat16* pd = chk_out(dxhat, "dxhat");
  const float* pinv = nullptr;
  if (inv_scale) {
    SB_CHECK(inv_scale->scalar_type() == at::kFloat && inv_scale->numel() == W.size(0), "decode_mse: inv_scale");
    pinv = inv_scale->data_ptr<float>();
  }
  const float* pb = nullptr;
  if (bias) {
    SB_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == D, "decode_mse: bias");
    pb = bias->data_ptr<float>();
  }
  const float* pgc = nullptr;
  if (grad_coef_dev) pgc = grad_coef_dev->data_ptr<float>();
  float* pl = loss_row ? loss_row->data_ptr<float>() : nullptr;
  float* pbs = bsum ? bsum->data_ptr<float>() : nullptr;
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(vals.device());
  const int vpt = pick_vpt(D, sparse::DEC_THREADS);
  const int64_t grid = std::min<int64_t>(M, int64_t(sm_count()) * 8);
  const size_t smem = size_t(2 * k + 32) * 4;
  auto stream = at::cuda::getCurrentCUDAStream();
#define SB_DEC(V)                                                                                  \
  sparse::decode_mse_kernel<V><<<dim3(grid), dim3(sparse::DEC_THREADS), smem, stream>>>(           \
      vals.data_ptr<float>(), idx.data_ptr<int>(), int(k), vals.stride(0), relu ? 1 : 0, pinv,      \
      reinterpret_cast<const __nv_bfloat16*>(W.data_ptr()), W.stride(0), pb,                      \
      reinterpret_cast<const __nv_bfloat16*>(target.data_ptr()), target.stride(0), po,             \
      out ? out->stride(0) : 0, pr, resid ? resid->stride(0) : 0, pd, dxhat ? dxhat->stride(0) : 0, \
      pgc, float(grad_coef), pl, pbs, int(M), int(D), int(W.size(0)))
  switch (vpt) {
    case 1: SB_DEC(1); break;
    case 2: SB_DEC(2); break;
    case 4: SB_DEC(4); break;
    default: SB_DEC(8); break;
  }
#undef SB_DEC
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Builds the latent-major pair lists.  Returns nothing; fills counts [N] (int32), colptr
// [N+1] (int64), pairs [nnz_capacity] (int64) and fire_counts [N] (int32, main pairs only).
void csc_count(const torch::Tensor& vals, const torch::Tensor& idx,
               const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& aux_idx,
               const torch::Tensor& counts, const c10::optional<torch::Tensor>& fire_counts) {
  const at::cuda::CUDAGuard guard(vals.device());
  const int64_t n_main = vals.numel();
  const int64_t n_aux = aux_vals ? aux_vals->numel() : 0;
  const int64_t total = n_main + n_aux;
  if (total == 0) return;
  const int64_t grid = std::min<int64_t>((total + 255) / 256, int64_t(sm_count()) * 16);
  sparse::csc_count_kernel<<<dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), idx.data_ptr<int>(), n_main,
      aux_vals ? aux_vals->data_ptr<float>() : nullptr, aux_idx ? aux_idx->data_ptr<int>() : nullptr,
      n_aux, counts.data_ptr<int>(), fire_counts ? fire_counts->data_ptr<int>() : nullptr, int(counts.numel()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void csc_fill(const torch::Tensor& vals, const torch::Tensor& idx,
              const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& aux_idx,
              const torch::Tensor& colptr, const torch::Tensor& cursor, const torch::Tensor& pairs) {
  const at::cuda::CUDAGuard guard(vals.device());
  const int64_t n_main = vals.numel();
  const int64_t n_aux = aux_vals ? aux_vals->numel() : 0;
  const int64_t total = n_main + n_aux;
  if (total == 0) return;
  SB_CHECK(colptr.scalar_type() == at::kLong && pairs.scalar_type() == at::kLong &&
                  cursor.scalar_type() == at::kInt,
              "csc_fill: dtypes");
  const int64_t grid = std::min<int64_t>((total + 255) / 256, int64_t(sm_count()) * 16);
  sparse::csc_fill_kernel<<<dim3(grid), dim3(256), 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), idx.data_ptr<int>(), n_main,
      aux_vals ? aux_vals->data_ptr<float>() : nullptr, aux_idx ? aux_idx->data_ptr<int>() : nullptr,
      n_aux, colptr.data_ptr<int64_t>(), cursor.data_ptr<int>(), pairs.data_ptr<int64_t>(),
      int(colptr.numel() - 1), pairs.numel());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void latent_grad_v1(const torch::Tensor& colptr, const torch::Tensor& pairs, const torch::Tensor& vals,
                 const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& inv_scale,
                 const torch::Tensor& dxhat, const c10::optional<torch::Tensor>& daux,
                 const torch::Tensor& x, const c10::optional<torch::Tensor>& b_dec,
                 const torch::Tensor& W_dec, const torch::Tensor& W_enc, const torch::Tensor& gW_dec,
                 const torch::Tensor& gW_enc, const torch::Tensor& gb_enc,
                 const c10::optional<torch::Tensor>& bterm, const c10::optional<torch::Tensor>& sumsq,
                 const c10::optional<torch::Tensor>& fire_counts,
                 const c10::optional<torch::Tensor>& act_freq,
                 const c10::optional<torch::Tensor>& since_fired) {
  const at::cuda::CUDAGuard guard(vals.device());
  const int64_t N = W_dec.size(0), D = W_dec.size(1);
  SB_CHECK(W_dec.is_contiguous() && W_enc.is_contiguous() && gW_dec.is_contiguous() &&
                  gW_enc.is_contiguous() && W_enc.size(0) == N && W_enc.size(1) == D,
              "latent_grad: weights must be contiguous [N, D]");
  SB_CHECK(dxhat.is_contiguous() && dxhat.size(1) == D && x.stride(1) == 1 && x.stride(0) % 8 == 0,
              "latent_grad: dxhat / x layout");
  SB_CHECK(D % 8 == 0, "latent_grad: d_in must be a multiple of 8");
  sparse::LatentGradArgs a{};
  a.colptr = colptr.data_ptr<int64_t>();
  a.pairs = pairs.data_ptr<int64_t>();
  a.P = pairs.numel();
  a.n_main = vals.numel();
  a.k = int(vals.size(1));
  a.k_aux = aux_vals ? int(aux_vals->size(1)) : 1;
  a.vals = vals.data_ptr<float>();
  a.aux_vals = aux_vals ? aux_vals->data_ptr<float>() : nullptr;
  a.inv_scale = inv_scale ? inv_scale->data_ptr<float>() : nullptr;
  a.dxhat = reinterpret_cast<const __nv_bfloat16*>(dxhat.data_ptr());
  a.daux = daux ? reinterpret_cast<const __nv_bfloat16*>(daux->data_ptr()) : nullptr;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.b_dec = b_dec ? b_dec->data_ptr<float>() : nullptr;
  a.W_dec = reinterpret_cast<const __nv_bfloat16*>(W_dec.data_ptr());
  a.W_enc = reinterpret_cast<const __nv_bfloat16*>(W_enc.data_ptr());
  a.gW_dec = reinterpret_cast<__nv_bfloat16*>(gW_dec.data_ptr());
  a.gW_enc = reinterpret_cast<__nv_bfloat16*>(gW_enc.data_ptr());
  a.gb_enc = gb_enc.data_ptr<float>();
  a.bterm = bterm ? bterm->data_ptr<float>() : nullptr;
  a.sumsq = sumsq ? sumsq->data_ptr<float>() : nullptr;
  a.fire_counts = fire_counts ? fire_counts->data_ptr<int>() : nullptr;
  a.act_freq = act_freq ? act_freq->data_ptr<float>() : nullptr;
  a.since_fired = since_fired ? since_fired->data_ptr<float>() : nullptr;
  a.N = int(N);
  a.D = int(D);
  if (N == 0) return;
  const int vpt = pick_vpt(D, sparse::LG_THREADS);
  const int64_t grid = std::min<int64_t>(N, int64_t(sm_count()) * 4);
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (vpt) {
    case 1: sparse::latent_grad_kernel<1><<<dim3(grid), dim3(sparse::LG_THREADS), 0, stream>>>(a); break;
    case 2: sparse::latent_grad_kernel<2><<<dim3(grid), dim3(sparse::LG_THREADS), 0, stream>>>(a); break;
    case 4: sparse::latent_grad_kernel<4><<<dim3(grid), dim3(sparse::LG_THREADS), 0, stream>>>(a); break;
    default: sparse::latent_grad_kernel<8><<<dim3(grid), dim3(sparse::LG_THREADS), 0, stream>>>(a); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Two-pass latent gradients (pair_dz_kernel + latent_rows_kernel); `idx` / `aux_idx` give the
// latent of every main / aux pair.  Same contract as the single-pass kernel.
void latent_grad(const torch::Tensor& colptr, const torch::Tensor& pairs, const torch::Tensor& vals,
                 const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& inv_scale,
                 const torch::Tensor& dxhat, const c10::optional<torch::Tensor>& daux,
                 const torch::Tensor& x, const c10::optional<torch::Tensor>& b_dec,
                 const torch::Tensor& W_dec, const torch::Tensor& W_enc, const torch::Tensor& gW_dec,
                 const torch::Tensor& gW_enc, const torch::Tensor& gb_enc,
                 const c10::optional<torch::Tensor>& bterm, const c10::optional<torch::Tensor>& sumsq,
                 const c10::optional<torch::Tensor>& fire_counts,
                 const c10::optional<torch::Tensor>& act_freq,
                 const c10::optional<torch::Tensor>& since_fired, const torch::Tensor& idx,
                 const c10::optional<torch::Tensor>& aux_idx, int64_t j0, int64_t j1, bool zero_empty,
                 const c10::optional<torch::Tensor>& jr_thr, const c10::optional<torch::Tensor>& jr_pre,
                 double jr_bandwidth, double jr_l0c, const c10::optional<torch::Tensor>& jr_gthr,
                 const std::vector<int64_t>& rs_bases, int64_t rs_rank, int64_t rs_dec_off, int64_t rs_enc_off,
                 int64_t rs_n) {
  static const bool v1 = [] {
    const char* e = std::getenv("SAELENS_B200_LATENT_GRAD");
    return e && std::string(e) == "v1";
  }();
  if (j1 < 0) j1 = W_dec.size(0);
  if (v1 && j0 == 0 && j1 == W_dec.size(0) && !zero_empty && !jr_thr && rs_n == 0) {
    latent_grad_v1(colptr, pairs, vals, aux_vals, inv_scale, dxhat, daux, x, b_dec, W_dec, W_enc, gW_dec, gW_enc,
                   gb_enc, bterm, sumsq, fire_counts, act_freq, since_fired);
    return;
  }
  const at::cuda::CUDAGuard guard(vals.device());
  const int64_t N = W_dec.size(0), D = W_dec.size(1);
  SB_CHECK(W_dec.is_contiguous() && W_enc.is_contiguous() && gW_dec.is_contiguous() &&
                  gW_enc.is_contiguous() && W_enc.size(0) == N && W_enc.size(1) == D,
              "latent_grad: weights must be contiguous [N, D]");
  SB_CHECK(dxhat.is_contiguous() && dxhat.size(1) == D && x.stride(1) == 1 && x.stride(0) % 8 == 0,
              "latent_grad: dxhat / x layout");
  SB_CHECK(D % 8 == 0 && D <= 8192, "latent_grad: d_in must be a multiple of 8 and at most 8192");
  SB_CHECK(idx.is_contiguous() && idx.scalar_type() == at::kInt && idx.sizes() == vals.sizes(), "latent_grad: idx");
  SB_CHECK(x.size(0) < (int64_t(1) << 31), "latent_grad: too many rows");
  if (N == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t P = pairs.numel();
  auto opt_f = vals.options().dtype(at::kFloat);
  auto prow = torch::empty({std::max<int64_t>(P, 1)}, vals.options().dtype(at::kInt));
  auto pcoef = torch::empty({std::max<int64_t>(P, 1)}, opt_f);
  auto pdz = torch::empty({std::max<int64_t>(P, 1)}, opt_f);
  if (P > 0) {
    sparse::PairDzArgs pa{};
    pa.pairs = pairs.data_ptr<int64_t>();
    SB_CHECK(colptr.numel() == N + 1 && colptr.scalar_type() == at::kLong, "latent_grad: colptr");
    SB_CHECK(j0 >= 0 && j0 <= j1 && j1 <= N, "latent_grad: latent range");
    pa.pos_begin = colptr.data_ptr<int64_t>() + j0;
    pa.pos_end = colptr.data_ptr<int64_t>() + j1;
    pa.P = P;
    pa.n_main = vals.numel();
    pa.k = int(vals.size(1));
    pa.k_aux = aux_vals ? int(aux_vals->size(1)) : 1;
    pa.vals = vals.data_ptr<float>();
    pa.idx = idx.data_ptr<int>();
    pa.aux_vals = aux_vals ? aux_vals->data_ptr<float>() : nullptr;
    pa.aux_idx = aux_idx ? aux_idx->data_ptr<int>() : nullptr;
    pa.inv_scale = inv_scale ? inv_scale->data_ptr<float>() : nullptr;
    pa.dxhat = reinterpret_cast<const __nv_bfloat16*>(dxhat.data_ptr());
    pa.daux = daux ? reinterpret_cast<const __nv_bfloat16*>(daux->data_ptr()) : nullptr;
    pa.W_dec = reinterpret_cast<const __nv_bfloat16*>(W_dec.data_ptr());
    pa.D = int(D);
    pa.N = int(N);
    pa.prow = prow.data_ptr<int>();
    pa.pcoef = pcoef.data_ptr<float>();
    pa.pdz = pdz.data_ptr<float>();
    if (jr_thr) {
      SB_CHECK(jr_pre && jr_gthr && jr_pre->sizes() == vals.sizes() && jr_thr->numel() == N &&
                      jr_gthr->numel() == N && jr_bandwidth > 0,
                  "latent_grad: JumpReLU mode needs jr_pre [M, k], jr_thr [N], jr_gthr [N], bandwidth > 0");
      pa.jr_thr = jr_thr->data_ptr<float>();
      pa.jr_pre = jr_pre->data_ptr<float>();
      pa.jr_inv_bw = float(1.0 / jr_bandwidth);
      pa.jr_l0c = float(jr_l0c);
      pa.jr_gthr = jr_gthr->data_ptr<float>();
    }
    const int64_t grid = std::min<int64_t>((P + sparse::LR_WARPS - 1) / sparse::LR_WARPS, int64_t(sm_count()) * 8);
    sparse::pair_dz_kernel<<<dim3(grid), dim3(sparse::LR_THREADS), 0, stream>>>(pa);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  const int nvec = int(D / 8);
  // d_in slices per latent (power of two <= 8): each warp owns one slice of every latent it visits.
  // SAELENS_B200_LR_SLICES caps it (fewer, wider slices: more loads in flight per warp item).
  static const int max_ns = [] {
    const char* e = std::getenv("SAELENS_B200_LR_SLICES");
    const int v = e ? std::atoi(e) : 8;
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 8;
  }();
  int ns = 1;
  while (ns < max_ns && ns * 64 < nvec) ns *= 2;
  SB_CHECK((nvec + 32 * ns - 1) / (32 * ns) <= 4, "latent_grad: d_in too wide for ", ns, " slices");
  const int vpl = (nvec + 32 * ns - 1) / (32 * ns);
  const int sw = 32 * vpl * 8;
  const int grid = sm_count() * 2;
  const int tw = grid * sparse::LR_WARPS;
  torch::Tensor bpart;
  if (bterm) bpart = torch::empty({int64_t(tw) * sw}, opt_f);
  sparse::LatentRowsArgs a{};
  a.colptr = colptr.data_ptr<int64_t>();
  a.prow = prow.data_ptr<int>();
  a.pcoef = pcoef.data_ptr<float>();
  a.pdz = pdz.data_ptr<float>();
  a.dxhat = reinterpret_cast<const __nv_bfloat16*>(dxhat.data_ptr());
  a.daux = daux ? reinterpret_cast<const __nv_bfloat16*>(daux->data_ptr()) : nullptr;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.b_dec = b_dec ? b_dec->data_ptr<float>() : nullptr;
  a.W_enc = reinterpret_cast<const __nv_bfloat16*>(W_enc.data_ptr());
  a.gW_dec = reinterpret_cast<__nv_bfloat16*>(gW_dec.data_ptr());
  a.gW_enc = reinterpret_cast<__nv_bfloat16*>(gW_enc.data_ptr());
  a.gb_enc = gb_enc.data_ptr<float>();
  a.bpart = bterm ? bpart.data_ptr<float>() : nullptr;
  a.sumsq = sumsq ? sumsq->data_ptr<float>() : nullptr;
  a.fire_counts = fire_counts ? fire_counts->data_ptr<int>() : nullptr;
  a.act_freq = act_freq ? act_freq->data_ptr<float>() : nullptr;
  a.since_fired = since_fired ? since_fired->data_ptr<float>() : nullptr;
  a.N = int(N);
  a.D = int(D);
  a.nslices = ns;
  a.M = int(x.size(0));
  a.n_pairs = P;
  a.j0 = int(j0);
  a.j1 = int(j1);
  a.zero_empty = zero_empty ? 1 : 0;
  if (rs_n > 0) {
    SB_CHECK(zero_empty && int64_t(rs_bases.size()) * rs_n == N && rs_dec_off % 16 == 0 && rs_enc_off % 16 == 0,
                "latent_grad: reduce-scatter destination needs zero_empty, S * rs_n == N and aligned offsets");
    a.P = p2p::make_peers(rs_bases, rs_rank);
    a.rs_dec_off = rs_dec_off;
    a.rs_enc_off = rs_enc_off;
    a.rs_n = int(rs_n);
  }
  switch (vpl) {
    case 1: sparse::latent_rows_kernel<1><<<dim3(grid), dim3(sparse::LR_THREADS), 0, stream>>>(a); break;
    case 2: sparse::latent_rows_kernel<2><<<dim3(grid), dim3(sparse::LR_THREADS), 0, stream>>>(a); break;
    case 3: sparse::latent_rows_kernel<3><<<dim3(grid), dim3(sparse::LR_THREADS), 0, stream>>>(a); break;
    default: sparse::latent_rows_kernel<4><<<dim3(grid), dim3(sparse::LR_THREADS), 0, stream>>>(a); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (bterm) {
    SB_CHECK(bterm->numel() == D && bterm->scalar_type() == at::kFloat, "latent_grad: bterm");
    sparse::col_reduce_kernel<<<dim3(int((D + 31) / 32)), dim3(32, sparse::CR_ROWS), 0, stream>>>(
        bpart.data_ptr<float>(), tw, ns, sw, int(D), bterm->data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void decode_partial(const torch::Tensor& vals, const torch::Tensor& idx, bool relu,
                    const c10::optional<torch::Tensor>& inv_scale, const torch::Tensor& W, const torch::Tensor& out) {
  SB_CHECK(vals.is_contiguous() && idx.is_contiguous() && vals.scalar_type() == at::kFloat &&
                  idx.scalar_type() == at::kInt, "decode_partial: vals/idx");
  SB_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.size(1) == W.size(1), "decode_partial: out");
  const int64_t M = vals.size(0), k = vals.size(1), D = W.size(1);
  SB_CHECK(D % 8 == 0 && W.stride(1) == 1, "decode_partial: W");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(vals.device());
  const int vpt = pick_vpt(D, sparse::DEC_THREADS);
  const int64_t grid = std::min<int64_t>(M, int64_t(sm_count()) * 8);
  const size_t smem = size_t(2 * k) * 4;
  auto stream = at::cuda::getCurrentCUDAStream();
  const float* pinv = inv_scale ? inv_scale->data_ptr<float>() : nullptr;
#define SB_DP(V) sparse::decode_partial_kernel<V><<<dim3(grid), dim3(sparse::DEC_THREADS), smem, stream>>>( \
      vals.data_ptr<float>(), idx.data_ptr<int>(), int(k), vals.stride(0), relu ? 1 : 0, pinv,                  \
      reinterpret_cast<const __nv_bfloat16*>(W.data_ptr()), W.stride(0), out.data_ptr<float>(), out.stride(0),  \
      int(M), int(D), int(W.size(0)))
  switch (vpt) {
    case 1: SB_DP(1); break;
    case 2: SB_DP(2); break;
    case 4: SB_DP(4); break;
    default: SB_DP(8); break;
  }
#undef SB_DP
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void finish_mse(const torch::Tensor& xsum, const c10::optional<torch::Tensor>& bias, const torch::Tensor& target,
                const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& resid,
                const c10::optional<torch::Tensor>& dxhat, const c10::optional<torch::Tensor>& grad_coef_dev,
                double grad_coef, const torch::Tensor& loss_row, const c10::optional<torch::Tensor>& bsum) {
  SB_CHECK(xsum.scalar_type() == at::kFloat && xsum.stride(1) == 1 && xsum.stride(0) % 8 == 0, "finish_mse: xsum");
  const int64_t M = xsum.size(0), D = xsum.size(1);
  SB_CHECK(target.size(0) == M && target.size(1) == D && target.stride(1) == 1, "finish_mse: target");
  for (const auto* o : {&out, &resid, &dxhat})
    if (*o) SB_CHECK((*o)->is_contiguous() && (*o)->size(0) == M && (*o)->size(1) == D, "finish_mse: outputs");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(xsum.device());
  const int64_t grid = std::min<int64_t>(M, int64_t(sm_count()) * 8);
  sparse::finish_mse_kernel<<<dim3(grid), dim3(sparse::DEC_THREADS), 0, at::cuda::getCurrentCUDAStream()>>>(
      xsum.data_ptr<float>(), xsum.stride(0), bias ? bias->data_ptr<float>() : nullptr,
      reinterpret_cast<const __nv_bfloat16*>(target.data_ptr()), target.stride(0),
      out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr,
      resid ? reinterpret_cast<__nv_bfloat16*>(resid->data_ptr()) : nullptr,
      dxhat ? reinterpret_cast<__nv_bfloat16*>(dxhat->data_ptr()) : nullptr,
      grad_coef_dev ? grad_coef_dev->data_ptr<float>() : nullptr, float(grad_coef), loss_row.data_ptr<float>(),
      bsum ? bsum->data_ptr<float>() : nullptr, int(M), int(D));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused TP decode (see decode_rs_kernel).  vals/idx [B, k] hold this rank's winners (local
// latent ids); target [Bo, D] are the rank's own input rows (or the aux residual).  Slab
// offsets: land fp32 [S, Bo, D], lcnt u32 [Bo/16], dx bf16 [B, D] (dx_off < 0: none), dcnt u32
// [B/16].  `epoch` counts the launches that used these buffers (1, 2, ...).
void decode_rs(const torch::Tensor& vals, const torch::Tensor& idx, bool relu,
               const c10::optional<torch::Tensor>& inv_scale, const torch::Tensor& W,
               const std::vector<int64_t>& peer_bases, int64_t rank, int64_t land_off, int64_t lcnt_off,
               int64_t dx_off, int64_t dcnt_off, int64_t epoch, const c10::optional<torch::Tensor>& bias,
               const torch::Tensor& target, const c10::optional<torch::Tensor>& out,
               const c10::optional<torch::Tensor>& resid, const c10::optional<torch::Tensor>& grad_coef_dev,
               double grad_coef, const torch::Tensor& loss_row, const c10::optional<torch::Tensor>& bsum,
               const torch::Tensor& ticket, const torch::Tensor& status) {
  const int64_t S = int64_t(peer_bases.size());
  SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "decode_rs: bad group");
  SB_CHECK(vals.is_contiguous() && idx.is_contiguous() && vals.scalar_type() == at::kFloat &&
                  idx.scalar_type() == at::kInt && vals.sizes() == idx.sizes(),
              "decode_rs: vals/idx");
  const int64_t B = vals.size(0), k = vals.size(1), D = W.size(1);
  SB_CHECK(W.scalar_type() == at::kBFloat16 && W.stride(1) == 1 && D % 8 == 0 && D <= 8 * 8 * sparse::DEC_THREADS,
              "decode_rs: W");
  SB_CHECK(B % (S * sparse::RS_RB) == 0, "decode_rs: batch must be a multiple of 16 * world");
  const int64_t Bo = B / S;
  SB_CHECK(target.scalar_type() == at::kBFloat16 && target.size(0) == Bo && target.size(1) == D &&
                  target.stride(1) == 1,
              "decode_rs: target");
  for (const auto* o : {&out, &resid})
    if (*o) SB_CHECK((*o)->is_contiguous() && (*o)->size(0) == Bo && (*o)->size(1) == D, "decode_rs: outputs");
  SB_CHECK(loss_row.numel() == Bo && loss_row.scalar_type() == at::kFloat, "decode_rs: loss_row");
  if (bias) SB_CHECK(bias->numel() == D && bias->scalar_type() == at::kFloat, "decode_rs: bias");
  if (bsum) SB_CHECK(bsum->numel() == D && bsum->scalar_type() == at::kFloat, "decode_rs: bsum");
  SB_CHECK(land_off % 16 == 0 && (dx_off < 0 || dx_off % 16 == 0), "decode_rs: offsets");
  const at::cuda::CUDAGuard guard(vals.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  sparse::DecodeRsArgs a{};
  a.vals = vals.data_ptr<float>();
  a.idx = idx.data_ptr<int>();
  a.k = int(k);
  a.ldk = k;
  a.relu = relu ? 1 : 0;
  a.inv_scale = inv_scale ? inv_scale->data_ptr<float>() : nullptr;
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.ldw = W.stride(0);
  a.n_lat = int(W.size(0));
  a.B = int(B);
  a.Bo = int(Bo);
  a.D = int(D);
  a.P = p2p::make_peers(peer_bases, rank);
  a.land_off = land_off;
  a.lcnt_off = lcnt_off;
  a.dx_off = dx_off;
  a.dcnt_off = dcnt_off;
  a.epoch = uint32_t(epoch);
  a.bias = bias ? bias->data_ptr<float>() : nullptr;
  a.target = reinterpret_cast<const __nv_bfloat16*>(target.data_ptr());
  a.ldt = target.stride(0);
  a.out = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  a.resid = resid ? reinterpret_cast<__nv_bfloat16*>(resid->data_ptr()) : nullptr;
  a.grad_coef_dev = grad_coef_dev ? grad_coef_dev->data_ptr<float>() : nullptr;
  a.grad_coef = float(grad_coef);
  a.loss_row = loss_row.data_ptr<float>();
  a.bsum = bsum ? bsum->data_ptr<float>() : nullptr;
  a.ticket = ticket.data_ptr<int>();
  a.status = status.data_ptr<int>();
  const size_t smem = size_t(2 * k + 32) * 4;
  const int nvec = int(D / 8);
  auto launch = [&](auto kern, int64_t work) {
    int occ = 0;
    C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, sparse::DEC_THREADS, smem));
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(work, int64_t(sm_count()) * std::max(occ, 1)));
    kern<<<dim3(grid), dim3(sparse::DEC_THREADS), smem, stream>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  };
  const int64_t nA = B / sparse::RS_RB, nB = Bo / sparse::RS_RB;
  // SAELENS_B200_DECODE_RS=split: phase A and phase B as two launches (phase A at the occupancy of
  // its own register count); default: one ticketed launch.
  static const bool split = [] {
    const char* e = std::getenv("SAELENS_B200_DECODE_RS");
    return e && std::string(e) == "split";
  }();
  if (!split) C10_CUDA_CHECK(cudaMemsetAsync(a.ticket, 0, sizeof(int), stream));
  auto run = [&](auto k0, auto k1, auto k2) {
    if (split) {
      launch(k1, nA);
      launch(k2, nB);
    } else {
      launch(k0, nA + nB);
    }
  };
  if (nvec <= sparse::DEC_THREADS) {
    run(sparse::decode_rs_kernel<1, 0>, sparse::decode_rs_kernel<1, 1>, sparse::decode_rs_kernel<1, 2>);
  } else if (nvec <= 2 * sparse::DEC_THREADS) {
    run(sparse::decode_rs_kernel<2, 0>, sparse::decode_rs_kernel<2, 1>, sparse::decode_rs_kernel<2, 2>);
  } else if (nvec <= 4 * sparse::DEC_THREADS) {
    run(sparse::decode_rs_kernel<4, 0>, sparse::decode_rs_kernel<4, 1>, sparse::decode_rs_kernel<4, 2>);
  } else {
    run(sparse::decode_rs_kernel<8, 0>, sparse::decode_rs_kernel<8, 1>, sparse::decode_rs_kernel<8, 2>);
  }
}


}  // namespace sb

#if SB_DEBUG_BOUNDS
namespace sb {
// {line, value, bound, violations} of this file's first bounds violation (debug module only).
std::vector<int64_t> sparse_bounds_info(bool reset) { return bounds_read(reset); }
}  // namespace sb
#endif

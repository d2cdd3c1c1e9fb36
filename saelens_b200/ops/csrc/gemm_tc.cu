// tcgen05 GEMM for the SAE encoder:  H[m, n] = epilogue( sum_k A[m, k] * B[n, k] )
//
// A (activations, [M, K]) and B (encoder weights stored latent-major, [N, K]) are both
// K-major bf16, which is the native operand layout of tcgen05.mma.  The kernel is persistent
// (one CTA per SM) and warp-specialised:
//   warp 0      TMA producer: 128x64 A tile + 256x64 B tile per stage, 4 stages, SWIZZLE_128B
//   warp 1      MMA issuer:   4 x tcgen05.mma (M=128, N=256, K=16) per stage, fp32 accumulate
//               into one of two 256-column TMEM accumulators
//   warps 2..5  epilogue:     tcgen05.ld a row per thread, bias / per-column scale / ReLU,
//               round to bf16, store, and optionally the max of every 32-column chunk
// Double-buffered TMEM lets the epilogue of tile i overlap the main loop of tile i+1.
//
// The fused epilogue replaces the reference's `sae_in @ W_enc + b_enc` followed by
// `hidden_pre * W_dec.norm(dim=-1)` (sae_lens/saes/topk_sae.py:626-630): with bias = b_enc -
// W_enc^T b_dec (b_dec folded, so A is the raw input) and scale = ||W_dec[j]||.  The chunk
// maxima let the row top-k kernel skip every 32-column chunk that cannot hold a top-k value.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tmap.h"

namespace sb {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_TILE_BYTES = BM * BK * 2;
constexpr int B_TILE_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
constexpr int NUM_EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;
constexpr int GROUP_N = 16;  // n-tiles per raster group (L2 reuse of A and B)
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct Epi {
  __nv_bfloat16* out;      // [M, ldo] or nullptr
  int64_t ldo;
  const float* bias;       // [N] or nullptr
  const float* scale;      // [N] or nullptr (applied after bias)
  int relu;                // apply max(., 0) after bias/scale
  __nv_bfloat16* cmax;     // [M, ldc] chunk maxima (one per 32 columns) or nullptr
  int64_t ldc;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mt, int& nt) {
  const int group = t / (num_m * GROUP_N);
  const int first_n = group * GROUP_N;
  const int gsize = min(GROUP_N, num_n - first_n);
  const int r = t - group * num_m * GROUP_N;
  mt = r / gsize;
  nt = first_n + r % gsize;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   int M, int N, int K, Epi ep, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_TILE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + STAGES * B_TILE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], NUM_EPI_WARPS * 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, num_m, num_n, mt, nt);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1, abort_flag, status, kTimeoutTmaProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
          tma_load_2d(sA + s * A_TILE_BYTES, &tmA, &full_bar[s], kb * BK, mt * BM);
          tma_load_2d(sB + s * B_TILE_BYTES, &tmB, &full_bar[s], kb * BK, nt * BN);
        }
      }
      if (!ok) {
        // drain the copies already issued before leaving (bounded)
        const uint32_t first = it > STAGES ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j) {
          volatile int dummy = 0;
          mbar_wait_bounded(&full_bar[j % STAGES], (j / STAGES) & 1, &dummy, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (elect_one()) {
      const uint32_t idesc = make_idesc_bf16_f32(BM, BN);
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tc) {
        const int acc = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], aph ^ 1, abort_flag, status,
                               kTimeoutMmaTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(&full_bar[s], ph, abort_flag, status, kTimeoutMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * A_TILE_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * B_TILE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16_ss(d_tmem, make_sdesc_sw128_kmajor(a_addr + k * 32),
                         make_sdesc_sw128_kmajor(b_addr + k * 32), idesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tc) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const int acc = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], aph, abort_flag, status, kTimeoutEpilogue)) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(trow + c * 32, r);
        tmem_ld_wait();
        const int col0 = nt * BN + c * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (ep.bias) {
          const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 b = __ldg(b4 + j);
            v[4 * j] += b.x;
            v[4 * j + 1] += b.y;
            v[4 * j + 2] += b.z;
            v[4 * j + 3] += b.w;
          }
        }
        if (ep.scale) {
          const float4* s4 = reinterpret_cast<const float4*>(ep.scale + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 s = __ldg(s4 + j);
            v[4 * j] *= s.x;
            v[4 * j + 1] *= s.y;
            v[4 * j + 2] *= s.z;
            v[4 * j + 3] *= s.w;
          }
        }
        if (ep.relu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
        }
        uint32_t packed[16];
        float cm = -INFINITY;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
          packed[j] = *reinterpret_cast<uint32_t*>(&h2);
          cm = fmaxf(cm, fmaxf(__low2float(h2), __high2float(h2)));
        }
        if (row < M) {
          if (ep.out) {
            uint4* dst = reinterpret_cast<uint4*>(ep.out + int64_t(row) * ep.ldo + col0);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                                  packed[4 * j + 3]);
          }
          if (ep.cmax) ep.cmax[int64_t(row) * ep.ldc + (col0 >> 5)] = __float2bfloat16_rn(cm);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm

// ------------------------------------------------------------------------------------------
// host entry
// ------------------------------------------------------------------------------------------
static int num_sms_cached() {
  static int n = -1;
  if (n < 0) {
    int dev;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// out = epilogue(A @ B^T).  A: [M, K] bf16 (row stride lda), B: [N, K] bf16.  Optional
// bias/scale fp32 [N].  Returns nothing; writes `out` [M, N] bf16 and/or `cmax` [M, N/32] bf16.
void gemm_tn_bf16(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& bias,
                  const c10::optional<torch::Tensor>& scale, bool relu,
                  const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                  const torch::Tensor& status, int64_t max_ctas) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "gemm_tn_bf16: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16,
              "gemm_tn_bf16: bf16 operands required");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_tn_bf16: shape");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_tn_bf16: K must be contiguous");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(K % gemm::BK == 0, "gemm_tn_bf16: K must be a multiple of 64, got ", K);
  TORCH_CHECK(N % gemm::BN == 0, "gemm_tn_bf16: N must be a multiple of 256, got ", N);
  TORCH_CHECK(M >= 1 && M < (1ll << 31) && N < (1ll << 31), "gemm_tn_bf16: size");
  const at::cuda::CUDAGuard guard(A.device());

  gemm::Epi ep{};
  if (out) {
    TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->size(0) == M && out->size(1) == N &&
                    out->stride(1) == 1 && out->stride(0) % 8 == 0,
                "gemm_tn_bf16: bad out");
    ep.out = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    ep.ldo = out->stride(0);
  }
  if (cmax) {
    TORCH_CHECK(cmax->scalar_type() == at::kBFloat16 && cmax->size(0) == M &&
                    cmax->size(1) == N / 32 && cmax->stride(1) == 1,
                "gemm_tn_bf16: bad cmax");
    ep.cmax = reinterpret_cast<__nv_bfloat16*>(cmax->data_ptr());
    ep.ldc = cmax->stride(0);
  }
  if (bias) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N && bias->is_contiguous(),
                "gemm_tn_bf16: bias must be fp32 [N]");
    ep.bias = bias->data_ptr<float>();
  }
  if (scale) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->numel() == N && scale->is_contiguous(),
                "gemm_tn_bf16: scale must be fp32 [N]");
    ep.scale = scale->data_ptr<float>();
  }
  ep.relu = relu ? 1 : 0;

  CUtensorMap tA = make_tmap_2d(A.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K,
                                A.stride(0) * 2, gemm::BM, gemm::BK,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tB = make_tmap_2d(B.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K,
                                B.stride(0) * 2, gemm::BN, gemm::BK,
                                CU_TENSOR_MAP_SWIZZLE_128B);

  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm::gemm_tn_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        gemm::SMEM_BYTES));
    attr_set = true;
  }
  const int64_t tiles = ((M + gemm::BM - 1) / gemm::BM) * (N / gemm::BN);
  int64_t grid = std::min<int64_t>(tiles, num_sms_cached());
  if (max_ctas > 0) grid = std::min<int64_t>(grid, max_ctas);
  auto stream = at::cuda::getCurrentCUDAStream();
  gemm::gemm_tn_kernel<<<dim3(grid), dim3(gemm::NUM_THREADS), gemm::SMEM_BYTES, stream>>>(
      tA, tB, int(M), int(N), int(K), ep, status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

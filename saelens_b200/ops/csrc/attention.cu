// Prefill attention for the activation-producing LM on tcgen05 (causal or full, grouped-query,
// optional logit soft-capping):
//
//   z[b, s, h, :] = sum_t softmax_t( cap(q[b,s,h] . k[b,t,h/g] * scale) ) v[b,t,h/g]      (t <= s if causal)
//
// q is [B, S, H, D] and k, v are [B, S, KV, D] (bf16, head dim contiguous, any token stride, so
// views into a fused QKV projection work); g = H / KV query heads share one K/V head, which is
// read from its own rows (no repeat of K/V).  `cap` is the identity or x -> c * tanh(x / c)
// (Gemma-2's attention soft-capping).  Replaces `F.scaled_dot_product_attention` and the eager
// soft-capped path of the producer (the reference runs its producer in HookedTransformer or in
// vLLM's kernels: sae_lens/vllm_model.py:626-743, sae_lens/load_model.py:17-67).
//
// One CTA computes 128 query rows of one head (the heaviest causal tiles are scheduled first):
//   warp 0      TMA: the Q tile once, then K and V tiles of BN rows through 2 stages (SWIZZLE_128B)
//   warp 1      MMA: S_j = Q K_j^T into one of two TMEM buffers (M=128, N=BN), and after the
//               softmax has produced P_j, O += P_j V_j (M=128, N=D, V read MN-major) in TMEM
//   warps 2..5  softmax, one query row per thread: tcgen05.ld of S_j, scale / soft-cap / causal
//               mask, running max and sum (online softmax), P_j as bf16 into shared memory in the
//               K-major SWIZZLE_128B layout the MMA reads; O is rescaled in TMEM only when the row
//               max grew by more than 2^8 since the last rescale (exact: the stale max only bounds
//               P by 256), and at the end O / l is written out as bf16.  Only the tiles that cross
//               the diagonal or the sequence end are masked; the row max and sum run as four
//               independent chains.  (With SAELENS_B200_ATTN_WARPS=8, warps 2..9 take half a row
//               each and exchange the row maxima and sums through shared memory on a bounded
//               mbarrier; measured slightly slower, so four warps are the default.)
// S_{j+1} is computed while the softmax works on S_j.  Every wait is bounded (status word).
#include <ATen/cuda/CUDAContext.h>
#include <cstdlib>
#include <string>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tmap.h"
#include "check.h"

namespace sb {
namespace attn {

constexpr int BM = 128;
// softmax warps: 4 (one per TMEM lane quadrant, whole rows) or 8 (two per quadrant, each with half
// of the columns; the halves exchange row maxima and sums through shared memory)
constexpr int threads_for(int smw) { return 64 + 32 * smw; }
constexpr int KV_STAGES = 2;
constexpr int TMEM_COLS = 512;
constexpr float kRescaleThreshold = 8.f;  // log2 units: rescale O once the max grew by 2^8

template <int D, int BN, int SMW = 4>
struct Cfg {
  static_assert(D % 64 == 0 && BN % 64 == 0, "tiles are made of 64-element swizzle rows");
  static_assert(2 * BN + D <= TMEM_COLS, "two S buffers and O must fit in TMEM");
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;  // one K or one V tile
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int NUM_BARS = 11;
  static constexpr int XBUF_FLOATS = 6 * BM;  // max exchange [2 tiles][2 halves][BM] + sums [2][BM]
  static constexpr int SMEM = Q_BYTES + 2 * KV_STAGES * KV_BYTES + P_BYTES + 4 * XBUF_FLOATS + 1024 + 8 * NUM_BARS + 16;
  static constexpr int HALVES = SMW / 4;
  static constexpr int CW = BN / HALVES;  // S / P columns per softmax thread
  static constexpr int DW = D / HALVES;   // O columns per softmax thread
  static_assert(SMW == 4 || SMW == 8, "4 or 8 softmax warps");
  static_assert(CW % 32 == 0 && DW % 32 == 0, "32-column TMEM loads");
};

struct Params {
  int B, S, H, KV;
  int causal;
  float scale_log2;      // softmax scale * log2(e) (no soft-cap)
  float cap_log2;        // soft-cap c * log2(e), 0 = no soft-cap
  float scale_over_cap;  // softmax scale / c
  __nv_bfloat16* out;    // [B, S, H, D] contiguous
  int* status;
};

// 2^x with the hardware's approximate base-2 exponential (PTX ex2.approx.ftz.f32): P is rounded
// to bf16 right after, far coarser than the instruction's error.
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// SOFTCAP is a template flag so the plain kernel carries no tanh code in its unrolled loops.
template <int D, int BN, bool SOFTCAP, int SMW>
__global__ void __launch_bounds__(threads_for(SMW), 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D, BN, SMW>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                // D/64 chunks of [BM rows x 128 B]
  uint8_t* sK = sQ + C::Q_BYTES;                     // stage s: D/64 chunks of [BN rows x 128 B]
  uint8_t* sV = sK + KV_STAGES * C::KV_BYTES;
  uint8_t* sP = sV + KV_STAGES * C::KV_BYTES;        // BN/64 chunks of [BM rows x 128 B]
  float* xbuf = reinterpret_cast<float*>(sP + C::P_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(xbuf + C::XBUF_FLOATS);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 8;
  uint64_t* drain = bars + 9;
  uint64_t* xchg = bars + 10;  // the softmax halves' exchange (8 softmax warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (p.S + BM - 1) / BM;
  const int qt = nqt - 1 - int(blockIdx.x);  // heaviest causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.H / p.KV);
  const int q0 = qt * BM;
  const int kv_tiles_all = (p.S + BN - 1) / BN;
  const int n_kv = p.causal ? min((q0 + BM + BN - 1) / BN, kv_tiles_all) : kv_tiles_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
    }
    mbar_init(p_full, SMW * 32);
    mbar_init(xchg, SMW * 32);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tO = tmem_base + 2 * BN;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int c = 0; c < D / 64; ++c) tma_load_3d(sQ + c * BM * 128, &tmQ, q_full, h * D + c * 64, q0, b);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait_bounded(&kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.status, kTimeoutTmaProducer)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * C::KV_BYTES);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sK + s * C::KV_BYTES + c * BN * 128, &tmK, &kv_full[s], kvh * D + c * 64, j * BN, b);
          tma_load_3d(sV + s * C::KV_BYTES + c * BN * 128, &tmV, &kv_full[s], kvh * D + c * 64, j * BN, b);
        }
        issued = j + 1;
      }
      // every copy issued lands before the CTA leaves (bounded, also after an abort; in a normal
      // run these phases completed long ago)
      volatile int keep_waiting = 0;
      mbar_wait_bounded(q_full, 0, &keep_waiting, nullptr, 0);
      for (int j = max(0, issued - KV_STAGES); j < issued; ++j)
        mbar_wait_bounded(&kv_full[j & 1], (j >> 1) & 1, &keep_waiting, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc_qk = make_idesc_bf16_f32(BM, BN);
      const uint32_t idesc_pv = make_idesc_bf16_f32(BM, D) | (1u << 16);  // B (= V) MN-major
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.status, kTimeoutMmaFull);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait_bounded(&kv_full[s], (j >> 1) & 1, abort_flag, p.status, kTimeoutMmaFull)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int chunk = kk >> 2, within = kk & 3;
          const uint64_t a = make_sdesc_sw128_kmajor(smem_u32(sQ + chunk * BM * 128 + within * 32));
          const uint64_t bd = make_sdesc_sw128_kmajor(smem_u32(sK + s * C::KV_BYTES + chunk * BN * 128 + within * 32));
          umma_bf16_ss(tmem_base + s * BN, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n_kv > 1) ok = issue_s(1);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (!mbar_wait_bounded(p_full, j & 1, abort_flag, p.status, kTimeoutMmaFull)) break;
        tc_fence_after();
        const int s = j & 1;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const int chunk = kk >> 2, within = kk & 3;
          const uint64_t a = make_sdesc_sw128_kmajor(smem_u32(sP + chunk * BM * 128 + within * 32));
          const uint64_t bd = make_sdesc_sw128_mnmajor(smem_u32(sV + s * C::KV_BYTES + kk * 16 * 128), BN * 128);
          umma_bf16_ss(tO, a, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[s]);
        umma_commit(o_done);
        if (j + 2 < n_kv) ok = issue_s(j + 2);
      }
      // every MMA issued above completes before TMEM is released
      umma_commit(drain);
      volatile int keep_waiting = 0;
      mbar_wait_bounded(drain, 0, &keep_waiting, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    // warp w handles TMEM lane quadrant w % 4 (rows 32 (w % 4) ..), columns of its half
    constexpr int HALVES = C::HALVES, CW = C::CW, DW = C::DW;
    const int quad = warp & 3;
    const int half = (warp - 2) / 4;
    const int row = quad * 32 + lane;
    const int q_idx = q0 + row;
    const uint32_t lane_base = uint32_t(quad * 32) << 16;
    const int col0 = half * CW;  // first S / P column of this thread
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // the halves of a row meet once per tile (and once at the end) on the exchange barrier;
    // a half that gave up stops arriving and the other's bounded wait ends too
    auto exchange = [&](int phase) -> bool {
      mbar_arrive(xchg);
      return __all_sync(0xffffffffu, mbar_wait_bounded(xchg, phase & 1, abort_flag, p.status, kTimeoutEpilogue));
    };
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      // warp-uniform outcome: the tcgen05.ld below is a whole-warp instruction
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[s], (j >> 1) & 1, abort_flag, p.status, kTimeoutEpilogue))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[CW];
      // two 32-column loads in flight per wait; scale (or soft-cap) in place
#pragma unroll
      for (int c = 0; c < CW / 32; c += 2) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(tmem_base + lane_base + s * BN + col0 + c * 32, r0);
        if (c + 1 < CW / 32) tmem_ld_32x32b_x32(tmem_base + lane_base + s * BN + col0 + (c + 1) * 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if constexpr (SOFTCAP) {
            v[c * 32 + e] = p.cap_log2 * tanhf(__uint_as_float(r0[e]) * p.scale_over_cap);
            if (c + 1 < CW / 32) v[(c + 1) * 32 + e] = p.cap_log2 * tanhf(__uint_as_float(r1[e]) * p.scale_over_cap);
          } else {
            v[c * 32 + e] = __uint_as_float(r0[e]) * p.scale_log2;
            if (c + 1 < CW / 32) v[(c + 1) * 32 + e] = __uint_as_float(r1[e]) * p.scale_log2;
          }
        }
      }
      // only tiles that cross the diagonal or the sequence end need the mask (warp-uniform test)
      if ((p.causal && (j + 1) * BN - 1 > q0) || (j + 1) * BN > p.S) {
        const int lim = min(p.causal ? q_idx : p.S - 1, p.S - 1) - j * BN - col0;  // last visible column
#pragma unroll
        for (int e = 0; e < CW; ++e)
          if (e > lim) v[e] = -INFINITY;
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
#pragma unroll
      for (int e = 0; e < CW; e += 4) {
        mx[0] = fmaxf(mx[0], v[e]);
        mx[1] = fmaxf(mx[1], v[e + 1]);
        mx[2] = fmaxf(mx[2], v[e + 2]);
        mx[3] = fmaxf(mx[3], v[e + 3]);
      }
      float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      if constexpr (HALVES == 2) {
        float* xb = xbuf + (j & 1) * 2 * BM;  // alternate buffers: a half is at most one tile ahead
        xb[half * BM + row] = tmax;
        if (!exchange(j)) {
          ok = false;
          break;
        }
        tmax = fmaxf(tmax, xb[(half ^ 1) * BM + row]);
      }
      // both halves take the same decisions from the same row maximum
      bool need = false;
      float m_new = m_run;
      if (tmax > m_run + kRescaleThreshold) {
        m_new = tmax;
        need = true;
      }
      const float alpha = need ? exp2f(m_run - m_new) : 1.f;  // m_run = -inf -> 0 (l_run is 0 then)
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      if (j > 0) {
        // P_{j-1} V_{j-1} has finished: the P buffer is free and O holds every earlier tile
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(o_done, (j - 1) & 1, abort_flag, p.status, kTimeoutEpilogue))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < DW / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tO + lane_base + half * DW + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st_32x32b_x32(tO + lane_base + half * DW + c * 32, r);
          }
          tmem_st_wait();
        }
      }
      l_run *= alpha;
      m_run = m_new;
      float rs[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums
#pragma unroll
      for (int g8 = 0; g8 < CW / 8; ++g8) {  // one 16-byte granule (8 columns) per step
        const int col = col0 + g8 * 8;
        uint8_t* prow = sP + (col / 64) * BM * 128 + row * 128;
        uint32_t packed[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float e0 = ex2_fast(v[g8 * 8 + 2 * i] - m_use);
          const float e1 = ex2_fast(v[g8 * 8 + 2 * i + 1] - m_use);
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(e0, e1);
          rs[i] += __low2float(h2) + __high2float(h2);
          packed[i] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(prow + ((((col % 64) / 8) ^ (row & 7)) << 4)) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
      l_run += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if constexpr (HALVES == 2) {
      // the row sum is the sum of the halves' sums (both halves are here only if neither gave up)
      if (ok) {
        xbuf[4 * BM + half * BM + row] = l_run;
        ok = exchange(n_kv);
        if (ok) l_run += xbuf[4 * BM + (half ^ 1) * BM + row];
      }
    }
    if (ok && n_kv > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(o_done, (n_kv - 1) & 1, abort_flag, p.status, kTimeoutEpilogue))) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* dst = p.out + ((int64_t(b) * p.S + q_idx) * p.H + h) * D + half * DW;
#pragma unroll 1
      for (int c = 0; c < DW / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tO + lane_base + half * DW + c * 32, r);
        tmem_ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const __nv_bfloat162 h2 =
              __floats2bfloat162_rn(__uint_as_float(r[2 * e]) * inv, __uint_as_float(r[2 * e + 1]) * inv);
          packed[e] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        if (q_idx < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = make_uint4(packed[4 * e], packed[4 * e + 1], packed[4 * e + 2], packed[4 * e + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int D, int BN, bool SOFTCAP, int SMW>
void launch(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const Params& prm) {
  using C = Cfg<D, BN, SMW>;
  const int B = prm.B, S = prm.S, H = prm.H, KV = prm.KV;
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq = make_tmap_3d(q.data_ptr(), bf, 2, uint64_t(H) * D, S, B, q.stride(1) * 2, q.stride(0) * 2, 64, BM, 1,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tk = make_tmap_3d(k.data_ptr(), bf, 2, uint64_t(KV) * D, S, B, k.stride(1) * 2, k.stride(0) * 2, 64, BN,
                                1, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = make_tmap_3d(v.data_ptr(), bf, 2, uint64_t(KV) * D, S, B, v.stride(1) * 2, v.stride(0) * 2, 64, BN,
                                1, CU_TENSOR_MAP_SWIZZLE_128B);
  auto kern = attn_fwd_kernel<D, BN, SOFTCAP, SMW>;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set = true;
  }
  const dim3 grid((S + BM - 1) / BM, H, B);
  kern<<<grid, threads_for(SMW), C::SMEM, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, prm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace attn

// q [B, S, H, D], k / v [B, S, KV, D] bf16 (head dim contiguous, heads adjacent within a token,
// token and batch strides multiples of 8 elements); out [B, S, H, D] contiguous bf16.
// softcap <= 0 disables soft-capping.  D must be 64, 128 or 256.
void attention_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& out,
                   double scale, double softcap, bool causal, const torch::Tensor& status) {
  SB_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && out.is_cuda(), "attention_fwd: CUDA tensors required");
  SB_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "attention_fwd: bf16 tensors required");
  SB_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention_fwd: q, k, v must be [B, S, heads, D]");
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), D = q.size(3), KV = k.size(2);
  SB_CHECK(D == 64 || D == 128 || D == 256, "attention_fwd: head dim must be 64, 128 or 256, got ", D);
  SB_CHECK(k.size(0) == B && k.size(1) == S && k.size(3) == D && v.sizes() == k.sizes(), "attention_fwd: k/v shape");
  SB_CHECK(KV >= 1 && H % KV == 0, "attention_fwd: query heads must be a multiple of the K/V heads");
  for (const auto* t : {&q, &k, &v}) {
    SB_CHECK(t->stride(3) == 1 && t->stride(2) == D && t->stride(1) % 8 == 0 && t->stride(0) % 8 == 0,
                "attention_fwd: head dim contiguous, heads adjacent, token/batch strides multiples of 8");
  }
  SB_CHECK(out.is_contiguous() && out.sizes() == q.sizes(), "attention_fwd: out must be contiguous [B, S, H, D]");
  SB_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "attention_fwd: status");
  SB_CHECK(B <= 65535 && H <= 65535 && S < (1 << 30), "attention_fwd: size");
  if (B == 0 || S == 0 || H == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  attn::Params prm{};
  prm.B = int(B);
  prm.S = int(S);
  prm.H = int(H);
  prm.KV = int(KV);
  prm.causal = causal ? 1 : 0;
  const float log2e = 1.4426950408889634f;
  prm.scale_log2 = float(scale) * log2e;
  prm.cap_log2 = softcap > 0 ? float(softcap) * log2e : 0.f;
  prm.scale_over_cap = softcap > 0 ? float(scale / softcap) : 0.f;
  prm.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  prm.status = status.data_ptr<int>();
  const bool cap = softcap > 0;
  // default four softmax warps (whole rows: measured faster); SAELENS_B200_ATTN_WARPS=8 takes
  // eight (half rows with exchanged row maxima and sums)
  const char* w = std::getenv("SAELENS_B200_ATTN_WARPS");
  const bool four = !(w && std::string(w) == "8");
#define SB_ATTN(DD, BB)                                                                              \
  (four ? (cap ? attn::launch<DD, BB, true, 4>(q, k, v, prm) : attn::launch<DD, BB, false, 4>(q, k, v, prm)) \
        : (cap ? attn::launch<DD, BB, true, 8>(q, k, v, prm) : attn::launch<DD, BB, false, 8>(q, k, v, prm)))
  switch (D) {
    case 64: SB_ATTN(64, 128); break;
    case 128: SB_ATTN(128, 128); break;
    default: SB_ATTN(256, 64); break;  // D == 256 (checked above)
  }
#undef SB_ATTN
}

}  // namespace sb

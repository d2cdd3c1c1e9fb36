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
//
// All-gather fused variant (tensor-parallel encoder, AG=true): A is the full input [B, K] in
// this rank's symmetric slab, of which only the rank's own rows [r*Bo, (r+1)*Bo) exist when
// the kernel starts.  Two extra warps per CTA push the own rows, one 128-row tile at a time, into
// every rank's slab over NVLink and publish a per-tile epoch flag on the receiver.  The TMA
// producer waits (acquire, bounded) for the flag of each m-tile before loading it, and the tile
// order starts with the rank's own rows, then the next rank's, so the transfers overlap the
// tensor-core work instead of preceding it (the reference all-gathers first and multiplies
// after: sae_lens/distributed.py:404-461 around sae_lens/saes/topk_sae.py:626).
//
// Parameter all-gather variant (sharded data parallel / FSDP, operand = B): B is the full
// encoder weight [N, K] in the slab, of which each rank owns the latents [r*n, (r+1)*n).  The
// copy warps push the own latent rows, one 256-row n-tile at a time, to every rank; the producer
// waits for each n-tile's flag, and the tile walk starts at the rank's own latents.  A second
// operand (the decoder shard) can ride along: its tiles are pushed and flagged after the first
// operand's, and nothing in this kernel waits for them (the decode does).  Replaces the
// parameter all-gather that torch FSDP runs before the forward
// (sae_lens/llm_sae_training_runner.py:449-463).
#include <ATen/cuda/CUDAContext.h>
#include <cstdlib>
#include <string>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "p2p.cuh"
#include "tmap.h"
#include "check.h"

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
constexpr int NUM_COPY_WARPS = 2;  // all-gather pushers (AG variant only)
constexpr int NUM_THREADS_AG = NUM_THREADS + 32 * NUM_COPY_WARPS;
constexpr int MAX_MTILES = 4096;   // ready bitmap capacity of the AG producer (524288 rows)
constexpr int TMEM_COLS = 2 * BN;
constexpr int GROUP_N = 16;  // n-tiles per raster group (L2 reuse of A and B)
constexpr int STAGE_OUT_BYTES = 32 * 64;  // one epilogue warp's 32 x 32 bf16 staging tile (dense stores)
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + NUM_EPI_WARPS * STAGE_OUT_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct Epi {
  __nv_bfloat16* out;      // [M, ldo] or nullptr
  int64_t ldo;
  const float* bias;       // [N] or nullptr
  const float* scale;      // [N] or nullptr (applied after bias)
  int relu;                // apply max(., 0) after bias/scale
  __nv_bfloat16* cmax;     // [M, ldc] chunk maxima (one per 32 columns) or nullptr
  int64_t ldc;
  __nv_bfloat16* tmax;     // [M, ldt] tile maxima (one per 256 columns) or nullptr
  int64_t ldt;
  int tma_out;             // 1: `out` is written by TMA tile stores from a per-warp staging tile
  unsigned long long* amax;  // [M] row argmax keys (atomicMax; see argmax_key) or nullptr
};

// Order-preserving 64-bit key of (value, column) for a row argmax by atomicMax: the high word maps
// the fp32 value to an unsigned integer with the same order (sign bit flipped for values >= 0,
// all bits flipped for negatives; -0 is taken as +0), the low word is 0xFFFFFFFF - column so that
// of equal values the smallest column wins.  A key of 0 means no column was seen.
__device__ __forceinline__ unsigned long long argmax_key(float v, int col) {
  uint32_t b = v == 0.f ? 0u : __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<unsigned long long>(0xFFFFFFFFu - uint32_t(col));
}

// Epilogue of the dense SAE steps (every field optional; order of application below).
//   v = acc - r1_row[row] * r1_col[col] + bias[col]                      (rank-1 correction, bias)
//   residual mode (target):  out2 = v (reconstruction), loss += (v - t)^2, v = res_coef * (v - t)
//   JumpReLU backward (hin): gthr[col] += rect((h - thr) / bw) * (-(thr / bw) * v - l0c),
//                            v = v * 1[h > thr]
//   JumpReLU forward (thr, no hin): out2 = v (pre-activation), v = v * 1[v > thr]
//   gated (gate_bias):       out2 = relu(acc + gate_bias) (gate path), v = 1[acc + gate_bias > 0] *
//                            relu(acc * mag_scale + bias)        (magnitude path: x (W * e^r) + b_mag)
//   relu;  colsum[col] += v;  hsum[col] += v * (h - hoff[col]) (backward mode);
//   colsum2[col] += out2 (gated: the gate activations);
//   combine (addend): v = v * oscale[col] + addend[row, col];
//   out = bf16(v);  then over the stored values: colcnt[col] += 1[v != 0], nnz += 1[v != 0],
//   sumsq += v^2 (rows >= M and columns >= N contribute nothing).
struct EpiD {
  __nv_bfloat16* out;
  int64_t ldo;
  __nv_bfloat16* out2;
  int64_t ldo2;
  const float* bias;
  const float* r1_row;
  const float* r1_col;
  const float* thr;
  int relu;
  const __nv_bfloat16* hin;
  int64_t ldh;
  float inv_bw, l0c;
  float* gthr;
  const __nv_bfloat16* target;
  int64_t ldtg;
  float res_coef;
  float* loss;
  float* colsum;
  float* colcnt;
  unsigned long long* nnz;
  float* sumsq;
  const float* gate_bias;
  const float* mag_scale;
  // reduce-scatter mode (rs_n > 0): output row `row` belongs to owner o = row / rs_n and is stored
  // over NVLink into o's slab at rs_off, slot [P.rank], row (row - o * rs_n) (ldo apart); the
  // stores are made visible system-wide before the kernel ends
  p2p::Peers P;
  int64_t rs_off;
  int rs_n;
  float* hsum;
  const float* hoff;
  float* colsum2;
  const __nv_bfloat16* addend;
  int64_t ldad;
  const float* oscale;
  int staged;  // 1: full 32-column chunks are stored through the warp's staging tile
};

// Sum over the 32 lanes of v[c] for every c; lane L returns the sum for column L.  Butterfly
// transpose-reduce: 16 + 8 + 4 + 2 + 1 shuffles; `v` is destroyed.
__device__ __forceinline__ float warp_colsum32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, float (&f)[32]) {
  const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = p4[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(h[j]);
      f[8 * q + 2 * j] = t.x;
      f[8 * q + 2 * j + 1] = t.y;
    }
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* p, const float (&f)[32], int n_valid) {
  if (n_valid >= 32) {
    uint4* p4 = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(f[8 * q + 2 * j], f[8 * q + 2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&h2);
      }
      p4[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n_valid) p[j] = __float2bfloat16_rn(f[j]);
  }
}

// Dense epilogue of one accumulator tile (see EpiD); `lane` is the thread's lane.
// A warp's 32 rows x 32 columns of bf16 (this lane holds row `lane` in `f`) stored row-contiguously
// through `stage` (2 KB): each lane writes its row's four 16-byte granules (XOR-swizzled so the
// 32 lanes spread over the banks), then every store instruction writes 8 rows x 64 contiguous
// bytes instead of 32 rows x 16 bytes.  `row_ptr` (16-byte aligned) and `rowok` are this lane's;
// the other lanes' are shuffled in.  Used for full 32-column chunks only.
__device__ __forceinline__ int stage_off(int r, int q) {
  return (r >> 1) * 128 + ((((r & 1) << 2) + (q ^ ((r >> 1) & 3))) << 4);
}
__device__ __forceinline__ void warp_store_rows_bf16x32(uint8_t* stage, const float (&f)[32],
                                                        __nv_bfloat16* row_ptr, bool rowok, int lane) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(f[8 * q + 2 * j], f[8 * q + 2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(stage + stage_off(lane, q)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  __syncwarp();
  const unsigned long long mine = reinterpret_cast<unsigned long long>(row_ptr);
  const int ok_mine = rowok ? 1 : 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2), q = lane & 3;
    const unsigned long long p = __shfl_sync(0xffffffffu, mine, r);
    const int ok = __shfl_sync(0xffffffffu, ok_mine, r);
    if (ok) reinterpret_cast<uint4*>(p)[q] = *reinterpret_cast<const uint4*>(stage + stage_off(r, q));
  }
  __syncwarp();  // the staging tile is free again
}

__device__ __forceinline__ void epilogue_tile_dense(const EpiD& e, uint32_t trow, int row, int M, int N, int nt,
                                                    int lane, uint8_t* stage = nullptr) {
  const bool rowok = row < M;
  // row stores: through the warp's staging tile for full 32-column chunks (`stage` given and every
  // lane calling), per thread otherwise; `p` points at this lane's row and column col0
  auto put = [&](__nv_bfloat16* p, const float (&f)[32], int nv, bool ok) {
    if (stage != nullptr && nv == 32) {
      warp_store_rows_bf16x32(stage, f, p, ok, lane);
    } else if (ok) {
      store_bf16x32(p, f, nv);
    }
  };
  float s_loss = 0.f, s_sq = 0.f, s_nnz = 0.f;
  const float rr = (e.r1_row && rowok) ? e.r1_row[row] : 0.f;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(trow + c * 32, r);
    tmem_ld_wait();
    const int col0 = nt * BN + c * 32;
    if (col0 >= N) continue;  // warp-uniform
    const int nv = min(32, N - col0);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if (e.r1_row) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nv) v[j] -= rr * __ldg(e.r1_col + col0 + j);
    }
    if (e.gate_bias) {
      float gate[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const bool ok = j < nv;
        const float pg = v[j] + (ok ? __ldg(e.gate_bias + col0 + j) : 0.f);
        const float pm = v[j] * (ok ? __ldg(e.mag_scale + col0 + j) : 0.f) + (ok && e.bias ? __ldg(e.bias + col0 + j) : 0.f);
        gate[j] = (rowok && ok) ? __bfloat162float(__float2bfloat16_rn(fmaxf(pg, 0.f))) : 0.f;
        v[j] = pg > 0.f ? fmaxf(pm, 0.f) : 0.f;
      }
      if (e.out2) put(e.out2 + int64_t(row) * e.ldo2 + col0, gate, nv, rowok);
      if (e.colsum2) {
        const float cs = warp_colsum32(gate, lane);
        if (lane < nv && cs != 0.f) atomicAdd(e.colsum2 + col0 + lane, cs);
      }
    } else if (e.bias) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nv) v[j] += __ldg(e.bias + col0 + j);
    }
    if (e.target) {
      float t[32];
      if (rowok && nv == 32) {
        load_bf16x32(e.target + int64_t(row) * e.ldtg + col0, t);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          t[j] = (rowok && j < nv) ? __bfloat162float(e.target[int64_t(row) * e.ldtg + col0 + j]) : 0.f;
      }
      if (e.out2) put(e.out2 + int64_t(row) * e.ldo2 + col0, v, nv, rowok);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        // the loss uses the bf16-rounded reconstruction the model outputs
        const float xh = __bfloat162float(__float2bfloat16_rn(v[j]));
        const float d = xh - t[j];
        if (rowok && j < nv) s_loss += d * d;
        v[j] = e.res_coef * d;
      }
    }
    float h[32];
    if (e.hin) {
      float g[32];
      if (rowok && nv == 32) {
        load_bf16x32(e.hin + int64_t(row) * e.ldh + col0, h);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          h[j] = (rowok && j < nv) ? __bfloat162float(e.hin[int64_t(row) * e.ldh + col0 + j]) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const bool ok = rowok && j < nv;
        const float th = j < nv ? __ldg(e.thr + col0 + j) : 0.f;
        const float x = (h[j] - th) * e.inv_bw;
        const bool inwin = ok && x > -0.5f && x < 0.5f;
        g[j] = inwin ? (-(th * e.inv_bw) * v[j] - e.l0c) : 0.f;
        v[j] = (ok && h[j] > th) ? v[j] : 0.f;
      }
      if (e.gthr) {
        const float gs = warp_colsum32(g, lane);
        if (lane < nv && gs != 0.f) atomicAdd(e.gthr + col0 + lane, gs);
      }
    } else if (e.thr) {
      // the gate compares the stored (bf16) pre-activation, as the backward does
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
      if (e.out2) put(e.out2 + int64_t(row) * e.ldo2 + col0, v, nv, rowok);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float th = j < nv ? __ldg(e.thr + col0 + j) : 0.f;
        v[j] = v[j] > th ? v[j] : 0.f;
      }
    }
    if (e.relu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (rowok && j < nv) ? v[j] : 0.f;
    if (e.colsum) {
      float t[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = v[j];
      const float cs = warp_colsum32(t, lane);
      if (lane < nv && cs != 0.f) atomicAdd(e.colsum + col0 + lane, cs);
    }
    if (e.hsum && e.hin) {
      float t[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = v[j] * (h[j] - (j < nv ? __ldg(e.hoff + col0 + j) : 0.f));
      const float cs = warp_colsum32(t, lane);
      if (lane < nv && cs != 0.f) atomicAdd(e.hsum + col0 + lane, cs);
    }
    if (e.addend) {
      float ad[32];
      if (rowok && nv == 32) {
        load_bf16x32(e.addend + int64_t(row) * e.ldad + col0, ad);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          ad[j] = (rowok && j < nv) ? __bfloat162float(e.addend[int64_t(row) * e.ldad + col0 + j]) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        v[j] = (rowok && j < nv) ? v[j] * (e.oscale ? __ldg(e.oscale + col0 + j) : 1.f) + ad[j] : 0.f;
    }
    // round to what is stored; the remaining statistics are taken over the stored values
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (rowok && j < nv) ? __bfloat162float(__float2bfloat16_rn(v[j])) : 0.f;
    if (e.rs_n > 0) {
      const int o = rowok ? row / e.rs_n : 0;  // rows past M name no owner (and store nothing)
      __nv_bfloat16* orow = p2p::at<__nv_bfloat16>(e.P, o, e.rs_off) +
                            (int64_t(e.P.rank) * e.rs_n + (rowok ? row - o * e.rs_n : 0)) * e.ldo;
      put(orow + col0, v, nv, rowok);
    } else if (e.out) {
      put(e.out + int64_t(row) * e.ldo + col0, v, nv, rowok);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      s_sq += v[j] * v[j];
      s_nnz += v[j] != 0.f ? 1.f : 0.f;
    }
    if (e.colcnt) {
      float cnt[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) cnt[j] = v[j] != 0.f ? 1.f : 0.f;
      const float cs = warp_colsum32(cnt, lane);
      if (lane < nv && cs != 0.f) atomicAdd(e.colcnt + col0 + lane, cs);
    }
  }
  if (e.rs_n > 0) __threadfence_system();  // peer rows visible before a later launch's release flag
  if (e.loss) {
    const float t = warp_sum(s_loss);
    if (lane == 0 && t != 0.f) atomicAdd(e.loss, t);
  }
  if (e.sumsq) {
    const float t = warp_sum(s_sq);
    if (lane == 0 && t != 0.f) atomicAdd(e.sumsq, t);
  }
  if (e.nnz) {
    const float t = warp_sum(s_nnz);
    if (lane == 0 && t != 0.f) atomicAdd(e.nnz, (unsigned long long)(t + 0.5f));
  }
}

// All-gather fusion parameters (byte offsets inside the symmetric slabs).
struct Ag {
  p2p::Peers P;
  const __nv_bfloat16* src;  // this rank's rows [rows_per_rank, K] (any device memory)
  int64_t x_off;             // offset of the full operand [S * rows_per_rank, K] bf16 in every slab
  int64_t flag_off;          // offset of the per-unit epoch flags u32 (unit = BM rows for A, BN for B)
  int rows_per_rank;         // multiple of the unit
  int m_base;                // first global row of this launch's A (multiple of BM; operand A)
  int rot;                   // tile rotation so that the tile walk starts at the own rows
  int push;                  // 1: this launch pushes the own rows (first launch of a step)
  uint32_t epoch;
  int* ticket;               // push-item counter, zero at launch: items go to whichever CTAs run
  int operand;               // 0: gather A rows (m-tiles); 1: gather B rows (n-tiles)
  const __nv_bfloat16* src2;  // optional second operand pushed along (same row split), or nullptr
  int64_t x2_off, flag2_off;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mt, int& nt, int rot = 0,
                                            int rot_n = 0) {
  const int group = t / (num_m * GROUP_N);
  const int first_n = group * GROUP_N;
  const int gsize = min(GROUP_N, num_n - first_n);
  const int r = t - group * num_m * GROUP_N;
  mt = r / gsize;
  if (rot) mt = (mt + rot) % num_m;
  nt = first_n + r % gsize;
  if (rot_n) nt = (nt + rot_n) % num_n;
}

// Epilogue of one accumulator tile: this thread's TMEM lane `trow` holds output row `row`
// (columns nt*BN .. nt*BN+255): bias, per-column scale, ReLU, bf16 store, 32-column maxima.
// Columns >= N (a partial last tile) are neither read from bias/scale nor stored.
//
// With `tmO` (CTA-pair kernel, ep.tma_out) the bf16 row chunk is not stored by the thread: the warp
// writes its 32 rows x 64 columns into `stage` (4 KB, 1024-aligned, 128-byte swizzle: 16-byte
// granule g of row r at granule g ^ (r % 8)) and one lane issues a TMA store of that box at
// (column nt*BN + 64 g, row row0); the tensor map clips rows >= M and columns >= N (the host takes
// this path only when N % 8 == 0, so every row ends on a 16-byte granule).  The staging
// tile is reused once the previous box's shared-memory read has completed.
__device__ __forceinline__ void epilogue_tile(const Epi& ep, uint32_t trow, int row, int M, int N, int nt,
                                              const CUtensorMap* tmO = nullptr, uint8_t* stage = nullptr,
                                              int row0 = 0, int lane = 0) {
  float tile_max = -INFINITY;
  float best_v = -INFINITY;  // row argmax over this tile (ep.amax): first column of the largest value
  int best_c = -1;
  const bool tma = tmO != nullptr && ep.out != nullptr;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    if (tma && (c & 1) == 0) {
      if (lane == 0) bulk_wait_read_all();  // the staging tile is free again
      __syncwarp();
    }
    uint32_t r[32];
    tmem_ld_32x32b_x32(trow + c * 32, r);
    tmem_ld_wait();
    const int col0 = nt * BN + c * 32;
    if (col0 >= N) continue;  // after the (warp-collective) load
    const bool full = col0 + 32 <= N;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if (ep.bias) {
      if (full) {
        const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 b = __ldg(b4 + j);
          v[4 * j] += b.x;
          v[4 * j + 1] += b.y;
          v[4 * j + 2] += b.z;
          v[4 * j + 3] += b.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] += __ldg(ep.bias + col0 + j);
      }
    }
    if (ep.scale) {
      if (full) {
        const float4* s4 = reinterpret_cast<const float4*>(ep.scale + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 s = __ldg(s4 + j);
          v[4 * j] *= s.x;
          v[4 * j + 1] *= s.y;
          v[4 * j + 2] *= s.z;
          v[4 * j + 3] *= s.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] *= __ldg(ep.scale + col0 + j);
      }
    }
    if (ep.relu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
    }
    if (ep.amax) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if ((full || col0 + j < N) && v[j] > best_v) {
          best_v = v[j];
          best_c = col0 + j;
        }
    }
    uint32_t packed[16];
    float cm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      packed[j] = *reinterpret_cast<uint32_t*>(&h2);
      if (full || col0 + 2 * j < N) cm = fmaxf(cm, __low2float(h2));
      if (full || col0 + 2 * j + 1 < N) cm = fmaxf(cm, __high2float(h2));
    }
    if (tma) {
      uint8_t* srow = stage + lane * 128;
      const int g0 = (c & 1) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(srow + (((g0 + j) ^ (lane & 7)) << 4)) =
            make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
      if ((c & 1) == 1 || col0 + 32 >= N) {  // the 64-column box is complete (or ends at N)
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmO, stage, nt * BN + (c & ~1) * 32, row0);
          bulk_commit_group();
        }
      }
    }
    if (row < M) {
      if (ep.out && !tma) {
        if (full) {
          uint4* dst = reinterpret_cast<uint4*>(ep.out + int64_t(row) * ep.ldo + col0);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        } else {
          __nv_bfloat16* dst = ep.out + int64_t(row) * ep.ldo + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < N) dst[j] = __float2bfloat16_rn(v[j]);
        }
      }
      if (ep.cmax) ep.cmax[int64_t(row) * ep.ldc + (col0 >> 5)] = __float2bfloat16_rn(cm);
    }
    tile_max = fmaxf(tile_max, cm);
  }
  if (ep.tmax && row < M) ep.tmax[int64_t(row) * ep.ldt + nt] = __float2bfloat16_rn(tile_max);
  if (ep.amax && row < M && best_c >= 0) atomicMax(ep.amax + row, argmax_key(best_v, best_c));
}

// All-gather pushers (two warps, ct = 0..63): claim (operand, distance d, own unit j) items from
// the launch's ticket counter, copy own rows [j*U, (j+1)*U) (U = BM for A, BN for B) into the
// slab of rank (r - d) mod S, which consumes them d-th in its rotated tile walk, and publish the
// unit's epoch flag there.  A copy whose source already is the destination (the own shard kept
// in place in the slab) only publishes.  Second-operand items come after all first-operand ones.
__device__ __forceinline__ void ag_push(const Ag& ag, int K, int ct) {
  if (!ag.push) return;
  __shared__ int s_item;
  const int S = ag.P.world, r = ag.P.rank;
  const int U = ag.operand ? BN : BM;
  const int upr = ag.rows_per_rank / U;
  const int64_t vec_per_unit = int64_t(U) * K / 8;
  const int per_op = S * upr;
  const int n_items = ag.src2 ? 2 * per_op : per_op;
  while (true) {
    if (ct == 0) s_item = atomicAdd(ag.ticket, 1);
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NUM_COPY_WARPS) : "memory");
    int item = s_item;
    if (item >= n_items) break;
    const bool second = item >= per_op;
    if (second) item -= per_op;
    const int d = item / upr, j = item - d * upr;
    const int dst = (r - d + S) % S;
    const __nv_bfloat16* base = second ? ag.src2 : ag.src;
    const uint4* src = reinterpret_cast<const uint4*>(base + int64_t(j) * U * K);
    uint4* out = reinterpret_cast<uint4*>(p2p::at<__nv_bfloat16>(ag.P, dst, second ? ag.x2_off : ag.x_off) +
                                          (int64_t(r) * ag.rows_per_rank + int64_t(j) * U) * K);
    if (reinterpret_cast<const void*>(out) != reinterpret_cast<const void*>(src)) {
      int64_t v = ct;
      for (; v + 3 * 64 < vec_per_unit; v += 4 * 64) {
        const uint4 a0 = __ldg(src + v), a1 = __ldg(src + v + 64), a2 = __ldg(src + v + 128),
                    a3 = __ldg(src + v + 192);
        out[v] = a0;
        out[v + 64] = a1;
        out[v + 128] = a2;
        out[v + 192] = a3;
      }
      for (; v < vec_per_unit; v += 64) out[v] = __ldg(src + v);
    }
    __threadfence_system();
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NUM_COPY_WARPS) : "memory");
    if (ct == 0)
      st_release_sys_u32(p2p::at<uint32_t>(ag.P, dst, second ? ag.flag2_off : ag.flag_off) + (r * upr + j),
                         ag.epoch);
  }
}

// A_MN / B_MN: the operand is stored MN-major ([K, M] / [K, N], M / N contiguous) and is loaded as
// 64 x 64 TMA boxes (64 MN elements by 64 k-rows, 8 KB each, LBO = 8 KB between MN chunks).
// DENSE: the epilogue is `epilogue_tile_dense` (EpiD) instead of the encoder epilogue (Epi).
template <bool AG, bool A_MN = false, bool B_MN = false, bool DENSE = false>
__global__ void __launch_bounds__(AG ? NUM_THREADS_AG : NUM_THREADS, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   int M, int N, int K, Epi ep, int* status, const __grid_constant__ Ag ag,
                   const __grid_constant__ EpiD ed) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_TILE_BYTES;
  uint8_t* sStage = sB + STAGES * B_TILE_BYTES;  // dense epilogue staging tiles, one per epilogue warp
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sStage + NUM_EPI_WARPS * STAGE_OUT_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ uint32_t ready_bits[AG ? MAX_MTILES / 32 : 1];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;  // a ragged last k-block reads zeros past K

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
  if (AG)
    for (int i = threadIdx.x; i < MAX_MTILES / 32; i += blockDim.x) ready_bits[i] = 0;
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
        tile_coords(t, num_m, num_n, mt, nt, AG && !ag.operand ? ag.rot : 0, AG && ag.operand ? ag.rot : 0);
        if (AG) {
          const int gm = ag.operand ? nt : ag.m_base / BM + mt;
          if (!(ready_bits[gm >> 5] & (1u << (gm & 31)))) {
            const uint32_t* f = p2p::at<uint32_t>(ag.P, ag.P.rank, ag.flag_off) + gm;
            if (!wait_geq_sys(f, ag.epoch, status, kTimeoutPeerFlag)) {
              *abort_flag = 1;
              ok = false;
              break;
            }
            fence_proxy_async_global();
            ready_bits[gm >> 5] |= 1u << (gm & 31);
          }
        }
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1, abort_flag, status, kTimeoutTmaProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_2d(sA + s * A_TILE_BYTES + c * 8192, &tmA, &full_bar[s], mt * BM + c * 64, kb * BK);
          } else {
            tma_load_2d(sA + s * A_TILE_BYTES, &tmA, &full_bar[s], kb * BK, mt * BM);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(sB + s * B_TILE_BYTES + c * 8192, &tmB, &full_bar[s], nt * BN + c * 64, kb * BK);
          } else {
            tma_load_2d(sB + s * B_TILE_BYTES, &tmB, &full_bar[s], kb * BK, nt * BN);
          }
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
      const uint32_t idesc = make_idesc_bf16_f32(BM, BN) | (A_MN ? (1u << 15) : 0u) | (B_MN ? (1u << 16) : 0u);
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
            const uint64_t ad = A_MN ? make_sdesc_sw128_mnmajor(a_addr + k * 2048, 8192)
                                     : make_sdesc_sw128_kmajor(a_addr + k * 32);
            const uint64_t bd = B_MN ? make_sdesc_sw128_mnmajor(b_addr + k * 2048, 8192)
                                     : make_sdesc_sw128_kmajor(b_addr + k * 32);
            umma_bf16_ss(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
    }
  } else if (AG && warp >= 2 + NUM_EPI_WARPS) {
    // ------------------------------ all-gather pushers ------------------------
    // Item i = (distance d, own m-tile j): copy own rows [j*BM, (j+1)*BM) into the slab of
    // rank (r - d) mod S, which consumes them d-th in its rotated tile walk; then publish.
    ag_push(ag, K, threadIdx.x - 32 * (2 + NUM_EPI_WARPS));
  } else {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tc) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt, AG && !ag.operand ? ag.rot : 0, AG && ag.operand ? ag.rot : 0);
      const int acc = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], aph, abort_flag, status, kTimeoutEpilogue)) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
      if (DENSE)
        epilogue_tile_dense(ed, trow, row, M, N, nt, lane, ed.staged ? sStage + (warp - 2) * STAGE_OUT_BYTES : nullptr);
      else
        epilogue_tile(ep, trow, row, M, N, nt);
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

// ------------------------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): a pair computes a 256 x 256 tile.
// CTA r of the pair stages rows [r*128, r*128+128) of the A tile and rows [r*128, r*128+128) of
// the B tile (i.e. output columns) per k-block, so each SM streams half as much B as the
// single-CTA kernel for the same tensor work; 6 stages of 32 KB.  The leader CTA (rank 0) issues
// the M=256 MMAs over both CTAs' shared memory; each CTA's TMEM holds its 128 output rows x 256
// columns.  Barriers: "stage full" lives in the leader (both CTAs' loads count on it), "stage
// empty" and "accumulator full" in both CTAs (the leader's commits arrive on both), "accumulator
// empty" in the leader (all 8 epilogue warps of the pair arrive on it).
// ------------------------------------------------------------------------------------------
constexpr int PSTAGES = 6;
constexpr int PA_BYTES = 128 * BK * 2;
constexpr int PB_BYTES = 128 * BK * 2;
constexpr int PSTAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int POUT_BYTES = 32 * 128;  // one epilogue warp's staging tile (32 rows x 64 bf16)
constexpr int PSMEM_BYTES = PSTAGES * PSTAGE_BYTES + NUM_EPI_WARPS * POUT_BYTES + 1024 + 256;

template <bool AG>
__global__ void __launch_bounds__(AG ? NUM_THREADS_AG : NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                     int N, int K, Epi ep, int* status, const __grid_constant__ Ag ag,
                     const __grid_constant__ CUtensorMap tmO) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + PSTAGES * PA_BYTES;
  uint8_t* sOut = sB + PSTAGES * PB_BYTES;  // NUM_EPI_WARPS staging tiles of 32 rows x 128 B (TMA stores)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sOut + NUM_EPI_WARPS * POUT_BYTES);
  uint64_t* empty_bar = full_bar + PSTAGES;
  uint64_t* tfull_bar = empty_bar + PSTAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ uint32_t ready_bits[AG ? MAX_MTILES / 32 : 1];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const bool leader = cta == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (M + 2 * BM - 1) / (2 * BM);
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * NUM_EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (AG)
    for (int i = threadIdx.x; i < MAX_MTILES / 32; i += blockDim.x) ready_bits[i] = 0;
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) ------------------
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        int mt, nt;
        tile_coords(t, num_m, num_n, mt, nt, AG && !ag.operand ? ag.rot : 0, AG && ag.operand ? ag.rot : 0);
        if (AG) {
          const int gm = ag.operand ? nt : ag.m_base / BM + 2 * mt + int(cta);
          if (!(ready_bits[gm >> 5] & (1u << (gm & 31)))) {
            const uint32_t* f = p2p::at<uint32_t>(ag.P, ag.P.rank, ag.flag_off) + gm;
            if (!wait_geq_sys(f, ag.epoch, status, kTimeoutPeerFlag)) {
              *abort_flag = 1;
              ok = false;
              break;
            }
            fence_proxy_async_global();
            ready_bits[gm >> 5] |= 1u << (gm & 31);
          }
        }
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % PSTAGES;
          const uint32_t ph = (it / PSTAGES) & 1;
          if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1, abort_flag, status, kTimeoutTmaProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * PSTAGE_BYTES);
          tma_load_2d_pair(sA + s * PA_BYTES, &tmA, fb, kb * BK, mt * 2 * BM + int(cta) * BM);
          tma_load_2d_pair(sB + s * PB_BYTES, &tmB, fb, kb * BK, nt * BN + int(cta) * 128);
        }
      }
      if (!ok && leader) {
        const uint32_t first = it > PSTAGES ? it - PSTAGES : 0;
        for (uint32_t j = first; j < it; ++j) {
          volatile int dummy = 0;
          mbar_wait_bounded(&full_bar[j % PSTAGES], (j / PSTAGES) & 1, &dummy, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader CTA) -------------------
    if (leader && elect_one()) {
      const uint32_t idesc = make_idesc_bf16_f32(2 * BM, BN);
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs, ++tc) {
        const int acc = tc & 1;
        const uint32_t aph = (tc >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], aph ^ 1, abort_flag, status, kTimeoutMmaTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % PSTAGES;
          const uint32_t ph = (it / PSTAGES) & 1;
          if (!mbar_wait_bounded(&full_bar[s], ph, abort_flag, status, kTimeoutMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * PA_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * PB_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16_ss_pair(d_tmem, make_sdesc_sw128_kmajor(a_addr + k * 32),
                              make_sdesc_sw128_kmajor(b_addr + k * 32), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          const uint32_t eb = smem_u32(&empty_bar[s]);
          umma_commit_pair(eb);
          umma_commit_pair(mapa_shared(eb, 1));
        }
        if (ok) {
          const uint32_t fb = smem_u32(&tfull_bar[acc]);
          umma_commit_pair(fb);
          umma_commit_pair(mapa_shared(fb, 1));
        }
      }
    }
  } else if (AG && warp >= 2 + NUM_EPI_WARPS) {
    ag_push(ag, K, threadIdx.x - 32 * (2 + NUM_EPI_WARPS));
  } else if (warp >= 2) {
    // ------------------------------ epilogue (both CTAs) ----------------------
    const int q = warp & 3;
    uint32_t tc = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tc) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt, AG && !ag.operand ? ag.rot : 0, AG && ag.operand ? ag.rot : 0);
      const int acc = tc & 1;
      const uint32_t aph = (tc >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], aph, abort_flag, status, kTimeoutEpilogue)) break;
      tc_fence_after();
      const int row0 = mt * 2 * BM + int(cta) * BM + q * 32;
      const int row = row0 + lane;
      const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
      epilogue_tile(ep, trow, row, M, N, nt, ep.tma_out ? &tmO : nullptr, sOut + (warp - 2) * POUT_BYTES, row0,
                    lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
    }
    if (ep.tma_out && lane == 0) bulk_wait_all();  // the tile stores have landed before the CTA ends
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its pair may still touch its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
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

static gemm::Epi make_epi(int64_t M, int64_t N, const c10::optional<torch::Tensor>& bias,
                          const c10::optional<torch::Tensor>& scale, bool relu,
                          const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                          const c10::optional<torch::Tensor>& tmax = c10::nullopt,
                          const c10::optional<torch::Tensor>& amax = c10::nullopt) {
  gemm::Epi ep{};
  if (amax) {
    SB_CHECK(amax->scalar_type() == at::kLong && amax->numel() == M && amax->is_contiguous(),
             "gemm_tn_bf16: amax must be int64 [M] (row argmax keys)");
    ep.amax = reinterpret_cast<unsigned long long*>(amax->data_ptr());
  }
  if (out) {
    SB_CHECK(out->scalar_type() == at::kBFloat16 && out->size(0) == M && out->size(1) == N &&
                    out->stride(1) == 1 && out->stride(0) % 8 == 0,
                "gemm_tn_bf16: bad out");
    ep.out = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    ep.ldo = out->stride(0);
  }
  if (cmax) {
    SB_CHECK(cmax->scalar_type() == at::kBFloat16 && cmax->size(0) == M &&
                    cmax->size(1) == N / 32 && cmax->stride(1) == 1,
                "gemm_tn_bf16: bad cmax");
    ep.cmax = reinterpret_cast<__nv_bfloat16*>(cmax->data_ptr());
    ep.ldc = cmax->stride(0);
  }
  if (bias) {
    SB_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N && bias->is_contiguous(),
                "gemm_tn_bf16: bias must be fp32 [N]");
    ep.bias = bias->data_ptr<float>();
  }
  if (scale) {
    SB_CHECK(scale->scalar_type() == at::kFloat && scale->numel() == N && scale->is_contiguous(),
                "gemm_tn_bf16: scale must be fp32 [N]");
    ep.scale = scale->data_ptr<float>();
  }
  if (tmax) {
    SB_CHECK(tmax->scalar_type() == at::kBFloat16 && tmax->size(0) == M && tmax->size(1) == N / gemm::BN &&
                    tmax->stride(1) == 1,
                "gemm_tn_bf16: bad tmax (bf16 [M, N/256])");
    ep.tmax = reinterpret_cast<__nv_bfloat16*>(tmax->data_ptr());
    ep.ldt = tmax->stride(0);
  }
  ep.relu = relu ? 1 : 0;
  return ep;
}

// CTA-pair kernel unless disabled (SAELENS_B200_GEMM_PAIR=0, read at every call) or M is too small
// to fill pairs.
static bool use_pair(int64_t M) {
  const char* e = std::getenv("SAELENS_B200_GEMM_PAIR");
  const bool off = e && e[0] == '0' && e[1] == 0;
  return !off && M >= 2 * gemm::BM;
}

// The dense epilogue stores its full 32-column chunks through the warp's staging tile (8 rows x 64
// contiguous bytes per store instruction, also into a peer's landing slot in reduce-scatter mode);
// SAELENS_B200_GEMM_STAGED_STORE=0 selects per-thread row stores
static bool staged_stores_enabled() {
  const char* e = std::getenv("SAELENS_B200_GEMM_STAGED_STORE");
  return !(e && e[0] == '0' && e[1] == 0);
}

template <bool AG>
static void launch_gemm(const void* a_ptr, int64_t lda, int64_t M, const torch::Tensor& B, const gemm::Epi& ep,
                        const torch::Tensor& status, int64_t max_ctas, const gemm::Ag& ag, bool pair) {
  const int64_t K = B.size(1), N = B.size(0);
  const int box_rows = pair ? 128 : gemm::BN;
  CUtensorMap tA = make_tmap_2d(const_cast<void*>(a_ptr), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda * 2,
                                gemm::BM, gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tB = make_tmap_2d(B.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, B.stride(0) * 2,
                                box_rows, gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = AG ? gemm::NUM_THREADS_AG : gemm::NUM_THREADS;
  int* st = status.data_ptr<int>();
  const int iM = int(M), iN = int(N), iK = int(K);
  if (!pair) {
    static bool attr_set = false;
    if (!attr_set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(gemm::gemm_tn_kernel<AG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          gemm::SMEM_BYTES));
      attr_set = true;
    }
    const int64_t tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
    int64_t grid = std::min<int64_t>(tiles, num_sms_cached());
    if (max_ctas > 0) grid = std::min<int64_t>(grid, max_ctas);
    gemm::gemm_tn_kernel<AG><<<dim3(grid), dim3(threads), gemm::SMEM_BYTES, stream>>>(tA, tB, iM, iN, iK, ep, st,
                                                                                         ag, gemm::EpiD{});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  auto kern = gemm::gemm_pair_kernel<AG>;
  static int max_pairs = -1;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = gemm::PSMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_pairs < 0) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::PSMEM_BYTES));
    cfg.gridDim = dim3(2 * (num_sms_cached() / 2));
    int n = 0;
    C10_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_pairs = std::max(1, n);
  }
  const int64_t tiles = ((M + 2 * gemm::BM - 1) / (2 * gemm::BM)) * ((N + gemm::BN - 1) / gemm::BN);
  int64_t pairs = std::min<int64_t>(tiles, max_pairs);
  if (max_ctas > 0) pairs = std::max<int64_t>(1, std::min<int64_t>(pairs, max_ctas / 2));
  cfg.gridDim = dim3(unsigned(2 * pairs));
  // TMA tile stores of `out` (SAELENS_B200_GEMM_TMA_STORE=0 keeps the per-thread row stores)
  gemm::Epi epp = ep;
  CUtensorMap tO = tA;  // unused unless epp.tma_out
  const char* ts = std::getenv("SAELENS_B200_GEMM_TMA_STORE");
  // rows must end on a 16-byte boundary (N % 8 == 0): the store writes whole 16-byte granules, so a
  // ragged row end would also write the padding past N
  const bool tma_ok = !(ts && ts[0] == '0' && ts[1] == 0) && ep.out != nullptr && (ep.ldo * 2) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(ep.out) % 16 == 0 && N % 8 == 0;
  if (tma_ok) {
    tO = make_tmap_2d(ep.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, N, ep.ldo * 2, 32, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    epp.tma_out = 1;
  }
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tA, tB, iM, iN, iK, epp, st, ag, tO));
}

// out = epilogue(A @ B^T).  A: [M, K] bf16 (row stride lda), B: [N, K] bf16.  Optional
// bias/scale fp32 [N].  Returns nothing; writes `out` [M, N] bf16 and/or `cmax` [M, N/32] bf16,
// and with `amax` (int64 [M], zeroed by the caller) folds each row's argmax of the fp32 epilogue
// values into an order-preserving key by atomicMax (value in the high word, 0xFFFFFFFF - column in
// the low word).
void gemm_tn_bf16(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& bias,
                  const c10::optional<torch::Tensor>& scale, bool relu,
                  const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                  const torch::Tensor& status, int64_t max_ctas, const c10::optional<torch::Tensor>& tmax,
                  const c10::optional<torch::Tensor>& amax) {
  SB_CHECK(A.is_cuda() && B.is_cuda(), "gemm_tn_bf16: CUDA tensors required");
  SB_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16,
              "gemm_tn_bf16: bf16 operands required");
  SB_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_tn_bf16: shape");
  SB_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_tn_bf16: K must be contiguous");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  SB_CHECK(K % 8 == 0, "gemm_tn_bf16: K must be a multiple of 8 (16-byte rows), got ", K);
  SB_CHECK(N >= 1 && ((!cmax && !tmax) || N % gemm::BN == 0),
              "gemm_tn_bf16: chunk / tile maxima need N to be a multiple of 256, got ", N);
  SB_CHECK(M >= 1 && M < (1ll << 31) && N < (1ll << 31), "gemm_tn_bf16: size");
  const at::cuda::CUDAGuard guard(A.device());
  const gemm::Epi ep = make_epi(M, N, bias, scale, relu, out, cmax, tmax, amax);
  launch_gemm<false>(A.data_ptr(), A.stride(0), M, B, ep, status, max_ctas, gemm::Ag{}, use_pair(M));
}

// All-gather fused encoder GEMM over rows [m_base, m_base + M) of the full input that lives at
// byte offset `x_off` of every rank's symmetric slab (`peer_bases[r]` = rank r's slab address).
// `x_own` [Bo, K] is this rank's part; with `push` the kernel also distributes it to every rank.
// Waits (bounded) for the epoch flag of each m-tile at `flag_off` before reading it.
void gemm_ag_tn_bf16(const torch::Tensor& x_own, const std::vector<int64_t>& peer_bases, int64_t rank,
                     int64_t x_off, int64_t flag_off, int64_t total_rows, int64_t m_base, int64_t M,
                     bool push, int64_t epoch, const torch::Tensor& B, const c10::optional<torch::Tensor>& bias,
                     const c10::optional<torch::Tensor>& scale, bool relu, const c10::optional<torch::Tensor>& out,
                     const c10::optional<torch::Tensor>& cmax, const torch::Tensor& status,
                     const torch::Tensor& ticket, int64_t max_ctas, const c10::optional<torch::Tensor>& tmax) {
  const int64_t S = int64_t(peer_bases.size());
  SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "gemm_ag: bad group");
  SB_CHECK(x_own.is_cuda() && x_own.scalar_type() == at::kBFloat16 && x_own.is_contiguous(),
              "gemm_ag: x_own must be contiguous CUDA bf16");
  SB_CHECK(B.scalar_type() == at::kBFloat16 && B.stride(1) == 1 && B.size(1) == x_own.size(1),
              "gemm_ag: weight");
  const int64_t Bo = x_own.size(0), K = x_own.size(1), N = B.size(0);
  SB_CHECK(Bo * S == total_rows, "gemm_ag: total_rows must be world * own rows");
  SB_CHECK(Bo % gemm::BM == 0 && m_base % gemm::BM == 0 && M % gemm::BM == 0 && M >= gemm::BM &&
                  m_base + M <= total_rows,
              "gemm_ag: rows must be multiples of 128");
  SB_CHECK(total_rows / gemm::BM <= gemm::MAX_MTILES, "gemm_ag: too many rows");
  SB_CHECK(K % gemm::BK == 0 && N % gemm::BN == 0, "gemm_ag: K % 64 and N % 256");
  SB_CHECK(x_off % 16 == 0 && flag_off % 4 == 0, "gemm_ag: slab offsets must be aligned");
  const at::cuda::CUDAGuard guard(x_own.device());
  const gemm::Epi ep = make_epi(M, N, bias, scale, relu, out, cmax, tmax);
  gemm::Ag ag{};
  ag.P = p2p::make_peers(peer_bases, rank);
  ag.src = reinterpret_cast<const __nv_bfloat16*>(x_own.data_ptr());
  ag.x_off = x_off;
  ag.flag_off = flag_off;
  ag.rows_per_rank = int(Bo);
  ag.m_base = int(m_base);
  const int64_t own0 = rank * Bo;
  const bool pair = use_pair(M) && Bo % (2 * gemm::BM) == 0 && M % (2 * gemm::BM) == 0 &&
                    m_base % (2 * gemm::BM) == 0;
  const int64_t tile_rows = pair ? 2 * gemm::BM : gemm::BM;
  const int num_m = int(M / tile_rows);
  ag.rot = (own0 >= m_base && own0 < m_base + M) ? int((own0 - m_base) / tile_rows) % num_m : 0;
  ag.push = push ? 1 : 0;
  ag.epoch = uint32_t(epoch);
  SB_CHECK(ticket.is_cuda() && ticket.scalar_type() == at::kInt && ticket.numel() >= 1, "gemm_ag: ticket");
  ag.ticket = ticket.data_ptr<int>();
  if (push) C10_CUDA_CHECK(cudaMemsetAsync(ag.ticket, 0, sizeof(int), at::cuda::getCurrentCUDAStream()));
  const char* a_ptr = reinterpret_cast<const char*>(peer_bases[rank]) + x_off + m_base * K * 2;
  launch_gemm<true>(a_ptr, K, M, B, ep, status, max_ctas, ag, pair);
}

// Parameter all-gather fused encoder GEMM (sharded data parallel): out = epilogue(A @ W^T) where
// W [N, K] is the full encoder weight at byte offset w_off of every rank's slab and this rank
// owns rows [rank*n, (rank+1)*n) of it (`w_own`, usually that very slab region).  With `push`,
// the kernel distributes the own rows (and, if given, the rows of `w2_own` into the [N, K] area
// at w2_off with flags at flag2_off) to every rank; it waits (bounded) for the epoch flag of each
// 256-row n-tile at flag_off before reading it.  A: [M, K] local rows.
void gemm_fsdp_tn_bf16(const torch::Tensor& A, const torch::Tensor& w_own, const std::vector<int64_t>& peer_bases,
                       int64_t rank, int64_t w_off, int64_t flag_off, bool push, int64_t epoch,
                       const c10::optional<torch::Tensor>& w2_own, int64_t w2_off, int64_t flag2_off,
                       const c10::optional<torch::Tensor>& bias, const c10::optional<torch::Tensor>& scale, bool relu,
                       const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                       const torch::Tensor& status, const torch::Tensor& ticket, int64_t max_ctas,
                       const c10::optional<torch::Tensor>& tmax) {
  const int64_t S = int64_t(peer_bases.size());
  SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "gemm_fsdp: bad group");
  SB_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && A.dim() == 2 && A.stride(1) == 1,
              "gemm_fsdp: A must be CUDA bf16 with contiguous rows");
  SB_CHECK(w_own.is_cuda() && w_own.scalar_type() == at::kBFloat16 && w_own.is_contiguous() &&
                  w_own.size(1) == A.size(1),
              "gemm_fsdp: w_own must be contiguous bf16 [n, K]");
  const int64_t M = A.size(0), K = A.size(1), n = w_own.size(0), N = n * S;
  SB_CHECK(n % gemm::BN == 0 && K % gemm::BK == 0, "gemm_fsdp: shard rows % 256 and K % 64");
  SB_CHECK(N / gemm::BN <= gemm::MAX_MTILES && M >= 1 && M < (1ll << 31), "gemm_fsdp: size");
  SB_CHECK(w_off % 16 == 0 && flag_off % 4 == 0 && w2_off % 16 == 0 && flag2_off % 4 == 0,
              "gemm_fsdp: slab offsets must be aligned");
  if (w2_own) {
    SB_CHECK(w2_own->is_cuda() && w2_own->scalar_type() == at::kBFloat16 && w2_own->is_contiguous() &&
                    w2_own->sizes() == w_own.sizes(),
                "gemm_fsdp: w2_own must be contiguous bf16 like w_own");
  }
  const at::cuda::CUDAGuard guard(A.device());
  const gemm::Epi ep = make_epi(M, N, bias, scale, relu, out, cmax, tmax);
  gemm::Ag ag{};
  ag.P = p2p::make_peers(peer_bases, rank);
  ag.src = reinterpret_cast<const __nv_bfloat16*>(w_own.data_ptr());
  ag.x_off = w_off;
  ag.flag_off = flag_off;
  ag.rows_per_rank = int(n);
  ag.operand = 1;
  ag.rot = int((rank * n) / gemm::BN);
  ag.push = push ? 1 : 0;
  ag.epoch = uint32_t(epoch);
  ag.src2 = w2_own ? reinterpret_cast<const __nv_bfloat16*>(w2_own->data_ptr()) : nullptr;
  ag.x2_off = w2_off;
  ag.flag2_off = flag2_off;
  SB_CHECK(ticket.is_cuda() && ticket.scalar_type() == at::kInt && ticket.numel() >= 1, "gemm_fsdp: ticket");
  ag.ticket = ticket.data_ptr<int>();
  if (push) C10_CUDA_CHECK(cudaMemsetAsync(ag.ticket, 0, sizeof(int), at::cuda::getCurrentCUDAStream()));
  // the full weight as seen in this rank's slab
  auto W = torch::from_blob(reinterpret_cast<char*>(peer_bases[rank]) + w_off, {N, K},
                            A.options().dtype(at::kBFloat16));
  launch_gemm<true>(A.data_ptr(), A.stride(0), M, W, ep, status, max_ctas, ag, use_pair(M));
}

}  // namespace sb

namespace sb {

template <bool A_MN, bool B_MN>
static void launch_dense(const CUtensorMap& tA, const CUtensorMap& tB, int M, int N, int K, const gemm::EpiD& ed,
                         int* st, int64_t max_ctas) {
  auto kern = gemm::gemm_tn_kernel<false, A_MN, B_MN, true>;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::SMEM_BYTES));
    attr_set = true;
  }
  const int64_t tiles = int64_t((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  int64_t grid = std::min<int64_t>(tiles, num_sms_cached());
  if (max_ctas > 0) grid = std::min<int64_t>(grid, max_ctas);
  kern<<<dim3(unsigned(grid)), dim3(gemm::NUM_THREADS), gemm::SMEM_BYTES, at::cuda::getCurrentCUDAStream()>>>(
      tA, tB, M, N, K, gemm::Epi{}, st, gemm::Ag{}, ed);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static const float* opt_f32(const c10::optional<torch::Tensor>& t, int64_t n, const char* what) {
  if (!t) return nullptr;
  SB_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n,
              "gemm_dense_bf16: ", what, " must be a contiguous CUDA fp32 tensor of ", n, " elements");
  return t->data_ptr<float>();
}

static __nv_bfloat16* opt_bf16_mat(const c10::optional<torch::Tensor>& t, int64_t M, int64_t N, int64_t* ld,
                                   const char* what) {
  if (!t) return nullptr;
  SB_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->size(0) == M &&
                  t->size(1) == N && t->stride(1) == 1 && t->stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
              "gemm_dense_bf16: ", what, " must be bf16 [M, N] with 16-byte aligned rows");
  *ld = t->stride(0);
  return reinterpret_cast<__nv_bfloat16*>(t->data_ptr());
}

// Dense GEMM of the dense SAE steps: C[M, N] = epilogue(sum_k A[m, k] B[n, k]) on tcgen05, with each
// operand either K-major (A [M, K], B [N, K]) or MN-major (A [K, M], B [K, N]; `a_mn` / `b_mn`),
// bf16 with contiguous inner dimension and 16-byte row strides.  The epilogue (EpiD) is assembled
// from the optional tensors; `nnz` is an int64 scalar, the other accumulators fp32.
void gemm_dense_bf16(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn,
                     const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& out2,
                     const c10::optional<torch::Tensor>& bias, const c10::optional<torch::Tensor>& r1_row,
                     const c10::optional<torch::Tensor>& r1_col, const c10::optional<torch::Tensor>& thr, bool relu,
                     const c10::optional<torch::Tensor>& hin, double bandwidth, double l0c,
                     const c10::optional<torch::Tensor>& gthr, const c10::optional<torch::Tensor>& target,
                     double res_coef, const c10::optional<torch::Tensor>& loss,
                     const c10::optional<torch::Tensor>& colsum, const c10::optional<torch::Tensor>& colcnt,
                     const c10::optional<torch::Tensor>& nnz, const c10::optional<torch::Tensor>& sumsq,
                     const c10::optional<torch::Tensor>& gate_bias, const c10::optional<torch::Tensor>& mag_scale,
                     const torch::Tensor& status, int64_t max_ctas, const std::vector<int64_t>& rs_bases,
                     int64_t rs_rank, int64_t rs_off, int64_t rs_n, const c10::optional<torch::Tensor>& hsum,
                     const c10::optional<torch::Tensor>& hoff, const c10::optional<torch::Tensor>& colsum2,
                     const c10::optional<torch::Tensor>& addend, const c10::optional<torch::Tensor>& oscale) {
  SB_CHECK(A.is_cuda() && B.is_cuda() && A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 &&
                  A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1,
              "gemm_dense_bf16: A and B must be 2-D CUDA bf16 with a contiguous inner dimension");
  const int64_t M = a_mn ? A.size(1) : A.size(0), K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0), Kb = b_mn ? B.size(0) : B.size(1);
  SB_CHECK(K == Kb && K >= 1 && M >= 1 && N >= 1, "gemm_dense_bf16: inner dimensions differ (", K, " vs ", Kb, ")");
  SB_CHECK(A.stride(0) % 8 == 0 && B.stride(0) % 8 == 0, "gemm_dense_bf16: row strides must be multiples of 8");
  SB_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_dense_bf16: size");
  gemm::EpiD ed{};
  ed.staged = staged_stores_enabled() ? 1 : 0;
  if (rs_n > 0) {
    const int64_t S = int64_t(rs_bases.size());
    SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rs_rank >= 0 && rs_rank < S && rs_n % gemm::BM == 0 &&
                    S * rs_n == M && rs_off % 16 == 0 && N % 8 == 0 && !out,
                "gemm_dense_bf16: reduce-scatter mode needs M = world * rs_n, rs_n % 128 == 0, N % 8 == 0, an "
                "aligned landing offset and no local out");
    ed.P = p2p::make_peers(rs_bases, rs_rank);
    ed.rs_off = rs_off;
    ed.rs_n = int(rs_n);
    ed.ldo = N;
  }
  ed.out = opt_bf16_mat(out, M, N, &ed.ldo, "out");
  ed.out2 = opt_bf16_mat(out2, M, N, &ed.ldo2, "out2");
  ed.bias = opt_f32(bias, N, "bias");
  ed.r1_row = opt_f32(r1_row, M, "r1_row");
  ed.r1_col = opt_f32(r1_col, N, "r1_col");
  SB_CHECK(!ed.r1_row == !ed.r1_col, "gemm_dense_bf16: r1_row and r1_col go together");
  ed.thr = opt_f32(thr, N, "thr");
  ed.relu = relu ? 1 : 0;
  ed.hin = opt_bf16_mat(hin, M, N, &ed.ldh, "hin");
  SB_CHECK(!ed.hin || (ed.thr && bandwidth > 0), "gemm_dense_bf16: hin needs thr and a positive bandwidth");
  ed.inv_bw = bandwidth > 0 ? float(1.0 / bandwidth) : 0.f;
  ed.l0c = float(l0c);
  ed.gthr = const_cast<float*>(opt_f32(gthr, N, "gthr"));
  ed.target = opt_bf16_mat(target, M, N, &ed.ldtg, "target");
  ed.res_coef = float(res_coef);
  ed.loss = const_cast<float*>(opt_f32(loss, 1, "loss"));
  ed.colsum = const_cast<float*>(opt_f32(colsum, N, "colsum"));
  ed.colcnt = const_cast<float*>(opt_f32(colcnt, N, "colcnt"));
  if (nnz) {
    SB_CHECK(nnz->is_cuda() && nnz->scalar_type() == at::kLong && nnz->numel() == 1, "gemm_dense_bf16: nnz int64[1]");
    ed.nnz = reinterpret_cast<unsigned long long*>(nnz->data_ptr<int64_t>());
  }
  ed.sumsq = const_cast<float*>(opt_f32(sumsq, 1, "sumsq"));
  ed.gate_bias = opt_f32(gate_bias, N, "gate_bias");
  ed.mag_scale = opt_f32(mag_scale, N, "mag_scale");
  SB_CHECK(!ed.gate_bias == !ed.mag_scale, "gemm_dense_bf16: gate_bias and mag_scale go together");
  ed.hsum = const_cast<float*>(opt_f32(hsum, N, "hsum"));
  ed.hoff = opt_f32(hoff, N, "hoff");
  SB_CHECK(!ed.hsum || (ed.hoff && ed.hin), "gemm_dense_bf16: hsum needs hoff and hin");
  ed.colsum2 = const_cast<float*>(opt_f32(colsum2, N, "colsum2"));
  SB_CHECK(!ed.colsum2 || ed.gate_bias, "gemm_dense_bf16: colsum2 is the gated epilogue's gate sum");
  int64_t ldad = 0;
  ed.addend = opt_bf16_mat(addend, M, N, &ldad, "addend");
  ed.ldad = ldad;
  ed.oscale = opt_f32(oscale, N, "oscale");
  SB_CHECK(!ed.oscale || ed.addend, "gemm_dense_bf16: oscale is applied with an addend");
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap tA = a_mn ? make_tmap_2d(A.data_ptr(), bf, 2, K, M, A.stride(0) * 2, 64, 64, sw)
                        : make_tmap_2d(A.data_ptr(), bf, 2, M, K, A.stride(0) * 2, gemm::BM, gemm::BK, sw);
  CUtensorMap tB = b_mn ? make_tmap_2d(B.data_ptr(), bf, 2, K, N, B.stride(0) * 2, 64, 64, sw)
                        : make_tmap_2d(B.data_ptr(), bf, 2, N, K, B.stride(0) * 2, gemm::BN, gemm::BK, sw);
  SB_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "gemm_dense_bf16: status");
  const at::cuda::CUDAGuard guard(A.device());
  int* st = status.data_ptr<int>();
  const int iM = int(M), iN = int(N), iK = int(K);
  if (a_mn && b_mn)
    launch_dense<true, true>(tA, tB, iM, iN, iK, ed, st, max_ctas);
  else if (a_mn)
    launch_dense<true, false>(tA, tB, iM, iN, iK, ed, st, max_ctas);
  else if (b_mn)
    launch_dense<false, true>(tA, tB, iM, iN, iK, ed, st, max_ctas);
  else
    launch_dense<false, false>(tA, tB, iM, iN, iK, ed, st, max_ctas);
}

// Sharded data-parallel encoder GEMM with the dense (JumpReLU / gated) epilogue: the parameter
// all-gather of `gemm_fsdp_tn_bf16` (own W_enc / W_dec latent tiles pushed to every rank, the
// TMA producer waiting per 256-latent tile) with the EpiD epilogue of the dense steps.
void gemm_fsdp_dense_bf16(const torch::Tensor& A, const torch::Tensor& w_own, const std::vector<int64_t>& peer_bases,
                          int64_t rank, int64_t w_off, int64_t flag_off, bool push, int64_t epoch,
                          const c10::optional<torch::Tensor>& w2_own, int64_t w2_off, int64_t flag2_off,
                          const torch::Tensor& out, const c10::optional<torch::Tensor>& out2,
                          const c10::optional<torch::Tensor>& bias, const c10::optional<torch::Tensor>& thr,
                          const c10::optional<torch::Tensor>& colcnt, const c10::optional<torch::Tensor>& nnz,
                          const torch::Tensor& status, const torch::Tensor& ticket) {
  const int64_t S = int64_t(peer_bases.size());
  SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "gemm_fsdp_dense: bad group");
  SB_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && A.dim() == 2 && A.stride(1) == 1 &&
                  A.stride(0) % 8 == 0,
              "gemm_fsdp_dense: A must be CUDA bf16 [M, K] with 16-byte rows");
  SB_CHECK(w_own.is_cuda() && w_own.scalar_type() == at::kBFloat16 && w_own.is_contiguous() &&
                  w_own.size(1) == A.size(1),
              "gemm_fsdp_dense: w_own must be contiguous bf16 [n, K]");
  const int64_t M = A.size(0), K = A.size(1), n = w_own.size(0), N = n * S;
  SB_CHECK(n % gemm::BN == 0 && K % gemm::BK == 0, "gemm_fsdp_dense: shard rows % 256 and K % 64");
  SB_CHECK(N / gemm::BN <= gemm::MAX_MTILES && M >= 1 && M < (1ll << 31), "gemm_fsdp_dense: size");
  SB_CHECK(w_off % 16 == 0 && flag_off % 4 == 0 && w2_off % 16 == 0 && flag2_off % 4 == 0,
              "gemm_fsdp_dense: slab offsets must be aligned");
  if (w2_own)
    SB_CHECK(w2_own->is_cuda() && w2_own->scalar_type() == at::kBFloat16 && w2_own->is_contiguous() &&
                    w2_own->sizes() == w_own.sizes(),
                "gemm_fsdp_dense: w2_own must be contiguous bf16 like w_own");
  gemm::EpiD ed{};
  ed.staged = staged_stores_enabled() ? 1 : 0;
  ed.out = opt_bf16_mat(out, M, N, &ed.ldo, "out");
  ed.out2 = opt_bf16_mat(out2, M, N, &ed.ldo2, "out2");
  ed.bias = opt_f32(bias, N, "bias");
  ed.thr = opt_f32(thr, N, "thr");
  ed.colcnt = const_cast<float*>(opt_f32(colcnt, N, "colcnt"));
  if (nnz) {
    SB_CHECK(nnz->is_cuda() && nnz->scalar_type() == at::kLong && nnz->numel() == 1, "gemm_fsdp_dense: nnz");
    ed.nnz = reinterpret_cast<unsigned long long*>(nnz->data_ptr<int64_t>());
  }
  SB_CHECK(ticket.is_cuda() && ticket.scalar_type() == at::kInt && ticket.numel() >= 1, "gemm_fsdp_dense: ticket");
  SB_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "gemm_fsdp_dense: status");
  const at::cuda::CUDAGuard guard(A.device());
  gemm::Ag ag{};
  ag.P = p2p::make_peers(peer_bases, rank);
  ag.src = reinterpret_cast<const __nv_bfloat16*>(w_own.data_ptr());
  ag.x_off = w_off;
  ag.flag_off = flag_off;
  ag.rows_per_rank = int(n);
  ag.operand = 1;
  ag.rot = int((rank * n) / gemm::BN);
  ag.push = push ? 1 : 0;
  ag.epoch = uint32_t(epoch);
  ag.src2 = w2_own ? reinterpret_cast<const __nv_bfloat16*>(w2_own->data_ptr()) : nullptr;
  ag.x2_off = w2_off;
  ag.flag2_off = flag2_off;
  ag.ticket = ticket.data_ptr<int>();
  auto stream = at::cuda::getCurrentCUDAStream();
  if (push) C10_CUDA_CHECK(cudaMemsetAsync(ag.ticket, 0, sizeof(int), stream));
  const char* wbase = reinterpret_cast<const char*>(peer_bases[rank]) + w_off;
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap tA = make_tmap_2d(A.data_ptr(), bf, 2, M, K, A.stride(0) * 2, gemm::BM, gemm::BK, sw);
  CUtensorMap tB = make_tmap_2d(wbase, bf, 2, N, K, K * 2, gemm::BN, gemm::BK, sw);
  auto kern = gemm::gemm_tn_kernel<true, false, false, true>;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::SMEM_BYTES));
    attr_set = true;
  }
  const int64_t tiles = ((M + gemm::BM - 1) / gemm::BM) * (N / gemm::BN);
  const int64_t grid = std::min<int64_t>(tiles, num_sms_cached());
  kern<<<dim3(unsigned(grid)), dim3(gemm::NUM_THREADS_AG), gemm::SMEM_BYTES, stream>>>(
      tA, tB, int(M), int(N), int(K), gemm::Epi{}, status.data_ptr<int>(), ag, ed);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

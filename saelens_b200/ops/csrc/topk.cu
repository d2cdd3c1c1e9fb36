// Row-wise exact top-k over bf16 pre-activations, pruned by per-chunk maxima.
//
// Replaces `torch.topk(hidden_pre, k, dim=-1, sorted=False)` + ReLU + scatter
// (sae_lens/saes/topk_sae.py:99-145) and the dead-latent top-k of the aux loss
// (sae_lens/saes/topk_sae.py:787-813).  No dense [B, d_sae] activation tensor is produced: the
// output is k (value, index) pairs per row.
//
// Algorithm (one CTA per row):
//  1. The encoder GEMM epilogue stored the max of every 32-column chunk.  The k-th largest
//     chunk max `klb` is a lower bound on the row's k-th largest value (k distinct chunks
//     each hold a value >= klb), so only chunks whose max >= klb can contribute.
//  2. Those chunks (about k of them) are read from H and every value >= klb is appended to a
//     shared-memory candidate list.
//  3. Two 8-bit radix-select passes over the 16-bit order-preserving keys give the exact k-th
//     largest key; values above it are emitted, and ties at it are broken by the smaller
//     column index so the selection is deterministic.
//  If the candidate list overflows (pathological ties), the row is selected directly from H
//  with the same radix select and an index-ordered tie scan.
// An optional column bitmask (one bit per column, 1 = eligible) restricts the selection to
// dead latents for the aux-k loss; the effective k can come from device memory so that the
// number of dead latents never has to be read on the host.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "p2p.cuh"
#include "check.h"
#include "bounds.cuh"

namespace sb {
namespace topk {

constexpr int THREADS = 256;
constexpr int CAP = 8192;
constexpr int MAX_NC = 32768;  // chunk keys cached in shared memory (N <= 1,048,576)

struct Sel {
  uint32_t key;   // k-th largest key
  int greater;    // number of keys strictly greater
};

// Warp 0: with hist[] over 256 bins, find the highest bin b with count(bins >= b) >= k.
// Writes sh[0] = b, sh[1] = count(bins > b).
__device__ __forceinline__ void scan_hist_desc(const uint32_t* hist, int k, uint32_t* sh) {
  const int lane = threadIdx.x & 31;
  uint32_t local[8];
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    local[j] = hist[255 - 8 * lane - j];
    s += local[j];
  }
  uint32_t incl = s;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  const uint32_t excl = incl - s;
  const unsigned m = __ballot_sync(0xffffffffu, excl < uint32_t(k) && uint32_t(k) <= incl);
  const int src = m ? __ffs(m) - 1 : -1;
  if (lane == src) {
    uint32_t cum = excl;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (cum + local[j] >= uint32_t(k)) {
        sh[0] = 255 - 8 * lane - j;
        sh[1] = cum;
        break;
      }
      cum += local[j];
    }
  }
  if (src < 0 && lane == 0) {  // k larger than the population: select everything
    sh[0] = 0;
    sh[1] = 0;
  }
}

// Block-wide: k-th largest of n 16-bit keys (keys with bit 16 set are "absent").
template <typename LoadKey>
__device__ Sel block_select16(int n, int k, LoadKey load, uint32_t* hist, uint32_t* sh) {
  for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t key = load(i);
    if (key < 0x10000u) atomicAdd(&hist[key >> 8], 1u);
  }
  __syncthreads();
  if (threadIdx.x < 32) scan_hist_desc(hist, k, sh);
  __syncthreads();
  const uint32_t b1 = sh[0];
  const int above1 = int(sh[1]);
  __syncthreads();
  for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t key = load(i);
    if (key < 0x10000u && (key >> 8) == b1) atomicAdd(&hist[key & 0xffu], 1u);
  }
  __syncthreads();
  if (threadIdx.x < 32) scan_hist_desc(hist, k - above1, sh);
  __syncthreads();
  Sel r;
  r.key = (b1 << 8) | sh[0];
  r.greater = above1 + int(sh[1]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ bool col_ok(const uint32_t* mask, int col) {
  return mask == nullptr || ((__ldg(mask + (col >> 5)) >> (col & 31)) & 1u);
}

__global__ void __launch_bounds__(THREADS)
    row_topk_kernel(const __nv_bfloat16* __restrict__ H, int64_t ldh,
                    const __nv_bfloat16* __restrict__ cmax, int64_t ldc, int N, int k_max,
                    const int* __restrict__ k_dev, const uint32_t* __restrict__ mask,
                    float* __restrict__ out_val, int* __restrict__ out_idx, int64_t ldo,
                    int* status, const __nv_bfloat16* __restrict__ tmax, int64_t ldtm) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh[4];
  __shared__ int n_cand, n_out;
  extern __shared__ uint8_t dyn[];
  const int NC = N >> 5;
  uint16_t* ckeys = reinterpret_cast<uint16_t*>(dyn);
  uint32_t* cand_key = reinterpret_cast<uint32_t*>(dyn + ((NC * 2 + 15) & ~15));
  int* cand_idx = reinterpret_cast<int*>(cand_key + CAP);

  const int row = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint16_t* hrow = reinterpret_cast<const uint16_t*>(H + int64_t(row) * ldh);
  const uint16_t* crow = reinterpret_cast<const uint16_t*>(cmax + int64_t(row) * ldc);
  float* vrow = out_val + int64_t(row) * ldo;
  int* irow = out_idx + int64_t(row) * ldo;

  int k = k_max;
  if (k_dev) k = min(k, *k_dev);
  // padding for rows with fewer eligible columns than k_max
  for (int i = tid; i < k_max; i += THREADS) {
    vrow[i] = 0.f;
    irow[i] = -1;
  }
  if (k <= 0) return;

  // Fast path (no column mask): chunk maxima bound the k-th value from below.  With a mask the
  // unmasked chunk maxima are no bound for the eligible columns, so masked rows go straight to
  // the exact full-row path below.
  if (tid == 0) {
    n_cand = 0;
    n_out = 0;
  }
  __syncthreads();
  if (mask == nullptr) {
  // Collect every value >= klb from the listed chunks (warps sweep 32 list entries at a time).
  auto collect = [&](int n_list, auto chunk_key, auto chunk_id, uint32_t klb) {
    for (int base = warp * 32; base < n_list; base += THREADS) {
      const int c = base + lane;
      const bool is_cand = c < n_list && chunk_key(c) >= klb;
      unsigned m = __ballot_sync(0xffffffffu, is_cand);
      while (m) {
        const int bit = __ffs(m) - 1;
        m &= m - 1;
        const int col = chunk_id(base + bit) * 32 + lane;
        const uint32_t key = bf16_to_key(hrow[col]);
        const bool keep = key >= klb;
        const unsigned km = __ballot_sync(0xffffffffu, keep);
        int basepos = 0;
        if (lane == 0 && km) basepos = atomicAdd(&n_cand, __popc(km));
        basepos = __shfl_sync(0xffffffffu, basepos, 0);
        const int pos = basepos + __popc(km & ((1u << lane) - 1u));
        if (keep && pos < CAP) {
          cand_key[pos] = key;
          cand_idx[pos] = col;
        }
      }
    }
  };
  bool collected = false;
  const int NT = N >> 8;
  if (tmax != nullptr && NT > k) {
    // Two levels: the k-th largest 256-column tile maximum bounds the k-th value from below; only
    // chunks of tiles at or above it can hold a top-k value, and the k-th largest chunk maximum
    // among them is the (tighter) bound used to collect candidates.
    const uint16_t* trow = reinterpret_cast<const uint16_t*>(tmax + int64_t(row) * ldtm);
    uint16_t* tkeys = ckeys;                  // NT tile keys
    const int lcap = ((NC - NT) / 2) & ~7;    // chunk-list capacity in the rest of ckeys
    uint16_t* lkey = ckeys + NT;
    uint16_t* lidx = lkey + lcap;
    __shared__ int n_list;
    for (int t = tid; t < NT; t += THREADS) tkeys[t] = uint16_t(bf16_to_key(trow[t]));
    if (tid == 0) n_list = 0;
    __syncthreads();
    const uint32_t klb0 = block_select16(NT, k, [&](int i) { return uint32_t(tkeys[i]); }, hist, sh).key;
    for (int t = tid; t < NT; t += THREADS) {
      if (uint32_t(tkeys[t]) >= klb0) {
        const int pos = atomicAdd(&n_list, 8);
        if (pos + 8 <= lcap) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            lkey[pos + j] = uint16_t(bf16_to_key(crow[t * 8 + j]));
            lidx[pos + j] = uint16_t(t * 8 + j);
          }
        }
      }
    }
    __syncthreads();
    const int nl = n_list;
    if (nl <= lcap) {
      const uint32_t klb =
          block_select16(nl, min(k, nl), [&](int i) { return uint32_t(lkey[i]); }, hist, sh).key;
      collect(nl, [&](int i) { return uint32_t(lkey[i]); }, [&](int i) { return int(lidx[i]); }, klb);
      collected = true;
    }
    __syncthreads();
  }
  if (!collected) {
    for (int c = tid; c < NC; c += THREADS) ckeys[c] = uint16_t(bf16_to_key(crow[c]));
    __syncthreads();
    uint32_t klb = 0;
    if (NC > k) klb = block_select16(NC, k, [&](int i) { return uint32_t(ckeys[i]); }, hist, sh).key;
    collect(NC, [&](int i) { return uint32_t(ckeys[i]); }, [&](int i) { return i; }, klb);
  }
  __syncthreads();
  const int C = n_cand;

  if (C <= CAP) {
    const int kk = min(k, C);
    const Sel r = block_select16(C, kk, [&](int i) { return cand_key[i]; }, hist, sh);
    const int need_ties = kk - r.greater;
    for (int i = tid; i < C; i += THREADS) {
      const uint32_t key = cand_key[i];
      bool take = key > r.key;
      if (!take && key == r.key) {
        const int my = cand_idx[i];
        int rank = 0;
        for (int j = 0; j < C; ++j) rank += (cand_key[j] == r.key && cand_idx[j] < my) ? 1 : 0;
        take = rank < need_ties;
      }
      if (take) {
        const int p = atomicAdd(&n_out, 1);
        if (p < k_max) {
          vrow[p] = key16_to_float(key);
          irow[p] = cand_idx[i];
        }
      }
    }
    return;
  }
  }  // fast path

  // ---- overflow fallback: exact select straight from H, ties in index order ----
  auto load_full = [&](int i) -> uint32_t {
    return col_ok(mask, i) ? bf16_to_key(hrow[i]) : 0x10000u;
  };
  int eligible = N;
  if (mask) {
    __shared__ int n_el;
    if (tid == 0) n_el = 0;
    __syncthreads();
    int cnt = 0;
    for (int c = tid; c < NC; c += THREADS) cnt += __popc(__ldg(mask + c));
    atomicAdd(&n_el, cnt);
    __syncthreads();
    eligible = n_el;
  }
  const int kk = min(k, eligible);
  const Sel r = block_select16(N, kk, load_full, hist, sh);
  const int need_ties = kk - r.greater;
  __shared__ int warp_tot[THREADS / 32];
  __shared__ int running;
  if (tid == 0) running = 0;
  __syncthreads();
  for (int base = 0; base < N; base += THREADS) {
    const int col = base + tid;
    const uint32_t key = col < N ? load_full(col) : 0x10000u;
    const bool gt = key < 0x10000u && key > r.key;
    const bool tie = key < 0x10000u && key == r.key;
    const unsigned tm = __ballot_sync(0xffffffffu, tie);
    if (lane == 0) warp_tot[warp] = __popc(tm);
    __syncthreads();
    int before = running;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    before += __popc(tm & ((1u << lane) - 1u));
    const bool take = gt || (tie && before < need_ties);
    if (take) {
      const int p = atomicAdd(&n_out, 1);
      if (p < k_max) {
        vrow[p] = key16_to_float(key);
        irow[p] = col;
      }
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < THREADS / 32; ++w) tot += warp_tot[w];
      running += tot;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// Tensor-parallel merge.  Every rank holds the per-row top-k of its own latent shard; after an
// all-gather of those candidates (cand_* [S, M, k], shard s owning global columns
// [s*n_local, (s+1)*n_local)), the global top-k of a row is the top-k of its S*k candidates.
// This kernel computes it for every row and keeps, in this rank's own (vals, idx), only the
// entries that made the global cut (the others become idx -1).  Ties at the k-th value are
// broken by the smaller global column index, matching the single-GPU kernel.
// ---------------------------------------------------------------------------------------
// Merge one row.  Candidate (s, i) of the row is at cv[s * s_stride + i] / ci[...]; the own
// candidates' output slots irow[i] become -1 when they miss the global cut.  key / gidx are
// S*k-entry shared arrays.  Starts with a barrier, so it may be called once per row in a loop.
__device__ __forceinline__ void merge_row(const float* cv, const int* ci, int64_t s_stride, int S, int k,
                                          int64_t n_local, int rank, int kk, int* irow, uint32_t* key,
                                          int64_t* gidx, uint32_t* hist, uint32_t* sh, int* n_valid) {
  const int C = S * k;
  const int tid = threadIdx.x;
  __syncthreads();
  if (tid == 0) *n_valid = 0;
  __syncthreads();
  int nv = 0;
  for (int c = tid; c < C; c += THREADS) {
    const int s = c / k, i = c - s * k;
    const int64_t off = int64_t(s) * s_stride + i;
    const int li = __ldcg(ci + off);
    if (li >= 0 && SB_IN_RANGE(li, n_local)) {  // debug builds: a peer id past its shard is dropped
      const uint32_t bits = __float_as_uint(__ldcg(cv + off)) >> 16;  // values are exact bf16
      key[c] = bf16_to_key(uint16_t(bits));
      gidx[c] = int64_t(s) * n_local + li;
      ++nv;
    } else {
      key[c] = 0x10000u;
      gidx[c] = -1;
    }
  }
  atomicAdd(n_valid, nv);
  __syncthreads();
  kk = min(kk, *n_valid);
  if (kk <= 0) {
    for (int i = tid; i < k; i += THREADS) irow[i] = -1;
    return;
  }
  const Sel r = block_select16(C, kk, [&](int i) { return key[i]; }, hist, sh);
  const int need_ties = kk - r.greater;
  for (int i = tid; i < k; i += THREADS) {
    const int c = rank * k + i;
    const uint32_t kc = key[c];
    bool keep = kc < 0x10000u && kc > r.key;
    if (!keep && kc == r.key) {
      const int64_t my = gidx[c];
      int rk = 0;
      for (int j = 0; j < C; ++j) rk += (key[j] == r.key && gidx[j] < my) ? 1 : 0;
      keep = rk < need_ties;
    }
    if (!keep) irow[i] = -1;
  }
}

__global__ void __launch_bounds__(THREADS)
    topk_merge_kernel(const float* __restrict__ cand_val, const int* __restrict__ cand_idx, int S, int M,
                      int k, int64_t n_local, int rank, const int* __restrict__ k_dev,
                      float* __restrict__ out_val, int* __restrict__ out_idx) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh[4];
  __shared__ int n_valid;
  extern __shared__ uint8_t dyn[];
  uint32_t* key = reinterpret_cast<uint32_t*>(dyn);
  int64_t* gidx = reinterpret_cast<int64_t*>(dyn + ((size_t(S * k) * 4 + 15) & ~size_t(15)));
  const int row = blockIdx.x;
  int kk = k;
  if (k_dev) kk = min(kk, *k_dev);
  (void)out_val;
  merge_row(cand_val + int64_t(row) * k, cand_idx + int64_t(row) * k, int64_t(M) * k, S, k, n_local, rank, kk,
            out_idx + int64_t(row) * k, key, gidx, hist, sh, &n_valid);
}

// ---------------------------------------------------------------------------------------
// Fused candidate all-gather + merge over NVLink (one launch per rank, ranks concurrent).
//   phase A (tickets [0, B/RB)): copy RB rows of this rank's candidates into slot [rank] of
//           every rank's candidate area (P2P stores), then release-add each receiver's arrival
//           counter of that row block.
//   phase B (tickets [B/RB, 2B/RB)): wait until all S slots of a row block arrived, then merge
//           its rows as topk_merge does, reading the S candidate lists from local memory.
// Slab layout: cand values fp32 [S, B, k] at cv_off, indices int32 [S, B, k] at ci_off, counters
// u32 [B/RB] at cnt_off.  Replaces the all-gather + merge of the TP top-k (the reference gathers
// the full [B, d_sae] pre-activations instead: sae_lens/distributed.py:404-461).
// ---------------------------------------------------------------------------------------
constexpr int XM_RB = 16;

struct XMergeArgs {
  const float* vals;
  int* idx;  // in: own candidates (local ids); out: -1 where they miss the global cut
  int B, k;
  int64_t n_local;
  const int* k_dev;
  p2p::Peers P;
  int64_t cv_off, ci_off, cnt_off;
  uint32_t epoch;
  int* ticket;
  int* status;
};

__global__ void __launch_bounds__(THREADS) topk_exchange_merge_kernel(const __grid_constant__ XMergeArgs a) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh[4];
  __shared__ int n_valid, s_tk, s_ok;
  extern __shared__ uint8_t dyn[];
  const int S = a.P.world, r = a.P.rank, k = a.k;
  uint32_t* key = reinterpret_cast<uint32_t*>(dyn);
  int64_t* gidx = reinterpret_cast<int64_t*>(dyn + ((size_t(S * k) * 4 + 15) & ~size_t(15)));
  const int t = threadIdx.x;
  const int nA = a.B / XM_RB;
  int kk = k;
  if (a.k_dev) kk = min(kk, *a.k_dev);
  while (true) {
    __syncthreads();
    if (t == 0) s_tk = atomicAdd(a.ticket, 1);
    __syncthreads();
    const int tk = s_tk;
    if (tk >= 2 * nA) break;
    if (tk < nA) {
      const int blk = tk;
      const int64_t row0 = int64_t(blk) * XM_RB;
      const int nv4 = XM_RB * k / 4;  // 16-byte vectors per block and array
      const uint4* sv = reinterpret_cast<const uint4*>(a.vals + row0 * k);
      const uint4* si = reinterpret_cast<const uint4*>(a.idx + row0 * k);
      for (int dd = 1; dd <= S; ++dd) {
        const int d = (r + dd) % S;
        uint4* dv = reinterpret_cast<uint4*>(p2p::at<float>(a.P, d, a.cv_off) + (int64_t(r) * a.B + row0) * k);
        uint4* di = reinterpret_cast<uint4*>(p2p::at<int>(a.P, d, a.ci_off) + (int64_t(r) * a.B + row0) * k);
        for (int v = t; v < nv4; v += THREADS) {
          dv[v] = __ldcg(sv + v);
          di[v] = __ldcg(si + v);
        }
      }
      __threadfence_system();
      __syncthreads();
      if (t < S) red_release_sys_add_u32(p2p::at<uint32_t>(a.P, t, a.cnt_off) + blk, 1u);
    } else {
      const int blk = tk - nA;
      if (t == 0)
        s_ok = wait_geq_sys(p2p::at<uint32_t>(a.P, r, a.cnt_off) + blk, uint32_t(S) * a.epoch, a.status,
                            kTimeoutPeerFlag)
                   ? 1
                   : 0;
      __syncthreads();
      if (!s_ok) continue;
      const float* cv = p2p::at<float>(a.P, r, a.cv_off);
      const int* ci = p2p::at<int>(a.P, r, a.ci_off);
      for (int rr = 0; rr < XM_RB; ++rr) {
        const int64_t row = int64_t(blk) * XM_RB + rr;
        merge_row(cv + row * k, ci + row * k, int64_t(a.B) * k, S, k, a.n_local, r, kk, a.idx + row * k, key,
                  gidx, hist, sh, &n_valid);
      }
    }
  }
}


// ---------------------------------------------------------------------------------------
// Batch top-k (BatchTopK SAEs: keep the k*B largest ReLU activations of the whole batch,
// sae_lens/saes/batchtopk_sae.py:13-33).  Input: per-row candidate lists (the per-row top-k_cap
// of the row top-k kernel, values exact bf16).  The global threshold comes from a 65536-bin
// histogram of the candidates' 16-bit keys (positive values only): the largest key whose
// suffix count reaches K.  Entries above the threshold are kept; ties at it are kept in (row,
// latent index) order until K entries are selected.  Unselected entries get idx -1.  A row
// whose k_cap-th candidate is still above the threshold may have lost entries to the per-row
// cap; those rows are counted in `truncated`.
// ---------------------------------------------------------------------------------------
__global__ void batch_hist_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int64_t n,
                                  uint32_t* __restrict__ hist) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float v = vals[i];
    if (idx[i] >= 0 && v > 0.f) atomicAdd(hist + bf16_to_key(uint16_t(__float_as_uint(v) >> 16)), 1u);
  }
}

// One CTA: find the threshold key and how many ties at it to keep.  sel[0] = key (0x8000 if fewer
// than K positive candidates: keep every positive one), sel[1] = ties to keep, sel[2] =
// strictly-above count, sel[3] = key of the smallest kept value (0 if nothing is kept).  With
// K >= 1 and the threshold found, at least one tie is kept, so the smallest kept value is the
// threshold key's; otherwise it is the smallest positive key present.
__global__ void batch_thresh_kernel(const uint32_t* __restrict__ hist, int64_t K, int* __restrict__ sel) {
  __shared__ uint32_t part[1024];
  __shared__ int s_found;
  __shared__ uint32_t s_min;
  const int t = threadIdx.x;  // 1024 threads x 64 bins, bins scanned from the top
  uint32_t sum = 0;
  for (int b = 0; b < 64; ++b) sum += hist[65535 - (t * 64 + b)];
  part[t] = sum;
  if (t == 0) {
    s_found = 0;
    s_min = 0x10000u;
  }
  __syncthreads();
  if (t == 0) {
    uint64_t acc = 0;
    int found = 0;
    for (int c = 0; c < 1024 && !found; ++c) {
      if (acc + part[c] >= uint64_t(K)) {
        for (int b = 0; b < 64; ++b) {
          const int key = 65535 - (c * 64 + b);
          const uint32_t h = hist[key];
          if (acc + h >= uint64_t(K)) {
            sel[0] = key;
            sel[1] = int(K - int64_t(acc));
            sel[2] = int(acc);
            sel[3] = K - int64_t(acc) > 0 ? key : 0;
            found = 1;
            break;
          }
          acc += h;
        }
      } else {
        acc += part[c];
      }
    }
    if (!found) {  // fewer than K positive candidates: keep them all
      sel[0] = 0x8000;  // key of +0.0: every positive value is strictly above it
      sel[1] = 0;
      sel[2] = int(acc);
    }
    s_found = found;
  }
  __syncthreads();
  if (!s_found) {
    uint32_t mn = 0x10000u;
    for (int b = 0; b < 64; ++b) {
      const uint32_t key = 65535u - uint32_t(t * 64 + b);
      if (key > 0x8000u && hist[key] > 0) mn = min(mn, key);
    }
    if (mn < 0x10000u) atomicMin(&s_min, mn);
    __syncthreads();
    if (t == 0) sel[3] = s_min < 0x10000u ? int(s_min) : 0;
  }
}

// Per row: ties at the threshold key (counted for the prefix over rows).
__global__ void batch_ties_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int M, int kc,
                                  const int* __restrict__ sel, int* __restrict__ ties) {
  const int key = sel[0];
  for (int row = blockIdx.x * blockDim.y + threadIdx.y; row < M; row += gridDim.x * blockDim.y) {
    int c = 0;
    for (int i = threadIdx.x; i < kc; i += 32) {
      const int64_t o = int64_t(row) * kc + i;
      const float v = vals[o];
      c += (idx[o] >= 0 && v > 0.f && int(bf16_to_key(uint16_t(__float_as_uint(v) >> 16))) == key) ? 1 : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (threadIdx.x == 0) ties[row] = c;
  }
}

// One CTA of 1024 threads: prefix[b] = ties of rows < b on every rank + ties of row b on ranks
// < rank, from the per-rank tie counts ties[S][M] (S = 1 on one GPU).  With latents sharded in
// contiguous blocks, (row, rank, local index) order is (row, global latent index) order.
__global__ void __launch_bounds__(1024) tie_prefix_kernel(const int* __restrict__ ties, int S, int M, int rank,
                                                          int64_t* __restrict__ prefix) {
  __shared__ int64_t part[1024];
  const int t = threadIdx.x;
  const int per = (M + 1023) / 1024;
  const int r0 = min(M, t * per), r1 = min(M, r0 + per);
  int64_t sum = 0;
  for (int b = r0; b < r1; ++b)
    for (int q = 0; q < S; ++q) sum += ties[int64_t(q) * M + b];
  part[t] = sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {  // inclusive scan
    const int64_t v = t >= o ? part[t - o] : 0;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  int64_t run = t > 0 ? part[t - 1] : 0;
  for (int b = r0; b < r1; ++b) {
    int64_t row_all = 0, row_before = 0;
    for (int q = 0; q < S; ++q) {
      const int c = ties[int64_t(q) * M + b];
      row_all += c;
      if (q < rank) row_before += c;
    }
    prefix[b] = run + row_before;
    run += row_all;
  }
}

// Per row: keep entries above the key, and ties while the global tie rank (rows before + smaller
// latent index within the row) is below the tie budget.  tie_prefix = exclusive prefix of ties.
__global__ void batch_filter_kernel(const float* __restrict__ vals, int* __restrict__ idx, int M, int kc,
                                    const int* __restrict__ sel, const int64_t* __restrict__ tie_prefix,
                                    int* __restrict__ truncated) {
  const int key = sel[0];
  const int64_t budget = sel[1];
  for (int row = blockIdx.x * blockDim.y + threadIdx.y; row < M; row += gridDim.x * blockDim.y) {
    const int64_t before = tie_prefix[row];
    uint32_t keep_bits = 0;  // bit m: entry lane + 32 m is kept (kc <= 1024)
    int kept = 0;
    for (int m = 0, i = threadIdx.x; i < kc; ++m, i += 32) {
      const int64_t o = int64_t(row) * kc + i;
      const int j = idx[o];
      const float v = vals[o];
      bool keep = false;
      if (j >= 0 && v > 0.f) {
        const int kk = int(bf16_to_key(uint16_t(__float_as_uint(v) >> 16)));
        if (kk > key) {
          keep = true;
        } else if (kk == key && budget > before) {
          int rank = 0;  // ties of this row with a smaller latent index
          for (int q = 0; q < kc; ++q) {
            const int64_t oq = int64_t(row) * kc + q;
            const float vq = vals[oq];
            rank += (idx[oq] >= 0 && idx[oq] < j && vq > 0.f &&
                     int(bf16_to_key(uint16_t(__float_as_uint(vq) >> 16))) == key) ? 1 : 0;
          }
          keep = before + rank < budget;
        }
      }
      keep_bits |= uint32_t(keep) << m;
      kept += keep;
    }
    __syncwarp();  // every lane has read the row before any slot is cleared
    for (int m = 0, i = threadIdx.x; i < kc; ++m, i += 32)
      if (!((keep_bits >> m) & 1u)) idx[int64_t(row) * kc + i] = -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kept += __shfl_xor_sync(0xffffffffu, kept, o);
    if (threadIdx.x == 0 && truncated && kept == kc) atomicAdd(truncated, 1);
  }
}

// ---------------------------------------------------------------------------------------
// JumpReLU candidates (sae_lens/saes/jumprelu_sae.py:19-85): per row, every column whose
// pre-activation exceeds lo[col] = threshold - bandwidth/2.  That covers the active entries
// (pre > threshold) and the rectangle window of the threshold's straight-through gradient.  A
// 32-column chunk can hold a candidate only if its maximum reaches the chunk's smallest lo, so the
// chunk maxima prune the row.  At most `cap` entries per row are kept (rows over the cap are
// counted in `truncated`); unused slots get idx -1.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS)
    threshold_select_kernel(const __nv_bfloat16* __restrict__ H, int64_t ldh, const __nv_bfloat16* __restrict__ cmax,
                            int64_t ldc, int N, const float* __restrict__ lo, const float* __restrict__ lo_cmin,
                            int cap, float* __restrict__ out_val, int* __restrict__ out_idx, int* __restrict__ counts,
                            int* __restrict__ truncated) {
  __shared__ int n_out;
  const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NC = N >> 5;
  const __nv_bfloat16* hrow = H + int64_t(row) * ldh;
  const __nv_bfloat16* crow = cmax + int64_t(row) * ldc;
  float* vrow = out_val + int64_t(row) * cap;
  int* irow = out_idx + int64_t(row) * cap;
  if (tid == 0) n_out = 0;
  __syncthreads();
  for (int base = warp * 32; base < NC; base += THREADS) {
    const int c = base + lane;
    const bool is_cand = c < NC && __bfloat162float(crow[c]) >= __ldg(lo_cmin + c);
    unsigned m = __ballot_sync(0xffffffffu, is_cand);
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      const int col = (base + bit) * 32 + lane;
      const float v = __bfloat162float(hrow[col]);
      const bool keep = v > __ldg(lo + col);
      const unsigned km = __ballot_sync(0xffffffffu, keep);
      int basepos = 0;
      if (lane == 0 && km) basepos = atomicAdd(&n_out, __popc(km));
      basepos = __shfl_sync(0xffffffffu, basepos, 0);
      const int pos = basepos + __popc(km & ((1u << lane) - 1u));
      if (keep && pos < cap) {
        vrow[pos] = v;
        irow[pos] = col;
      }
    }
  }
  __syncthreads();
  const int n = n_out;
  for (int i = n + tid; i < cap; i += THREADS) {
    vrow[i] = 0.f;
    irow[i] = -1;
  }
  if (tid == 0) {
    counts[row] = min(n, cap);
    if (n > cap && truncated) atomicAdd(truncated, 1);
  }
}
}  // namespace topk

void topk_merge(const torch::Tensor& cand_val, const torch::Tensor& cand_idx, int64_t n_local, int64_t rank,
                const c10::optional<torch::Tensor>& k_dev, const torch::Tensor& out_val,
                const torch::Tensor& out_idx) {
  SB_CHECK(cand_val.dim() == 3 && cand_val.sizes() == cand_idx.sizes() && cand_val.is_contiguous() &&
                  cand_idx.is_contiguous() && cand_val.scalar_type() == at::kFloat &&
                  cand_idx.scalar_type() == at::kInt,
              "topk_merge: candidates must be contiguous fp32/int32 [S, M, k]");
  const int64_t S = cand_val.size(0), M = cand_val.size(1), k = cand_val.size(2);
  SB_CHECK(out_val.size(0) == M && out_val.size(1) == k && out_idx.is_contiguous(), "topk_merge: outputs");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(cand_val.device());
  const size_t smem = ((size_t(S * k) * 4 + 15) & ~size_t(15)) + size_t(S * k) * 8;
  SB_CHECK(smem <= 227 * 1024, "topk_merge: S*k too large for one CTA");
  C10_CUDA_CHECK(cudaFuncSetAttribute(topk::topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(smem)));
  topk::topk_merge_kernel<<<dim3(M), dim3(topk::THREADS), smem, at::cuda::getCurrentCUDAStream()>>>(
      cand_val.data_ptr<float>(), cand_idx.data_ptr<int>(), int(S), int(M), int(k), n_local, int(rank),
      k_dev ? k_dev->data_ptr<int>() : nullptr, out_val.data_ptr<float>(), out_idx.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// H [M, N] bf16, cmax [M, N/32] bf16 -> (val fp32 [M, k_max], idx int32 [M, k_max]).
// `k_dev` (int32 scalar on device) optionally lowers k below k_max; `mask` (int32 bit words,
// [N/32]) optionally restricts the eligible columns.  Unused output slots hold idx -1, val 0.
void row_topk(const torch::Tensor& H, const torch::Tensor& cmax, int64_t k_max,
              const c10::optional<torch::Tensor>& k_dev, const c10::optional<torch::Tensor>& mask,
              const torch::Tensor& out_val, const torch::Tensor& out_idx, const torch::Tensor& status,
              const c10::optional<torch::Tensor>& tmax) {
  SB_CHECK(H.is_cuda() && H.scalar_type() == at::kBFloat16 && H.dim() == 2 && H.stride(1) == 1,
              "row_topk: H must be a CUDA bf16 matrix with contiguous rows");
  const int64_t M = H.size(0), N = H.size(1);
  SB_CHECK(N % 32 == 0 && N / 32 <= topk::MAX_NC, "row_topk: N must be a multiple of 32 and <= 2^20");
  SB_CHECK(cmax.scalar_type() == at::kBFloat16 && cmax.size(0) == M && cmax.size(1) == N / 32 &&
                  cmax.stride(1) == 1,
              "row_topk: bad cmax");
  SB_CHECK(k_max >= 1 && k_max <= N, "row_topk: k out of range");
  SB_CHECK(out_val.scalar_type() == at::kFloat && out_idx.scalar_type() == at::kInt &&
                  out_val.size(0) == M && out_val.size(1) == k_max && out_idx.size(0) == M &&
                  out_idx.size(1) == k_max && out_val.is_contiguous() && out_idx.is_contiguous(),
              "row_topk: bad outputs");
  const int* kd = nullptr;
  if (k_dev) {
    SB_CHECK(k_dev->scalar_type() == at::kInt && k_dev->numel() == 1, "row_topk: k_dev");
    kd = k_dev->data_ptr<int>();
  }
  const uint32_t* mk = nullptr;
  if (mask) {
    SB_CHECK(mask->scalar_type() == at::kInt && mask->numel() == N / 32 && mask->is_contiguous(),
                "row_topk: mask must be int32 [N/32]");
    mk = reinterpret_cast<const uint32_t*>(mask->data_ptr<int>());
  }
  if (tmax) {
    SB_CHECK(N % 256 == 0 && tmax->scalar_type() == at::kBFloat16 && tmax->size(0) == M &&
                    tmax->size(1) == N / 256 && tmax->stride(1) == 1,
                "row_topk: tmax must be bf16 [M, N/256]");
  }
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(H.device());
  const int NC = int(N / 32);
  const size_t smem = ((NC * 2 + 15) & ~15) + size_t(topk::CAP) * 8;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(topk::row_topk_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(((topk::MAX_NC * 2 + 15) & ~15) + topk::CAP * 8)));
    attr = true;
  }
  topk::row_topk_kernel<<<dim3(M), dim3(topk::THREADS), smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(H.data_ptr()), H.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(cmax.data_ptr()), cmax.stride(0), int(N), int(k_max),
      kd, mk, out_val.data_ptr<float>(), out_idx.data_ptr<int>(), out_val.stride(0),
      status.data_ptr<int>(), tmax ? reinterpret_cast<const __nv_bfloat16*>(tmax->data_ptr()) : nullptr,
      tmax ? tmax->stride(0) : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused candidate exchange + merge (see topk_exchange_merge_kernel).  vals/idx [B, k]: this
// rank's per-row top-k of its shard (local ids); on return idx is -1 wherever an entry missed
// the global top-k.  `epoch` counts the launches that used these slab buffers (1, 2, ...).
void topk_exchange_merge(const torch::Tensor& vals, const torch::Tensor& idx, int64_t n_local,
                         const c10::optional<torch::Tensor>& k_dev, const std::vector<int64_t>& peer_bases,
                         int64_t rank, int64_t cv_off, int64_t ci_off, int64_t cnt_off, int64_t epoch,
                         const torch::Tensor& ticket, const torch::Tensor& status) {
  const int64_t S = int64_t(peer_bases.size());
  SB_CHECK(S >= 1 && S <= p2p::kMaxRanks && rank >= 0 && rank < S, "topk_exchange_merge: bad group");
  SB_CHECK(vals.is_contiguous() && idx.is_contiguous() && vals.scalar_type() == at::kFloat &&
                  idx.scalar_type() == at::kInt && vals.sizes() == idx.sizes(),
              "topk_exchange_merge: vals/idx");
  const int64_t B = vals.size(0), k = vals.size(1);
  SB_CHECK(B % topk::XM_RB == 0, "topk_exchange_merge: batch must be a multiple of 16");
  SB_CHECK(cv_off % 16 == 0 && ci_off % 16 == 0, "topk_exchange_merge: offsets");
  const size_t smem = ((size_t(S * k) * 4 + 15) & ~size_t(15)) + size_t(S * k) * 8;
  SB_CHECK(smem <= 200 * 1024, "topk_exchange_merge: S*k too large for one CTA");
  const at::cuda::CUDAGuard guard(vals.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  topk::XMergeArgs a{};
  a.vals = vals.data_ptr<float>();
  a.idx = idx.data_ptr<int>();
  a.B = int(B);
  a.k = int(k);
  a.n_local = n_local;
  a.k_dev = k_dev ? k_dev->data_ptr<int>() : nullptr;
  a.P = p2p::make_peers(peer_bases, rank);
  a.cv_off = cv_off;
  a.ci_off = ci_off;
  a.cnt_off = cnt_off;
  a.epoch = uint32_t(epoch);
  a.ticket = ticket.data_ptr<int>();
  a.status = status.data_ptr<int>();
  C10_CUDA_CHECK(cudaMemsetAsync(a.ticket, 0, sizeof(int), stream));
  C10_CUDA_CHECK(cudaFuncSetAttribute(topk::topk_exchange_merge_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  int occ = 0;
  C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, topk::topk_exchange_merge_kernel,
                                                               topk::THREADS, smem));
  int dev = 0, nsm = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(2 * B / topk::XM_RB, int64_t(nsm) * std::max(occ, 1)));
  topk::topk_exchange_merge_kernel<<<dim3(grid), dim3(topk::THREADS), smem, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void check_cands(const torch::Tensor& vals, const torch::Tensor& idx, const char* what) {
  SB_CHECK(vals.is_cuda() && vals.is_contiguous() && idx.is_contiguous() && vals.scalar_type() == at::kFloat &&
                  idx.scalar_type() == at::kInt && vals.sizes() == idx.sizes() && vals.dim() == 2,
              what, ": vals/idx must be contiguous fp32/int32 [M, kc]");
  SB_CHECK(vals.size(1) <= 1024, what, ": at most 1024 candidates per row");
}

static int sm_count_here() {
  int dev = 0, nsm = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  return nsm;
}

// 65536-bin histogram (int32, zeroed here) of the positive candidates' bf16 keys.
void batch_hist(const torch::Tensor& vals, const torch::Tensor& idx, const torch::Tensor& hist) {
  check_cands(vals, idx, "batch_hist");
  SB_CHECK(hist.is_cuda() && hist.is_contiguous() && hist.scalar_type() == at::kInt && hist.numel() == 65536,
              "batch_hist: hist must be int32 [65536]");
  const at::cuda::CUDAGuard guard(vals.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemsetAsync(hist.data_ptr<int>(), 0, 65536 * sizeof(int), stream));
  const int64_t n = vals.numel();
  if (n == 0) return;
  topk::batch_hist_kernel<<<dim3(int(std::min<int64_t>((n + 255) / 256, int64_t(sm_count_here()) * 8))), 256, 0,
                            stream>>>(vals.data_ptr<float>(), idx.data_ptr<int>(), n,
                                      reinterpret_cast<uint32_t*>(hist.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Threshold of the K largest from a (possibly group-summed) histogram; sel int32 [4] (see
// batch_thresh_kernel).
void batch_thresh(const torch::Tensor& hist, int64_t K, const torch::Tensor& sel) {
  SB_CHECK(hist.is_cuda() && hist.is_contiguous() && hist.scalar_type() == at::kInt && hist.numel() == 65536 &&
                  sel.is_cuda() && sel.scalar_type() == at::kInt && sel.numel() >= 4,
              "batch_thresh: hist int32 [65536], sel int32 [4]");
  const at::cuda::CUDAGuard guard(hist.device());
  topk::batch_thresh_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(hist.data_ptr<int>()), K, sel.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Ties at the threshold key per row (int32 [M], contiguous).
void batch_ties(const torch::Tensor& vals, const torch::Tensor& idx, const torch::Tensor& sel,
                const torch::Tensor& ties) {
  check_cands(vals, idx, "batch_ties");
  const int64_t M = vals.size(0), kc = vals.size(1);
  SB_CHECK(ties.is_cuda() && ties.is_contiguous() && ties.scalar_type() == at::kInt && ties.numel() == M,
              "batch_ties: ties must be int32 [M]");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(vals.device());
  const int grid = int(std::min<int64_t>((M + 7) / 8, int64_t(sm_count_here()) * 16));
  topk::batch_ties_kernel<<<grid, dim3(32, 8), 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), idx.data_ptr<int>(), int(M), int(kc), sel.data_ptr<int>(), ties.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Keep the selected entries (idx -1 elsewhere), with ties ranked in (row, rank, local index)
// order from every rank's per-row tie counts ties_all [S, M].  prefix: int64 [M] scratch.
void batch_filter(const torch::Tensor& vals, const torch::Tensor& idx, const torch::Tensor& sel,
                  const torch::Tensor& ties_all, int64_t rank, const torch::Tensor& prefix,
                  const c10::optional<torch::Tensor>& truncated) {
  check_cands(vals, idx, "batch_filter");
  const int64_t M = vals.size(0), kc = vals.size(1);
  SB_CHECK(ties_all.is_cuda() && ties_all.is_contiguous() && ties_all.scalar_type() == at::kInt &&
                  ties_all.dim() == 2 && ties_all.size(1) == M && rank >= 0 && rank < ties_all.size(0),
              "batch_filter: ties_all must be int32 [S, M]");
  SB_CHECK(prefix.is_cuda() && prefix.is_contiguous() && prefix.scalar_type() == at::kLong && prefix.numel() >= M,
              "batch_filter: prefix must be int64 [M]");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(vals.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  topk::tie_prefix_kernel<<<1, 1024, 0, stream>>>(ties_all.data_ptr<int>(), int(ties_all.size(0)), int(M), int(rank),
                                                   prefix.data_ptr<int64_t>());
  const int grid = int(std::min<int64_t>((M + 7) / 8, int64_t(sm_count_here()) * 16));
  topk::batch_filter_kernel<<<grid, dim3(32, 8), 0, stream>>>(vals.data_ptr<float>(), idx.data_ptr<int>(), int(M),
                                                               int(kc), sel.data_ptr<int>(),
                                                               prefix.data_ptr<int64_t>(),
                                                               truncated ? truncated->data_ptr<int>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Keep the K = round(k * rows) largest positive candidate values of the whole batch (see
// batch_hist_kernel).  vals/idx [M, kc] from row_topk; idx is updated in place (-1 = dropped).
// Returns int32 [4] on the device (see batch_thresh_kernel); counts rows whose whole candidate
// list was kept into `truncated` (int32 [1], optional).  Five launches, no host sync.
torch::Tensor batch_topk_select(const torch::Tensor& vals, const torch::Tensor& idx, int64_t K,
                                const c10::optional<torch::Tensor>& truncated) {
  check_cands(vals, idx, "batch_topk_select");
  const int64_t M = vals.size(0);
  auto opts = vals.options();
  auto sel = torch::zeros({4}, opts.dtype(at::kInt));
  if (M == 0) return sel;
  auto hist = torch::empty({65536}, opts.dtype(at::kInt));
  auto ties = torch::empty({1, M}, opts.dtype(at::kInt));
  auto prefix = torch::empty({M}, opts.dtype(at::kLong));
  batch_hist(vals, idx, hist);
  batch_thresh(hist, K, sel);
  auto ties_row = ties.select(0, 0);
  batch_ties(vals, idx, sel, ties_row);
  batch_filter(vals, idx, sel, ties, 0, prefix, truncated);
  return sel;
}

// JumpReLU candidate lists (see threshold_select_kernel).  H [M, N] bf16 pre-activations, cmax
// [M, N/32], lo [N] fp32 (threshold - bandwidth/2), lo_cmin [N/32] (per-chunk minimum of lo).
void threshold_select(const torch::Tensor& H, const torch::Tensor& cmax, const torch::Tensor& lo,
                      const torch::Tensor& lo_cmin, const torch::Tensor& out_val, const torch::Tensor& out_idx,
                      const torch::Tensor& counts, const c10::optional<torch::Tensor>& truncated) {
  SB_CHECK(H.is_cuda() && H.scalar_type() == at::kBFloat16 && H.dim() == 2 && H.stride(1) == 1,
              "threshold_select: H must be CUDA bf16 [M, N]");
  const int64_t M = H.size(0), N = H.size(1);
  SB_CHECK(N % 32 == 0 && cmax.size(0) == M && cmax.size(1) == N / 32 && cmax.stride(1) == 1,
              "threshold_select: cmax");
  SB_CHECK(lo.numel() == N && lo_cmin.numel() == N / 32 && lo.scalar_type() == at::kFloat &&
                  lo_cmin.scalar_type() == at::kFloat && lo.is_contiguous() && lo_cmin.is_contiguous(),
              "threshold_select: lo / lo_cmin");
  SB_CHECK(out_val.is_contiguous() && out_idx.is_contiguous() && out_val.size(0) == M && out_idx.size(0) == M &&
                  out_val.size(1) == out_idx.size(1) && counts.numel() == M,
              "threshold_select: outputs");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(H.device());
  topk::threshold_select_kernel<<<dim3(M), dim3(topk::THREADS), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(H.data_ptr()), H.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(cmax.data_ptr()), cmax.stride(0), int(N), lo.data_ptr<float>(),
      lo_cmin.data_ptr<float>(), int(out_val.size(1)), out_val.data_ptr<float>(), out_idx.data_ptr<int>(),
      counts.data_ptr<int>(), truncated ? truncated->data_ptr<int>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

#if SB_DEBUG_BOUNDS
namespace sb {
// {line, value, bound, violations} of this file's first bounds violation (debug module only).
std::vector<int64_t> topk_bounds_info(bool reset) { return bounds_read(reset); }
}  // namespace sb
#endif

// Allocation-free CSC build (see noalloc_csc.h for the contract and who needs it).
//
// Same result as the allocating path used by the training engine (csc_count, an exclusive scan
// of the per-latent counts, csc_fill), with all working memory in one file-scope device array:
//   [0, MAX)               per-latent counts
//   [MAX, 2*MAX)           per-latent fill cursors
//   [2*MAX, 2*MAX + MAX/1024)  per-block partial sums of the scan
//   [2*MAX + MAX/1024]     number of pairs skipped for a latent index >= n_latents
#include <mutex>

#include "noalloc_csc.h"

namespace {

constexpr int kMax = SB_NOALLOC_CSC_MAX_LATENTS;
constexpr int kScanBlock = 1024;
constexpr int kScanBlocksMax = kMax / kScanBlock;
constexpr int kMaxDevices = 64;

// 8 MiB + 4 KiB per device that loads the library, held until exit.
static __device__ __align__(256) int32_t g_csc_scratch[2 * kMax + kScanBlocksMax + 1];

__global__ void zero_kernel(int32_t* p, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = 0;
}

// Counts kept pairs per latent; an index >= n_latents is skipped and counted in *bad.
__global__ void count_kernel(const float* __restrict__ vals, const int32_t* __restrict__ idx, int64_t n_pairs,
                             int32_t n_latents, int32_t* __restrict__ counts, int32_t* __restrict__ bad) {
  int32_t nbad = 0;
  for (int64_t p = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; p < n_pairs; p += int64_t(gridDim.x) * blockDim.x) {
    const int32_t j = idx[p];
    if (j < 0 || !(vals[p] > 0.f)) continue;
    if (j >= n_latents) {
      ++nbad;
      continue;
    }
    atomicAdd(counts + j, 1);
  }
  if (nbad) atomicAdd(bad, nbad);
}

// inclusive warp scan helper
__device__ __forceinline__ int32_t warp_incl(int32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

// Block-wide exclusive scan of one value per thread (blockDim.x == kScanBlock); returns the
// exclusive prefix and writes the block total to *total.
__device__ __forceinline__ int32_t block_excl(int32_t v, int32_t* total) {
  __shared__ int32_t warp_sums[kScanBlock / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int32_t incl = warp_incl(v);
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int32_t s = warp_sums[lane];
    warp_sums[lane] = warp_incl(s) - s;  // exclusive over warps
  }
  __syncthreads();
  const int32_t out = warp_sums[warp] + incl - v;
  if (threadIdx.x == blockDim.x - 1) *total = out + v;
  __syncthreads();
  return out;
}

__global__ void copy_count_kernel(const int32_t* __restrict__ src, int32_t* __restrict__ dst) { *dst = *src; }

__global__ void __launch_bounds__(kScanBlock) block_sum_kernel(const int32_t* __restrict__ counts, int n,
                                                               int32_t* __restrict__ block_sums) {
  __shared__ int32_t tot;
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  block_excl(i < n ? counts[i] : 0, &tot);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kScanBlock) scan_block_sums_kernel(int32_t* __restrict__ block_sums, int nb) {
  __shared__ int32_t tot;
  const int i = threadIdx.x;
  const int32_t e = block_excl(i < nb ? block_sums[i] : 0, &tot);
  if (i < nb) block_sums[i] = e;
}

__global__ void __launch_bounds__(kScanBlock) colptr_kernel(const int32_t* __restrict__ counts, int n,
                                                            const int32_t* __restrict__ block_offs,
                                                            int64_t* __restrict__ colptr) {
  __shared__ int32_t tot;
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  const int32_t c = i < n ? counts[i] : 0;
  const int32_t e = block_excl(c, &tot);
  const int64_t off = block_offs[blockIdx.x];
  if (i < n) colptr[i] = off + e;
  if (i == n - 1) colptr[n] = off + e + c;
}

__global__ void fill_kernel(const float* __restrict__ vals, const int32_t* __restrict__ idx, int64_t n_pairs,
                            int32_t n_latents, const int64_t* __restrict__ colptr, int32_t* __restrict__ cursor,
                            int64_t* __restrict__ pairs) {
  for (int64_t p = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; p < n_pairs; p += int64_t(gridDim.x) * blockDim.x) {
    const int32_t j = idx[p];
    if (j >= 0 && j < n_latents && vals[p] > 0.f) {
      const int32_t pos = atomicAdd(cursor + j, 1);
      pairs[colptr[j] + pos] = p;
    }
  }
}

std::mutex g_setup_mutex;
int32_t* g_scratch_dev[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device (looked up once per device).
int scratch_for_current_device(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SB_NOALLOC_ERR_SYMBOL_ADDRESS;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_dev[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_csc_scratch);
    if (e != cudaSuccess || p == nullptr) return SB_NOALLOC_ERR_SYMBOL_ADDRESS;
    g_scratch_dev[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_dev[dev];
  return SB_NOALLOC_OK;
}

}  // namespace

extern "C" int sb_csc_build_noalloc(const float* vals, const int32_t* idx, int64_t n_pairs, int32_t n_latents,
                                    int64_t* colptr, int64_t* pairs, int32_t* bad_pairs, cudaStream_t stream) {
  if (n_latents < 1 || n_latents > kMax) return SB_NOALLOC_ERR_TOO_MANY_LATENTS;
  if (n_pairs > SB_NOALLOC_CSC_MAX_PAIRS) return SB_NOALLOC_ERR_TOO_MANY_PAIRS;
  if (n_pairs < 0 || colptr == nullptr || (n_pairs > 0 && (vals == nullptr || idx == nullptr || pairs == nullptr)))
    return SB_NOALLOC_ERR_BAD_ARGUMENT;
  if (cudaGetLastError() != cudaSuccess) return SB_NOALLOC_ERR_PENDING;
  int32_t* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != SB_NOALLOC_OK) return rc;
  int32_t* counts = scratch;
  int32_t* cursor = scratch + kMax;
  int32_t* block_sums = scratch + 2 * kMax;
  int32_t* bad = scratch + 2 * kMax + kScanBlocksMax;
  const int n = n_latents;
  const int nb = (n + kScanBlock - 1) / kScanBlock;
  const int zb = (n + 255) / 256;
  const int zgrid = zb < 1024 ? zb : 1024;
  const int64_t g = (n_pairs + 255) / 256;
  const int pgrid = int(g < 4096 ? g : 4096);
#define SB_NOALLOC_CHECK_LAUNCH() \
  if (cudaGetLastError() != cudaSuccess) return SB_NOALLOC_ERR_LAUNCH
  zero_kernel<<<zgrid, 256, 0, stream>>>(counts, n);
  SB_NOALLOC_CHECK_LAUNCH();
  zero_kernel<<<zgrid, 256, 0, stream>>>(cursor, n);
  SB_NOALLOC_CHECK_LAUNCH();
  zero_kernel<<<1, 32, 0, stream>>>(bad, 1);
  SB_NOALLOC_CHECK_LAUNCH();
  if (n_pairs > 0) {
    count_kernel<<<pgrid, 256, 0, stream>>>(vals, idx, n_pairs, n, counts, bad);
    SB_NOALLOC_CHECK_LAUNCH();
  }
  block_sum_kernel<<<nb, kScanBlock, 0, stream>>>(counts, n, block_sums);
  SB_NOALLOC_CHECK_LAUNCH();
  scan_block_sums_kernel<<<1, kScanBlock, 0, stream>>>(block_sums, nb);
  SB_NOALLOC_CHECK_LAUNCH();
  colptr_kernel<<<nb, kScanBlock, 0, stream>>>(counts, n, block_sums, colptr);
  SB_NOALLOC_CHECK_LAUNCH();
  if (n_pairs > 0) {
    fill_kernel<<<pgrid, 256, 0, stream>>>(vals, idx, n_pairs, n, colptr, cursor, pairs);
    SB_NOALLOC_CHECK_LAUNCH();
  }
  if (bad_pairs != nullptr) {
    copy_count_kernel<<<1, 1, 0, stream>>>(bad, bad_pairs);
    SB_NOALLOC_CHECK_LAUNCH();
  }
#undef SB_NOALLOC_CHECK_LAUNCH
  return SB_NOALLOC_OK;
}

extern "C" const char* sb_noalloc_strerror(int code) {
  switch (code) {
    case SB_NOALLOC_OK:
      return "ok";
    case SB_NOALLOC_ERR_TOO_MANY_LATENTS:
      return "n_latents must be between 1 and SB_NOALLOC_CSC_MAX_LATENTS (1048576)";
    case SB_NOALLOC_ERR_BAD_ARGUMENT:
      return "null pointer or negative n_pairs";
    case SB_NOALLOC_ERR_SYMBOL_ADDRESS:
      return "could not look up the device address of the scratch array (cudaGetSymbolAddress)";
    case SB_NOALLOC_ERR_LAUNCH:
      return "kernel launch failed";
    case SB_NOALLOC_ERR_TOO_MANY_PAIRS:
      return "n_pairs must be at most SB_NOALLOC_CSC_MAX_PAIRS (2147483647)";
    case SB_NOALLOC_ERR_PENDING:
      return "a CUDA error was already pending when the call started (taken with cudaGetLastError); nothing was launched";
    default:
      return "unknown error";
  }
}

// Debug bounds checks for the kernels that dereference data-dependent indices: the sparse
// decode / CSC build / latent gradients (latent ids, pair ids, CSC offsets, pair rows), the top-k
// candidate merges (peer-local latent ids) and the ring gather / row router (permutation rows,
// routing-table row ranges).
//
// In the normal build (`SB_DEBUG_BOUNDS` undefined or 0) `SB_IN_RANGE(v, n)` is the constant
// `true` and compiles away.  The debug module `_C_debug` compiles the same kernel sources with
// `-DSB_DEBUG_BOUNDS=1`: each such index is tested against its bound before it is used, and a
// value outside [0, n) makes the kernel skip that access (the entry is treated as absent) and
// record, in a per-source-file device record, how many violations happened and the source line,
// value and bound of the first one.  The host reads and clears the record with the unit's
// `<unit>_bounds_info(reset)` binding.  Nothing traps or asserts; the kernel runs to its end.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#ifndef SB_DEBUG_BOUNDS
#define SB_DEBUG_BOUNDS 0
#endif

namespace sb {

#if SB_DEBUG_BOUNDS
// [0] first violating source line + 1 (0: none), [1] its value, [2] its bound, [3] violations
// (distinct (line, value) per warp).
// `static`: one record per translation unit (the module is built without relocatable device code).
static __device__ unsigned long long g_bounds_rec[4];

// Lanes of a warp that report the same (line, value) together (a warp checking one shared index)
// count as one violation: the lowest such lane records it.
static __device__ __noinline__ void bounds_record(long long v, long long n, int line) {
  const unsigned long long key = (static_cast<unsigned long long>(line) << 44) ^ static_cast<unsigned long long>(v);
  const unsigned same = __match_any_sync(__activemask(), key);
  if ((threadIdx.x & 31) != __ffs(same) - 1) return;
  atomicAdd(&g_bounds_rec[3], 1ull);
  if (atomicCAS(&g_bounds_rec[0], 0ull, static_cast<unsigned long long>(line) + 1ull) == 0ull) {
    g_bounds_rec[1] = static_cast<unsigned long long>(v);
    g_bounds_rec[2] = static_cast<unsigned long long>(n);
  }
}

// {line, value, bound, violations}; line 0 means no violation since the last reset.
static inline std::vector<int64_t> bounds_read(bool reset) {
  unsigned long long h[4] = {0, 0, 0, 0};
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(h, g_bounds_rec, sizeof(h));
  if (reset) {
    const unsigned long long z[4] = {0, 0, 0, 0};
    cudaMemcpyToSymbol(g_bounds_rec, z, sizeof(z));
  }
  return {h[0] == 0 ? 0 : static_cast<int64_t>(h[0] - 1), static_cast<int64_t>(h[1]),
          static_cast<int64_t>(h[2]), static_cast<int64_t>(h[3])};
}
#endif

__device__ __forceinline__ bool in_range(long long v, long long n, int line) {
#if SB_DEBUG_BOUNDS
  if (v < 0 || v >= n) {
    bounds_record(v, n, line);
    return false;
  }
#else
  (void)v;
  (void)n;
  (void)line;
#endif
  return true;
}

}  // namespace sb

#if SB_DEBUG_BOUNDS
#define SB_IN_RANGE(v, n) (::sb::in_range(static_cast<long long>(v), static_cast<long long>(n), __LINE__))
#else
// the arguments are not evaluated: a check may read the index it tests
#define SB_IN_RANGE(v, n) true
#endif

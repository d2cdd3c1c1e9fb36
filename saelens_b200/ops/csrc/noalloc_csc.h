// Allocation-free entry point for building the latent-major (CSC) pair lists of a TopK step.
//
// This entry point has no counterpart in the reference (SAELens has no native code); it exists
// for callers of this library that cannot allocate device memory themselves: embedders whose
// device memory is fully reserved up front by a host framework (so a cudaMalloc would fail or
// fight that framework's pool), and plain C/C++ programs that link this library without
// PyTorch's caching allocator and may not call into it.  The caller passes inputs and outputs; the working
// memory (per-latent counters, cursors and scan partials) lives in a fixed-size device array
// inside this library.
//
// Contract:
//   * n_latents must be in [1, SB_NOALLOC_CSC_MAX_LATENTS]; larger sizes are rejected with
//     SB_NOALLOC_ERR_TOO_MANY_LATENTS before anything is launched.
//   * vals/idx are the [n_rows, k] outputs of the row top-k (fp32 values, int32 latent indices,
//     -1 = empty slot), flattened to n_pairs = n_rows * k.  A pair is kept when idx >= 0 and
//     vals > 0, exactly like the allocating path (`csc_count` + scan + `csc_fill`).
//   * n_pairs must be in [0, SB_NOALLOC_CSC_MAX_PAIRS] (2^31 - 1: the offsets are summed in
//     32-bit integers); larger values return SB_NOALLOC_ERR_TOO_MANY_PAIRS.
//   * A latent index >= n_latents is not a valid pair: it is skipped (nothing is written for it)
//     and counted.  When `bad_pairs` (a device int32 the caller owns, or NULL) is given, the call
//     stores the number of skipped pairs there, so the caller can check it after the stream
//     reaches this call.
//   * An error already pending on this thread when the call starts (cudaGetLastError) is taken
//     and reported as SB_NOALLOC_ERR_PENDING, and nothing is launched; each launch is checked on
//     its own, so SB_NOALLOC_ERR_LAUNCH names a failure of this call only.
//   * Calls must run in the device's primary context (the runtime API's context), since the
//     scratch address is looked up once per device ordinal.
//   * colptr receives n_latents + 1 int64 offsets; pairs receives the kept pair ids grouped by
//     latent (capacity n_pairs).  Within one latent the order of its pairs is unspecified.
//   * The first call on a device looks up the device address of the scratch array for that
//     device (cudaGetSymbolAddress with that device current).  Make that first call before any
//     stream capture begins.
//   * Every call on a device shares the one scratch array, and the scratch keeps the previous
//     call's contents (each call clears what must start at zero).  Calls whose execution
//     overlaps on the GPU race on the scratch: serialise them (one stream, or events).
//   * No cudaMalloc, cudaFree or allocating library routine is called.
#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

#define SB_NOALLOC_CSC_MAX_LATENTS (1 << 20)

#define SB_NOALLOC_OK 0
#define SB_NOALLOC_ERR_TOO_MANY_LATENTS 1
#define SB_NOALLOC_ERR_BAD_ARGUMENT 2
#define SB_NOALLOC_ERR_SYMBOL_ADDRESS 3
#define SB_NOALLOC_ERR_LAUNCH 4
#define SB_NOALLOC_ERR_TOO_MANY_PAIRS 5
#define SB_NOALLOC_ERR_PENDING 6

#define SB_NOALLOC_CSC_MAX_PAIRS 2147483647LL

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int sb_csc_build_noalloc(const float* vals, const int32_t* idx,
                                                                  int64_t n_pairs, int32_t n_latents,
                                                                  int64_t* colptr, int64_t* pairs,
                                                                  int32_t* bad_pairs, cudaStream_t stream);

__attribute__((visibility("default"))) const char* sb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif

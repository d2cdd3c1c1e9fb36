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

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int sb_csc_build_noalloc(const float* vals, const int32_t* idx,
                                                                  int64_t n_pairs, int32_t n_latents,
                                                                  int64_t* colptr, int64_t* pairs,
                                                                  cudaStream_t stream);

__attribute__((visibility("default"))) const char* sb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif

// Symmetric slab allocation for peer-memory kernels: one cudaMalloc per rank, exported with a
// CUDA IPC handle that the other ranks of the node open once.  The Python side
// (saelens_b200/parallel/symm_heap.py) exchanges the 64-byte handles over the process group
// and places buffers at identical offsets inside every rank's slab.
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include "check.h"

namespace sb {

// Allocates `nbytes` of zeroed device memory on the current device.  Returns (address, handle)
// where handle is a CPU uint8 tensor holding the cudaIpcMemHandle_t.
std::tuple<int64_t, torch::Tensor> symm_alloc(int64_t nbytes) {
  SB_CHECK(nbytes > 0, "symm_alloc: size must be positive");
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, size_t(nbytes)));
  C10_CUDA_CHECK(cudaMemset(p, 0, size_t(nbytes)));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto t = torch::empty({int64_t(sizeof(h))}, torch::dtype(torch::kUInt8));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), t};
}

// Page-locks [ptr, ptr + bytes) of host memory (for example a shared-memory activation ring mapped
// by several processes) for the copy engines of every device (cudaHostRegisterPortable).  Returns
// the cudaError_t code; a refusal (a mapping the driver cannot pin) leaves no error pending for the
// next CUDA call.
int64_t host_register(int64_t ptr, int64_t bytes) {
  const cudaError_t e = cudaHostRegister(reinterpret_cast<void*>(ptr), size_t(bytes), cudaHostRegisterPortable);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return int64_t(e);
}

int64_t host_unregister(int64_t ptr) {
  const cudaError_t e = cudaHostUnregister(reinterpret_cast<void*>(ptr));
  if (e != cudaSuccess) (void)cudaGetLastError();
  return int64_t(e);
}

// Maps a peer's slab into this process (peer access is enabled lazily by the driver).
int64_t symm_open(const torch::Tensor& handle) {
  SB_CHECK(handle.numel() == int64_t(sizeof(cudaIpcMemHandle_t)) && handle.scalar_type() == torch::kUInt8,
              "symm_open: expected a 64-byte uint8 handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t addr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(addr))); }

void symm_free(int64_t addr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(addr))); }

// A tensor view of device memory at `addr` (no ownership; the slab outlives its views).
torch::Tensor tensor_at(int64_t addr, std::vector<int64_t> sizes, torch::ScalarType dtype, int64_t device) {
  return torch::from_blob(reinterpret_cast<void*>(addr), sizes,
                          torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device));
}

}  // namespace sb

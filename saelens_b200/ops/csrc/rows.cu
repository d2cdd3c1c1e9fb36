// Row gather from two sources with a permutation: the shuffle step of the activation mixing
// buffer (sae_lens/training/mixing_buffer.py:35-96 concatenates the held rows with the new batch
// and then indexes the result with a random permutation; here both happen in one pass).
//
//   out[i] = perm[i] < n_a ? a[perm[i]] : b[perm[i] - n_a]        (perm absent: perm[i] = i)
//
// Rows are moved as raw bytes, one warp per output row, with the widest vector (16, 8 or 4
// bytes) that the row size and the three base addresses and strides allow.  An index outside
// [0, n_a + n_b) leaves its output row untouched and is counted in `bad` (the host reads it
// when it wants to know; nothing traps).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "check.h"

namespace sb {
namespace rows {

constexpr int WARPS = 8;

template <typename V>
__global__ void __launch_bounds__(32 * WARPS)
    gather_kernel(const char* __restrict__ a, int64_t lda, int64_t n_a, const char* __restrict__ b, int64_t ldb,
                  int64_t n_b, const int64_t* __restrict__ perm, int64_t n_out, char* __restrict__ out, int64_t ldo,
                  int64_t row_vecs, int* __restrict__ bad) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = int64_t(gridDim.x) * WARPS;
  for (int64_t i = int64_t(blockIdx.x) * WARPS + (threadIdx.x >> 5); i < n_out; i += nw) {
    const int64_t s = perm ? __ldg(perm + i) : i;
    if (s < 0 || s >= n_a + n_b) {
      if (lane == 0 && bad) atomicAdd(bad, 1);
      continue;
    }
    const V* src = reinterpret_cast<const V*>(s < n_a ? a + s * lda : b + (s - n_a) * ldb);
    V* dst = reinterpret_cast<V*>(out + i * ldo);
    constexpr int U = 4;
    int64_t v = lane;
    for (; v + 32 * (U - 1) < row_vecs; v += 32 * U) {
      V t[U];
#pragma unroll
      for (int u = 0; u < U; ++u) t[u] = __ldg(src + v + 32 * u);
#pragma unroll
      for (int u = 0; u < U; ++u) dst[v + 32 * u] = t[u];
    }
    for (; v < row_vecs; v += 32) dst[v] = __ldg(src + v);
  }
}

}  // namespace rows

// out [n_out, ...] = rows of cat([a, b]) picked by `perm` (int64 [n_out]; absent: the first n_out
// rows).  a, b and out: same dtype and row shape, rows contiguous within themselves (dim 0 may be
// strided).  `bad` (int32 [1], optional) counts indices outside the two sources.
void gather_rows(const torch::Tensor& a, const c10::optional<torch::Tensor>& b, const c10::optional<torch::Tensor>& perm,
                 const torch::Tensor& out, const c10::optional<torch::Tensor>& bad) {
  SB_CHECK(a.is_cuda() && out.is_cuda() && a.dim() >= 1 && out.dim() == a.dim(), "gather_rows: CUDA tensors");
  SB_CHECK(a.scalar_type() == out.scalar_type(), "gather_rows: a and out must have the same dtype");
  const int64_t row_elems = a.dim() == 1 ? 1 : a.numel() / std::max<int64_t>(a.size(0), 1);
  auto rows_ok = [&](const torch::Tensor& t) {
    if (t.dim() == 1) return true;
    int64_t expect = 1;
    for (int64_t d = t.dim() - 1; d >= 1; --d) {
      if (t.size(d) != 1 && t.stride(d) != expect) return false;
      expect *= t.size(d);
    }
    return true;
  };
  for (int64_t d = 1; d < a.dim(); ++d) SB_CHECK(out.size(d) == a.size(d), "gather_rows: row shapes differ");
  SB_CHECK(rows_ok(a) && rows_ok(out), "gather_rows: rows must be contiguous");
  const int64_t es = a.element_size();
  const int64_t row_bytes = row_elems * es;
  const int64_t n_a = a.size(0);
  int64_t n_b = 0;
  const char* pb = nullptr;
  int64_t ldb = 0;
  if (b) {
    SB_CHECK(b->is_cuda() && b->scalar_type() == a.scalar_type() && b->dim() == a.dim() && rows_ok(*b),
             "gather_rows: b must match a");
    for (int64_t d = 1; d < a.dim(); ++d) SB_CHECK(b->size(d) == a.size(d), "gather_rows: row shapes differ");
    n_b = b->size(0);
    pb = static_cast<const char*>(b->data_ptr());
    ldb = (b->dim() == 1 ? 1 : b->stride(0)) * es;
  }
  const int64_t n_out = out.size(0);
  const int64_t* pp = nullptr;
  if (perm) {
    SB_CHECK(perm->is_cuda() && perm->scalar_type() == at::kLong && perm->is_contiguous() && perm->numel() == n_out,
             "gather_rows: perm must be int64 [n_out] on the device");
    pp = perm->data_ptr<int64_t>();
  } else {
    SB_CHECK(n_out <= n_a + n_b, "gather_rows: out has more rows than the sources");
  }
  int* pbad = nullptr;
  if (bad) {
    SB_CHECK(bad->is_cuda() && bad->scalar_type() == at::kInt && bad->numel() >= 1, "gather_rows: bad int32 [1]");
    pbad = bad->data_ptr<int>();
  }
  if (n_out == 0 || row_bytes == 0) return;
  const char* pa = static_cast<const char*>(a.data_ptr());
  char* po = static_cast<char*>(out.data_ptr());
  const int64_t lda = (a.dim() == 1 ? 1 : a.stride(0)) * es;
  const int64_t ldo = (out.dim() == 1 ? 1 : out.stride(0)) * es;
  auto aligned = [&](int64_t w) {
    auto ok = [w](const void* p) { return reinterpret_cast<uintptr_t>(p) % w == 0; };
    return row_bytes % w == 0 && lda % w == 0 && ldo % w == 0 && ok(pa) && ok(po) &&
           (pb == nullptr || (ok(pb) && ldb % w == 0));
  };
  const at::cuda::CUDAGuard guard(a.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  int sms = 0, dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t blocks = std::min<int64_t>((n_out + rows::WARPS - 1) / rows::WARPS, int64_t(sms) * 16);
  const dim3 grid(unsigned(std::max<int64_t>(blocks, 1))), block(32 * rows::WARPS);
  if (aligned(16))
    rows::gather_kernel<uint4><<<grid, block, 0, stream>>>(pa, lda, n_a, pb, ldb, n_b, pp, n_out, po, ldo,
                                                           row_bytes / 16, pbad);
  else if (aligned(8))
    rows::gather_kernel<uint2><<<grid, block, 0, stream>>>(pa, lda, n_a, pb, ldb, n_b, pp, n_out, po, ldo,
                                                           row_bytes / 8, pbad);
  else if (aligned(4))
    rows::gather_kernel<uint32_t><<<grid, block, 0, stream>>>(pa, lda, n_a, pb, ldb, n_b, pp, n_out, po, ldo,
                                                              row_bytes / 4, pbad);
  else
    rows::gather_kernel<uint8_t><<<grid, block, 0, stream>>>(pa, lda, n_a, pb, ldb, n_b, pp, n_out, po, ldo,
                                                             row_bytes, pbad);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sb

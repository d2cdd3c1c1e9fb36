// Python bindings of the saelens_b200 native kernels (module `saelens_b200.ops._C`).
#include <torch/extension.h>

namespace sb {
void gemm_tn_bf16(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& bias,
                  const c10::optional<torch::Tensor>& scale, bool relu,
                  const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                  const torch::Tensor& status, int64_t max_ctas);
void row_topk(const torch::Tensor& H, const torch::Tensor& cmax, int64_t k_max,
              const c10::optional<torch::Tensor>& k_dev, const c10::optional<torch::Tensor>& mask,
              const torch::Tensor& out_val, const torch::Tensor& out_idx, const torch::Tensor& status);
void decode_mse(const torch::Tensor& vals, const torch::Tensor& idx, bool relu,
                const c10::optional<torch::Tensor>& inv_scale, const torch::Tensor& W,
                const c10::optional<torch::Tensor>& bias, const torch::Tensor& target,
                const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& resid,
                const c10::optional<torch::Tensor>& dxhat, const c10::optional<torch::Tensor>& grad_coef_dev,
                double grad_coef, const c10::optional<torch::Tensor>& loss_row,
                const c10::optional<torch::Tensor>& bsum);
void csc_count(const torch::Tensor& vals, const torch::Tensor& idx,
               const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& aux_idx,
               const torch::Tensor& counts, const c10::optional<torch::Tensor>& fire_counts);
void csc_fill(const torch::Tensor& vals, const torch::Tensor& idx,
              const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& aux_idx,
              const torch::Tensor& colptr, const torch::Tensor& cursor, const torch::Tensor& pairs);
void latent_grad(const torch::Tensor& colptr, const torch::Tensor& pairs, const torch::Tensor& vals,
                 const c10::optional<torch::Tensor>& aux_vals, const c10::optional<torch::Tensor>& inv_scale,
                 const torch::Tensor& dxhat, const c10::optional<torch::Tensor>& daux,
                 const torch::Tensor& x, const c10::optional<torch::Tensor>& b_dec,
                 const torch::Tensor& W_dec, const torch::Tensor& W_enc, const torch::Tensor& gW_dec,
                 const torch::Tensor& gW_enc, const torch::Tensor& gb_enc,
                 const c10::optional<torch::Tensor>& bterm, const c10::optional<torch::Tensor>& sumsq,
                 const c10::optional<torch::Tensor>& fire_counts,
                 const c10::optional<torch::Tensor>& act_freq,
                 const c10::optional<torch::Tensor>& since_fired);
void adam_bdec(const c10::optional<torch::Tensor>& bsum, const c10::optional<torch::Tensor>& bterm,
               const torch::Tensor& gb_dec, const c10::optional<torch::Tensor>& sumsq,
               const c10::optional<torch::Tensor>& clip_out, const torch::Tensor& p, const torch::Tensor& m,
               const torch::Tensor& v, double lr, double beta1, double beta2, double eps, int64_t step,
               double max_norm, bool update);
void adam_rows(const torch::Tensor& pd, const torch::Tensor& md, const torch::Tensor& vd,
               const torch::Tensor& pe, const torch::Tensor& me, const torch::Tensor& ve,
               const torch::Tensor& wd, const torch::Tensor& we,
               const c10::optional<torch::Tensor>& gd, const c10::optional<torch::Tensor>& ge,
               const torch::Tensor& pb, const torch::Tensor& mb, const torch::Tensor& vb,
               const c10::optional<torch::Tensor>& gb, const c10::optional<torch::Tensor>& colptr,
               const c10::optional<torch::Tensor>& clip, const c10::optional<torch::Tensor>& b_dec,
               const c10::optional<torch::Tensor>& scale, const c10::optional<torch::Tensor>& inv_scale,
               const c10::optional<torch::Tensor>& bias_eff, double lr, double beta1, double beta2,
               double eps, int64_t step, bool update);
void topk_merge(const torch::Tensor& cand_val, const torch::Tensor& cand_idx, int64_t n_local, int64_t rank,
                const c10::optional<torch::Tensor>& k_dev, const torch::Tensor& out_val,
                const torch::Tensor& out_idx);
void decode_partial(const torch::Tensor& vals, const torch::Tensor& idx, bool relu,
                    const c10::optional<torch::Tensor>& inv_scale, const torch::Tensor& W, const torch::Tensor& out);
void finish_mse(const torch::Tensor& xsum, const c10::optional<torch::Tensor>& bias, const torch::Tensor& target,
                const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& resid,
                const c10::optional<torch::Tensor>& dxhat, const c10::optional<torch::Tensor>& grad_coef_dev,
                double grad_coef, const torch::Tensor& loss_row, const c10::optional<torch::Tensor>& bsum);
}  // namespace sb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "saelens_b200 sm_100a kernels";
  m.def("gemm_tn_bf16", &sb::gemm_tn_bf16);
  m.def("row_topk", &sb::row_topk);
  m.def("decode_mse", &sb::decode_mse);
  m.def("csc_count", &sb::csc_count);
  m.def("csc_fill", &sb::csc_fill);
  m.def("latent_grad", &sb::latent_grad);
  m.def("adam_bdec", &sb::adam_bdec);
  m.def("adam_rows", &sb::adam_rows);
  m.def("topk_merge", &sb::topk_merge);
  m.def("decode_partial", &sb::decode_partial);
  m.def("finish_mse", &sb::finish_mse);
}

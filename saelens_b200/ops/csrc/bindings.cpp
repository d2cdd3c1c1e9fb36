// Python bindings of the saelens_b200 native kernels (module `saelens_b200.ops._C`).
#include <torch/extension.h>

// SB_DEBUG_BOUNDS=1 builds the debug-bounds module: only the index-dereferencing kernels, checked
#ifndef SB_DEBUG_BOUNDS
#define SB_DEBUG_BOUNDS 0
#endif

#include <tuple>
#include <vector>

namespace sb {
void gemm_tn_bf16(const torch::Tensor& A, const torch::Tensor& B, const c10::optional<torch::Tensor>& bias,
                  const c10::optional<torch::Tensor>& scale, bool relu,
                  const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                  const torch::Tensor& status, int64_t max_ctas, const c10::optional<torch::Tensor>& tmax,
                  const c10::optional<torch::Tensor>& amax);
void row_topk(const torch::Tensor& H, const torch::Tensor& cmax, int64_t k_max,
              const c10::optional<torch::Tensor>& k_dev, const c10::optional<torch::Tensor>& mask,
              const torch::Tensor& out_val, const torch::Tensor& out_idx, const torch::Tensor& status,
              const c10::optional<torch::Tensor>& tmax);
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
                 const c10::optional<torch::Tensor>& since_fired, const torch::Tensor& idx,
                 const c10::optional<torch::Tensor>& aux_idx, int64_t j0, int64_t j1, bool zero_empty,
                 const c10::optional<torch::Tensor>& jr_thr, const c10::optional<torch::Tensor>& jr_pre,
                 double jr_bandwidth, double jr_l0c, const c10::optional<torch::Tensor>& jr_gthr,
                 const std::vector<int64_t>& rs_bases, int64_t rs_rank, int64_t rs_dec_off, int64_t rs_enc_off,
                 int64_t rs_n);
void threshold_select(const torch::Tensor& H, const torch::Tensor& cmax, const torch::Tensor& lo,
                      const torch::Tensor& lo_cmin, const torch::Tensor& out_val, const torch::Tensor& out_idx,
                      const torch::Tensor& counts, const c10::optional<torch::Tensor>& truncated);
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
void gemm_ag_tn_bf16(const torch::Tensor& x_own, const std::vector<int64_t>& peer_bases, int64_t rank,
                     int64_t x_off, int64_t flag_off, int64_t total_rows, int64_t m_base, int64_t M,
                     bool push, int64_t epoch, const torch::Tensor& B, const c10::optional<torch::Tensor>& bias,
                     const c10::optional<torch::Tensor>& scale, bool relu, const c10::optional<torch::Tensor>& out,
                     const c10::optional<torch::Tensor>& cmax, const torch::Tensor& status,
                     const torch::Tensor& ticket, int64_t max_ctas, const c10::optional<torch::Tensor>& tmax);
void gemm_fsdp_tn_bf16(const torch::Tensor& A, const torch::Tensor& w_own, const std::vector<int64_t>& peer_bases,
                       int64_t rank, int64_t w_off, int64_t flag_off, bool push, int64_t epoch,
                       const c10::optional<torch::Tensor>& w2_own, int64_t w2_off, int64_t flag2_off,
                       const c10::optional<torch::Tensor>& bias, const c10::optional<torch::Tensor>& scale, bool relu,
                       const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& cmax,
                       const torch::Tensor& status, const torch::Tensor& ticket, int64_t max_ctas,
                       const c10::optional<torch::Tensor>& tmax);
void decode_rs(const torch::Tensor& vals, const torch::Tensor& idx, bool relu,
               const c10::optional<torch::Tensor>& inv_scale, const torch::Tensor& W,
               const std::vector<int64_t>& peer_bases, int64_t rank, int64_t land_off, int64_t lcnt_off,
               int64_t dx_off, int64_t dcnt_off, int64_t epoch, const c10::optional<torch::Tensor>& bias,
               const torch::Tensor& target, const c10::optional<torch::Tensor>& out,
               const c10::optional<torch::Tensor>& resid, const c10::optional<torch::Tensor>& grad_coef_dev,
               double grad_coef, const torch::Tensor& loss_row, const c10::optional<torch::Tensor>& bsum,
               const torch::Tensor& ticket, const torch::Tensor& status);
void topk_exchange_merge(const torch::Tensor& vals, const torch::Tensor& idx, int64_t n_local,
                         const c10::optional<torch::Tensor>& k_dev, const std::vector<int64_t>& peer_bases,
                         int64_t rank, int64_t cv_off, int64_t ci_off, int64_t cnt_off, int64_t epoch,
                         const torch::Tensor& ticket, const torch::Tensor& status);
std::vector<int64_t> p2p_allreduce_sizes(int64_t n, int64_t elem_bytes, int64_t world, int64_t chunk);
void p2p_allreduce(const torch::Tensor& x, double scale, const std::vector<int64_t>& peer_bases, int64_t rank,
                   int64_t land_off, int64_t cnt_off, int64_t out_off, int64_t flag_off, int64_t epoch,
                   const torch::Tensor& ticket, const torch::Tensor& status, int64_t sq_off, int64_t chunk,
                   int64_t max_ctas, const c10::optional<torch::Tensor>& x_out);
void p2p_slot_reduce(const torch::Tensor& land, double scale, const torch::Tensor& out,
                     const c10::optional<torch::Tensor>& sumsq);
void ring_claim(const std::vector<int64_t>& peer_bases, int64_t rank, int64_t owner, int64_t state_off,
                int64_t n_slots, int64_t from, int64_t to, int64_t start, double timeout_ms, const torch::Tensor& slot);
void ring_write(const torch::Tensor& src, const std::vector<int64_t>& peer_bases, int64_t rank, int64_t owner,
                int64_t data_off, int64_t chunk_rows, const torch::Tensor& slot, int64_t mode, double scale);
void ring_publish(const std::vector<int64_t>& peer_bases, int64_t rank, int64_t owner, int64_t state_off,
                  int64_t meta_off, const torch::Tensor& slot, int64_t rows, int64_t producer, int64_t seq,
                  int64_t value);
void ring_gather(const torch::Tensor& data, const torch::Tensor& slot, const c10::optional<torch::Tensor>& perm,
                 const torch::Tensor& out);
void p2p_wait_flags(const torch::Tensor& flags, int64_t target, const torch::Tensor& status);
std::tuple<int64_t, torch::Tensor> symm_alloc(int64_t nbytes);
int64_t symm_open(const torch::Tensor& handle);
int64_t host_register(int64_t ptr, int64_t bytes);
int64_t host_unregister(int64_t ptr);
void symm_close(int64_t addr);
void symm_free(int64_t addr);
torch::Tensor tensor_at(int64_t addr, std::vector<int64_t> sizes, torch::ScalarType dtype, int64_t device);
void p2p_route_rows(const torch::Tensor& src, const torch::Tensor& routes, const std::vector<int64_t>& peer_bases,
                    int64_t rank, int64_t land_off, int64_t rows_cap, int64_t slot, int64_t cnt_off,
                    int64_t cnt_slot, int64_t free_off, const std::vector<int64_t>& free_slots, int64_t mode,
                    double scale, int64_t epoch, const torch::Tensor& status);
void p2p_wait_targets(const torch::Tensor& counters, const torch::Tensor& targets, const torch::Tensor& status);
void p2p_signal(const std::vector<int64_t>& peer_bases, int64_t rank, int64_t off, int64_t index,
                int64_t rank_mask, int64_t value);
torch::Tensor rmsnorm(const torch::Tensor& x, const torch::Tensor& w, double eps, bool one_plus);
void rope_(const torch::Tensor& x, const torch::Tensor& cos, const torch::Tensor& sin, int64_t pos0);
torch::Tensor gated_act(const torch::Tensor& gate, const torch::Tensor& up, int64_t kind);
torch::Tensor layernorm(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& b,
                        double eps);
torch::Tensor embed(const torch::Tensor& tokens, const torch::Tensor& table, double scale,
                    const c10::optional<torch::Tensor>& pos, const torch::Tensor& bad);
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
                     const c10::optional<torch::Tensor>& addend, const c10::optional<torch::Tensor>& oscale);
void gemm_fsdp_dense_bf16(const torch::Tensor& A, const torch::Tensor& w_own, const std::vector<int64_t>& peer_bases,
                          int64_t rank, int64_t w_off, int64_t flag_off, bool push, int64_t epoch,
                          const c10::optional<torch::Tensor>& w2_own, int64_t w2_off, int64_t flag2_off,
                          const torch::Tensor& out, const c10::optional<torch::Tensor>& out2,
                          const c10::optional<torch::Tensor>& bias, const c10::optional<torch::Tensor>& thr,
                          const c10::optional<torch::Tensor>& colcnt, const c10::optional<torch::Tensor>& nnz,
                          const torch::Tensor& status, const torch::Tensor& ticket);
void gather_rows(const torch::Tensor& a, const c10::optional<torch::Tensor>& b, const c10::optional<torch::Tensor>& perm,
                 const torch::Tensor& out, const c10::optional<torch::Tensor>& bad);
void mp_step(const torch::Tensor& resid, const torch::Tensor& resid_bf, const torch::Tensor& key,
             const torch::Tensor& acts, const torch::Tensor& done, const c10::optional<torch::Tensor>& idx_out,
             const c10::optional<torch::Tensor>& val_out, const torch::Tensor& n_active, const torch::Tensor& W,
             double thresh, bool stop_dup, const c10::optional<torch::Tensor>& rows);
void mp_backward(const torch::Tensor& resid, const torch::Tensor& g_resid, const torch::Tensor& g_acts,
                 const torch::Tensor& idx, const torch::Tensor& val, const c10::optional<torch::Tensor>& g_W,
                 const torch::Tensor& W);
void attention_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& out,
                   double scale, double softcap, bool causal, const torch::Tensor& status);
torch::Tensor batch_topk_select(const torch::Tensor& vals, const torch::Tensor& idx, int64_t K,
                                const c10::optional<torch::Tensor>& truncated);
void batch_hist(const torch::Tensor& vals, const torch::Tensor& idx, const torch::Tensor& hist);
void batch_thresh(const torch::Tensor& hist, int64_t K, const torch::Tensor& sel);
void batch_ties(const torch::Tensor& vals, const torch::Tensor& idx, const torch::Tensor& sel,
                const torch::Tensor& ties);
void batch_filter(const torch::Tensor& vals, const torch::Tensor& idx, const torch::Tensor& sel,
                  const torch::Tensor& ties_all, int64_t rank, const torch::Tensor& prefix,
                  const c10::optional<torch::Tensor>& truncated);
#if SB_DEBUG_BOUNDS
std::vector<int64_t> sparse_bounds_info(bool reset);
std::vector<int64_t> topk_bounds_info(bool reset);
std::vector<int64_t> p2p_bounds_info(bool reset);
#endif
}  // namespace sb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "saelens_b200 sm_100a kernels";
  // kernels that dereference data-dependent indices (also built into the debug-bounds module)
  m.def("row_topk", &sb::row_topk, py::arg("H"), py::arg("cmax"), py::arg("k_max"), py::arg("k_dev"),
        py::arg("mask"), py::arg("out_val"), py::arg("out_idx"), py::arg("status"), py::arg("tmax") = py::none());
  m.def("decode_mse", &sb::decode_mse);
  m.def("csc_count", &sb::csc_count);
  m.def("csc_fill", &sb::csc_fill);
  m.def("latent_grad", &sb::latent_grad, py::arg("colptr"), py::arg("pairs"), py::arg("vals"), py::arg("aux_vals"),
        py::arg("inv_scale"), py::arg("dxhat"), py::arg("daux"), py::arg("x"), py::arg("b_dec"), py::arg("W_dec"),
        py::arg("W_enc"), py::arg("gW_dec"), py::arg("gW_enc"), py::arg("gb_enc"), py::arg("bterm"),
        py::arg("sumsq"), py::arg("fire_counts"), py::arg("act_freq"), py::arg("since_fired"), py::arg("idx"),
        py::arg("aux_idx"), py::arg("j0") = 0, py::arg("j1") = -1, py::arg("zero_empty") = false,
        py::arg("jr_thr") = py::none(), py::arg("jr_pre") = py::none(), py::arg("jr_bandwidth") = 0.0,
        py::arg("jr_l0c") = 0.0, py::arg("jr_gthr") = py::none(), py::arg("rs_bases") = std::vector<int64_t>{},
        py::arg("rs_rank") = 0, py::arg("rs_dec_off") = 0, py::arg("rs_enc_off") = 0, py::arg("rs_n") = 0);
  m.def("threshold_select", &sb::threshold_select);
  m.def("topk_merge", &sb::topk_merge);
  m.def("decode_partial", &sb::decode_partial);
  m.def("finish_mse", &sb::finish_mse);
  m.def("decode_rs", &sb::decode_rs);
  m.def("topk_exchange_merge", &sb::topk_exchange_merge);
  m.def("p2p_allreduce_sizes", &sb::p2p_allreduce_sizes, py::arg("n"), py::arg("elem_bytes"), py::arg("world"),
        py::arg("chunk") = 0);
  m.def("p2p_allreduce", &sb::p2p_allreduce, py::arg("x"), py::arg("scale"), py::arg("peer_bases"),
        py::arg("rank"), py::arg("land_off"), py::arg("cnt_off"), py::arg("out_off"), py::arg("flag_off"),
        py::arg("epoch"), py::arg("ticket"), py::arg("status"), py::arg("sq_off") = -1, py::arg("chunk") = 0, py::arg("max_ctas") = 0, py::arg("x_out") = py::none());
  m.def("p2p_wait_flags", &sb::p2p_wait_flags);
  m.def("p2p_slot_reduce", &sb::p2p_slot_reduce);
  m.def("ring_claim", &sb::ring_claim);
  m.def("ring_write", &sb::ring_write);
  m.def("ring_publish", &sb::ring_publish);
  m.def("ring_gather", &sb::ring_gather);
  m.def("p2p_route_rows", &sb::p2p_route_rows);
  m.def("p2p_wait_targets", &sb::p2p_wait_targets);
  m.def("p2p_signal", &sb::p2p_signal);
  m.def("batch_topk_select", &sb::batch_topk_select);
  m.def("batch_hist", &sb::batch_hist);
  m.def("batch_thresh", &sb::batch_thresh);
  m.def("batch_ties", &sb::batch_ties);
  m.def("batch_filter", &sb::batch_filter);
#if SB_DEBUG_BOUNDS
  m.attr("debug_bounds") = true;
  m.def("sparse_bounds_info", &sb::sparse_bounds_info, py::arg("reset") = true);
  m.def("topk_bounds_info", &sb::topk_bounds_info, py::arg("reset") = true);
  m.def("p2p_bounds_info", &sb::p2p_bounds_info, py::arg("reset") = true);
#else
  m.attr("debug_bounds") = false;
  m.def("gemm_tn_bf16", &sb::gemm_tn_bf16, py::arg("A"), py::arg("B"), py::arg("bias"), py::arg("scale"),
        py::arg("relu"), py::arg("out"), py::arg("cmax"), py::arg("status"), py::arg("max_ctas"),
        py::arg("tmax") = py::none(), py::arg("amax") = py::none());
  m.def("adam_bdec", &sb::adam_bdec);
  m.def("adam_rows", &sb::adam_rows);
  m.def("gemm_ag_tn_bf16", &sb::gemm_ag_tn_bf16, py::arg("x_own"), py::arg("peer_bases"), py::arg("rank"),
        py::arg("x_off"), py::arg("flag_off"), py::arg("total_rows"), py::arg("m_base"), py::arg("M"), py::arg("push"),
        py::arg("epoch"), py::arg("B"), py::arg("bias"), py::arg("scale"), py::arg("relu"), py::arg("out"),
        py::arg("cmax"), py::arg("status"), py::arg("ticket"), py::arg("max_ctas"), py::arg("tmax") = py::none());
  m.def("gemm_fsdp_tn_bf16", &sb::gemm_fsdp_tn_bf16, py::arg("A"), py::arg("w_own"), py::arg("peer_bases"),
        py::arg("rank"), py::arg("w_off"), py::arg("flag_off"), py::arg("push"), py::arg("epoch"), py::arg("w2_own"),
        py::arg("w2_off"), py::arg("flag2_off"), py::arg("bias"), py::arg("scale"), py::arg("relu"), py::arg("out"),
        py::arg("cmax"), py::arg("status"), py::arg("ticket"), py::arg("max_ctas") = 0, py::arg("tmax") = py::none());
  m.def("rmsnorm", &sb::rmsnorm);
  m.def("rope_", &sb::rope_);
  m.def("gated_act", &sb::gated_act);
  m.def("layernorm", &sb::layernorm);
  m.def("embed", &sb::embed);
  m.def("gemm_dense_bf16", &sb::gemm_dense_bf16, py::arg("A"), py::arg("a_mn"), py::arg("B"), py::arg("b_mn"),
        py::arg("out") = py::none(), py::arg("out2") = py::none(), py::arg("bias") = py::none(),
        py::arg("r1_row") = py::none(), py::arg("r1_col") = py::none(), py::arg("thr") = py::none(),
        py::arg("relu") = false, py::arg("hin") = py::none(), py::arg("bandwidth") = 0.0, py::arg("l0c") = 0.0,
        py::arg("gthr") = py::none(), py::arg("target") = py::none(), py::arg("res_coef") = 1.0,
        py::arg("loss") = py::none(), py::arg("colsum") = py::none(), py::arg("colcnt") = py::none(),
        py::arg("nnz") = py::none(), py::arg("sumsq") = py::none(), py::arg("gate_bias") = py::none(),
        py::arg("mag_scale") = py::none(), py::arg("status"), py::arg("max_ctas") = 0,
        py::arg("rs_bases") = std::vector<int64_t>{}, py::arg("rs_rank") = 0, py::arg("rs_off") = 0,
        py::arg("rs_n") = 0, py::arg("hsum") = py::none(), py::arg("hoff") = py::none(),
        py::arg("colsum2") = py::none(), py::arg("addend") = py::none(), py::arg("oscale") = py::none());
  m.def("gemm_fsdp_dense_bf16", &sb::gemm_fsdp_dense_bf16);
  m.def("gather_rows", &sb::gather_rows, py::arg("a"), py::arg("b"), py::arg("perm"), py::arg("out"),
        py::arg("bad") = py::none());
  m.def("mp_step", &sb::mp_step, py::arg("resid"), py::arg("resid_bf"), py::arg("key"), py::arg("acts"),
        py::arg("done"), py::arg("idx_out"), py::arg("val_out"), py::arg("n_active"), py::arg("W"), py::arg("thresh"),
        py::arg("stop_dup"), py::arg("rows") = py::none());
  m.def("mp_backward", &sb::mp_backward, py::arg("resid"), py::arg("g_resid"), py::arg("g_acts"), py::arg("idx"),
        py::arg("val"), py::arg("g_W"), py::arg("W"));
  m.def("attention_fwd", &sb::attention_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"),
        py::arg("scale"), py::arg("softcap"), py::arg("causal"), py::arg("status"));
  m.def("symm_alloc", &sb::symm_alloc);
  m.def("symm_open", &sb::symm_open);
  m.def("host_register", &sb::host_register, py::arg("ptr"), py::arg("bytes"));
  m.def("host_unregister", &sb::host_unregister, py::arg("ptr"));
  m.def("symm_close", &sb::symm_close);
  m.def("symm_free", &sb::symm_free);
  m.def("tensor_at", &sb::tensor_at);
#endif
}

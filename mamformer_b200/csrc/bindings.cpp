// Python bindings of the native sm_100a kernels (module mamformer_b200._C).
#include <torch/extension.h>

#include <vector>

namespace mamf {
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps);
std::vector<at::Tensor> rmsnorm_bwd(at::Tensor x, at::Tensor w, at::Tensor dy, at::Tensor rstd);
at::Tensor swiglu_fwd(at::Tensor g, at::Tensor u);
std::vector<at::Tensor> swiglu_bwd(at::Tensor g, at::Tensor u, at::Tensor dy);
at::Tensor rope_apply(at::Tensor x, at::Tensor cos, at::Tensor sin, bool inverse);
at::Tensor conv_silu_fwd(at::Tensor x, at::Tensor w);
std::vector<at::Tensor> conv_silu_bwd(at::Tensor x, at::Tensor w, at::Tensor dy);
std::vector<at::Tensor> head_groupnorm_fwd(at::Tensor x, int64_t H, at::Tensor w, at::Tensor b, double eps);
std::vector<at::Tensor> head_groupnorm_bwd(at::Tensor x, int64_t H, at::Tensor w, at::Tensor mr, at::Tensor dy);
std::vector<at::Tensor> selective_scan_fwd(at::Tensor x, at::Tensor dt, at::Tensor A_log, at::Tensor Bm,
                                           at::Tensor Cm, at::Tensor D, c10::optional<at::Tensor> z,
                                           c10::optional<at::Tensor> h0, bool softplus, bool need_hs,
                                           bool need_final);
std::vector<at::Tensor> selective_scan_bwd(at::Tensor x, at::Tensor dt, at::Tensor A_log, at::Tensor Bm,
                                           at::Tensor Cm, at::Tensor D, c10::optional<at::Tensor> z,
                                           at::Tensor ckpt, at::Tensor dy, c10::optional<at::Tensor> dhs,
                                           bool softplus);
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> out16,
                double lr, double b1, double b2, double eps, double wd, int64_t step,
                c10::optional<at::Tensor> gscale);
void sq_norm_accumulate(at::Tensor g, at::Tensor out);
void clip_scale(at::Tensor sq, at::Tensor scale, double max_norm, double inv_world, at::Tensor norm_out);
void grad_accumulate(at::Tensor dst, at::Tensor src);
void embedding_grad_accumulate(at::Tensor mg, at::Tensor ids, at::Tensor dy);
void gemm_tn(at::Tensor A, bool a_mn, at::Tensor B, bool b_mn, at::Tensor D, bool accumulate,
             c10::optional<at::Tensor> seg, c10::optional<at::Tensor> tile_off, int64_t mode, double alpha);
int64_t gemm_error();
void gemm_clear_error();
void ce_stats(at::Tensor logits, at::Tensor labels, int64_t ignore_index, at::Tensor loss, at::Tensor lse);
void ce_grad_inplace(at::Tensor logits, at::Tensor labels, int64_t ignore_index, at::Tensor lse,
                     at::Tensor scale, at::Tensor n_valid);
void moe_scatter_rows(at::Tensor dst, at::Tensor dst_idx, at::Tensor src, int64_t k);
void moe_combine(at::Tensor out, std::vector<int64_t> table, int64_t ld_src, int64_t src_rows,
                 at::ScalarType src_dtype, c10::optional<at::Tensor> owner, at::Tensor pos,
                 c10::optional<at::Tensor> w, int64_t k, c10::optional<at::Tensor> rows_out);
void moe_combine_bwd(at::Tensor dout, at::Tensor y, c10::optional<at::Tensor> y_idx, at::Tensor gate,
                     at::Tensor dgate, at::Tensor dy, c10::optional<at::Tensor> dy_idx, int64_t k);
void ep_pull_runs(at::Tensor dst, std::vector<int64_t> table, int64_t ld_src, at::Tensor runs, int64_t max_len);
void ep_barrier(std::vector<int64_t> signal, int64_t me, int64_t epoch, int64_t slot0);
std::vector<at::Tensor> moe_sort_plan(at::Tensor idx, int64_t E, bool padded);
int64_t plan_error();
void ep_exchange_counts(std::vector<int64_t> mats, std::vector<int64_t> signal, at::Tensor counts, int64_t me,
                        int64_t epoch, int64_t slot0);
void ep_layout(at::Tensor C, int64_t me, int64_t cap, at::Tensor plan, at::Tensor status);
void ep_positions(at::Tensor idx, at::Tensor srow, at::Tensor start, at::Tensor plan, int64_t P, int64_t cap,
                  at::Tensor pos, at::Tensor owner);
void ep_pull_rows(at::Tensor dst, std::vector<int64_t> table, int64_t ld_src, int64_t src_rows, at::Tensor plan,
                  int64_t P);
int64_t bounds_error_moe_rows();
int64_t bounds_error_ce();
bool bounds_check_built();
int64_t ep_plan_size(int64_t P, int64_t El);
void moe_zero_pad_rows(at::Tensor buf, at::Tensor seg, at::Tensor counts);
void moe_bias_update(at::Tensor counts, double n_assign, int64_t E, double speed, at::Tensor bias, at::Tensor ema);
int64_t dp_slice(int64_t lo, int64_t hi, int64_t P);
at::Tensor dp_reduce_scatter(std::vector<int64_t> bufs, int64_t me, int64_t lo, int64_t hi, double scale, bool want_sq);
void dp_all_gather(std::vector<int64_t> bufs, int64_t me, int64_t lo, int64_t hi);
at::Tensor dp_allreduce_nvls(int64_t mc_base, int64_t P, int64_t me, int64_t lo, int64_t hi, double scale, bool want_sq);
int64_t comm_error();
void comm_clear_error();
std::vector<at::Tensor> linear_attn_fwd(at::Tensor q1, at::Tensor q2, at::Tensor k, at::Tensor v, at::Tensor lam,
                                        int64_t kernel_dim);
std::vector<at::Tensor> linear_attn_bwd(at::Tensor q1, at::Tensor q2, at::Tensor k, at::Tensor v, at::Tensor lam,
                                        int64_t kernel_dim, at::Tensor Sst, at::Tensor zst, at::Tensor dout);
std::vector<at::Tensor> router_topk(at::Tensor scores, int64_t k);
at::Tensor router_topk_bwd(at::Tensor dg, at::Tensor gates, at::Tensor idx, int64_t E);
at::Tensor expert_histogram(at::Tensor idx, int64_t E);
std::vector<at::Tensor> flash_tc_fwd(at::Tensor q1, c10::optional<at::Tensor> q2, at::Tensor k, at::Tensor v,
                                     c10::optional<at::Tensor> lam, int64_t lo, int64_t hi, double scale);
int64_t flash_tc_error();
std::vector<at::Tensor> flash_tc_bwd(at::Tensor q1, c10::optional<at::Tensor> q2, at::Tensor k, at::Tensor v,
                                     at::Tensor o1, c10::optional<at::Tensor> o2, at::Tensor lse1,
                                     c10::optional<at::Tensor> lse2, at::Tensor dout, c10::optional<at::Tensor> coef,
                                     int64_t lo, int64_t hi, double scale);
int64_t flash_tc_bwd_error();
std::vector<at::Tensor> flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, int64_t lo, int64_t hi, double scale);
std::vector<at::Tensor> flash_attn_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor lse,
                                       at::Tensor dout, int64_t lo, int64_t hi, double scale);
void gemm_ag(std::vector<int64_t> a_ptrs, int64_t shard_rows, int64_t lda, int64_t rank, at::Tensor B, bool b_mn,
             at::Tensor D);
void gemm_rs(at::Tensor A, at::Tensor B, bool b_mn, std::vector<int64_t> d_ptrs, int64_t shard_rows, int64_t ldd,
             int64_t rank);
}  // namespace mamf

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mamformer_b200 native kernels for sm_100a (B200)";
  m.def("rmsnorm_fwd", &mamf::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &mamf::rmsnorm_bwd);
  m.def("swiglu_fwd", &mamf::swiglu_fwd);
  m.def("swiglu_bwd", &mamf::swiglu_bwd);
  m.def("rope_apply", &mamf::rope_apply);
  m.def("conv_silu_fwd", &mamf::conv_silu_fwd);
  m.def("conv_silu_bwd", &mamf::conv_silu_bwd);
  m.def("head_groupnorm_fwd", &mamf::head_groupnorm_fwd);
  m.def("head_groupnorm_bwd", &mamf::head_groupnorm_bwd);
  m.def("selective_scan_fwd", &mamf::selective_scan_fwd);
  m.def("selective_scan_bwd", &mamf::selective_scan_bwd);
  m.def("adamw_step", &mamf::adamw_step);
  m.def("sq_norm_accumulate", &mamf::sq_norm_accumulate);
  m.def("clip_scale", &mamf::clip_scale);
  m.def("grad_accumulate", &mamf::grad_accumulate);
  m.def("embedding_grad_accumulate", &mamf::embedding_grad_accumulate);
  m.def("gemm_tn", &mamf::gemm_tn);
  m.def("gemm_error", &mamf::gemm_error);
  m.def("gemm_clear_error", &mamf::gemm_clear_error);
  m.def("ce_stats", &mamf::ce_stats);
  m.def("ce_grad_inplace", &mamf::ce_grad_inplace);
  m.def("moe_scatter_rows", &mamf::moe_scatter_rows);
  m.def("moe_combine", &mamf::moe_combine);
  m.def("moe_combine_bwd", &mamf::moe_combine_bwd);
  m.def("ep_pull_runs", &mamf::ep_pull_runs);
  m.def("ep_barrier", &mamf::ep_barrier);
  m.def("moe_sort_plan", &mamf::moe_sort_plan);
  m.def("plan_error", &mamf::plan_error);
  m.def("ep_exchange_counts", &mamf::ep_exchange_counts);
  m.def("ep_layout", &mamf::ep_layout);
  m.def("ep_positions", &mamf::ep_positions);
  m.def("ep_pull_rows", &mamf::ep_pull_rows);
  m.def("ep_plan_size", &mamf::ep_plan_size);
  m.def("moe_zero_pad_rows", &mamf::moe_zero_pad_rows);
  m.def("bounds_error_moe_rows", &mamf::bounds_error_moe_rows);
  m.def("bounds_error_ce", &mamf::bounds_error_ce);
  m.def("bounds_check_built", &mamf::bounds_check_built);
  m.def("moe_bias_update", &mamf::moe_bias_update);
  m.def("dp_slice", &mamf::dp_slice);
  m.def("dp_reduce_scatter", &mamf::dp_reduce_scatter);
  m.def("dp_all_gather", &mamf::dp_all_gather);
  m.def("dp_allreduce_nvls", &mamf::dp_allreduce_nvls);
  m.def("comm_error", &mamf::comm_error);
  m.def("comm_clear_error", &mamf::comm_clear_error);
  m.def("linear_attn_fwd", &mamf::linear_attn_fwd);
  m.def("linear_attn_bwd", &mamf::linear_attn_bwd);
  m.def("router_topk", &mamf::router_topk);
  m.def("router_topk_bwd", &mamf::router_topk_bwd);
  m.def("expert_histogram", &mamf::expert_histogram);
  m.def("flash_tc_fwd", &mamf::flash_tc_fwd);
  m.def("flash_tc_error", &mamf::flash_tc_error);
  m.def("flash_tc_bwd", &mamf::flash_tc_bwd);
  m.def("flash_tc_bwd_error", &mamf::flash_tc_bwd_error);
  m.def("flash_attn_fwd", &mamf::flash_attn_fwd);
  m.def("flash_attn_bwd", &mamf::flash_attn_bwd);
  m.def("gemm_ag", &mamf::gemm_ag);
  m.def("gemm_rs", &mamf::gemm_rs);
}

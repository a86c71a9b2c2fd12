// Bounds-checked build of the index-driven kernels (module mamformer_b200._C_check): the row
// movement of the routed experts and the cross-entropy rows, compiled with MAMF_BOUNDS_CHECK so
// every guarded index is tested against its buffer and a bad one is recorded in an error word
// and skipped instead of being accessed.  The main module _C is built without the checks (unless
// MAMF_BOUNDS_CHECK=1 is set for the whole build); this one exists so the guards are compiled
// and tested in every build.
#include <torch/extension.h>

#include <vector>

namespace mamf {
void moe_scatter_rows(at::Tensor dst, at::Tensor dst_idx, at::Tensor src, int64_t k);
void moe_combine(at::Tensor out, std::vector<int64_t> table, int64_t ld_src, int64_t src_rows,
                 at::ScalarType src_dtype, c10::optional<at::Tensor> owner, at::Tensor pos,
                 c10::optional<at::Tensor> w, int64_t k, c10::optional<at::Tensor> rows_out);
void moe_combine_bwd(at::Tensor dout, at::Tensor y, c10::optional<at::Tensor> y_idx, at::Tensor gate,
                     at::Tensor dgate, at::Tensor dy, c10::optional<at::Tensor> dy_idx, int64_t k);
void ep_pull_rows(at::Tensor dst, std::vector<int64_t> table, int64_t ld_src, int64_t src_rows, at::Tensor plan,
                  int64_t P);
void ep_layout(at::Tensor C, int64_t me, int64_t cap, at::Tensor plan, at::Tensor status);
int64_t ep_plan_size(int64_t P, int64_t El);
void ce_stats(at::Tensor logits, at::Tensor labels, int64_t ignore_index, at::Tensor loss, at::Tensor lse);
int64_t bounds_error_moe_rows();
int64_t bounds_error_ce();
bool bounds_check_built();
}  // namespace mamf

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "bounds-checked build of the mamformer_b200 row-movement and cross-entropy kernels";
  m.def("moe_scatter_rows", &mamf::moe_scatter_rows);
  m.def("moe_combine", &mamf::moe_combine);
  m.def("moe_combine_bwd", &mamf::moe_combine_bwd);
  m.def("ep_pull_rows", &mamf::ep_pull_rows);
  m.def("ep_layout", &mamf::ep_layout);
  m.def("ep_plan_size", &mamf::ep_plan_size);
  m.def("ce_stats", &mamf::ce_stats);
  m.def("bounds_error_moe_rows", &mamf::bounds_error_moe_rows);
  m.def("bounds_error_ce", &mamf::bounds_error_ce);
  m.def("bounds_check_built", &mamf::bounds_check_built);
}

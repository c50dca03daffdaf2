// Bindings of the elementwise / routing / attention / GDN / sampling kernels.
#include "binding_utils.h"
#include "kernels.h"

using namespace afb_bind;

namespace {

void rmsnorm_op(const at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w, at::Tensor& y,
                double eps, bool zero_centered) {
  AFB_CHECK_CUDA(x);
  AFB_CHECK_DT(x, at::kBFloat16);
  AFB_CHECK_CONTIG(x);
  AFB_CHECK_CONTIG(y);
  const int H = x.size(-1), rows = x.numel() / H;
  check_rc(afb::rmsnorm(x.data_ptr(), optr<void>(residual), w.data_ptr(), y.data_ptr(), rows, H, (float)eps,
                        zero_centered, stream()),
           "rmsnorm");
}

void qk_norm_rope_store_op(const at::Tensor& qkv, int64_t Hq, int64_t Hkv, int64_t D, int64_t rot,
                           const at::Tensor& qw, const at::Tensor& kw, const at::Tensor& positions,
                           const at::Tensor& slots, const at::Tensor& cos_t, const at::Tensor& sin_t, double eps,
                           at::Tensor& q_out, at::Tensor& kcache, at::Tensor& vcache) {
  AFB_CHECK_DT(positions, at::kInt);
  AFB_CHECK_DT(slots, at::kInt);
  AFB_CHECK_DT(cos_t, at::kFloat);
  const int T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) == Hq * 2 * D + 2 * Hkv * D, "qkv width");
  const int page_size = kcache.size(2);
  check_rc(afb::qk_norm_rope_store(qkv.data_ptr(), T, Hq, Hkv, D, rot, qw.data_ptr(), kw.data_ptr(),
                                   ptr<int>(positions), ptr<int>(slots), ptr<float>(cos_t), ptr<float>(sin_t),
                                   (float)eps, q_out.data_ptr(), kcache.data_ptr(), vcache.data_ptr(), page_size,
                                   stream()),
           "qk_norm_rope_store");
}

void router_topk_op(const at::Tensor& logits, int64_t E, int64_t k, bool renorm, at::Tensor& ids,
                    at::Tensor& weights) {
  AFB_CHECK_DT(logits, at::kFloat);
  AFB_CHECK_DT(ids, at::kInt);
  AFB_CHECK_DT(weights, at::kFloat);
  TORCH_CHECK(logits.stride(1) == 1, "router logits need unit inner stride");
  check_rc(afb::router_topk(ptr<float>(logits), logits.stride(0), logits.size(0), E, k, renorm, ptr<int>(ids),
                            ptr<float>(weights), stream()),
           "router_topk");
}

void expert_sort_op(const at::Tensor& ids, int64_t E, c10::optional<at::Tensor> expert_map, at::Tensor& offsets,
                    at::Tensor& row_token, at::Tensor& row_entry, at::Tensor& entry_row) {
  AFB_CHECK_DT(ids, at::kInt);
  AFB_CHECK_CONTIG(ids);
  const int k = ids.size(-1);
  check_rc(afb::expert_sort(ptr<int>(ids), ids.numel(), E, optr<int>(expert_map), ptr<int>(offsets),
                            ptr<int>(row_token), ptr<int>(row_entry), ptr<int>(entry_row), k, stream()),
           "expert_sort");
}

void quant_rows_e4m3_op(const at::Tensor& x, c10::optional<at::Tensor> row_token, c10::optional<at::Tensor> nrows_dev,
                        int64_t nrows, at::Tensor& q, at::Tensor& scales) {
  AFB_CHECK_DT(x, at::kBFloat16);
  TORCH_CHECK(x.stride(-1) == 1, "x inner stride");
  check_rc(afb::quant_rows_e4m3(x.data_ptr(), x.stride(0), optr<int>(row_token), optr<int>(nrows_dev), nrows,
                                x.size(1), q.data_ptr(), ptr<float>(scales), stream()),
           "quant_rows_e4m3");
}

void moe_combine_op(const at::Tensor& y, const at::Tensor& entry_row, int64_t k, c10::optional<at::Tensor> shared,
                    c10::optional<at::Tensor> router_logits, int64_t sg_col, c10::optional<at::Tensor> resid,
                    at::Tensor& out) {
  const int T = out.size(0), H = out.size(1);
  const int ld = router_logits.has_value() ? router_logits->stride(0) : 0;
  check_rc(afb::moe_combine(y.data_ptr(), ptr<int>(entry_row), k, optr<void>(shared), optr<float>(router_logits), ld,
                            sg_col, optr<void>(resid), out.data_ptr(), T, H, stream()),
           "moe_combine");
}

void swiglu_op(const at::Tensor& x, at::Tensor& y) {
  const int T = x.size(0), I = x.size(1) / 2;
  check_rc(afb::swiglu(x.data_ptr(), y.data_ptr(), T, I, stream()), "swiglu");
}

void embedding_op(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out) {
  AFB_CHECK_DT(ids, at::kInt);
  check_rc(afb::embedding(ptr<int>(ids), table.data_ptr(), out.data_ptr(), ids.numel(), table.size(1), table.size(0),
                          status_ptr(ids.get_device()), stream()),
           "embedding");
}

}  // namespace

void register_kernel_ops(pybind11::module& m) {
  m.def("rmsnorm", &rmsnorm_op);
  m.def("qk_norm_rope_store", &qk_norm_rope_store_op);
  m.def("router_topk", &router_topk_op);
  m.def("expert_sort", &expert_sort_op);
  m.def("quant_rows_e4m3", &quant_rows_e4m3_op);
  m.def("moe_combine", &moe_combine_op);
  m.def("swiglu", &swiglu_op);
  m.def("embedding", &embedding_op);
}

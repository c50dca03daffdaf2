// Python bindings of the native library: tensor checks + launches on the current torch stream.
// Kernels are declared in the csrc headers and take raw pointers; this is the only file that includes torch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <vector>

#include "binding_utils.h"
#include "gemm.h"
#include "kernels.h"

namespace {
// One 16-word status buffer per device: bounded waits and bounds checks OR their error codes into word 0.
std::mutex g_status_mu;
std::vector<at::Tensor> g_status;
}  // namespace

namespace afb_bind {
uint32_t* status_ptr(int dev) {
  std::lock_guard<std::mutex> lk(g_status_mu);
  if ((int)g_status.size() <= dev) g_status.resize(dev + 1);
  if (!g_status[dev].defined())
    g_status[dev] = torch::zeros({16}, torch::dtype(torch::kInt32).device(torch::kCUDA, dev));
  return reinterpret_cast<uint32_t*>(g_status[dev].data_ptr<int32_t>());
}
int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}
}  // namespace afb_bind

namespace {
using namespace afb_bind;

at::Tensor status_tensor(int64_t dev) {
  status_ptr((int)dev);
  return g_status[dev];
}

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_DT(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has dtype ", (x).scalar_type(), ", expected ", dt)
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).dim() == 2 && (x).stride(1) == 1, #x " must be 2-D with unit inner stride")

// ------------------------------------------------------------------------------------------ GEMM
at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, c10::optional<at::Tensor> out,
                c10::optional<at::Tensor> residual, double alpha, bool out_fp32, int64_t bn, int64_t splits,
                c10::optional<at::Tensor> bias, int64_t act) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  CHECK_DT(a, at::kBFloat16);
  CHECK_DT(b, at::kBFloat16);
  CHECK_ROWMAJOR(a);
  CHECK_ROWMAJOR(b);
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K, "gemm: K mismatch");
  c10::cuda::CUDAGuard g(a.device());
  at::Tensor o = out.has_value() ? *out
                                 : torch::empty({M, N}, a.options().dtype(out_fp32 ? at::kFloat : at::kBFloat16));
  CHECK_ROWMAJOR(o);
  TORCH_CHECK(o.size(0) == M && o.size(1) == N, "gemm: out shape");
  TORCH_CHECK(o.scalar_type() == (out_fp32 ? at::kFloat : at::kBFloat16), "gemm: out dtype");
  afb::GemmEpilogue epi;
  epi.out = o.data_ptr();
  epi.ldo = o.stride(0);
  epi.out_fp32 = out_fp32;
  epi.alpha = (float)alpha;
  if (residual.has_value()) {
    CHECK_DT((*residual), at::kBFloat16);
    CHECK_ROWMAJOR((*residual));
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N, "gemm: residual shape");
    epi.residual = residual->data_ptr();
    epi.ldr = residual->stride(0);
  }
  if (bias.has_value()) {
    CHECK_DT((*bias), at::kBFloat16);
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == N, "gemm: bias is bf16 [N]");
    epi.bias = bias->data_ptr();
  }
  TORCH_CHECK(act >= 0 && act <= 2, "gemm: act is 0 (none), 1 (tanh-GELU) or 2 (erf-GELU)");
  epi.act = (int)act;
  afb::GemmPlan p = afb::plan_gemm(M, N, K, num_sms());
  if (bn > 0) p.bn = (int)bn;
  if (splits > 0) p.splits = (int)splits;
  at::Tensor part;
  if (p.splits > 1) {
    part = torch::empty({p.splits, M, N}, a.options().dtype(at::kFloat));
    epi.partial = part.data_ptr();
  }
  check_rc(afb::gemm_bf16_tn(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), M, N, K, epi, p.bn, p.splits,
                             status_ptr(a.get_device()), stream()),
           "gemm_bf16_tn");
  return o;
}

// Grouped GEMM over the experts of a MoE layer (modes of afb::GemmGroups). ROWS: a [R, K] rows sorted by group,
// b [E * group_rows, K], out [R, group_rows]. REDUCE: a [group_rows, R_pad], b [Kd, R_pad], out [E, group_rows, Kd],
// seg entries multiples of 64.
void gemm_grouped(const at::Tensor& a, const at::Tensor& b, const at::Tensor& seg, c10::optional<at::Tensor> tiles,
                  int64_t mode, int64_t group_rows, int64_t max_tiles, at::Tensor& out) {
  CHECK_CUDA(a);
  CHECK_DT(a, at::kBFloat16);
  CHECK_DT(b, at::kBFloat16);
  CHECK_ROWMAJOR(a);
  CHECK_ROWMAJOR(b);
  if (mode == 1) {
    CHECK_ROWMAJOR(out);
  } else {
    TORCH_CHECK(out.is_contiguous(), "gemm_grouped REDUCE: contiguous [E, group_rows, Kd] out");
  }
  TORCH_CHECK(seg.scalar_type() == at::kInt && seg.is_contiguous(), "gemm_grouped: seg int32");
  TORCH_CHECK(a.size(1) == b.size(1), "gemm_grouped: K mismatch");
  c10::cuda::CUDAGuard g(a.device());
  afb::GemmEpilogue epi;
  epi.out = out.data_ptr();
  epi.out_fp32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(epi.out_fp32 || out.scalar_type() == at::kBFloat16, "gemm_grouped: bf16 or fp32 out");
  afb::GemmGroups grp;
  grp.mode = (int)mode;
  grp.seg = seg.data_ptr<int>();
  grp.E = (int)seg.numel() - 1;
  grp.group_rows = (int)group_rows;
  int N;
  if (mode == 1) {
    TORCH_CHECK(tiles.has_value() && tiles->scalar_type() == at::kInt && tiles->numel() == seg.numel(),
                "gemm_grouped ROWS: tiles int32 [E + 1]");
    TORCH_CHECK(b.size(0) == (int64_t)grp.E * group_rows && out.size(0) == a.size(0) && out.size(1) == group_rows,
                "gemm_grouped ROWS shapes");
    grp.tiles = tiles->data_ptr<int>();
    N = (int)group_rows;
    epi.ldo = out.stride(0);
  } else {
    TORCH_CHECK(out.dim() == 3 && out.size(0) == grp.E && out.size(1) == group_rows && out.size(2) == b.size(0) &&
                    a.size(0) == group_rows,
                "gemm_grouped REDUCE shapes");
    N = (int)b.size(0);
    epi.ldo = (int)out.size(2);
    grp.group_out_stride = (int64_t)group_rows * out.size(2);
  }
  check_rc(afb::gemm_bf16_grouped(a.data_ptr(), a.stride(0), a.size(0), b.data_ptr(), b.stride(0), b.size(0), N,
                                  a.size(1), epi, grp, (int)max_tiles, status_ptr(a.get_device()), stream()),
           "gemm_grouped");
}

std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K) {
  afb::GemmPlan p = afb::plan_gemm(M, N, K, num_sms());
  return {p.bn, p.splits};
}

}  // namespace

void register_kernel_ops(pybind11::module& m);  // defined in ops_bindings.cpp
void register_runtime(pybind11::module& m);     // defined in runtime.cpp
void register_symm(pybind11::module& m);        // defined in symm.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "arc_forge_2026_b200 native kernels (sm_100a)";
  m.def("status_tensor", &status_tensor, "per-device kernel status words (int32[16])");
  m.def("gemm_grouped", &gemm_grouped, py::arg("a"), py::arg("b"), py::arg("seg"), py::arg("tiles"), py::arg("mode"),
        py::arg("group_rows"), py::arg("max_tiles"), py::arg("out"));
  m.def("gemm", &gemm, "bf16 tcgen05 GEMM: out = act(alpha * a @ b.T + bias) (+ residual)", py::arg("a"), py::arg("b"),
        py::arg("out") = py::none(), py::arg("residual") = py::none(), py::arg("alpha") = 1.0,
        py::arg("out_fp32") = false, py::arg("bn") = 0, py::arg("splits") = 0, py::arg("bias") = py::none(),
        py::arg("act") = 0);
  m.def("gemm_plan", &gemm_plan);
  register_kernel_ops(m);
  register_runtime(m);
  register_symm(m);
}

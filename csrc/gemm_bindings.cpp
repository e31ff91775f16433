// Python bindings of the primus_dlrm_b200 tensor-core kernels (module `_gemm`):
// pyramid attention (attn_fmha.cu) and the tcgen05 GEMMs (gemm_*.cu).
#include <torch/extension.h>

namespace pd {
std::vector<at::Tensor> fmha_fwd(at::Tensor, at::Tensor, at::Tensor, double, int64_t);
void fmha_bwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
              at::Tensor, double);
long long launches();
std::vector<at::Tensor> fmha_fwd_tc(at::Tensor, int64_t, double, at::Tensor);
void fmha_bwd_tc(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, double, at::Tensor,
                 c10::optional<at::Tensor>);
int64_t fmha_bwd_tc_max_q();
void tc_gemm(at::Tensor, at::Tensor, at::Tensor, int64_t, c10::optional<at::Tensor>, c10::optional<at::Tensor>,
             at::Tensor, bool, c10::optional<at::Tensor>);
void tc_wgrad(at::Tensor, at::Tensor, at::Tensor, at::Tensor, bool);
at::Tensor tc_mma_rate(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, at::Tensor);
at::Tensor tc_mma_burst(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, at::Tensor);
}  // namespace pd

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "primus_dlrm_b200 sm_100a tensor-core kernels";
  m.def("fmha_fwd", &pd::fmha_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("scale"), py::arg("warps") = 0,
        "pyramid causal attention forward -> (o, lse); warps (d = 32): 4 (64-query CTAs), 8 (128), 0 = default");
  m.def("fmha_fwd_tc", &pd::fmha_fwd_tc, "tcgen05 pyramid causal attention forward from qkv [B,T,3,H,d] -> (o, lse)");
  m.def("fmha_bwd_tc", &pd::fmha_bwd_tc, py::arg("qkv"), py::arg("o"), py::arg("lse"), py::arg("dout"),
        py::arg("dqkv"), py::arg("q_len"), py::arg("scale"), py::arg("err"), py::arg("dbg") = py::none(),
        "tcgen05 attention backward (d=32) into dqkv [B,T,3,H,d]; dbg: optional int64 stage stamps of CTA 0");
  m.def("fmha_bwd_tc_max_q", &pd::fmha_bwd_tc_max_q, "largest q_len the tcgen05 backward supports");
  m.def("fmha_bwd", &pd::fmha_bwd, "pyramid causal attention backward into dq/dk/dv views");
  m.def("tc_gemm", &pd::tc_gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("epi") = 0,
        py::arg("R") = py::none(), py::arg("AUX") = py::none(), py::arg("err"), py::arg("b_kn") = false,
        py::arg("R2") = py::none(),
        "C[l] = epi(A[l] @ B[l]^T) on tcgen05 (A [L,M,K], B [L|1,N,K] or with b_kn [L|1,K,N], C [L,M,N] bf16 views); "
        "epi 0 none, 1 gelu, 2 +R, 3 dgelu(R), 4 gelu+gelu' to AUX, 5 *R, 6 relu(+R), 7 acc where R>0, 8 R*acc+R2");
  m.def("tc_wgrad", &pd::tc_wgrad, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("err"), py::arg("l_sum") = false,
        "C[l] (fp32, zeroed) += A[l]^T B[l] over rows on tcgen05, split over rows (A [L,K,M], B [L,K,N] bf16 views); "
        "l_sum: one C summed over the batches too");
  m.def("tc_mma_rate", &pd::tc_mma_rate, py::arg("mode"), py::arg("n"), py::arg("iters"), py::arg("nacc"),
        py::arg("swz"), py::arg("issue"), py::arg("err"),
        "tcgen05.mma probe: int64 [SMs, 2] (issue cycles, issue + execution cycles) for `iters` M=128 x n x 16 "
        "MMAs; mode 0 SS K/K, 1 SS K/MN, 2 SS MN/MN, 3 TS B K-major, 4 TS B MN-major; swz 2 = 128 B, 4 = 64 B; "
        "issue 0 = lone lane, 1 = converged warp + elect.sync, 2 = as 1 with the lane-mask operand form");
  m.def("tc_mma_burst", &pd::tc_mma_burst, py::arg("n"), py::arg("iters"), py::arg("issuers"), py::arg("per_sm"),
        py::arg("ts"), py::arg("wstride"), py::arg("lanes"), py::arg("var"), py::arg("err"),
        "unrolled tcgen05.mma probe: int64 [CTAs, 8] (issue, total cycles per issuing warp) for iters x 16 MMAs; "
        "issuers are warps 0, wstride, 2 wstride, ...; var: 0 fixed operands, 1 B advances, 2 A advances, "
        "3 run-time accumulate flag, 4 not unrolled, 5 = 1 + 2 + 3");
  m.def("launch_count", &pd::launches);
}

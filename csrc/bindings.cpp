// Python bindings of the primus_dlrm_b200 core kernels (module `_C`).
#include <torch/extension.h>

namespace pd {
// embedding.cu
void emb_gather(std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, std::vector<at::Tensor>,
                std::vector<at::Tensor>, at::Tensor, int64_t, at::Tensor);
void emb_pooled(std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, std::vector<at::Tensor>,
                std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, int64_t, at::Tensor);
void emb_gather_planned(std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, std::vector<at::Tensor>,
                        std::vector<at::Tensor>, at::Tensor, int64_t, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                        at::Tensor);
at::Tensor emb_keys(std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, std::vector<at::Tensor>,
                    std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, int64_t);
std::vector<at::Tensor> emb_pooled_scale(std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor,
                                         std::vector<at::Tensor>, std::vector<at::Tensor>,
                                         std::vector<at::Tensor>, at::Tensor, int64_t);
void emb_reduce_update(std::vector<at::Tensor>, at::Tensor, std::vector<at::Tensor>, std::vector<at::Tensor>,
                       std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, int64_t, at::Tensor,
                       at::Tensor, c10::optional<at::Tensor>, c10::optional<at::Tensor>, int64_t, double,
                       double, double, double, double, double, double, at::Tensor, c10::optional<at::Tensor>,
                       c10::optional<at::Tensor>);
// norm.cu
std::vector<at::Tensor> norm_fwd(at::Tensor, c10::optional<at::Tensor>, at::Tensor, c10::optional<at::Tensor>,
                                 double, int64_t);
std::vector<at::Tensor> norm_bwd(at::Tensor, at::Tensor, c10::optional<at::Tensor>, at::Tensor, at::Tensor,
                                 c10::optional<at::Tensor>, int64_t, int64_t);
// loss.cu
std::vector<at::Tensor> heads_loss_fwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, std::vector<double>,
                                       std::vector<int64_t>);
std::vector<at::Tensor> heads_loss_bwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor);
// optim.cu
void grad_sqnorm(at::Tensor, at::Tensor);
void adamw_step(at::Tensor, at::Tensor, at::Tensor, at::Tensor, double, double, double, double, double, double,
                double, double, c10::optional<at::Tensor>);
void scale_(at::Tensor, double);
long long launches();
// comm.cu
at::Tensor alloc_shared(int64_t, int64_t);
at::Tensor ipc_handle(at::Tensor);
std::vector<int64_t> ipc_open(at::Tensor);
void ipc_close(int64_t);
void push_rows(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor);
void signal_barrier(at::Tensor, int64_t, int64_t, int64_t, at::Tensor);
void peer_put_row(at::Tensor, at::Tensor, int64_t);
at::Tensor owner_keys(at::Tensor, at::Tensor, int64_t);
void peer_reduce_slice(at::Tensor, int64_t, at::Tensor, int64_t, int64_t, double, int64_t);
void peer_gather_slices(at::Tensor, int64_t, at::Tensor, at::Tensor, int64_t, int64_t);
}  // namespace pd

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "primus_dlrm_b200 sm_100a core kernels";
  m.def("emb_gather", &pd::emb_gather);
  m.def("emb_pooled", &pd::emb_pooled);
  m.def("emb_keys", &pd::emb_keys);
  m.def("emb_gather_planned", &pd::emb_gather_planned,
        "deduplicated gather from an owner-sorted routing plan (unique rows once, then expanded)");
  m.def("emb_pooled_scale", &pd::emb_pooled_scale);
  m.def("emb_reduce_update", &pd::emb_reduce_update, py::arg("grads"), py::arg("slot_meta"), py::arg("weights"),
        py::arg("shard_ptrs"), py::arg("state1"), py::arg("state2"), py::arg("table_meta"), py::arg("dim"),
        py::arg("sorted_keys"), py::arg("perm"), py::arg("scale"), py::arg("grad_row"), py::arg("opt_kind"),
        py::arg("lr"), py::arg("eps"), py::arg("weight_decay"), py::arg("beta1"), py::arg("beta2"),
        py::arg("bc1"), py::arg("bc2"), py::arg("err"), py::arg("out_rows") = py::none(),
        py::arg("seg") = py::none());
  m.def("norm_fwd", &pd::norm_fwd);
  m.def("norm_bwd", &pd::norm_bwd, py::arg("xin"), py::arg("dy"), py::arg("dz_extra"), py::arg("w"),
        py::arg("rstd"), py::arg("mean"), py::arg("kind"), py::arg("ex_off") = 0);
  m.def("heads_loss_fwd", &pd::heads_loss_fwd);
  m.def("heads_loss_bwd", &pd::heads_loss_bwd);
  m.def("grad_sqnorm", &pd::grad_sqnorm);
  m.def("adamw_step", &pd::adamw_step);
  m.def("scale_", &pd::scale_);
  m.def("alloc_shared", &pd::alloc_shared);
  m.def("ipc_handle", &pd::ipc_handle);
  m.def("ipc_open", &pd::ipc_open);
  m.def("ipc_close", &pd::ipc_close);
  m.def("push_rows", &pd::push_rows);
  m.def("signal_barrier", &pd::signal_barrier);
  m.def("peer_put_row", &pd::peer_put_row, "row `rank` of every rank's int64 [W, n] board = src (peer stores)");
  m.def("owner_keys", &pd::owner_keys);
  m.def("peer_reduce_slice", &pd::peer_reduce_slice, py::arg("ptrs"), py::arg("rank"), py::arg("own"), py::arg("a"),
        py::arg("b"), py::arg("scale"), py::arg("max_blocks") = 0,
        "own[a:b) = scale * sum over ranks of peer[a:b) (NVLink P2P loads); max_blocks > 0 caps the grid");
  m.def("peer_gather_slices", &pd::peer_gather_slices, py::arg("ptrs"), py::arg("rank"), py::arg("own"),
        py::arg("bounds"), py::arg("span") = 0, py::arg("max_blocks") = 0,
        "copy every other rank's slice [bounds[q], bounds[q+1]) from that rank (all-gather); span sizes the grid");
  m.def("launch_count", &pd::launches, "kernels launched by this extension so far");
}

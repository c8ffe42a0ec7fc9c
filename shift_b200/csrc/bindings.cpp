// Python bindings for the sm_100a kernels of shift_b200 (module shift_b200._C).
#include <torch/extension.h>

#include "gemm_sm100.h"

namespace sb {
namespace norm {
std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& delta, const at::Tensor& w,
                                    double eps, const c10::optional<at::Tensor>& delta2,
                                    const c10::optional<at::Tensor>& y_out, const std::vector<int64_t>& xchg,
                                    const c10::optional<at::Tensor>& status);
at::Tensor rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& w,
                       const c10::optional<at::Tensor>& dres, at::Tensor& dw_out, bool accumulate,
                       const c10::optional<at::Tensor>& dy2, const c10::optional<at::Tensor>& dx_out,
                       const std::vector<int64_t>& xchg, const c10::optional<at::Tensor>& status);
void column_reduce(const at::Tensor& partial, at::Tensor& out, bool accumulate);
void rope_(at::Tensor& qkv, const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t S, int64_t n_rot_heads,
           int64_t head_dim, int64_t pos0, bool inverse);
}  // namespace norm
namespace moe {
std::vector<at::Tensor> router_fwd(const at::Tensor& x, const at::Tensor& wr, int64_t k, bool normalize);
at::Tensor router_bwd(const at::Tensor& probs, const at::Tensor& topk_idx, const at::Tensor& topk_w,
                      const at::Tensor& d_topk_w, const c10::optional<at::Tensor>& aux_grad, bool normalize);
at::Tensor router_input_weight_grad(const at::Tensor& x, const at::Tensor& wr, const at::Tensor& dlogits,
                                    at::Tensor& dx, const std::vector<int64_t>& peer_rows,
                                    const std::vector<int64_t>& xchg);
std::vector<at::Tensor> bucket_sort(const at::Tensor& keys, int64_t lo, int64_t hi, int64_t pad, int64_t src_div);
void gather_rows(const at::Tensor& src, const at::Tensor& row_src, const c10::optional<at::Tensor>& total,
                 at::Tensor& out);
at::Tensor combine(const at::Tensor& y, const at::Tensor& pos, const at::Tensor& w, int64_t T,
                   const c10::optional<at::Tensor>& out, const std::vector<int64_t>& split,
                   const std::vector<int64_t>& xchg);
std::vector<at::Tensor> combine_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& pos,
                                    const at::Tensor& w, const at::Tensor& row_src, const at::Tensor& slot_of_row,
                                    const at::Tensor& total);
void scatter_back(const at::Tensor& dperm, const at::Tensor& pos, at::Tensor& dx, bool accumulate);
at::Tensor invert_pos(const at::Tensor& pos, int64_t cap);
void embedding_bwd(const at::Tensor& dout, const at::Tensor& ids, at::Tensor& dW, int64_t vocab_lo);
at::Tensor embedding_fwd(const at::Tensor& W, const at::Tensor& ids, int64_t vocab_lo);
at::Tensor swiglu_fwd(const at::Tensor& h);
at::Tensor swiglu_bwd(const at::Tensor& h, const at::Tensor& da);
}  // namespace moe
namespace xent {
at::Tensor xent_fwd_bwd(at::Tensor& logits, const at::Tensor& labels, double scale, int64_t label_lo);
}
namespace adam {
void adamw_step(const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, const std::vector<at::Tensor>& grads,
                at::Tensor& master_out, at::Tensor& m_out, at::Tensor& v_out, at::Tensor& param_out, double lr,
                double beta1, double beta2, double eps, double wd, int64_t step, double grad_scale,
                const c10::optional<at::Tensor>& nonfinite, const c10::optional<at::Tensor>& step_dev);
void nonfinite_check(const at::Tensor& x, at::Tensor& flag);
}  // namespace adam
namespace fa {
std::vector<at::Tensor> fwd(const at::Tensor& qkv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, double scale,
                            const at::Tensor& status);
at::Tensor bwd(const at::Tensor& qkv, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dout, int64_t B,
               int64_t S, int64_t Hq, int64_t Hkv, double scale, const at::Tensor& status);
}  // namespace fa
namespace coll {
at::Tensor sym_alloc(int64_t nbytes, int64_t device);
at::Tensor ipc_handle(const at::Tensor& t);
at::Tensor ipc_open(const at::Tensor& handle, int64_t nbytes, int64_t device);
void fused_reduce_adamw(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& flag_ptrs,
                        const at::Tensor& step_dev, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v,
                        at::Tensor& master_out, at::Tensor& m_out, at::Tensor& v_out, at::Tensor& param_out,
                        double beta1, double beta2, double eps, double wd, double grad_scale,
                        const at::Tensor& nonfinite, const at::Tensor& status, double timeout_s, int64_t blocks_per_sm);
void flag_set(int64_t flag_ptr, const at::Tensor& step_dev, int64_t delta);
void reduce_slice_scatter(const std::vector<int64_t>& src_ptrs, const std::vector<int64_t>& dst_ptrs, int64_t lo,
                          int64_t hi, const std::vector<int64_t>& flag_ptrs, const at::Tensor& step_dev,
                          double scale, const at::Tensor& status, double timeout_s, int64_t blocks_per_sm);
void flag_wait(const std::vector<int64_t>& flag_ptrs, const at::Tensor& step_dev, int64_t delta,
               const at::Tensor& status, double timeout_s);
void peer_copy(int64_t src_ptr, int64_t dst_ptr, int64_t nbytes);
void xcopy(int64_t src_ptr, int64_t dst_ptr, int64_t nbytes, const std::vector<int64_t>& xchg,
           const at::Tensor& status);
std::string fingerprint(const at::Tensor& t);
}  // namespace coll
namespace digest {
at::Tensor sha256_leaves(const at::Tensor& t, int64_t leaf, const at::Tensor& consts);
}  // namespace digest
}  // namespace sb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "shift_b200 sm_100a kernels";
  m.def("gemm", &sb::gemm::gemm, "tcgen05 GEMM (dense / grouped, optional tensor-parallel exchange)",
        py::arg("A"), py::arg("B"), py::arg("D"), py::arg("D2"), py::arg("offs"), py::arg("M"), py::arg("N"),
        py::arg("K"), py::arg("G"), py::arg("mode"), py::arg("a_mn"), py::arg("b_mn"), py::arg("epi"),
        py::arg("alpha"), py::arg("bn"), py::arg("status"), py::arg("max_rows_hint"),
        py::arg("xchg") = std::vector<int64_t>{}, py::arg("tp") = std::vector<int64_t>{});
  m.def("rmsnorm_fwd", &sb::norm::rmsnorm_fwd, py::arg("x"), py::arg("delta"), py::arg("w"), py::arg("eps"),
        py::arg("delta2") = py::none(), py::arg("y_out") = py::none(), py::arg("xchg") = std::vector<int64_t>{},
        py::arg("status") = py::none());
  m.def("rmsnorm_bwd", &sb::norm::rmsnorm_bwd, py::arg("dy"), py::arg("x"), py::arg("rstd"), py::arg("w"),
        py::arg("dres"), py::arg("dw_out"), py::arg("accumulate"), py::arg("dy2") = py::none(),
        py::arg("dx_out") = py::none(), py::arg("xchg") = std::vector<int64_t>{}, py::arg("status") = py::none());
  m.def("column_reduce", &sb::norm::column_reduce);
  m.def("rope_", &sb::norm::rope_);
  m.def("router_fwd", &sb::moe::router_fwd);
  m.def("router_bwd", &sb::moe::router_bwd);
  m.def("router_input_weight_grad", &sb::moe::router_input_weight_grad, py::arg("x"), py::arg("wr"),
        py::arg("dlogits"), py::arg("dx"), py::arg("peer_rows") = std::vector<int64_t>{},
        py::arg("xchg") = std::vector<int64_t>{});
  m.def("bucket_sort", &sb::moe::bucket_sort);
  m.def("gather_rows", &sb::moe::gather_rows);
  m.def("combine", &sb::moe::combine, py::arg("y"), py::arg("pos"), py::arg("w"), py::arg("T"),
        py::arg("out") = py::none(), py::arg("split") = std::vector<int64_t>{},
        py::arg("xchg") = std::vector<int64_t>{});
  m.def("combine_bwd", &sb::moe::combine_bwd);
  m.def("scatter_back", &sb::moe::scatter_back);
  m.def("invert_pos", &sb::moe::invert_pos);
  m.def("embedding_fwd", &sb::moe::embedding_fwd);
  m.def("embedding_bwd", &sb::moe::embedding_bwd);
  m.def("swiglu_fwd", &sb::moe::swiglu_fwd);
  m.def("swiglu_bwd", &sb::moe::swiglu_bwd);
  m.def("xent_fwd_bwd", &sb::xent::xent_fwd_bwd);
  m.def("adamw_step", &sb::adam::adamw_step, py::arg("master"), py::arg("m"), py::arg("v"), py::arg("grads"),
        py::arg("master_out"), py::arg("m_out"), py::arg("v_out"), py::arg("param_out"), py::arg("lr"), py::arg("beta1"),
        py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("step"), py::arg("grad_scale"),
        py::arg("nonfinite") = py::none(), py::arg("step_dev") = py::none());
  m.def("nonfinite_check", &sb::adam::nonfinite_check);
  m.def("attn_fwd", &sb::fa::fwd, "tcgen05 causal flash attention forward");
  m.def("attn_bwd", &sb::fa::bwd, "tcgen05 causal flash attention backward (dK/dV + dQ kernels)");
  m.def("sym_alloc", &sb::coll::sym_alloc);
  m.def("ipc_handle", &sb::coll::ipc_handle);
  m.def("ipc_open", &sb::coll::ipc_open);
  m.def("fused_reduce_adamw", &sb::coll::fused_reduce_adamw, "K1: cross-replica reduce + cast + scale + AdamW");
  m.def("flag_set", &sb::coll::flag_set);
  m.def("reduce_slice_scatter", &sb::coll::reduce_slice_scatter, "K1 phase A: reduce-scatter + all-gather via P2P");
  m.def("flag_wait", &sb::coll::flag_wait);
  m.def("peer_copy", &sb::coll::peer_copy, "K10: SM-driven peer-memory copy");
  m.def("xcopy", &sb::coll::xcopy, "copy to a local and a peer destination with TP exchange wait/signal");
  m.def("fingerprint", &sb::coll::fingerprint, "deterministic 64-bit fingerprint of a tensor's bytes");
  m.def("sha256_leaves", &sb::digest::sha256_leaves, "SHA-256 of each fixed-size leaf of a device buffer");
}

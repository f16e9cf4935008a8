// Python bindings of the sm_100a kernel library (module titans_pytorch_b200._C).
#include <torch/extension.h>

#include <vector>

namespace tb {
// norm.cu
std::vector<at::Tensor> rms_norm_fwd(const at::Tensor& x, const at::Tensor& w, double eps);
std::vector<at::Tensor> rms_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                     const at::Tensor& rstd, bool need_dw, const c10::optional<at::Tensor>& dadd);
std::vector<at::Tensor> rms_norm_add_fwd(const at::Tensor& x, const at::Tensor& res, const at::Tensor& w, double eps);
// conv.cu
at::Tensor conv_silu_norm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w,
                              const c10::optional<at::Tensor>& b, bool normalize);
std::vector<at::Tensor> conv_silu_norm_bwd(const at::Tensor& dy, const at::Tensor& x,
                                           const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b,
                                           bool normalize, bool need_wgrad);
// elementwise.cu
at::Tensor swiglu_fwd(const at::Tensor& gu);
at::Tensor swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu);
at::Tensor silu_mul(const at::Tensor& g, const at::Tensor& u);
at::Tensor memory_gates(const at::Tensor& x, const std::vector<at::Tensor>& ws, const std::vector<at::Tensor>& bs,
                        double lr, double mom);
void act_inplace(const at::Tensor& z, at::Tensor& a, const std::string& act);
void act_grad_mul(at::Tensor& gr, const at::Tensor& z, const std::string& act);
void act_grad_out(const at::Tensor& g, const at::Tensor& z, at::Tensor& out, const std::string& act);
void scaled_err(at::Tensor& p, const at::Tensor& v, double scale);
std::vector<at::Tensor> mem_update(const at::Tensor& w, const at::Tensor& m, const at::Tensor& grad,
                                   const at::Tensor& gates);
// loss.cu
std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& labels, int64_t ignore_index);
at::Tensor cross_entropy_bwd(const at::Tensor& logits, const at::Tensor& labels, const at::Tensor& lse,
                             const at::Tensor& stats, const at::Tensor& gout, int64_t ignore_index);
// optim.cu
at::Tensor grad_norm_clip(const at::Tensor& grads, const at::Tensor& tab, int64_t nseg, int64_t items, double gscale,
                          double max_norm);
void adamw_step(at::Tensor& master, at::Tensor& exp_avg, at::Tensor& exp_avg_sq, const at::Tensor& grads,
                const c10::optional<at::Tensor>& params_out, const at::Tensor& tab, int64_t nseg, int64_t items,
                const c10::optional<at::Tensor>& clip, double gscale, double lr, double beta1, double beta2,
                double eps, double wd, int64_t step, const c10::optional<at::Tensor>& hyper);
void adamw_hyper_step(at::Tensor& hyper, double base_lr, double beta1, double beta2, int64_t warmup, int64_t total,
                      double min_ratio, bool use_schedule);
// attention.cu
std::vector<at::Tensor> attn_pack(const at::Tensor& qkv, const c10::optional<at::Tensor>& pkv, int64_t H,
                                  const c10::optional<at::Tensor>& inv_freq, int64_t pos0);
std::vector<at::Tensor> attn_fwd_packed(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, int64_t window,
                                        double scale);
std::vector<at::Tensor> attn_bwd_packed(const at::Tensor& dO, const at::Tensor& Q, const at::Tensor& K,
                                        const at::Tensor& V, const at::Tensor& O, const at::Tensor& LSE,
                                        int64_t window, double scale);
std::vector<at::Tensor> attn_unpack(const at::Tensor& dQa, const at::Tensor& dKa, const at::Tensor& dVa,
                                    const c10::optional<at::Tensor>& inv_freq, int64_t Bp, at::ScalarType dtype,
                                    int64_t pos0);
// attention_tc.cu
std::vector<at::Tensor> attn_fwd_tc(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, int64_t window,
                                    double scale);
bool attn_tc_fwd_supported(int64_t head_dim);
bool attn_tc_supported(int64_t head_dim);
std::vector<at::Tensor> attn_bwd_tc(const at::Tensor& dO, const at::Tensor& Q, const at::Tensor& K,
                                    const at::Tensor& V, const at::Tensor& O, const at::Tensor& LSE, int64_t window,
                                    double scale);
int64_t kernel_error_status(int64_t device, bool reset);
at::Tensor exp2_poly_eval(const at::Tensor& x);
at::Tensor memory_scan_fwd(at::Tensor& W1, at::Tensor& S1, at::Tensor& W2T, at::Tensor& S2T, const at::Tensor& k,
                           const at::Tensor& v, const at::Tensor& q, const at::Tensor& theta, const at::Tensor& eta,
                           const at::Tensor& alpha);
// comm.cu
std::vector<at::Tensor> comm_alloc(int64_t nbytes, int64_t device);
int64_t comm_ipc_open(const at::Tensor& handle, int64_t device);
void comm_ipc_close(int64_t ptr);
void comm_barrier(const at::Tensor& sig_ptrs, int64_t slot, at::Tensor& epoch, bool bump, int64_t world, int64_t me,
                  at::Tensor& err, int64_t budget);
void comm_reduce_shard(const at::Tensor& grad_ptrs, int64_t lo, int64_t n, at::Tensor& gsum, double gscale,
                       const at::Tensor& slot_ptrs, int64_t world, int64_t me);
void comm_adamw_shard(const at::Tensor& gsum, at::Tensor& master, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                      const at::Tensor& param_ptrs, int64_t lo, int64_t world, const at::Tensor& tab, int64_t nseg,
                      int64_t items, const at::Tensor& norm_slots, double gscale, double max_norm, double lr,
                      double beta1, double beta2, double eps, double wd, int64_t step, at::Tensor& norm_out,
                      const c10::optional<at::Tensor>& hyper, const c10::optional<at::Tensor>& seg_aux, int64_t me);
void comm_reduce_segments(const at::Tensor& grad_ptrs, const at::Tensor& tab, int64_t nseg, int64_t items,
                          at::Tensor& gsum, double gscale, const at::Tensor& slot_ptrs, int64_t world, int64_t me);
void comm_reduce_into(const at::Tensor& grad_ptrs, const at::Tensor& tab, int64_t nseg, int64_t items,
                      at::Tensor& gsum, double gscale, at::Tensor& part, int64_t part_off, int64_t blocks,
                      bool accumulate);
void comm_norm_publish(const at::Tensor& part, int64_t nparts, const at::Tensor& slot_ptrs, int64_t world,
                       int64_t me);
std::vector<at::Tensor> quantize_int8_rows(const at::Tensor& w);
at::Tensor dequantize_int8_rows(const at::Tensor& q, const at::Tensor& s);
at::Tensor int8_gemm_small(const at::Tensor& x, const at::Tensor& q, const at::Tensor& s);
// gemm_tc.cu
at::Tensor gemm_tc(const at::Tensor& A, const at::Tensor& B);
at::Tensor gemm_gather_tc(const at::Tensor& A, const at::Tensor& B, at::Tensor& flat, const at::Tensor& src_ptrs,
                          int64_t u0, int64_t len, int64_t shard, int64_t me, bool consume, bool copy_own);
void fsdp_gather(at::Tensor& flat, const at::Tensor& src_ptrs, int64_t u0, int64_t len, int64_t shard, int64_t me,
                 bool copy_own);
// gemm_sm100.cu
void gemm_sm100(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t M, int64_t N, int64_t K,
                int64_t mode, const at::Tensor& Cout, const c10::optional<at::Tensor>& R,
                const c10::optional<at::Tensor>& C2, const c10::optional<at::Tensor>& R2,
                const c10::optional<at::Tensor>& gates, double scale, int64_t act, int64_t ffn_f, int64_t splits);
}  // namespace tb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "titans_pytorch_b200 sm_100a kernels";
  m.def("rms_norm_fwd", &tb::rms_norm_fwd);
  m.def("rms_norm_bwd", &tb::rms_norm_bwd, pybind11::arg("dy"), pybind11::arg("x"), pybind11::arg("w"),
        pybind11::arg("rstd"), pybind11::arg("need_dw"), pybind11::arg("dadd") = pybind11::none());
  m.def("rms_norm_add_fwd", &tb::rms_norm_add_fwd);
  m.def("conv_silu_norm_fwd", &tb::conv_silu_norm_fwd);
  m.def("conv_silu_norm_bwd", &tb::conv_silu_norm_bwd);
  m.def("swiglu_fwd", &tb::swiglu_fwd);
  m.def("swiglu_bwd", &tb::swiglu_bwd);
  m.def("silu_mul", &tb::silu_mul);
  m.def("memory_gates", &tb::memory_gates);
  m.def("act_inplace", &tb::act_inplace);
  m.def("act_grad_mul", &tb::act_grad_mul);
  m.def("act_grad_out", &tb::act_grad_out);
  m.def("scaled_err", &tb::scaled_err);
  m.def("mem_update", &tb::mem_update);
  m.def("cross_entropy_fwd", &tb::cross_entropy_fwd);
  m.def("cross_entropy_bwd", &tb::cross_entropy_bwd);
  m.def("grad_norm_clip", &tb::grad_norm_clip);
  m.def("adamw_step", &tb::adamw_step, pybind11::arg("master"), pybind11::arg("exp_avg"), pybind11::arg("exp_avg_sq"),
        pybind11::arg("grads"), pybind11::arg("params_out"), pybind11::arg("tab"), pybind11::arg("nseg"),
        pybind11::arg("items"), pybind11::arg("clip"), pybind11::arg("gscale"), pybind11::arg("lr"),
        pybind11::arg("beta1"), pybind11::arg("beta2"), pybind11::arg("eps"), pybind11::arg("wd"),
        pybind11::arg("step"), pybind11::arg("hyper") = pybind11::none());
  m.def("adamw_hyper_step", &tb::adamw_hyper_step);
  m.def("attn_pack", &tb::attn_pack, py::arg("qkv"), py::arg("pkv"), py::arg("H"), py::arg("inv_freq"),
        py::arg("pos0") = 0);
  m.def("attn_fwd_packed", &tb::attn_fwd_packed);
  m.def("attn_bwd_packed", &tb::attn_bwd_packed);
  m.def("attn_unpack", &tb::attn_unpack, py::arg("dQa"), py::arg("dKa"), py::arg("dVa"), py::arg("inv_freq"),
        py::arg("Bp"), py::arg("dtype"), py::arg("pos0") = 0);
  m.def("attn_fwd_tc", &tb::attn_fwd_tc);
  m.def("attn_tc_supported", &tb::attn_tc_supported);
  m.def("attn_tc_fwd_supported", &tb::attn_tc_fwd_supported);
  m.def("attn_bwd_tc", &tb::attn_bwd_tc);
  m.def("memory_scan_fwd", &tb::memory_scan_fwd);
  m.def("comm_alloc", &tb::comm_alloc);
  m.def("comm_ipc_open", &tb::comm_ipc_open);
  m.def("comm_ipc_close", &tb::comm_ipc_close);
  m.def("comm_barrier", &tb::comm_barrier, pybind11::arg("sig_ptrs"), pybind11::arg("slot"), pybind11::arg("epoch"),
        pybind11::arg("bump"), pybind11::arg("world"), pybind11::arg("me"), pybind11::arg("err"),
        pybind11::arg("budget") = (int64_t)1 << 31);
  m.def("comm_reduce_shard", &tb::comm_reduce_shard);
  m.def("comm_adamw_shard", &tb::comm_adamw_shard, pybind11::arg("gsum"), pybind11::arg("master"),
        pybind11::arg("exp_avg"), pybind11::arg("exp_avg_sq"), pybind11::arg("param_ptrs"), pybind11::arg("lo"),
        pybind11::arg("world"), pybind11::arg("tab"), pybind11::arg("nseg"), pybind11::arg("items"),
        pybind11::arg("norm_slots"), pybind11::arg("gscale"), pybind11::arg("max_norm"), pybind11::arg("lr"),
        pybind11::arg("beta1"), pybind11::arg("beta2"), pybind11::arg("eps"), pybind11::arg("wd"),
        pybind11::arg("step"), pybind11::arg("norm_out"), pybind11::arg("hyper") = pybind11::none(),
        pybind11::arg("seg_aux") = pybind11::none(), pybind11::arg("me") = 0);
  m.def("comm_reduce_segments", &tb::comm_reduce_segments);
  m.def("comm_reduce_into", &tb::comm_reduce_into);
  m.def("comm_norm_publish", &tb::comm_norm_publish);
  m.def("quantize_int8_rows", &tb::quantize_int8_rows);
  m.def("dequantize_int8_rows", &tb::dequantize_int8_rows);
  m.def("int8_gemm_small", &tb::int8_gemm_small);
  m.def("gemm_tc", &tb::gemm_tc);
  m.def("gemm_gather_tc", &tb::gemm_gather_tc, pybind11::arg("A"), pybind11::arg("B"), pybind11::arg("flat"),
        pybind11::arg("src_ptrs"), pybind11::arg("u0"), pybind11::arg("len"), pybind11::arg("shard"),
        pybind11::arg("me"), pybind11::arg("consume"), pybind11::arg("copy_own") = false);
  m.def("fsdp_gather", &tb::fsdp_gather, pybind11::arg("flat"), pybind11::arg("src_ptrs"), pybind11::arg("u0"),
        pybind11::arg("len"), pybind11::arg("shard"), pybind11::arg("me"), pybind11::arg("copy_own") = false);
  m.def("gemm_sm100", &tb::gemm_sm100, pybind11::arg("A"), pybind11::arg("a_mn"), pybind11::arg("B"),
        pybind11::arg("b_mn"), pybind11::arg("M"), pybind11::arg("N"), pybind11::arg("K"), pybind11::arg("mode"),
        pybind11::arg("C"), pybind11::arg("R") = pybind11::none(), pybind11::arg("C2") = pybind11::none(),
        pybind11::arg("R2") = pybind11::none(), pybind11::arg("gates") = pybind11::none(),
        pybind11::arg("scale") = 1.0, pybind11::arg("act") = 0, pybind11::arg("ffn_f") = 0,
        pybind11::arg("splits") = 0);
  m.def("exp2_poly_eval", &tb::exp2_poly_eval);
  m.def("kernel_error_status", &tb::kernel_error_status, pybind11::arg("device") = 0, pybind11::arg("reset") = true);
}

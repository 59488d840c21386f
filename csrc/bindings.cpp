// Python bindings of the sm_100a extension nanospec_b200._C.
#include <torch/extension.h>

#include <vector>

#include "common.h"

namespace ns {
void linear(at::Tensor x, at::Tensor w, at::Tensor out, c10::optional<at::Tensor> residual);
void linear_dgrad(at::Tensor dy, at::Tensor w, at::Tensor out, bool accumulate);
int64_t linear_wgrad(at::Tensor dy, at::Tensor x, at::Tensor out, bool accumulate, c10::optional<at::Tensor> nfac,
                     c10::optional<at::Tensor> npart, int64_t offset);
void gemm_test(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor out, int splits);
void gemm_trace(c10::optional<at::Tensor> buf);
void rms_norm_fwd(at::Tensor x, at::Tensor w, double eps, at::Tensor y, at::Tensor inv);
void rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor inv, at::Tensor w, at::Tensor dx, at::Tensor dw,
                  c10::optional<at::Tensor> res);
void head_norm_rope_fwd(at::Tensor x, at::Tensor w, double eps, at::Tensor cs, at::Tensor sn, at::Tensor y,
                        at::Tensor inv);
void head_norm_rope_bwd(at::Tensor dy, at::Tensor x, at::Tensor inv, at::Tensor w, at::Tensor cs, at::Tensor sn,
                        at::Tensor dx, at::Tensor dw);
void swiglu_fwd(at::Tensor gu, at::Tensor out);
void swiglu_bwd(at::Tensor dp, at::Tensor gu, at::Tensor dgu);
void embedding_fwd(at::Tensor ids, at::Tensor w, at::Tensor out);
void embedding_bwd(at::Tensor dy, at::Tensor ids, at::Tensor grad);
void grad_norm_sq(at::Tensor grad, at::Tensor factor, at::Tensor norm2);
void grad_norm_sq_ranges(std::vector<at::Tensor> ranges, at::Tensor factor, at::Tensor norm2);
void adamw_update(at::Tensor param, at::Tensor master, at::Tensor m, at::Tensor v, at::Tensor grad,
                  at::Tensor factor, at::Tensor norm2, double lr, double wd, double b1, double b2, double eps,
                  double bc1, double bc2, double max_norm, c10::optional<at::Tensor> bc_dev, bool zero_grad);
void adam_prepare(at::Tensor norm2, at::Tensor step, double b1, double b2, at::Tensor bc);
void attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs,
              at::Tensor out, at::Tensor lse);
void attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor lse,
              at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs, at::Tensor dq, at::Tensor dk,
              at::Tensor dv);
std::vector<at::Tensor> head_loss(at::Tensor hcat, int64_t T, at::Tensor lm_head, c10::optional<at::Tensor> e,
                                  c10::optional<at::Tensor> w2, c10::optional<at::Tensor> target_logits,
                                  at::Tensor labels, at::Tensor weights, double ce_w, double kl_w,
                                  double inv_accum, c10::optional<at::Tensor> dw2_out, int64_t chunk);
void fp8_linear(at::Tensor x, at::Tensor w, at::Tensor scale_inv, at::Tensor out);
void add_bf16(at::Tensor a, at::Tensor b, at::Tensor o);
void silu_mul(at::Tensor g, at::Tensor u, at::Tensor o);
void qwen_norm(at::Tensor x, at::Tensor w, double eps, at::Tensor y);
void gated_norm(at::Tensor x, at::Tensor gate, at::Tensor w, double eps, at::Tensor y);
void conv_silu(at::Tensor x, at::Tensor w, at::Tensor y);
void gdn_gates(at::Tensor a, at::Tensor b, at::Tensor alog, at::Tensor dtb, at::Tensor g, at::Tensor beta);
void gdn_chunk_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, int64_t groups, at::Tensor out);
void causal_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor gate, at::Tensor cs, at::Tensor sn, int64_t rd,
                     at::Tensor out);
std::vector<int64_t> window_create(int64_t bytes, int64_t rank, int64_t world);
at::Tensor window_ipc_handle(int64_t id);
void window_open(int64_t id, at::Tensor handles);
void window_close(int64_t id);
at::Tensor window_view(int64_t id, int64_t offset, int64_t numel, at::ScalarType dtype);
void peer_reduce_avg_ce(int64_t id, int64_t slot_off, int64_t ss_elems, at::Tensor grad, at::Tensor staging);
void peer_allgather_ce(int64_t id, int64_t src_off, int64_t ss_elems, at::Tensor out);
void peer_allgather(int64_t id, int64_t src_off, int64_t ss_elems, at::Tensor out);
void peer_reduce_avg(int64_t id, int64_t slot_off, int64_t ss_elems, at::Tensor grad);
void peer_reduce_local(int64_t id, int64_t slot_off, int64_t ss_elems, at::Tensor grad);
void ag_gemm(int64_t id, int64_t src_off, int64_t ss, at::Tensor resident, int64_t w_off, int64_t N, int64_t K,
             at::Tensor x, at::Tensor out, at::Tensor flags, at::Tensor claim, int64_t epoch, int64_t poll_limit);
void gemm_rs(int64_t id, int64_t slot_off, int64_t ss, int64_t g_off, at::Tensor dy, at::Tensor x);
void peer_push(int64_t id, int64_t slot_off, int64_t ss, at::Tensor src, int64_t lo, int64_t hi);
void peer_put(int64_t id, int64_t dst, int64_t dst_off, at::Tensor src);
void peer_signal_to(int64_t id, int64_t flags_off, int64_t channel, int64_t dst, int64_t seq);
void peer_wait_from(int64_t id, int64_t flags_off, int64_t channel, int64_t src, int64_t seq, int64_t poll_limit);
void peer_signal(int64_t id, int64_t flags_off, int64_t channel, int64_t seq);
void peer_wait(int64_t id, int64_t flags_off, int64_t channel, int64_t seq, int64_t poll_limit);
std::vector<at::Tensor> gdn_chunk_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                                      at::Tensor dout, int64_t groups);
int64_t device_error();
void clear_device_error();
void fp8_gemm(at::Tensor q, at::Tensor sa, at::Tensor w, at::Tensor scale_inv, at::Tensor out);
void quant_e4m3(at::Tensor x, at::Tensor q, at::Tensor s);
void add_norm(at::Tensor x, c10::optional<at::Tensor> y, at::Tensor w, double eps, c10::optional<at::Tensor> x_out,
              c10::optional<at::Tensor> n_out, c10::optional<at::Tensor> q_out, c10::optional<at::Tensor> s_out);
void add_norm_peer(at::Tensor x, c10::optional<at::Tensor> y, at::Tensor w, double eps,
                   c10::optional<at::Tensor> x_out, c10::optional<at::Tensor> n_out, c10::optional<at::Tensor> q_out,
                   c10::optional<at::Tensor> s_out, int64_t win, int64_t x_dst, int64_t x_off, int64_t n_dst,
                   int64_t n_off);
void silu_mul_quant(at::Tensor gu, at::Tensor q, at::Tensor s);
void gated_norm_quant(at::Tensor x, at::Tensor z, int64_t nv, int64_t z_ts, at::Tensor w, double eps, at::Tensor q,
                      at::Tensor s);
void conv_silu_vec(at::Tensor x, int64_t ld, at::Tensor w, at::Tensor y);
void head_norm_rope(at::Tensor x, int64_t H, int64_t x_ts, int64_t x_hs, int64_t S, at::Tensor w, double eps,
                    at::Tensor cs, at::Tensor sn, int64_t rd, at::Tensor y);
void vattn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor gate, int64_t g_ts, int64_t g_hs, at::Tensor out);
at::Tensor device_error_tensor();
void reset_device_error_state();
}  // namespace ns

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nanospec_b200 sm_100a kernels";
  m.def("linear", &ns::linear);
  m.def("linear_dgrad", &ns::linear_dgrad);
  m.def("linear_wgrad", &ns::linear_wgrad, py::arg("dy"), py::arg("x"), py::arg("out"), py::arg("accumulate") = false,
        py::arg("nfac") = py::none(), py::arg("npart") = py::none(), py::arg("offset") = 0);
  m.def("gemm_test", &ns::gemm_test);
  m.def("gemm_trace", &ns::gemm_trace);
  m.def("rms_norm_fwd", &ns::rms_norm_fwd);
  m.def("rms_norm_bwd", &ns::rms_norm_bwd);
  m.def("head_norm_rope_fwd", &ns::head_norm_rope_fwd);
  m.def("head_norm_rope_bwd", &ns::head_norm_rope_bwd);
  m.def("swiglu_fwd", &ns::swiglu_fwd);
  m.def("swiglu_bwd", &ns::swiglu_bwd);
  m.def("embedding_fwd", &ns::embedding_fwd);
  m.def("embedding_bwd", &ns::embedding_bwd);
  m.def("grad_norm_sq", &ns::grad_norm_sq);
  m.def("grad_norm_sq_ranges", &ns::grad_norm_sq_ranges);
  m.def("adamw_update", &ns::adamw_update, py::arg("param"), py::arg("master"), py::arg("m"), py::arg("v"),
        py::arg("grad"), py::arg("factor"), py::arg("norm2"), py::arg("lr"), py::arg("wd"), py::arg("b1"),
        py::arg("b2"), py::arg("eps"), py::arg("bc1"), py::arg("bc2"), py::arg("max_norm"),
        py::arg("bc_dev") = py::none(), py::arg("zero_grad") = true);
  m.def("adam_prepare", &ns::adam_prepare);
  m.def("attn_fwd", &ns::attn_fwd);
  m.def("attn_bwd", &ns::attn_bwd);
  m.def("head_loss", &ns::head_loss);
  m.def("fp8_linear", &ns::fp8_linear);
  m.def("add_bf16", &ns::add_bf16);
  m.def("silu_mul", &ns::silu_mul);
  m.def("qwen_norm", &ns::qwen_norm);
  m.def("gated_norm", &ns::gated_norm);
  m.def("conv_silu", &ns::conv_silu);
  m.def("gdn_gates", &ns::gdn_gates);
  m.def("gdn_chunk_fwd", &ns::gdn_chunk_fwd);
  m.def("causal_attn_fwd", &ns::causal_attn_fwd);
  m.def("window_create", &ns::window_create);
  m.def("window_ipc_handle", &ns::window_ipc_handle);
  m.def("window_open", &ns::window_open);
  m.def("window_close", &ns::window_close);
  m.def("window_view", &ns::window_view);
  m.def("peer_reduce_avg_ce", &ns::peer_reduce_avg_ce);
  m.def("peer_allgather_ce", &ns::peer_allgather_ce);
  m.def("peer_allgather", &ns::peer_allgather);
  m.def("peer_reduce_avg", &ns::peer_reduce_avg);
  m.def("peer_reduce_local", &ns::peer_reduce_local);
  m.def("ag_gemm", &ns::ag_gemm);
  m.def("gemm_rs", &ns::gemm_rs);
  m.def("peer_push", &ns::peer_push);
  m.def("peer_put", &ns::peer_put);
  m.def("peer_signal_to", &ns::peer_signal_to);
  m.def("peer_wait_from", &ns::peer_wait_from);
  m.def("peer_signal", &ns::peer_signal);
  m.def("peer_wait", &ns::peer_wait);
  m.def("gdn_chunk_bwd", &ns::gdn_chunk_bwd);
  m.def("fp8_gemm", &ns::fp8_gemm, "block-scaled FP8 GEMM of pre-quantised activations");
  m.def("quant_e4m3", &ns::quant_e4m3);
  m.def("add_norm", &ns::add_norm, py::arg("x"), py::arg("y"), py::arg("w"), py::arg("eps"), py::arg("x_out"),
        py::arg("n_out"), py::arg("q_out"), py::arg("s_out"));
  m.def("add_norm_peer", &ns::add_norm_peer);
  m.def("silu_mul_quant", &ns::silu_mul_quant);
  m.def("gated_norm_quant", &ns::gated_norm_quant);
  m.def("conv_silu_vec", &ns::conv_silu_vec);
  m.def("head_norm_rope", &ns::head_norm_rope, "(1+w)-RMSNorm per head row + partial RoPE");
  m.def("vattn_fwd", &ns::vattn_fwd, "causal GQA flash attention (tcgen05) with sigmoid output gate");
  m.def("device_error", &ns::device_error, "read the kernels' bounded-wait error word");
  m.def("clear_device_error", &ns::clear_device_error);
  m.def("device_error_tensor", &ns::device_error_tensor, "the error word as a 1-element int32 CUDA view");
  m.def("reset_device_error_state", &ns::reset_device_error_state,
        "after a timed-out wait: clear split-K counters and the error word");
}

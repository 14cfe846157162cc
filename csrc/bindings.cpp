// Python bindings of the sm_100a kernels (module dmad_b200._C).
#include <torch/extension.h>
#include <vector>

namespace dmad {
void register_h2d_stream(pybind11::module& m);
void fsdp_reduce_scatter(std::vector<int64_t> slot_ptrs, at::Tensor& acc, int64_t off, int64_t len, bool accumulate);
void flash_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
               double scale);
void flash_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
               const at::Tensor& dout, const at::Tensor& lse2, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
               at::Tensor& dd_scratch, double scale);
void flash_bwd_fused(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                     const at::Tensor& dout, const at::Tensor& lse2, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
                     at::Tensor& dd_scratch, at::Tensor& dq_acc, double scale);
int64_t flash_lse_pad(int64_t L);
int64_t device_status(int64_t device, bool reset);
void ln_mod_fwd(const at::Tensor& x, at::Tensor& y, c10::optional<at::Tensor> mean, at::Tensor& rstd,
                c10::optional<at::Tensor> a, c10::optional<at::Tensor> c, double a_add, int64_t rows_per_group,
                c10::optional<at::Tensor> gidx, double eps, bool rms);
void ln_mod_bwd(const at::Tensor& dy, const at::Tensor& x, c10::optional<at::Tensor> mean, const at::Tensor& rstd,
                c10::optional<at::Tensor> a, double a_add, int64_t rows_per_group, c10::optional<at::Tensor> gidx,
                bool rms, at::Tensor& dx, c10::optional<at::Tensor> dres, c10::optional<at::Tensor> da,
                c10::optional<at::Tensor> dc, c10::optional<at::Tensor> gate, c10::optional<at::Tensor> yg,
                c10::optional<at::Tensor> dyg, c10::optional<at::Tensor> dgate);
void gate_res_fwd(const at::Tensor& x, const at::Tensor& y, at::Tensor& out, c10::optional<at::Tensor> gate,
                  int64_t rows_per_group, c10::optional<at::Tensor> gidx);
void gate_res_bwd(const at::Tensor& dout, const at::Tensor& y, at::Tensor& dy, const at::Tensor& gate,
                  at::Tensor& dgate, int64_t rows_per_group, c10::optional<at::Tensor> gidx);
void qk_norm_rope_fwd(const at::Tensor& src, at::Tensor& dst, const at::Tensor& wq, const at::Tensor& wk,
                      const at::Tensor& cosT, const at::Tensor& sinT, at::Tensor& rstd_q, at::Tensor& rstd_k,
                      int64_t D, int64_t hd, double eps);
void qk_norm_rope_bwd(const at::Tensor& gq, const at::Tensor& gk, const at::Tensor& src, at::Tensor& dx,
                      const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& cosT, const at::Tensor& sinT,
                      const at::Tensor& rstd_q, const at::Tensor& rstd_k, at::Tensor& dwq, at::Tensor& dwk, int64_t D,
                      int64_t hd);
void rope_apply(const at::Tensor& x, at::Tensor& y, const at::Tensor& cosT, const at::Tensor& sinT, int64_t hd,
                bool inverse);
void gelu_fwd(const at::Tensor& x, at::Tensor& y);
at::Tensor sn_weight_fwd(const at::Tensor& w, at::Tensor& u, at::Tensor& v, const at::Tensor& gain,
                         at::Tensor& scale, at::Tensor& sigma, std::vector<int64_t> offsets, std::vector<int64_t> on,
                         bool train);
at::Tensor sn_weight_bwd(const at::Tensor& g, const at::Tensor& w, const at::Tensor& u, const at::Tensor& v,
                         const at::Tensor& gain, const at::Tensor& scale, const at::Tensor& sigma,
                         std::vector<int64_t> offsets, std::vector<int64_t> on);
void gelu_bwd(const at::Tensor& g, const at::Tensor& x, at::Tensor& dx);
void fused_adamw(std::vector<at::Tensor> master, std::vector<at::Tensor> grads, std::vector<at::Tensor> exp_avg,
                 std::vector<at::Tensor> exp_avg_sq, std::vector<at::Tensor> lowp, std::vector<at::Tensor> ema,
                 double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step,
                 c10::optional<at::Tensor> grad_scale, double ema_beta);
void multi_sumsq(std::vector<at::Tensor> grads, at::Tensor& out);
void clip_scale(const at::Tensor& sumsq, at::Tensor& scale, double max_norm);
void sinusoid_embed(const at::Tensor& t, at::Tensor& out, int64_t dim, double max_period);
void small_linear(const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> bias, at::Tensor& y,
                  int64_t act_in);
void flash_jvp_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& tq,
                   c10::optional<at::Tensor> tk, c10::optional<at::Tensor> tv, at::Tensor& o, at::Tensor& to,
                   at::Tensor& lse, double scale);
void flash_jvp_accumulate(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& tq,
                          c10::optional<at::Tensor> tk, c10::optional<at::Tensor> tv, at::Tensor& o, at::Tensor& to,
                          at::Tensor& lse, at::Tensor& acc_o, at::Tensor& acc_u, at::Tensor& acc_lse,
                          at::Tensor& acc_mu, bool read, bool final_, double scale);
void flash_fwd_scatter(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                       double scale, std::vector<int64_t> scatter, int64_t ld, int64_t col);
void cp_qkv_push(const at::Tensor& src, std::vector<int64_t> dst, const at::Tensor& wq, const at::Tensor& wk,
                 const at::Tensor& cosT, const at::Tensor& sinT, at::Tensor& rstd_q, at::Tensor& rstd_k, int64_t B,
                 int64_t D, int64_t hd, int64_t rank, double eps);
void cp_seq_to_head(const at::Tensor& src, std::vector<int64_t> dst, int64_t B, int64_t D, int64_t n, int64_t hd,
                    int64_t rank);
void cp_head_to_seq(std::vector<at::Tensor> srcs, std::vector<int64_t> dst, int64_t ld, int64_t D, int64_t rank);
void gemm_bf16(const at::Tensor& a, const at::Tensor& b, c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2,
               c10::optional<at::Tensor> bias, at::Tensor& d, double alpha, int64_t act);
void gemm_bf16_ex(const at::Tensor& a, const at::Tensor& b, c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2,
                  c10::optional<at::Tensor> bias, c10::optional<at::Tensor> d, c10::optional<at::Tensor> d32,
                  double alpha, int64_t act, bool a_mn, bool b_mn, int64_t split);
void fsdp_gather(std::vector<int64_t> shard_ptrs, at::Tensor& dst, int64_t len, int64_t numel);
void flash_fwd_accumulate(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                          at::Tensor& lse, at::Tensor& acc_o, at::Tensor& acc_lse, bool read, bool final_,
                          double scale);
void peer_copy(at::Tensor& dst, int64_t src_ptr, int64_t nbytes);
void peer_copy_to(int64_t dst_ptr, const at::Tensor& src, int64_t nbytes);
void symm_barrier(const at::Tensor& buf_ptrs, int64_t rank, int64_t epoch, c10::optional<at::Tensor> payload,
                  double timeout_s);
void dp_sumsq(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs, int64_t mc_grads, int64_t mc_params,
              int64_t elem_size, int64_t off, int64_t len, at::Tensor& acc, bool force_finite);
void dp_adamw(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs, int64_t mc_grads, int64_t mc_params,
              int64_t elem_size, at::Tensor& master, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
              c10::optional<at::Tensor> ema, int64_t off, int64_t len, double lr, double beta1, double beta2,
              double eps, double weight_decay, int64_t step, double ema_beta, c10::optional<at::Tensor> slots,
              double max_norm, bool force_finite);
}  // namespace dmad

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dmad_b200 sm_100a kernels";
  m.def("flash_fwd", &dmad::flash_fwd);
  m.def("flash_bwd", &dmad::flash_bwd);
  m.def("flash_bwd_fused", &dmad::flash_bwd_fused);
  m.def("flash_lse_pad", &dmad::flash_lse_pad);
  m.def("device_status", &dmad::device_status);
  m.def("ln_mod_fwd", &dmad::ln_mod_fwd);
  m.def("ln_mod_bwd", &dmad::ln_mod_bwd);
  m.def("gate_res_fwd", &dmad::gate_res_fwd);
  m.def("gate_res_bwd", &dmad::gate_res_bwd);
  m.def("qk_norm_rope_fwd", &dmad::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &dmad::qk_norm_rope_bwd);
  m.def("rope_apply", &dmad::rope_apply);
  m.def("gelu_fwd", &dmad::gelu_fwd);
  m.def("sn_weight_fwd", &dmad::sn_weight_fwd);
  m.def("sn_weight_bwd", &dmad::sn_weight_bwd);
  m.def("gelu_bwd", &dmad::gelu_bwd);
  m.def("fused_adamw", &dmad::fused_adamw);
  m.def("multi_sumsq", &dmad::multi_sumsq);
  m.def("clip_scale", &dmad::clip_scale);
  m.def("sinusoid_embed", &dmad::sinusoid_embed);
  m.def("small_linear", &dmad::small_linear);
  m.def("flash_jvp_fwd", &dmad::flash_jvp_fwd);
  m.def("flash_jvp_accumulate", &dmad::flash_jvp_accumulate);
  m.def("flash_fwd_scatter", &dmad::flash_fwd_scatter);
  m.def("cp_qkv_push", &dmad::cp_qkv_push);
  m.def("cp_seq_to_head", &dmad::cp_seq_to_head);
  m.def("cp_head_to_seq", &dmad::cp_head_to_seq);
  m.def("gemm_bf16", &dmad::gemm_bf16);
  m.def("gemm_bf16_ex", &dmad::gemm_bf16_ex);
  m.def("fsdp_gather", &dmad::fsdp_gather);
  m.def("fsdp_reduce_scatter", &dmad::fsdp_reduce_scatter);
  m.def("flash_fwd_accumulate", &dmad::flash_fwd_accumulate);
  m.def("peer_copy", &dmad::peer_copy);
  m.def("peer_copy_to", &dmad::peer_copy_to);
  m.def("symm_barrier", &dmad::symm_barrier);
  m.def("dp_sumsq", &dmad::dp_sumsq);
  m.def("dp_adamw", &dmad::dp_adamw);
  dmad::register_h2d_stream(m);
}

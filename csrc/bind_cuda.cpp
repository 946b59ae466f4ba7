// Python bindings of the sm_100a kernels (module mtorus._cuda).
#include <torch/extension.h>

#include "kernels/launch_counter.h"

namespace mtorus {
// layernorm.cu
std::vector<at::Tensor> layernorm_fwd(const at::Tensor& x, const at::Tensor& gamma,
                                      const at::Tensor& beta, double eps);
std::vector<at::Tensor> layernorm_fwd_fp8(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta,
                                          double eps, at::Tensor y8, const at::Tensor& scale, at::Tensor amax,
                                          int64_t fmt, const c10::optional<at::Tensor>& counter,
                                          const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap,
                                          int64_t slot, int64_t parity, int64_t epoch, int64_t ep_ptr);
at::Tensor layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& gamma,
                         const at::Tensor& mean, const at::Tensor& rstd, at::Tensor dgamma,
                         at::Tensor dbeta, bool accumulate, const c10::optional<at::Tensor>& dres);
// xent.cu
at::Tensor xent_fused(at::Tensor logits, const at::Tensor& targets,
                      const c10::optional<at::Tensor>& grad_scale, double scale_mul,
                      bool write_grad, const c10::optional<at::Tensor>& out8,
                      const c10::optional<at::Tensor>& out8_scale, const c10::optional<at::Tensor>& out8_amax);
// optim.cu
void optim_grad_sumsq(const at::Tensor& g, at::Tensor st);
void optim_finalize(at::Tensor st, bool dynamic, int64_t growth_interval, double max_norm,
                    bool unscale);
void adam_step(at::Tensor p, at::Tensor m, at::Tensor v, const at::Tensor& g,
               c10::optional<at::Tensor> w16, const at::Tensor& st, double lr, double beta1,
               double beta2, double eps, double weight_decay, double step_override);
void sgd_step(at::Tensor p, const at::Tensor& g, c10::optional<at::Tensor> w16,
              const at::Tensor& st, double lr);
// elementwise.cu
at::Tensor embed_fwd(const at::Tensor& ids, const at::Tensor& wte, const at::Tensor& wpe, int64_t S,
                     const c10::optional<at::Tensor>& drop_rng, int64_t drop_site, int64_t drop_thr16,
                     double drop_scale);
void dropout_apply(const at::Tensor& x, at::Tensor out, const at::Tensor& rng, int64_t site, int64_t thr16,
                   double scale);
void dropout_advance(at::Tensor rng, int64_t base);
void embed_bwd(const at::Tensor& ids, const at::Tensor& dy, at::Tensor dwte, at::Tensor dwpe,
               int64_t S, bool accumulate);
at::Tensor bias_gelu_fwd(at::Tensor pre, const c10::optional<at::Tensor>& bias);
void gelu_bwd_(at::Tensor dact, const at::Tensor& pre);
void colsum_e5m2_(const at::Tensor& codes, at::Tensor out, bool accumulate, const c10::optional<at::Tensor>& scale,
                  const c10::optional<at::Tensor>& scale2);
void colsum_(const at::Tensor& x, at::Tensor out, bool accumulate,
             const c10::optional<at::Tensor>& scale);
// gemm.cu
void gemm_bf16(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor D,
               const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
               const c10::optional<at::Tensor>& act, const c10::optional<at::Tensor>& aux,
               const c10::optional<at::Tensor>& alpha, bool beta);
int64_t gemm_status(bool reset);
void gemm_set_reserved_sms(int64_t n);
void gemm_fp8(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
              int64_t b_fmt, at::Tensor D, const c10::optional<at::Tensor>& bias,
              const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
              const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha,
              const c10::optional<at::Tensor>& alpha2, bool beta);
void gemm_fp8_act8(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
                   int64_t b_fmt, at::Tensor D, const c10::optional<at::Tensor>& bias,
                   const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
                   const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha,
                   const c10::optional<at::Tensor>& alpha2, bool beta,
                   const c10::optional<at::Tensor>& act8, const c10::optional<at::Tensor>& act8_scale,
                   const c10::optional<at::Tensor>& act8_amax, int64_t act8_fmt);
void gemm_mxfp8(const at::Tensor& A, int64_t a_fmt, const at::Tensor& sfa, const at::Tensor& B,
                int64_t b_fmt, const at::Tensor& sfb, at::Tensor D, const c10::optional<at::Tensor>& bias,
                const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
                const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha, bool beta,
                const c10::optional<at::Tensor>& out_rc, const c10::optional<at::Tensor>& out_rsf,
                const c10::optional<at::Tensor>& out_cc, const c10::optional<at::Tensor>& out_csf, int64_t out_fmt,
                double out_fmax, const c10::optional<at::Tensor>& out_colsum, bool out_gelu, bool store_d);
void mx_quantize(const at::Tensor& x, at::Tensor codes, at::Tensor sf, int64_t fmt, double fmax);
void copy_async(int64_t dst, int64_t src, int64_t bytes);
void dp_quant_e5m2(int64_t grad, int64_t codes, int64_t sf, int64_t nelem);
void dp_decode_mean_e5m2(const at::Tensor& codes, const at::Tensor& sf, at::Tensor out);
void symm_rs_bucket_e5m2(const std::vector<int64_t>& codes, const std::vector<int64_t>& sfs,
                         const std::vector<int64_t>& flags, int64_t me, int64_t start, int64_t len, int64_t clen,
                         int64_t slot, int64_t epoch, at::Tensor st, int64_t ctas, double inv_n, int64_t mine,
                         int64_t ep_ptr);
void layernorm_fwd_mx_rc(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta, double eps,
                         at::Tensor rc, at::Tensor rsf, at::Tensor cc, at::Tensor csf, at::Tensor mean,
                         at::Tensor rstd, int64_t fmt, double fmax);
void mx_quantize_rc(const at::Tensor& x, at::Tensor rc, at::Tensor rsf, at::Tensor cc, at::Tensor csf, int64_t fmt,
                    double fmax, const c10::optional<at::Tensor>& colsum, const c10::optional<at::Tensor>& xq,
                    int64_t act, const c10::optional<at::Tensor>& aux);
void gemm_fp8_gather_b(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
                       int64_t b_fmt, const std::vector<int64_t>& b_peers, int64_t shard_rows, at::Tensor D,
                       const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
                       const c10::optional<at::Tensor>& act, const c10::optional<at::Tensor>& aux,
                       const c10::optional<at::Tensor>& alpha, const c10::optional<at::Tensor>& alpha2, bool beta);
// attention.cu
std::vector<at::Tensor> attn_fwd(const at::Tensor& qkv, int64_t B, int64_t S, int64_t H,
                                 const c10::optional<at::Tensor>& drop_rng, int64_t drop_site, int64_t drop_thr16,
                                 double drop_scale, const c10::optional<at::Tensor>& mx_rc,
                                 const c10::optional<at::Tensor>& mx_rsf, const c10::optional<at::Tensor>& mx_cc,
                                 const c10::optional<at::Tensor>& mx_csf, int64_t mx_fmt, double mx_fmax);
at::Tensor attn_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& lse,
                    int64_t B, int64_t S, int64_t H, const c10::optional<at::Tensor>& drop_rng, int64_t drop_site,
                    int64_t drop_thr16, double drop_scale, const c10::optional<at::Tensor>& dq_out);
int64_t attn_status(bool reset);
// fp8.cu
void fp8_quantize(const at::Tensor& x, at::Tensor out, const c10::optional<at::Tensor>& scale,
                  const c10::optional<at::Tensor>& amax, int64_t fmt);
void fp8_amax(const at::Tensor& x, at::Tensor amax);
void fp8_quantize_ar(const at::Tensor& x, at::Tensor out, const at::Tensor& scale, at::Tensor amax,
                     at::Tensor counter, const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap,
                     int64_t slot, int64_t parity, int64_t epoch, int64_t fmt, int64_t ep_ptr);
void fp8_amax_gather(const at::Tensor& table, at::Tensor amax, int64_t world, int64_t cap, int64_t parity,
                     int64_t epoch, int64_t ep_ptr);
void fp8_amax_publish(const at::Tensor& amax, const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap,
                      int64_t parity, int64_t epoch, int64_t ep_ptr);
void fp8_quantize_colsum(const at::Tensor& x, at::Tensor out, const at::Tensor& scale, at::Tensor amax,
                         at::Tensor colsum, bool accumulate, const c10::optional<at::Tensor>& counter,
                         const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap, int64_t slot,
                         int64_t parity, int64_t epoch, int64_t fmt, int64_t ep_ptr);
void fp8_scaling_update(at::Tensor hist, at::Tensor amax, at::Tensor scale, at::Tensor inv,
                        const at::Tensor& fmax, int64_t cursor, bool current,
                        const c10::optional<at::Tensor>& cursor_dev);
void fp8_dequantize(const at::Tensor& q, at::Tensor out, const at::Tensor& inv_scale, int64_t fmt);
void fp8_quantize_blocks(const at::Tensor& x, at::Tensor out, at::Tensor scales, int64_t block_size,
                         double fmax, int64_t fmt);
// symm.cu
int64_t symm_status(bool reset);
void symm_rs_bucket(const std::vector<int64_t>& grads, const std::vector<int64_t>& flags,
                    int64_t me, int64_t start, int64_t len, int64_t clen, int64_t slot,
                    int64_t epoch, at::Tensor st, int64_t ctas, double inv_n, int64_t ep_ptr);
void symm_rs_bucket_mc(int64_t grads_mc, const std::vector<int64_t>& grads, const std::vector<int64_t>& flags,
                       int64_t me, int64_t start, int64_t len, int64_t clen, int64_t slot, int64_t epoch,
                       at::Tensor st, int64_t ctas, double inv_n, int64_t ep_ptr);
void symm_scalars_ar(const std::vector<int64_t>& scal, const std::vector<int64_t>& flags,
                     int64_t me, int64_t slot, int64_t epoch, at::Tensor st, int64_t ep_ptr);
void symm_epoch_advance(at::Tensor ep);
void symm_adam_shard_ag(const at::Tensor& ranges, at::Tensor master, at::Tensor m, at::Tensor v,
                        const at::Tensor& grad, const std::vector<int64_t>& w16, const at::Tensor& st,
                        double lr, double beta1, double beta2, double eps, double wd, int64_t w16_mc);
void symm_barrier(const std::vector<int64_t>& flags, int64_t me, int64_t slot, int64_t epoch,
                  int64_t code, int64_t ep_ptr);
void symm_allreduce(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t me,
                    int64_t numel, int64_t dtype, int64_t slot, int64_t epoch, int64_t ctas);
void symm_allgather(int64_t src, const std::vector<int64_t>& dst, int64_t me, int64_t bytes,
                    int64_t ctas);
void symm_broadcast(const std::vector<int64_t>& bufs, int64_t root, int64_t bytes, int64_t ctas);
void symm_allreduce_mc(int64_t mc, const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags,
                       int64_t me, int64_t numel, int64_t dtype, int64_t slot, int64_t epoch, int64_t ctas);
void symm_broadcast_mc(int64_t src, int64_t mc, int64_t bytes, int64_t ctas);
void gemm_profile(bool on);
void gemm_set_dropout(const c10::optional<at::Tensor>& rng, int64_t site, int64_t thr16, double scale, int64_t mode);
std::vector<int64_t> gemm_profile_read();
void fp8_wire_encode(const at::Tensor& x, at::Tensor codes, at::Tensor sf, int64_t fmt);
void fp8_wire_decode(const at::Tensor& codes, const at::Tensor& sf, at::Tensor out, int64_t fmt);
void symm_pull_msgs(const std::vector<int64_t>& src, int64_t src_off, int64_t dst, int64_t slot_bytes,
                    const std::vector<int64_t>& peers, const std::vector<int64_t>& slots, int64_t ctas_per_msg);
void symm_allreduce_msgs(const std::vector<int64_t>& src, int64_t src_off, int64_t dst, int64_t dtype, int64_t op,
                         int64_t cap, int64_t ctas);
void symm_flag(int64_t signal_addr, int64_t signal_value, int64_t wait_addr, int64_t wait_value, int64_t code);
void symm_halo(int64_t src, const std::vector<int64_t>& recv, const at::Tensor& nbr_rank,
               const at::Tensor& nbr_slot, int64_t bytes, int64_t ctas);
void install_segv_handler();
void wait_flag(const at::Tensor& flag, int64_t target, double limit_ms, at::Tensor status, int64_t code,
               at::Tensor waited);
}  // namespace mtorus

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace mtorus;
  namespace py = pybind11;
  m.doc() = "mtorus sm_100a kernels";
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("gamma"), py::arg("mean"),
        py::arg("rstd"), py::arg("dgamma"), py::arg("dbeta"), py::arg("accumulate"),
        py::arg("dres") = py::none());
  m.def("xent_fused", &xent_fused, py::arg("logits"), py::arg("targets"),
        py::arg("grad_scale") = py::none(), py::arg("scale_mul") = 1.0,
        py::arg("write_grad") = true, py::arg("out8") = py::none(), py::arg("out8_scale") = py::none(),
        py::arg("out8_amax") = py::none());
  m.def("optim_grad_sumsq", &optim_grad_sumsq);
  m.def("optim_finalize", &optim_finalize);
  m.def("adam_step", &adam_step);
  m.def("sgd_step", &sgd_step);
  m.def("embed_fwd", &embed_fwd, py::arg("ids"), py::arg("wte"), py::arg("wpe"), py::arg("S"),
        py::arg("drop_rng") = py::none(), py::arg("drop_site") = 0, py::arg("drop_thr16") = 0,
        py::arg("drop_scale") = 1.0);
  m.def("dropout_apply", &dropout_apply);
  m.def("dropout_advance", &dropout_advance);
  m.def("embed_bwd", &embed_bwd);
  m.def("bias_gelu_fwd", &bias_gelu_fwd);
  m.def("gelu_bwd_", &gelu_bwd_);
  m.def("colsum_e5m2_", &colsum_e5m2_, py::arg("codes"), py::arg("out"), py::arg("accumulate"),
        py::arg("scale") = py::none(), py::arg("scale2") = py::none());
  m.def("colsum_", &colsum_, py::arg("x"), py::arg("out"), py::arg("accumulate"),
        py::arg("scale") = py::none());
  m.def("gemm_bf16", &gemm_bf16, py::arg("A"), py::arg("a_mn"), py::arg("B"), py::arg("b_mn"),
        py::arg("D"), py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("act") = py::none(), py::arg("aux") = py::none(), py::arg("alpha") = py::none(),
        py::arg("beta") = false);
  m.def("gemm_status", &gemm_status, py::arg("reset") = true);
  m.def("gemm_set_reserved_sms", &gemm_set_reserved_sms);
  m.def("gemm_fp8", &gemm_fp8, py::arg("A"), py::arg("a_mn"), py::arg("a_fmt"), py::arg("B"), py::arg("b_mn"),
        py::arg("b_fmt"), py::arg("D"), py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("act") = py::none(), py::arg("aux") = py::none(), py::arg("alpha") = py::none(),
        py::arg("alpha2") = py::none(), py::arg("beta") = false);
  m.def("fp8_quantize", &fp8_quantize, py::arg("x"), py::arg("out"), py::arg("scale") = py::none(),
        py::arg("amax") = py::none(), py::arg("fmt") = 0);
  m.def("fp8_amax", &fp8_amax);
  m.def("fp8_scaling_update", &fp8_scaling_update, py::arg("hist"), py::arg("amax"), py::arg("scale"),
        py::arg("inv"), py::arg("fmax"), py::arg("cursor"), py::arg("current"), py::arg("cursor_dev") = py::none());
  m.def("fp8_dequantize", &fp8_dequantize);
  m.def("fp8_quantize_blocks", &fp8_quantize_blocks);
  m.def("symm_status", &symm_status, py::arg("reset") = true);
  // ep_ptr: address of a device-resident uint32 step counter added to `epoch` in the
  // kernels (0: none), which lets a captured CUDA graph replay with fresh epochs
  m.def("symm_rs_bucket", &symm_rs_bucket, py::arg("grads"), py::arg("flags"), py::arg("me"), py::arg("start"),
        py::arg("len"), py::arg("clen"), py::arg("slot"), py::arg("epoch"), py::arg("st"), py::arg("ctas"),
        py::arg("inv_n"), py::arg("ep_ptr") = 0);
  m.def("symm_rs_bucket_mc", &symm_rs_bucket_mc, py::arg("grads_mc"), py::arg("grads"), py::arg("flags"),
        py::arg("me"), py::arg("start"), py::arg("len"), py::arg("clen"), py::arg("slot"), py::arg("epoch"),
        py::arg("st"), py::arg("ctas"), py::arg("inv_n"), py::arg("ep_ptr") = 0);
  m.def("symm_scalars_ar", &symm_scalars_ar, py::arg("scal"), py::arg("flags"), py::arg("me"), py::arg("slot"),
        py::arg("epoch"), py::arg("st"), py::arg("ep_ptr") = 0);
  m.def("symm_adam_shard_ag", &symm_adam_shard_ag, py::arg("ranges"), py::arg("master"), py::arg("m"),
        py::arg("v"), py::arg("grad"), py::arg("w16"), py::arg("st"), py::arg("lr"), py::arg("beta1"),
        py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("w16_mc") = 0);
  m.def("symm_barrier", &symm_barrier, py::arg("flags"), py::arg("me"), py::arg("slot"), py::arg("epoch"),
        py::arg("code"), py::arg("ep_ptr") = 0);
  m.def("symm_epoch_advance", &symm_epoch_advance);
  m.def("symm_allreduce", &symm_allreduce);
  m.def("symm_allgather", &symm_allgather);
  m.def("symm_broadcast", &symm_broadcast);
  m.def("symm_halo", &symm_halo);
  m.def("symm_pull_msgs", &symm_pull_msgs);
  m.def("fp8_wire_encode", &fp8_wire_encode);
  m.def("gemm_profile", &gemm_profile);
  m.def("gemm_set_dropout", &gemm_set_dropout);
  m.def("gemm_profile_read", &gemm_profile_read);
  m.def("fp8_wire_decode", &fp8_wire_decode);
  m.def("symm_allreduce_msgs", &symm_allreduce_msgs);
  m.def("symm_flag", &symm_flag);
  m.def("symm_allreduce_mc", &symm_allreduce_mc);
  m.def("symm_broadcast_mc", &symm_broadcast_mc);
  m.def("install_segv_handler", &install_segv_handler);
  m.def("wait_flag", &wait_flag);
  m.def("launch_count", []() { return mtorus::launch_counter(); });
  m.def("fp8_quantize_ar", &fp8_quantize_ar, py::arg("x"), py::arg("out"), py::arg("scale"), py::arg("amax"),
        py::arg("counter"), py::arg("table_ptrs"), py::arg("me"), py::arg("cap"), py::arg("slot"), py::arg("parity"),
        py::arg("epoch"), py::arg("fmt"), py::arg("ep_ptr") = 0);
  m.def("layernorm_fwd_fp8", &layernorm_fwd_fp8, py::arg("x"), py::arg("gamma"), py::arg("beta"), py::arg("eps"),
        py::arg("y8"), py::arg("scale"), py::arg("amax"), py::arg("fmt"), py::arg("counter"), py::arg("table_ptrs"),
        py::arg("me"), py::arg("cap"), py::arg("slot"), py::arg("parity"), py::arg("epoch"), py::arg("ep_ptr") = 0);
  m.def("gemm_fp8_act8", &gemm_fp8_act8);
  m.def("gemm_mxfp8", &gemm_mxfp8, py::arg("A"), py::arg("a_fmt"), py::arg("sfa"), py::arg("B"), py::arg("b_fmt"),
        py::arg("sfb"), py::arg("D"), py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("act") = py::none(), py::arg("aux") = py::none(), py::arg("alpha") = py::none(),
        py::arg("beta") = false, py::arg("out_rc") = py::none(), py::arg("out_rsf") = py::none(),
        py::arg("out_cc") = py::none(), py::arg("out_csf") = py::none(), py::arg("out_fmt") = 0,
        py::arg("out_fmax") = 448.0, py::arg("out_colsum") = py::none(), py::arg("out_gelu") = false,
        py::arg("store_d") = true);
  m.def("mx_quantize", &mx_quantize);
  m.def("copy_async", &copy_async);
  m.def("dp_quant_e5m2", &dp_quant_e5m2);
  m.def("dp_decode_mean_e5m2", &dp_decode_mean_e5m2);
  m.def("symm_rs_bucket_e5m2", &symm_rs_bucket_e5m2, py::arg("codes"), py::arg("sfs"), py::arg("flags"),
        py::arg("me"), py::arg("start"), py::arg("len"), py::arg("clen"), py::arg("slot"), py::arg("epoch"),
        py::arg("st"), py::arg("ctas"), py::arg("inv_n"), py::arg("mine"), py::arg("ep_ptr") = 0);
  m.def("layernorm_fwd_mx_rc", &layernorm_fwd_mx_rc);
  m.def("mx_quantize_rc", &mx_quantize_rc, py::arg("x"), py::arg("rc"), py::arg("rsf"), py::arg("cc"),
        py::arg("csf"), py::arg("fmt"), py::arg("fmax"), py::arg("colsum") = py::none(), py::arg("xq") = py::none(),
        py::arg("act") = 0, py::arg("aux") = py::none());
  m.def("gemm_fp8_gather_b", &gemm_fp8_gather_b, py::arg("A"), py::arg("a_mn"), py::arg("a_fmt"), py::arg("B"),
        py::arg("b_mn"), py::arg("b_fmt"), py::arg("b_peers"), py::arg("shard_rows"), py::arg("D"),
        py::arg("bias") = py::none(), py::arg("residual") = py::none(), py::arg("act") = py::none(),
        py::arg("aux") = py::none(), py::arg("alpha") = py::none(), py::arg("alpha2") = py::none(),
        py::arg("beta") = false);
  m.def("fp8_amax_gather", &fp8_amax_gather, py::arg("table"), py::arg("amax"), py::arg("world"), py::arg("cap"),
        py::arg("parity"), py::arg("epoch"), py::arg("ep_ptr") = 0);
  m.def("fp8_amax_publish", &fp8_amax_publish, py::arg("amax"), py::arg("table_ptrs"), py::arg("me"), py::arg("cap"),
        py::arg("parity"), py::arg("epoch"), py::arg("ep_ptr") = 0);
  m.def("fp8_quantize_colsum", &fp8_quantize_colsum, py::arg("x"), py::arg("out"), py::arg("scale"), py::arg("amax"),
        py::arg("colsum"), py::arg("accumulate"), py::arg("counter"), py::arg("table_ptrs"), py::arg("me"),
        py::arg("cap"), py::arg("slot"), py::arg("parity"), py::arg("epoch"), py::arg("fmt"), py::arg("ep_ptr") = 0);
  m.def("attn_fwd", &attn_fwd, py::arg("qkv"), py::arg("B"), py::arg("S"), py::arg("H"),
        py::arg("drop_rng") = py::none(), py::arg("drop_site") = 0, py::arg("drop_thr16") = 0,
        py::arg("drop_scale") = 1.0, py::arg("mx_rc") = py::none(), py::arg("mx_rsf") = py::none(),
        py::arg("mx_cc") = py::none(), py::arg("mx_csf") = py::none(), py::arg("mx_fmt") = 0,
        py::arg("mx_fmax") = 448.0);
  m.def("attn_bwd", &attn_bwd, py::arg("dout"), py::arg("qkv"), py::arg("out"), py::arg("lse"), py::arg("B"),
        py::arg("S"), py::arg("H"), py::arg("drop_rng") = py::none(), py::arg("drop_site") = 0,
        py::arg("drop_thr16") = 0, py::arg("drop_scale") = 1.0, py::arg("dq_out") = py::none());
  m.def("attn_status", &attn_status, py::arg("reset") = true);
}

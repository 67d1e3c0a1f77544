// Python bindings of the cq_pretrain_b200 sm_100a kernel library.
#include <torch/extension.h>

#include <atomic>
#include <vector>

namespace cqb {
std::atomic<long long>& launch_counter() {
  static std::atomic<long long> counter{0};
  return counter;
}
long long launch_count() { return launch_counter().load(); }

// rowops.cu
std::vector<at::Tensor> rms_norm_fwd(at::Tensor x, at::Tensor w, double eps, c10::optional<at::Tensor> add);
std::vector<at::Tensor> rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                                     c10::optional<at::Tensor> dres);
std::vector<at::Tensor> gated_norm_fwd(at::Tensor x, at::Tensor z, at::Tensor w, double eps);
std::vector<at::Tensor> gated_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor z, at::Tensor w, at::Tensor rstd);
std::vector<at::Tensor> ln_modulate_fwd(at::Tensor x, at::Tensor scale, at::Tensor shift, at::Tensor idx, double eps);
std::vector<at::Tensor> ln_modulate_bwd(at::Tensor dy, at::Tensor x, at::Tensor scale, at::Tensor idx, at::Tensor mean,
                                        at::Tensor rstd);
at::Tensor gated_add_fwd(at::Tensor x, at::Tensor branch, at::Tensor gate, at::Tensor idx);
std::vector<at::Tensor> gated_add_bwd(at::Tensor dy, at::Tensor branch, at::Tensor gate, at::Tensor idx);
at::Tensor swiglu_fwd(at::Tensor x);
at::Tensor column_sum(at::Tensor x);
at::Tensor rope_pairs(at::Tensor x, at::Tensor cos_t, at::Tensor sin_t, bool inverse);
at::Tensor swiglu_bwd(at::Tensor dy, at::Tensor x);
// gemm.cu
at::Tensor gemm_nt(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias);
at::Tensor gemm_dual(at::Tensor x, at::Tensor w, at::Tensor x2, at::Tensor w2, bool w_mn_major);
at::Tensor gemm_nn(at::Tensor a, at::Tensor b);
void gemm_tn_acc(at::Tensor a, at::Tensor b, at::Tensor out);
int gemm_status(bool reset);
std::vector<at::Tensor> ce_partials(at::Tensor h, at::Tensor w, at::Tensor targets, int64_t lo);
std::vector<at::Tensor> ce_stats(at::Tensor h, at::Tensor w, at::Tensor targets, int64_t lo);
at::Tensor ce_grad_logits(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor lse, int64_t lo,
                          at::Tensor scale);
void gemm_scatter(at::Tensor x, at::Tensor w, bool w_mn_major, at::Tensor peer_out_ptrs, int64_t rows_per_rank,
                  int64_t src_rank, int64_t tp);
at::Tensor gather_gemm(at::Tensor a_local, at::Tensor w, c10::optional<at::Tensor> bias, at::Tensor peer_in_ptrs,
                       int64_t ready_ptr, at::Tensor chunk_flags, int64_t epoch, int64_t rows_per_rank, int64_t src_rank,
                       int64_t tp, bool mn_major, c10::optional<at::Tensor> x_local, int64_t send_mine,
                       c10::optional<at::Tensor> peer_ready, int64_t own_done, int64_t epoch_ctr, int64_t epoch_done,
                       c10::optional<at::Tensor> peer_in_odd, int64_t send_mine_odd);
// comm.cu
std::vector<at::Tensor> symm_alloc(int64_t bytes);
int64_t symm_open(at::Tensor handle_bytes);
void symm_close(int64_t ptr);
void symm_free(int64_t ptr);
at::Tensor symm_view(int64_t base, int64_t offset, std::vector<int64_t> shape, at::ScalarType dtype);
void signal_wait(at::Tensor peer_flag_ptrs, int64_t my_flags, int64_t rank, int64_t tp, int64_t epoch, bool wait);
at::Tensor gemm_scatter_reduce(at::Tensor x, at::Tensor w, bool w_mn_major, c10::optional<at::Tensor> x2,
                               c10::optional<at::Tensor> w2, c10::optional<at::Tensor> bias, at::Tensor peer_recv,
                               int64_t my_recv, at::Tensor peer_flags, int64_t my_flags, int64_t flag_slots,
                               int64_t epoch, int64_t rows_per_rank, int64_t src_rank, int64_t tp,
                               int64_t epoch_ctr, int64_t epoch_done, c10::optional<at::Tensor> peer_recv_odd,
                               int64_t my_recv_odd);
at::Tensor rs_reduce(at::Tensor recv, c10::optional<at::Tensor> bias, int64_t tp, int64_t rows, int64_t cols);
int comm_status_read(bool reset);
std::vector<at::Tensor> ce_combine_tp(at::Tensor part, at::Tensor tgt_local, at::Tensor peer_recv, int64_t my_recv,
                                      at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp,
                                      int64_t max_rows, int64_t epoch, int64_t epoch_ctr, int64_t epoch_done,
                                      c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd);
std::vector<at::Tensor> tp_rms_fwd(at::Tensor x, at::Tensor w, at::Tensor peer_recv, int64_t my_recv,
                                   at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp, int64_t max_rows,
                                   int64_t epoch, int64_t total_dim, double eps, int64_t epoch_ctr, int64_t epoch_done,
                                   c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd);
std::vector<at::Tensor> tp_rms_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, at::Tensor peer_recv,
                                   int64_t my_recv, at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp,
                                   int64_t max_rows, int64_t epoch, int64_t total_dim, int64_t epoch_ctr, int64_t epoch_done,
                                   c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd);
std::vector<at::Tensor> qk_norm_rope_fwd(at::Tensor q, at::Tensor k, at::Tensor wq, at::Tensor wk,
                                         c10::optional<at::Tensor> cos_t, c10::optional<at::Tensor> sin_t,
                                         int64_t head_dim, int64_t total_dim, double eps,
                                         c10::optional<at::Tensor> peer_recv, int64_t my_recv,
                                         c10::optional<at::Tensor> peer_flags, int64_t my_flags, int64_t rank,
                                         int64_t tp, int64_t max_rows, int64_t epoch_ctr, int64_t epoch_done,
                                         c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd);
std::vector<at::Tensor> qk_norm_rope_bwd(at::Tensor dyq, at::Tensor dyk, at::Tensor q, at::Tensor k, at::Tensor wq,
                                         at::Tensor wk, at::Tensor rstd, c10::optional<at::Tensor> cos_t,
                                         c10::optional<at::Tensor> sin_t, int64_t head_dim, int64_t total_dim,
                                         c10::optional<at::Tensor> peer_recv, int64_t my_recv,
                                         c10::optional<at::Tensor> peer_flags, int64_t my_flags, int64_t rank,
                                         int64_t tp, int64_t max_rows, int64_t epoch_ctr, int64_t epoch_done,
                                         c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd);
// gdn.cu
std::vector<at::Tensor> gdn_fwd(at::Tensor W, at::Tensor U, at::Tensor P, at::Tensor Qd, at::Tensor Kt, at::Tensor gamma,
                                at::Tensor start, at::Tensor count, bool want_final);
void gdn_decode_step(at::Tensor state, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                     at::Tensor out);
at::Tensor gdn_bwd(at::Tensor dO, at::Tensor W, at::Tensor P, at::Tensor Qd, at::Tensor Kt, at::Tensor gamma,
                   at::Tensor start, at::Tensor count);
// moss.cu
at::Tensor moss_pointwise_fwd(int64_t kind, at::Tensor a, at::Tensor b, at::Tensor c);
std::vector<at::Tensor> moss_pointwise_bwd(int64_t kind, at::Tensor dy, at::Tensor a, at::Tensor b, at::Tensor c);
// attention.cu
std::vector<at::Tensor> attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor kstart, at::Tensor kend,
                                    double scale);
std::vector<at::Tensor> attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                                    at::Tensor lse, at::Tensor kstart, at::Tensor kend, double scale);
int attn_status(bool reset);
// gdn_chunk.cu
std::vector<at::Tensor> gdn_prep(at::Tensor Q, at::Tensor K, at::Tensor V, at::Tensor G, at::Tensor B);
int64_t gdn_status(bool reset);
std::vector<at::Tensor> gdn_chunk_bwd(at::Tensor Q, at::Tensor K, at::Tensor V, at::Tensor dO, at::Tensor G,
                                      at::Tensor B, at::Tensor S, at::Tensor dS, c10::optional<at::Tensor> dgamma);
// gather.cu
at::Tensor gather_rows(at::Tensor src0, c10::optional<at::Tensor> src1, at::Tensor idx);
std::vector<at::Tensor> gather_rows_bwd(at::Tensor grad, at::Tensor inv, int64_t n0, int64_t n1);
// conv.cu
at::Tensor conv_fwd(at::Tensor x, at::Tensor w, at::Tensor pos);
std::vector<at::Tensor> conv_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor pos);
std::vector<at::Tensor> chunk_gather(at::Tensor x, at::Tensor idx, int64_t chunks, bool normalize, double scale);
at::Tensor qconv_fwd(at::Tensor raw, at::Tensor updates, at::Tensor w, at::Tensor qs, at::Tensor qh);
std::vector<at::Tensor> qconv_bwd(at::Tensor dy, at::Tensor raw, at::Tensor updates, at::Tensor w, at::Tensor qs,
                                  at::Tensor qh, at::Tensor hist_rows, at::Tensor hist_offsets,
                                  at::Tensor hist_entries);
std::vector<at::Tensor> qconv_bwd_into(at::Tensor dy, at::Tensor raw, at::Tensor updates, at::Tensor w,
                                       at::Tensor qs, at::Tensor qh, at::Tensor hist_rows, at::Tensor hist_offsets,
                                       at::Tensor hist_entries, at::Tensor d_upd);
void qconv_raw_grad(at::Tensor g, at::Tensor w, at::Tensor qs, at::Tensor d_raw);
at::Tensor chunk_scatter(at::Tensor dyc, at::Tensor slot_of, at::Tensor x, at::Tensor rnorm, bool normalize,
                         double scale);
// optim.cu
void adamw_step(std::vector<at::Tensor> masters, std::vector<at::Tensor> grads, std::vector<at::Tensor> exp_avg,
                std::vector<at::Tensor> exp_avg_sq, std::vector<at::Tensor> decay, std::vector<at::Tensor> params,
                at::Tensor gscale, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                std::vector<at::Tensor> ema, double ema_weight);
at::Tensor sum_squares(std::vector<at::Tensor> xs);
}  // namespace cqb

namespace cqb {
void rows_accumulate(at::Tensor grad, at::Tensor order, at::Tensor seg_start, at::Tensor run_seg, at::Tensor ids,
                     at::Tensor out);
}  // namespace cqb

#ifdef CQB_DEBUG_BOUNDS
namespace cqb {
std::vector<int64_t> debug_status_gather(bool reset);
std::vector<int64_t> debug_status_conv(bool reset);
}  // namespace cqb
#endif

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "cq_pretrain_b200 sm_100a kernels";
  m.def("launch_count", &cqb::launch_count);
  m.def("rms_norm_fwd", &cqb::rms_norm_fwd, py::arg("x"), py::arg("w"), py::arg("eps"), py::arg("add") = py::none());
  m.def("rms_norm_bwd", &cqb::rms_norm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("dres") = py::none());
  m.def("gated_norm_fwd", &cqb::gated_norm_fwd);
  m.def("gated_norm_bwd", &cqb::gated_norm_bwd);
  m.def("ln_modulate_fwd", &cqb::ln_modulate_fwd);
  m.def("ln_modulate_bwd", &cqb::ln_modulate_bwd);
  m.def("gated_add_fwd", &cqb::gated_add_fwd);
  m.def("gated_add_bwd", &cqb::gated_add_bwd);
  m.def("swiglu_fwd", &cqb::swiglu_fwd);
  m.def("column_sum", &cqb::column_sum);
  m.def("rope_pairs", &cqb::rope_pairs);
  m.def("swiglu_bwd", &cqb::swiglu_bwd);
  m.def("gemm_dual", &cqb::gemm_dual);
  m.def("gemm_nt", &cqb::gemm_nt, py::arg("x"), py::arg("w"), py::arg("bias") = py::none());
  m.def("gemm_nn", &cqb::gemm_nn);
  m.def("gemm_tn_acc", &cqb::gemm_tn_acc);
  m.def("gemm_status", &cqb::gemm_status, py::arg("reset") = false);
  m.def("ce_stats", &cqb::ce_stats);
  m.def("ce_partials", &cqb::ce_partials);
  m.def("ce_grad_logits", &cqb::ce_grad_logits);
  m.def("gemm_scatter", &cqb::gemm_scatter);
  m.def("gather_gemm", &cqb::gather_gemm, py::arg("a_local"), py::arg("w"), py::arg("bias"), py::arg("peer_in_ptrs"),
        py::arg("ready_ptr"), py::arg("chunk_flags"), py::arg("epoch"), py::arg("rows_per_rank"), py::arg("src_rank"),
        py::arg("tp"), py::arg("mn_major") = false, py::arg("x_local") = py::none(), py::arg("send_mine") = 0,
        py::arg("peer_ready") = py::none(), py::arg("own_done") = 0, py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0,
        py::arg("peer_in_odd") = py::none(), py::arg("send_mine_odd") = 0);
  m.def("symm_alloc", &cqb::symm_alloc);
  m.def("symm_open", &cqb::symm_open);
  m.def("symm_close", &cqb::symm_close);
  m.def("symm_free", &cqb::symm_free);
  m.def("symm_view", &cqb::symm_view);
  m.def("signal_wait", &cqb::signal_wait);
  m.def("rows_accumulate", &cqb::rows_accumulate);
#ifdef CQB_DEBUG_BOUNDS
  // First out-of-range index seen by the checked kernels: {site, index, bound} (zeros when none).
  m.def("debug_bounds_status", [](bool reset) {
    for (auto* fn : {&cqb::debug_status_gather, &cqb::debug_status_conv}) {
      auto v = fn(reset);
      if (v[0] != 0) return v;
    }
    return std::vector<int64_t>{0, 0, 0};
  }, py::arg("reset") = true);
#endif
  m.def("gemm_scatter_reduce", &cqb::gemm_scatter_reduce, py::arg("x"), py::arg("w"), py::arg("w_mn_major"),
        py::arg("x2"), py::arg("w2"), py::arg("bias"), py::arg("peer_recv"), py::arg("my_recv"), py::arg("peer_flags"),
        py::arg("my_flags"), py::arg("flag_slots"), py::arg("epoch"), py::arg("rows_per_rank"), py::arg("src_rank"),
        py::arg("tp"), py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0, py::arg("peer_recv_odd") = py::none(),
        py::arg("my_recv_odd") = 0);
  m.def("qk_norm_rope_fwd", &cqb::qk_norm_rope_fwd, py::arg("q"), py::arg("k"), py::arg("wq"), py::arg("wk"),
        py::arg("cos") = py::none(), py::arg("sin") = py::none(), py::arg("head_dim") = 0, py::arg("total_dim"),
        py::arg("eps"), py::arg("peer_recv") = py::none(), py::arg("my_recv") = 0, py::arg("peer_flags") = py::none(),
        py::arg("my_flags") = 0, py::arg("rank") = 0, py::arg("tp") = 1, py::arg("max_rows") = 0,
        py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0, py::arg("peer_recv_odd") = py::none(),
        py::arg("my_recv_odd") = 0);
  m.def("qk_norm_rope_bwd", &cqb::qk_norm_rope_bwd, py::arg("dyq"), py::arg("dyk"), py::arg("q"), py::arg("k"),
        py::arg("wq"), py::arg("wk"), py::arg("rstd"), py::arg("cos") = py::none(), py::arg("sin") = py::none(),
        py::arg("head_dim") = 0, py::arg("total_dim"), py::arg("peer_recv") = py::none(), py::arg("my_recv") = 0, py::arg("peer_flags") = py::none(),
        py::arg("my_flags") = 0, py::arg("rank") = 0, py::arg("tp") = 1, py::arg("max_rows") = 0,
        py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0, py::arg("peer_recv_odd") = py::none(),
        py::arg("my_recv_odd") = 0);
  m.def("rs_reduce", &cqb::rs_reduce);
  m.def("comm_status_read", &cqb::comm_status_read, py::arg("reset") = false);
  m.def("tp_rms_fwd", &cqb::tp_rms_fwd, py::arg("x"), py::arg("w"), py::arg("peer_recv"), py::arg("my_recv"),
        py::arg("peer_flags"), py::arg("my_flags"), py::arg("rank"), py::arg("tp"), py::arg("max_rows"),
        py::arg("epoch"), py::arg("total_dim"), py::arg("eps"), py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0,
        py::arg("peer_recv_odd") = py::none(), py::arg("my_recv_odd") = 0);
  m.def("ce_combine_tp", &cqb::ce_combine_tp, py::arg("part"), py::arg("tgt_local"), py::arg("peer_recv"),
        py::arg("my_recv"), py::arg("peer_flags"), py::arg("my_flags"), py::arg("rank"), py::arg("tp"),
        py::arg("max_rows"), py::arg("epoch"), py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0,
        py::arg("peer_recv_odd") = py::none(), py::arg("my_recv_odd") = 0);
  m.def("tp_rms_bwd", &cqb::tp_rms_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("peer_recv"), py::arg("my_recv"), py::arg("peer_flags"), py::arg("my_flags"), py::arg("rank"),
        py::arg("tp"), py::arg("max_rows"), py::arg("epoch"), py::arg("total_dim"), py::arg("epoch_ctr") = 0, py::arg("epoch_done") = 0,
        py::arg("peer_recv_odd") = py::none(), py::arg("my_recv_odd") = 0);
  m.def("gdn_fwd", &cqb::gdn_fwd, py::arg("W"), py::arg("U"), py::arg("P"), py::arg("Qd"), py::arg("Kt"),
        py::arg("gamma"), py::arg("start"), py::arg("count"), py::arg("want_final") = false);
  m.def("gdn_decode_step", &cqb::gdn_decode_step);
  m.def("gdn_bwd", &cqb::gdn_bwd);
  m.def("moss_pointwise_fwd", &cqb::moss_pointwise_fwd);
  m.def("moss_pointwise_bwd", &cqb::moss_pointwise_bwd);
  m.def("attn_fwd", &cqb::attn_fwd);
  m.def("attn_bwd", &cqb::attn_bwd);
  m.def("attn_status", &cqb::attn_status, py::arg("reset") = false);
  m.def("adamw_step", &cqb::adamw_step, py::arg("masters"), py::arg("grads"), py::arg("exp_avg"),
        py::arg("exp_avg_sq"), py::arg("decay"), py::arg("params"), py::arg("gscale"), py::arg("lr"), py::arg("b1"),
        py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("bc1"), py::arg("bc2"),
        py::arg("ema") = std::vector<at::Tensor>{}, py::arg("ema_weight") = 0.0);
  m.def("sum_squares", &cqb::sum_squares);
  m.def("gdn_prep", &cqb::gdn_prep);
  m.def("gdn_status", &cqb::gdn_status, py::arg("reset") = false);
  m.def("gdn_chunk_bwd", &cqb::gdn_chunk_bwd, py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("dO"), py::arg("G"),
        py::arg("B"), py::arg("S"), py::arg("dS"), py::arg("dgamma") = py::none());
  m.def("gather_rows", &cqb::gather_rows);
  m.def("gather_rows_bwd", &cqb::gather_rows_bwd);
  m.def("conv_fwd", &cqb::conv_fwd);
  m.def("conv_bwd", &cqb::conv_bwd);
  m.def("chunk_gather", &cqb::chunk_gather);
  m.def("qconv_fwd", &cqb::qconv_fwd);
  m.def("qconv_bwd", &cqb::qconv_bwd);
  m.def("qconv_bwd_into", &cqb::qconv_bwd_into);
  m.def("qconv_raw_grad", &cqb::qconv_raw_grad);
  m.def("chunk_scatter", &cqb::chunk_scatter);
}

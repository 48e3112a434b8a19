// Python bindings of the art_mlx_b200 native kernels.
#include <torch/extension.h>

namespace art {
void ep_gemm(torch::Tensor x, torch::Tensor w, std::vector<int64_t> offs, int64_t N, bool w_transposed,
             c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> src,
             c10::optional<torch::Tensor> src_ext, c10::optional<torch::Tensor> push_tok,
             c10::optional<torch::Tensor> push_scale, c10::optional<torch::Tensor> push_rank,
             c10::optional<torch::Tensor> push_row, c10::optional<torch::Tensor> push_expert,
             c10::optional<torch::Tensor> push_meta, std::vector<int64_t> recv_x_ptrs,
             std::vector<int64_t> recv_ext_ptrs, std::vector<int64_t> recv_meta_ptrs, std::vector<int64_t> arrive_ptrs,
             c10::optional<torch::Tensor> arrive_local, c10::optional<torch::Tensor> arrive_target,
             c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> row_dst, std::vector<int64_t> slot_ptrs,
             std::vector<int64_t> slot_count_ptrs);
torch::Tensor ep_wait_combine(torch::Tensor slots, c10::optional<torch::Tensor> w, int64_t k, torch::Tensor counter,
                              int64_t target);
torch::Tensor lowrank_rows(torch::Tensor x, c10::optional<torch::Tensor> src, c10::optional<torch::Tensor> scale,
                           std::vector<int64_t> seg_off, std::vector<int64_t> seg_group, torch::Tensor w,
                           int64_t R, int64_t w_gs, int64_t w_rs, int64_t w_ks, int64_t K,
                           c10::optional<torch::Tensor> out);
void lowrank_wgrad(torch::Tensor p, torch::Tensor q, std::vector<int64_t> seg_off, std::vector<int64_t> seg_group,
                   torch::Tensor g, int64_t R, int64_t C, int64_t g_gs, int64_t g_rs, int64_t g_cs, double alpha);
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> res,
                                       torch::Tensor w, double eps, bool legacy);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor xs, torch::Tensor w, torch::Tensor rstd,
                          c10::optional<torch::Tensor> dres, bool legacy);
std::vector<torch::Tensor> rope_fwd(torch::Tensor qkv, torch::Tensor pos, torch::Tensor inv_freq,
                                    int64_t nq, int64_t nkv, int64_t D,
                                    c10::optional<torch::Tensor> qn_w,
                                    c10::optional<torch::Tensor> kn_w, double eps,
                                    c10::optional<torch::Tensor> perm);
void rope_bwd(torch::Tensor dqk, torch::Tensor qkv, torch::Tensor pos, torch::Tensor inv_freq,
              int64_t nq, int64_t nkv, int64_t D, c10::optional<torch::Tensor> qn_w,
              c10::optional<torch::Tensor> kn_w, c10::optional<torch::Tensor> rstd,
              torch::Tensor dqkv, c10::optional<torch::Tensor> perm);
void rope_bwd_f32(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv, torch::Tensor pos,
                  torch::Tensor inv_freq, int64_t nq, int64_t nkv, int64_t D, c10::optional<torch::Tensor> qn_w,
                  c10::optional<torch::Tensor> kn_w, c10::optional<torch::Tensor> rstd, torch::Tensor dqkv,
                  c10::optional<torch::Tensor> perm);
torch::Tensor swiglu_fwd(torch::Tensor gu);
torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu);
std::vector<torch::Tensor> logits_stats(torch::Tensor logits, torch::Tensor targets, bool entropy);
void logits_grad_(torch::Tensor logits, torch::Tensor targets, torch::Tensor lse, torch::Tensor g);
std::vector<torch::Tensor> grpo_token_loss(torch::Tensor newlp, torch::Tensor oldlp,
                                           torch::Tensor adv, torch::Tensor w, torch::Tensor mask,
                                           c10::optional<torch::Tensor> reflp,
                                           c10::optional<torch::Tensor> origlp, torch::Tensor cfg);
torch::Tensor grad_sumsq(torch::Tensor g);
void adamw_step(torch::Tensor p, torch::Tensor p16, torch::Tensor g, torch::Tensor m,
                torch::Tensor v, torch::Tensor hp, torch::Tensor norm_sq, torch::Tensor norm_out);
std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                    torch::Tensor kend, torch::Tensor tile_kmax, double scale, int64_t q_off);
std::vector<torch::Tensor> attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor kend,
                                       torch::Tensor tile_kmax, torch::Tensor tile_kmin, double scale, int64_t q_off,
                                       c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> tile_pmax,
                                       int64_t window, c10::optional<torch::Tensor> sinks,
                                       c10::optional<torch::Tensor> diag);
std::vector<torch::Tensor> attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                       torch::Tensor out, torch::Tensor lse, torch::Tensor kend, torch::Tensor units,
                                       double scale, int64_t q_off, c10::optional<torch::Tensor> pos, int64_t window,
                                       c10::optional<torch::Tensor> diag);
torch::Tensor gemm_tc_grouped(torch::Tensor x, torch::Tensor w, std::vector<int64_t> offs, int64_t N,
                              c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2, bool w_transposed);
void peer_copy(torch::Tensor dst, int64_t src_ptr, int64_t nbytes);
torch::Tensor decode_attn(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor lens,
                          double scale);
void kv_append(torch::Tensor k, torch::Tensor v, torch::Tensor slot, torch::Tensor pos, torch::Tensor k_cache,
               torch::Tensor v_cache);
std::vector<torch::Tensor> attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k,
                                    torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                                    torch::Tensor kend, torch::Tensor units, double scale, int64_t q_off);
std::vector<torch::Tensor> ipc_alloc(int64_t nbytes);
int64_t ipc_open(torch::Tensor handle);
void ipc_close(int64_t ptr);
void peer_barrier(torch::Tensor flag_bases, int64_t rank, int64_t world, int64_t epoch,
                  int64_t timeout_ns, torch::Tensor status);
void dp_reduce_sumsq(torch::Tensor grad_bases, int64_t world, int64_t off, int64_t n,
                     torch::Tensor partial);
void dp_publish_norm(torch::Tensor norm_bases, int64_t rank, int64_t world, torch::Tensor partial);
void dp_adamw_allgather(torch::Tensor compute_bases, int64_t world, int64_t off, int64_t n,
                        torch::Tensor grad_shard, torch::Tensor master, torch::Tensor m,
                        torch::Tensor v, torch::Tensor hp, torch::Tensor norms,
                        torch::Tensor norm_out);
torch::Tensor gemm_tc(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2,
                      c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> bias,
                      c10::optional<torch::Tensor> out, bool accumulate);
int64_t tc_error_code();
torch::Tensor tc_error_word();
torch::Tensor gemm_tc_ag(std::vector<int64_t> a_ptrs, int64_t rows, int64_t K, int64_t lda, torch::Tensor b,
                         c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                         c10::optional<torch::Tensor> bias);
void gemm_tc_rs(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                std::vector<int64_t> c_ptrs, int64_t rows, int64_t ldc, int64_t slot);
torch::Tensor slot_sum(torch::Tensor staging, int64_t nslots, int64_t rows, c10::optional<torch::Tensor> res);
void scatter_rows(torch::Tensor src, c10::optional<torch::Tensor> dst_rank, torch::Tensor dst_row,
                  c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_dst,
                  c10::optional<torch::Tensor> dst_limit);
void scatter_rows_idx(torch::Tensor src, torch::Tensor src_idx, torch::Tensor dst_rank, torch::Tensor dst_row,
                      c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_dst);
void gather_rows(torch::Tensor dst, c10::optional<torch::Tensor> src_rank, torch::Tensor src_row,
                 c10::optional<torch::Tensor> scale, torch::Tensor bases, int64_t ld_src);
torch::Tensor combine_rows(torch::Tensor slots, c10::optional<torch::Tensor> w, int64_t k);
std::vector<torch::Tensor> gdn_scan_fwd(torch::Tensor gq, torch::Tensor W, torch::Tensor U0, torch::Tensor QKM,
                                        torch::Tensor Kd, torch::Tensor gC, c10::optional<torch::Tensor> S0,
                                        bool want_out, bool save, c10::optional<torch::Tensor> peer_out);
std::vector<torch::Tensor> gdn_scan_bwd(c10::optional<torch::Tensor> dO, c10::optional<torch::Tensor> dS_end,
                                        torch::Tensor gq, torch::Tensor W, torch::Tensor QKM, torch::Tensor Kd,
                                        torch::Tensor gC, int64_t DV);
torch::Tensor gdn_conv_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor prev);
torch::Tensor gemm_pair(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2,
                        c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> bias,
                        c10::optional<torch::Tensor> out, bool accumulate, c10::optional<torch::Tensor> diag,
                        bool b_transposed);
std::vector<torch::Tensor> lm_head_fwd(torch::Tensor h, torch::Tensor w, torch::Tensor targets, bool entropy,
                                       c10::optional<torch::Tensor> logits_out);
torch::Tensor glu_clamp_fwd(torch::Tensor gu, double alpha, double limit);
torch::Tensor glu_clamp_bwd(torch::Tensor da, torch::Tensor gu, double alpha, double limit);
void gemm_pair_rs(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2,
                  std::vector<int64_t> c_ptrs, int64_t rows, int64_t ldc, int64_t slot);
void gemm_pair_mainloop(torch::Tensor a, torch::Tensor b, torch::Tensor diag);
void lm_head_grad_logits(torch::Tensor h, torch::Tensor w, torch::Tensor targets, torch::Tensor lse, torch::Tensor g,
                         torch::Tensor out);
std::vector<torch::Tensor> gdn_conv_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor prev,
                                        torch::Tensor succ_ptr, torch::Tensor succ_idx, torch::Tensor succ_tap);
}  // namespace art

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "art_mlx_b200 sm_100a kernels";
  // legacy=True: the block-per-row kernels (kept for comparison)
  m.def("rmsnorm_fwd", &art::rmsnorm_fwd, py::arg("x"), py::arg("res"), py::arg("w"), py::arg("eps"),
        py::arg("legacy") = false);
  m.def("rmsnorm_bwd", &art::rmsnorm_bwd, py::arg("dy"), py::arg("xs"), py::arg("w"), py::arg("rstd"),
        py::arg("dres"), py::arg("legacy") = false);
  m.def("rope_fwd", &art::rope_fwd, py::arg("qkv"), py::arg("pos"), py::arg("inv_freq"), py::arg("nq"),
        py::arg("nkv"), py::arg("D"), py::arg("qn_w"), py::arg("kn_w"), py::arg("eps"), py::arg("perm") = py::none());
  m.def("rope_bwd", &art::rope_bwd, py::arg("dqk"), py::arg("qkv"), py::arg("pos"), py::arg("inv_freq"),
        py::arg("nq"), py::arg("nkv"), py::arg("D"), py::arg("qn_w"), py::arg("kn_w"), py::arg("rstd"),
        py::arg("dqkv"), py::arg("perm") = py::none());
  m.def("rope_bwd_f32", &art::rope_bwd_f32, py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("qkv"),
        py::arg("pos"), py::arg("inv_freq"), py::arg("nq"), py::arg("nkv"), py::arg("D"), py::arg("qn_w"),
        py::arg("kn_w"), py::arg("rstd"), py::arg("dqkv"), py::arg("perm") = py::none());
  m.def("swiglu_fwd", &art::swiglu_fwd);
  m.def("swiglu_bwd", &art::swiglu_bwd);
  m.def("logits_stats", &art::logits_stats);
  m.def("logits_grad_", &art::logits_grad_);
  m.def("grpo_token_loss", &art::grpo_token_loss);
  m.def("grad_sumsq", &art::grad_sumsq);
  m.def("adamw_step", &art::adamw_step);
  m.def("attn_fwd", &art::attn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("kend"), py::arg("tile_kmax"),
        py::arg("scale"), py::arg("q_off") = 0);
  m.def("attn_fwd_tc", &art::attn_fwd_tc, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("kend"),
        py::arg("tile_kmax"), py::arg("tile_kmin"), py::arg("scale"), py::arg("q_off") = 0,
        py::arg("pos") = py::none(), py::arg("tile_pmax") = py::none(), py::arg("window") = 0,
        py::arg("sinks") = py::none(), py::arg("diag") = py::none());
  m.def("attn_bwd_tc", &art::attn_bwd_tc, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("out"), py::arg("lse"), py::arg("kend"), py::arg("units"), py::arg("scale"), py::arg("q_off") = 0,
        py::arg("pos") = py::none(), py::arg("window") = 0, py::arg("diag") = py::none());
  m.def("gemm_tc_grouped", &art::gemm_tc_grouped, py::arg("x"), py::arg("w"), py::arg("offs"), py::arg("N"),
        py::arg("a2") = py::none(), py::arg("b2") = py::none(), py::arg("w_transposed") = false);
  m.def("peer_copy", &art::peer_copy);
  m.def("decode_attn", &art::decode_attn);
  m.def("kv_append", &art::kv_append);
  m.def("attn_bwd", &art::attn_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"),
        py::arg("lse"), py::arg("kend"), py::arg("units"), py::arg("scale"), py::arg("q_off") = 0);
  m.def("gemm_tc", &art::gemm_tc);
  m.def("tc_error_code", &art::tc_error_code);
  m.def("tc_error_word", &art::tc_error_word);
  m.def("gemm_tc_ag", &art::gemm_tc_ag);
  m.def("gemm_tc_rs", &art::gemm_tc_rs);
  m.def("slot_sum", &art::slot_sum);
  m.def("scatter_rows", &art::scatter_rows);
  m.def("gather_rows", &art::gather_rows);
  m.def("scatter_rows_idx", &art::scatter_rows_idx);
  m.def("combine_rows", &art::combine_rows);
  m.def("ipc_alloc", &art::ipc_alloc);
  m.def("ipc_open", &art::ipc_open);
  m.def("ipc_close", &art::ipc_close);
  m.def("peer_barrier", &art::peer_barrier);
  m.def("dp_reduce_sumsq", &art::dp_reduce_sumsq);
  m.def("dp_publish_norm", &art::dp_publish_norm);
  m.def("dp_adamw_allgather", &art::dp_adamw_allgather);
  m.def("gdn_scan_fwd", &art::gdn_scan_fwd, py::arg("gq"), py::arg("W"), py::arg("U0"), py::arg("QKM"),
        py::arg("Kd"), py::arg("gC"), py::arg("S0") = py::none(), py::arg("want_out") = true,
        py::arg("save") = false, py::arg("peer_out") = py::none());
  m.def("gdn_scan_bwd", &art::gdn_scan_bwd, py::arg("dO"), py::arg("dS_end"), py::arg("gq"), py::arg("W"),
        py::arg("QKM"), py::arg("Kd"), py::arg("gC"), py::arg("DV"));
  m.def("gdn_conv_fwd", &art::gdn_conv_fwd);
  m.def("gemm_pair", &art::gemm_pair, py::arg("a"), py::arg("b"), py::arg("a2") = py::none(),
        py::arg("b2") = py::none(), py::arg("bias") = py::none(), py::arg("out") = py::none(),
        py::arg("accumulate") = false, py::arg("diag") = py::none(), py::arg("b_transposed") = false);
  m.def("lm_head_fwd", &art::lm_head_fwd, py::arg("h"), py::arg("w"), py::arg("targets"), py::arg("entropy"),
        py::arg("logits_out") = py::none());
  m.def("lm_head_grad_logits", &art::lm_head_grad_logits);
  m.def("gemm_pair_mainloop", &art::gemm_pair_mainloop);
  m.def("gemm_pair_rs", &art::gemm_pair_rs);
  m.def("glu_clamp_fwd", &art::glu_clamp_fwd);
  m.def("glu_clamp_bwd", &art::glu_clamp_bwd);
  m.def("gdn_conv_bwd", &art::gdn_conv_bwd);
  m.def("ep_gemm", &art::ep_gemm);
  m.def("ep_wait_combine", &art::ep_wait_combine);
  m.def("lowrank_rows", &art::lowrank_rows, py::arg("x"), py::arg("src"), py::arg("scale"), py::arg("seg_off"),
        py::arg("seg_group"), py::arg("w"), py::arg("R"), py::arg("w_gs"), py::arg("w_rs"), py::arg("w_ks"),
        py::arg("K"), py::arg("out") = py::none());
  m.def("lowrank_wgrad", &art::lowrank_wgrad, py::arg("p"), py::arg("q"), py::arg("seg_off"), py::arg("seg_group"),
        py::arg("g"), py::arg("R"), py::arg("C"), py::arg("g_gs"), py::arg("g_rs"), py::arg("g_cs"),
        py::arg("alpha"));
}

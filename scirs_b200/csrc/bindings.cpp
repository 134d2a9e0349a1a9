// Python bindings of the sm_100a kernels (module scirs_b200._C).
#include "host_common.h"

namespace scirs {
void gemm_tc(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t a_mn, int64_t b_mn, int64_t epi,
             c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> out2,
             bool accumulate, int64_t splits, int64_t bn_force, c10::optional<torch::Tensor> bias_grad,
             c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin, int64_t rope_S,
             int64_t rope_hd, int64_t rope_cols);
void layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, torch::Tensor y, torch::Tensor mean,
                   torch::Tensor rstd, double eps);
void layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                   c10::optional<torch::Tensor> dresid, torch::Tensor dx, torch::Tensor dw, torch::Tensor db,
                   torch::Tensor part, c10::optional<torch::Tensor> dsum);
void xent_fwd_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss, int64_t V, double grad_scale,
                  int64_t ignore_index);
void xent_fwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss, int64_t V, int64_t ignore_index);
void embedding_fwd(torch::Tensor tok, torch::Tensor wte, c10::optional<torch::Tensor> wpe, torch::Tensor out,
                   int64_t S);
void embedding_bwd(torch::Tensor tok, torch::Tensor dout, c10::optional<torch::Tensor> dwte, c10::optional<torch::Tensor> dwpe,
                   int64_t S);
void bias_grad(torch::Tensor dy, torch::Tensor out);
void optim_step(int64_t mode, torch::Tensor params, torch::Tensor state1, torch::Tensor state2, torch::Tensor grads,
                c10::optional<torch::Tensor> params16, int64_t n_decay, c10::optional<torch::Tensor> decay_mask,
                torch::Tensor hp, c10::optional<torch::Tensor> part, c10::optional<torch::Tensor> norm_out,
                int64_t parts_ready);
int64_t grad_sumsq(torch::Tensor grads, torch::Tensor part, torch::Tensor hp);
void patchify(torch::Tensor img, torch::Tensor out, int64_t patch);
void vit_embed_fwd(torch::Tensor pe, torch::Tensor cls, torch::Tensor pos, torch::Tensor x, int64_t B);
void vit_embed_bwd(torch::Tensor dx, torch::Tensor dpe, torch::Tensor dpos, torch::Tensor dcls, int64_t B);
void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    bool causal, double scale);
torch::Tensor attn_bwd_trace();
void flash_attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc,
                    torch::Tensor delta, bool causal, double scale, int64_t impl,
                    c10::optional<torch::Tensor> blk_ptr, c10::optional<torch::Tensor> blk_idx,
                    c10::optional<torch::Tensor> bmap, int64_t wl, int64_t wr, int64_t ng);
void flash_attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       bool causal, double scale);
void gemm_tp(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t a_mn, int64_t b_mn, int64_t epi,
             c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> out2,
             bool accumulate, int64_t splits, int64_t rank, int64_t world, std::vector<int64_t> a_peers,
             std::vector<int64_t> b_peers, std::vector<int64_t> rs_dst, c10::optional<torch::Tensor> flags,
             c10::optional<torch::Tensor> epoch, int64_t wait_idx, std::vector<int64_t> sig_flags, int64_t sig_idx,
             double timeout_s, c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
             int64_t rope_S, int64_t rope_hd, int64_t rope_cols);
void tp_signal(std::vector<int64_t> sig_flags, torch::Tensor epoch, int64_t idx);
void ep_dispatch(torch::Tensor src, torch::Tensor idx, c10::optional<torch::Tensor> scale, std::vector<int64_t> dst,
                 int64_t L, int64_t C, int64_t sl, int64_t sr, int64_t rank, std::vector<int64_t> sig_flags,
                 torch::Tensor epoch, int64_t sig_idx);
void ep_combine(std::vector<int64_t> srcs, torch::Tensor expert, torch::Tensor slot, c10::optional<torch::Tensor> wt,
                torch::Tensor out, int64_t L, int64_t C, int64_t rank, c10::optional<torch::Tensor> flags,
                torch::Tensor epoch, int64_t wait_idx, double timeout_s);
void ep_grad_w(std::vector<int64_t> srcs, torch::Tensor expert, torch::Tensor slot, torch::Tensor dout,
               torch::Tensor gw, int64_t L, int64_t C, int64_t rank);
void tp_wait(torch::Tensor flags, torch::Tensor epoch, int64_t idx, int64_t rank, int64_t world, double timeout_s);
void conv_im2col(torch::Tensor x, torch::Tensor cols, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t ph,
                 int64_t pw, int64_t dh, int64_t dw);
void conv_col2im(torch::Tensor dcols, torch::Tensor dx, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t ph,
                 int64_t pw, int64_t dh, int64_t dw);
void conv_rows_nchw(torch::Tensor rows, torch::Tensor y, bool to_nchw);
void pool2d_fwd(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> arg, int64_t KH, int64_t KW,
                int64_t sh, int64_t sw, int64_t ph, int64_t pw, bool is_max, bool count_pad);
void pool2d_bwd(torch::Tensor dy, torch::Tensor dx, c10::optional<torch::Tensor> arg, int64_t KH, int64_t KW,
                int64_t sh, int64_t sw, int64_t ph, int64_t pw, bool is_max, bool count_pad);
void dgelu_mul(torch::Tensor gy, torch::Tensor pre, torch::Tensor out);
void scale_by(torch::Tensor x, torch::Tensor g, torch::Tensor count, torch::Tensor out);
void lstm_cell_fwd(torch::Tensor gx, c10::optional<torch::Tensor> gh, c10::optional<torch::Tensor> c_prev,
                   torch::Tensor c_out, torch::Tensor h_out, torch::Tensor acts);
void lstm_cell_bwd(torch::Tensor dh, c10::optional<torch::Tensor> dc_in, torch::Tensor acts,
                   c10::optional<torch::Tensor> c_prev, torch::Tensor c, torch::Tensor dc_out, torch::Tensor dgates);
void gru_cell_fwd(torch::Tensor gx, c10::optional<torch::Tensor> gh, c10::optional<torch::Tensor> h_prev,
                  torch::Tensor h_out, torch::Tensor acts);
void gru_cell_bwd(torch::Tensor dh, torch::Tensor acts, c10::optional<torch::Tensor> h_prev, torch::Tensor dgx,
                  torch::Tensor dgh, torch::Tensor dh_prev);
void rnn_cell_fwd(torch::Tensor gx, c10::optional<torch::Tensor> gh, torch::Tensor h_out);
void rnn_cell_bwd(torch::Tensor dh, torch::Tensor h, torch::Tensor dg);
void add_bf16_f32(torch::Tensor a, c10::optional<torch::Tensor> b, torch::Tensor out);
void vocab_route(torch::Tensor tok, torch::Tensor dout, int64_t R, int64_t V, std::vector<int64_t> rows,
                 std::vector<int64_t> ids, int64_t rank, std::vector<int64_t> sig_flags, torch::Tensor epoch,
                 int64_t sig_idx);
void vocab_accum(torch::Tensor rows, torch::Tensor ids, torch::Tensor shard, double scale, int64_t rank,
                 torch::Tensor flags, torch::Tensor epoch, int64_t wait_idx, double timeout_s);
void paged_kv_append(torch::Tensor k_new, torch::Tensor v_new, torch::Tensor k_pool, torch::Tensor v_pool,
                     torch::Tensor block_tables, torch::Tensor seq, torch::Tensor pos);
void paged_attention_decode(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor block_tables,
                            torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                            int64_t tokens_per_split, double scale);
void flash_attn_fwd_pp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       bool causal, double scale, bool poly, c10::optional<torch::Tensor> trace, bool x2,
                       c10::optional<torch::Tensor> blk_ptr, c10::optional<torch::Tensor> blk_idx,
                       c10::optional<torch::Tensor> bmap, int64_t wl, int64_t wr, int64_t ng, bool bf2,
                       int64_t persist);
void tp_step_begin(torch::Tensor epoch, c10::optional<torch::Tensor> vals);
void tp_reduce(torch::Tensor recv, torch::Tensor out, c10::optional<torch::Tensor> bias,
               c10::optional<torch::Tensor> resid, int64_t rank, c10::optional<torch::Tensor> flags,
               torch::Tensor epoch, int64_t wait_idx, std::vector<int64_t> sig_flags, int64_t sig_idx,
               double timeout_s);
void rope_apply(torch::Tensor qkv, torch::Tensor cos_t, torch::Tensor sin_t, int64_t S, int64_t H, int64_t hd,
                bool inverse);
void tp_xent_stats(torch::Tensor logits, torch::Tensor targets, int64_t nvalid, int64_t v0, int64_t rank,
                   std::vector<int64_t> stats_dst, std::vector<int64_t> sig_flags, torch::Tensor epoch,
                   int64_t sig_idx);
void tp_xent_finish(torch::Tensor logits, torch::Tensor targets, torch::Tensor stats, c10::optional<torch::Tensor> loss,
                    int64_t nvalid, int64_t v0, int64_t rank, double scale, torch::Tensor flags, torch::Tensor epoch,
                    int64_t wait_idx, double timeout_s);
}  // namespace scirs

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "scirs_b200 sm_100a kernels";
  m.def("gemm", &scirs::gemm_tc, "tcgen05 GEMM with fused epilogue", py::arg("a"), py::arg("b"), py::arg("out"),
        py::arg("a_mn"), py::arg("b_mn"), py::arg("epi"), py::arg("bias") = py::none(), py::arg("aux") = py::none(),
        py::arg("out2") = py::none(), py::arg("accumulate") = false, py::arg("splits") = 0,
        py::arg("bn_force") = 0, py::arg("bias_grad") = py::none(), py::arg("rope_cos") = py::none(),
        py::arg("rope_sin") = py::none(), py::arg("rope_S") = 0, py::arg("rope_hd") = 0, py::arg("rope_cols") = 0);
  m.def("layernorm_fwd", &scirs::layernorm_fwd);
  m.def("layernorm_bwd", &scirs::layernorm_bwd);
  m.def("xent_fwd_bwd", &scirs::xent_fwd_bwd);
  m.def("xent_fwd", &scirs::xent_fwd);
  m.def("embedding_fwd", &scirs::embedding_fwd);
  m.def("embedding_bwd", &scirs::embedding_bwd);
  m.def("bias_grad", &scirs::bias_grad);
  m.def("optim_step", &scirs::optim_step, py::arg("mode"), py::arg("params"), py::arg("state1"), py::arg("state2"),
        py::arg("grads"), py::arg("params16"), py::arg("n_decay"), py::arg("decay_mask"), py::arg("hp"),
        py::arg("part"), py::arg("norm_out"), py::arg("parts_ready") = 0);
  m.def("grad_sumsq", &scirs::grad_sumsq);
  m.def("gemm_tp", &scirs::gemm_tp, "tensor-parallel tcgen05 GEMM (fused all-gather / reduce-scatter)",
        py::arg("a"), py::arg("b"), py::arg("out"), py::arg("a_mn"), py::arg("b_mn"), py::arg("epi"),
        py::arg("bias") = py::none(), py::arg("aux") = py::none(), py::arg("out2") = py::none(),
        py::arg("accumulate") = false, py::arg("splits") = 0, py::arg("rank") = 0, py::arg("world") = 1,
        py::arg("a_peers") = std::vector<int64_t>{}, py::arg("b_peers") = std::vector<int64_t>{},
        py::arg("rs_dst") = std::vector<int64_t>{}, py::arg("flags") = py::none(), py::arg("epoch") = py::none(),
        py::arg("wait_idx") = 0, py::arg("sig_flags") = std::vector<int64_t>{}, py::arg("sig_idx") = 0,
        py::arg("timeout_s") = 10.0, py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none(),
        py::arg("rope_S") = 0, py::arg("rope_hd") = 0, py::arg("rope_cols") = 0);
  m.def("tp_signal", &scirs::tp_signal);
  m.def("tp_wait", &scirs::tp_wait);
  m.def("conv_im2col", &scirs::conv_im2col, "NCHW input -> im2col rows for the convolution GEMM");
  m.def("conv_col2im", &scirs::conv_col2im, "im2col-row gradients -> NCHW input gradient (deterministic gather)");
  m.def("conv_rows_nchw", &scirs::conv_rows_nchw, "GEMM rows (NHWC) <-> NCHW");
  m.def("pool2d_fwd", &scirs::pool2d_fwd, "2-D max / average pooling forward");
  m.def("pool2d_bwd", &scirs::pool2d_bwd, "2-D max / average pooling backward");
  m.def("dgelu_mul", &scirs::dgelu_mul, "out = gy * gelu'(pre)");
  m.def("scale_by", &scirs::scale_by, "out = x * g / count (device scalars)");
  m.def("lstm_cell_fwd", &scirs::lstm_cell_fwd);
  m.def("lstm_cell_bwd", &scirs::lstm_cell_bwd);
  m.def("gru_cell_fwd", &scirs::gru_cell_fwd);
  m.def("gru_cell_bwd", &scirs::gru_cell_bwd);
  m.def("rnn_cell_fwd", &scirs::rnn_cell_fwd);
  m.def("rnn_cell_bwd", &scirs::rnn_cell_bwd);
  m.def("add_bf16_f32", &scirs::add_bf16_f32);
  m.def("vocab_route", &scirs::vocab_route, "send embedding-gradient rows to the rank owning each vocabulary row");
  m.def("vocab_accum", &scirs::vocab_accum, "add the routed embedding-gradient rows into this rank's shard");
  m.def("ep_dispatch", &scirs::ep_dispatch, "expert-parallel dispatch: gather rows and store them into peers");
  m.def("ep_combine", &scirs::ep_combine, "expert-parallel combine: read expert outputs from peers, weighted sum");
  m.def("ep_grad_w", &scirs::ep_grad_w, "routing-weight gradient against peers' expert outputs");
  m.def("paged_kv_append", &scirs::paged_kv_append);
  m.def("paged_attention_decode", &scirs::paged_attention_decode);
  m.def("flash_attn_fwd_pp", &scirs::flash_attn_fwd_pp, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"),
        py::arg("lse"), py::arg("causal"), py::arg("scale"), py::arg("poly") = false,
        py::arg("trace") = py::none(), py::arg("x2") = false, py::arg("blk_ptr") = py::none(),
        py::arg("blk_idx") = py::none(), py::arg("bmap") = py::none(), py::arg("wl") = -1, py::arg("wr") = -1,
        py::arg("ng") = 0, py::arg("bf2") = false, py::arg("persist") = -1);
  m.def("tp_step_begin", &scirs::tp_step_begin, py::arg("epoch"), py::arg("vals") = py::none());
  m.def("tp_reduce", &scirs::tp_reduce);
  m.def("rope_apply", &scirs::rope_apply);
  m.def("tp_xent_stats", &scirs::tp_xent_stats);
  m.def("tp_xent_finish", &scirs::tp_xent_finish);
  m.def("patchify", &scirs::patchify);
  m.def("vit_embed_fwd", &scirs::vit_embed_fwd);
  m.def("vit_embed_bwd", &scirs::vit_embed_bwd);
  m.def("flash_attn_fwd", &scirs::flash_attn_fwd);
  m.def("attn_bwd_trace", &scirs::attn_bwd_trace, "phase trace of the last traced attention backward launch");
  m.def("flash_attn_bwd", &scirs::flash_attn_bwd, "attention backward", py::arg("dout"), py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("out"), py::arg("lse"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("dq_acc"),
        py::arg("delta"), py::arg("causal"), py::arg("scale"), py::arg("impl") = 1, py::arg("blk_ptr") = py::none(),
        py::arg("blk_idx") = py::none(), py::arg("bmap") = py::none(), py::arg("wl") = -1, py::arg("wr") = -1,
        py::arg("ng") = 0);
  m.def("flash_attn_fwd_tc", &scirs::flash_attn_fwd_tc);
  m.def("status_read_and_clear", &scirs::status_read_and_clear);
  m.def("num_sms", &scirs::num_sms);
}

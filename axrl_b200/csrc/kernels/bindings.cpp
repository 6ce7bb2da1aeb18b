// Python bindings of the sm_100a kernels (module axrl_b200._C).
#include <torch/extension.h>

#include <vector>

namespace ax {
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps);
std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd);
std::vector<at::Tensor> qknorm_rope_fwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, int64_t, double);
std::vector<at::Tensor> qknorm_rope_cache(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, int64_t, double,
                                          at::Tensor, at::Tensor, at::Tensor);
std::vector<at::Tensor> qknorm_rope_bwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                                        at::Tensor, at::Tensor, int64_t, int64_t);
at::Tensor swiglu_fwd(at::Tensor gu);
at::Tensor swiglu_bwd(at::Tensor dy, at::Tensor gu);
void logprob_fwd(at::Tensor, at::Tensor, double, at::Tensor, at::Tensor, at::Tensor);
void logprob_bwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, double);
void sample_tokens(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, c10::optional<at::Tensor>, c10::optional<at::Tensor>);
at::Tensor linear_fwd(at::Tensor x, at::Tensor w);
at::Tensor linear_dgrad(at::Tensor dy, at::Tensor w);
at::Tensor linear_wgrad(at::Tensor dy, at::Tensor x);
void linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor acc);
at::Tensor gemm_bf16(at::Tensor a, at::Tensor b, bool trans_b);
std::vector<at::Tensor> attn_fwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, double);
std::vector<at::Tensor> attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles,
                                    double scale, int64_t variant);
std::vector<at::Tensor> attn_fwd_mma(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles,
                                     double scale);
int64_t attn_tc_error();
std::vector<at::Tensor> attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse2,
                                 at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale, c10::optional<at::Tensor> tiles_tc,
                                 c10::optional<at::Tensor> qseg, c10::optional<at::Tensor> kr, c10::optional<at::Tensor> fwd_tiles);
void set_attn_deterministic(bool on);
bool attn_deterministic();
at::Tensor attn_bwd_dsum(at::Tensor o, at::Tensor dout);
std::vector<at::Tensor> attn_bwd_partial(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor lse2, at::Tensor dsum,
                                         at::Tensor dq_acc, at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale,
                                         c10::optional<at::Tensor> tiles_tc);
std::vector<at::Tensor> attn_merge(std::vector<at::Tensor> os, std::vector<at::Tensor> lses);
at::Tensor gdn_step(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, at::Tensor pool, at::Tensor slots);
int64_t attn_bwd_tc_error();
void set_attn_bwd_tc(bool on);
void set_attn_bwd_blocks64(bool on);
void set_attn_bwd_dbl(bool on);
void paged_decode_attn(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t,
                       double, c10::optional<at::Tensor>,
                       c10::optional<at::Tensor>);
void decode_plan(at::Tensor seq_lens, at::Tensor prefix);
void set_decode_attn_tma(bool on);
void kv_store(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor);
void sqnorm_accumulate(at::Tensor x, at::Tensor acc);
void adamw_step(at::Tensor, at::Tensor, at::Tensor, at::Tensor, c10::optional<at::Tensor>, int64_t, double, double, double, double,
                double, int64_t, c10::optional<at::Tensor>, double, double);
at::Tensor embed_fwd(at::Tensor ids, at::Tensor table);
void embed_bwd(at::Tensor ids, at::Tensor dout, at::Tensor grad);
void p2p_reduce_shard(at::Tensor, at::Tensor, int64_t, int64_t, int64_t, at::Tensor);
void p2p_broadcast_shard(at::Tensor, at::Tensor, int64_t, int64_t, int64_t);
void mc_reduce_shard(int64_t, at::Tensor, int64_t, int64_t, at::Tensor);
void mc_broadcast_shard(int64_t, at::Tensor, int64_t, int64_t);
void flag_signal(int64_t, int64_t, int64_t);
void flag_wait_bounded(at::Tensor, int64_t, int64_t, int64_t, at::Tensor);
void sync_push(at::Tensor, at::Tensor, at::Tensor, int64_t);
at::Tensor linear_residual(at::Tensor x, at::Tensor w, at::Tensor residual);
void linear_fwd_into(at::Tensor x, at::Tensor w, at::Tensor out);
void set_streamk_decomposition(int64_t mode, int64_t splits);
void set_pdl(bool on);
bool get_pdl();
void set_weights_static(bool on);
void set_decode_gemm(std::string mode);
at::Tensor linear_rms_stream(at::Tensor h, at::Tensor g, double eps, at::Tensor w, c10::optional<at::Tensor> residual);
at::Tensor linear_swiglu_stream(at::Tensor gu, at::Tensor w, c10::optional<at::Tensor> residual);
at::Tensor skinny_tma_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual);
int64_t skinny_tma_error();
at::Tensor moe_combine(at::Tensor y, at::Tensor w, at::Tensor pos);
std::vector<at::Tensor> moe_combine_bwd(at::Tensor y, at::Tensor w, at::Tensor pos, at::Tensor dout);
std::vector<at::Tensor> router_topk(at::Tensor, int64_t, bool, c10::optional<at::Tensor>, c10::optional<at::Tensor>);
void tp_ar_rms(at::Tensor, int64_t, int64_t, int64_t, c10::optional<at::Tensor>, at::Tensor, double, c10::optional<at::Tensor>, at::Tensor,
               at::Tensor, at::Tensor, at::Tensor, int64_t, int64_t, at::Tensor);
void tp_gather_cols(at::Tensor, int64_t, int64_t, int64_t, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, int64_t, at::Tensor);
void linear_dgrad_into(at::Tensor dy, at::Tensor w, at::Tensor out);
void tp_push(at::Tensor, int64_t, int64_t, at::Tensor, int64_t, at::Tensor, at::Tensor, int64_t, int64_t, int64_t, int64_t, at::Tensor,
             int64_t, at::Tensor, int64_t);
void tp_wait(at::Tensor, int64_t, int64_t, int64_t, int64_t, at::Tensor);
at::Tensor grouped_linear_fwd(at::Tensor x, at::Tensor w, at::Tensor offsets);
at::Tensor grouped_linear_dgrad(at::Tensor dy, at::Tensor w, at::Tensor offsets);
void grouped_linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor offsets, at::Tensor acc);
void ep_plan(at::Tensor, int64_t, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor);
std::vector<at::Tensor> grpo_pg_fwd(at::Tensor, at::Tensor, at::Tensor, at::Tensor, double, double, double);
at::Tensor grpo_pg_bwd(at::Tensor, at::Tensor);
std::vector<at::Tensor> quant_fp8_rows(at::Tensor x);
at::Tensor fp8_block_linear(at::Tensor xq, at::Tensor xs, at::Tensor wq, at::Tensor ws);
void ep_transfer(int64_t, at::Tensor, at::Tensor, int64_t, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t,
                 at::Tensor, at::Tensor, int64_t, int64_t, at::Tensor, int64_t, at::Tensor, int64_t, c10::optional<at::Tensor>);
void tp_reduce_slots(at::Tensor, int64_t, int64_t, c10::optional<at::Tensor>, at::Tensor);
at::Tensor linear_variant(at::Tensor x, at::Tensor w, std::string variant);
at::Tensor skinny_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual);
void decode_advance(int64_t, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, at::Tensor,
                    at::Tensor, at::Tensor, int64_t, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, at::Tensor);
at::Tensor tc_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual);
void tc_linear_ag(at::Tensor gather, at::Tensor w, at::Tensor out, at::Tensor src_ptrs, int64_t rank, int64_t rows_per_rank,
                  at::Tensor flag_ptrs, at::Tensor my_flags, int64_t ch, int64_t epoch, at::Tensor ag_cnt, int64_t call, int64_t timeout_ns,
                  at::Tensor status);
void tc_linear_to_slots(at::Tensor x, at::Tensor w, at::Tensor peer_ptrs, int64_t rank, int64_t rows_per_rank, at::Tensor flag_ptrs,
                        at::Tensor my_flags, int64_t ch, int64_t epoch, at::Tensor ticket, int64_t timeout_ns, at::Tensor status);
int64_t tc_linear_error();
at::Tensor tc_stream_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual);
int64_t tc_stream_error();
std::vector<int64_t> stream_cluster_fit(int64_t ntok);
int64_t decode_tma_error();
at::Tensor tc_linear_dgrad(at::Tensor dy, at::Tensor w);
void adamw_p2p_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, at::Tensor ptrs, int64_t s0, int64_t decay_end, double lr,
                    double b1, double b2, double eps, double wd, int64_t step, at::Tensor sqnorm, double clip, double extra_scale);
void tc_linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor acc, bool accumulate);
}  // namespace ax

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("rmsnorm_fwd", &ax::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &ax::rmsnorm_bwd);
  m.def("qknorm_rope_fwd", &ax::qknorm_rope_fwd);
  m.def("qknorm_rope_cache", &ax::qknorm_rope_cache);
  m.def("qknorm_rope_bwd", &ax::qknorm_rope_bwd);
  m.def("swiglu_fwd", &ax::swiglu_fwd);
  m.def("swiglu_bwd", &ax::swiglu_bwd);
  m.def("logprob_fwd", &ax::logprob_fwd);
  m.def("logprob_bwd", &ax::logprob_bwd);
  m.def("sample_tokens", &ax::sample_tokens, py::arg("logits"), py::arg("temperature"), py::arg("seed"), py::arg("out_tok"),
        py::arg("out_lp"), py::arg("row_ids") = py::none(), py::arg("forced") = py::none());
  m.def("linear_fwd", &ax::linear_fwd);
  m.def("linear_fwd_into", &ax::linear_fwd_into);
  m.def("set_streamk_decomposition", &ax::set_streamk_decomposition);
  m.def("set_pdl", &ax::set_pdl);
  m.def("get_pdl", &ax::get_pdl);
  m.def("set_weights_static", &ax::set_weights_static);
  m.def("linear_rms_stream", &ax::linear_rms_stream, "RMSNorm(h) @ w^T (+ residual), <= 64 rows, norm folded into the streaming GEMM",
        py::arg("h"), py::arg("g"), py::arg("eps"), py::arg("w"), py::arg("residual") = py::none());
  m.def("linear_swiglu_stream", &ax::linear_swiglu_stream, "SwiGLU(gu) @ w^T (+ residual), <= 64 rows, activation folded into the streaming GEMM",
        py::arg("gu"), py::arg("w"), py::arg("residual") = py::none());
  m.def("set_decode_gemm", &ax::set_decode_gemm, "force the decode GEMM for <= 64 rows: skinny, tma, tcgen05, tcstream, tccluster; \"\" = by shape");
  m.def("moe_combine", &ax::moe_combine);
  m.def("moe_combine_bwd", &ax::moe_combine_bwd);
  m.def("router_topk", &ax::router_topk);
  m.def("decode_plan", &ax::decode_plan);
  m.def("skinny_tma_linear", &ax::skinny_tma_linear);
  m.def("skinny_tma_error", &ax::skinny_tma_error);
  m.def("tp_ar_rms", &ax::tp_ar_rms);
  m.def("tp_gather_cols", &ax::tp_gather_cols);
  m.def("linear_dgrad_into", &ax::linear_dgrad_into);
  m.def("tp_push", &ax::tp_push);
  m.def("tp_wait", &ax::tp_wait);
  m.def("grouped_linear_fwd", &ax::grouped_linear_fwd);
  m.def("grouped_linear_dgrad", &ax::grouped_linear_dgrad);
  m.def("grouped_linear_wgrad_acc", &ax::grouped_linear_wgrad_acc);
  m.def("ep_plan", &ax::ep_plan);
  m.def("grpo_pg_fwd", &ax::grpo_pg_fwd);
  m.def("grpo_pg_bwd", &ax::grpo_pg_bwd);
  m.def("quant_fp8_rows", &ax::quant_fp8_rows);
  m.def("fp8_block_linear", &ax::fp8_block_linear);
  m.def("ep_transfer", &ax::ep_transfer, py::arg("mode"), py::arg("rows"), py::arg("C"), py::arg("self"), py::arg("dst_start"),
        py::arg("offsets"), py::arg("blk_pos"), py::arg("blk_src"), py::arg("totals"), py::arg("dst_ptrs"), py::arg("dst_cap_rows"),
        py::arg("flag_ptrs"), py::arg("my_flags"), py::arg("ch"), py::arg("epoch"), py::arg("ticket"), py::arg("timeout_ns"),
        py::arg("status"), py::arg("ctas"), py::arg("src_idx") = py::none());
  m.def("tp_reduce_slots", &ax::tp_reduce_slots);
  m.def("linear_dgrad", &ax::linear_dgrad);
  m.def("linear_wgrad", &ax::linear_wgrad);
  m.def("linear_wgrad_acc", &ax::linear_wgrad_acc);
  m.def("gemm", &ax::gemm_bf16);
  m.def("attn_fwd", &ax::attn_fwd);
  m.def("attn_fwd_tc", &ax::attn_fwd_tc, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("qseg"), py::arg("kr"), py::arg("tiles"),
        py::arg("scale"), py::arg("variant") = 0);
  m.def("attn_fwd_mma", &ax::attn_fwd_mma);
  m.def("attn_tc_error", &ax::attn_tc_error);
  m.def("attn_bwd", &ax::attn_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse2"),
        py::arg("kseg"), py::arg("qr"), py::arg("tiles"), py::arg("scale"), py::arg("tiles_tc") = py::none(), py::arg("qseg") = py::none(),
        py::arg("kr") = py::none(), py::arg("fwd_tiles") = py::none());
  m.def("set_attn_deterministic", &ax::set_attn_deterministic);
  m.def("attn_deterministic", &ax::attn_deterministic);
  m.def("attn_bwd_dsum", &ax::attn_bwd_dsum);
  m.def("attn_bwd_partial", &ax::attn_bwd_partial, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("lse2"),
        py::arg("dsum"), py::arg("dq_acc"), py::arg("kseg"), py::arg("qr"), py::arg("tiles"), py::arg("scale"),
        py::arg("tiles_tc") = py::none());
  m.def("attn_merge", &ax::attn_merge);
  m.def("gdn_step", &ax::gdn_step);
  m.def("attn_bwd_tc_error", &ax::attn_bwd_tc_error);
  m.def("set_attn_bwd_tc", &ax::set_attn_bwd_tc);
  m.def("set_attn_bwd_blocks64", &ax::set_attn_bwd_blocks64);
  m.def("set_attn_bwd_dbl", &ax::set_attn_bwd_dbl);
  m.def("set_decode_attn_tma", &ax::set_decode_attn_tma);
  m.def("paged_decode_attn", &ax::paged_decode_attn, py::arg("q"), py::arg("kc"), py::arg("vc"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("out"), py::arg("part_o"), py::arg("part_ml"), py::arg("splits"), py::arg("scale"),
        py::arg("prefix") = py::none(), py::arg("chunk_cnt") = py::none());
  m.def("kv_store", &ax::kv_store);
  m.def("sqnorm_accumulate", &ax::sqnorm_accumulate);
  m.def("adamw_step", &ax::adamw_step);
  m.def("embed_fwd", &ax::embed_fwd);
  m.def("embed_bwd", &ax::embed_bwd);
  m.def("p2p_reduce_shard", &ax::p2p_reduce_shard);
  m.def("p2p_broadcast_shard", &ax::p2p_broadcast_shard);
  m.def("mc_reduce_shard", &ax::mc_reduce_shard);
  m.def("mc_broadcast_shard", &ax::mc_broadcast_shard);
  m.def("flag_signal", &ax::flag_signal);
  m.def("flag_wait_bounded", &ax::flag_wait_bounded);
  m.def("sync_push", &ax::sync_push);
  m.def("linear_residual", &ax::linear_residual);
  m.def("linear_variant", &ax::linear_variant);
  m.def("decode_advance", &ax::decode_advance);
  m.def("tc_linear", &ax::tc_linear, py::arg("x"), py::arg("w"), py::arg("residual") = py::none());
  m.def("tc_linear_to_slots", &ax::tc_linear_to_slots);
  m.def("tc_linear_ag", &ax::tc_linear_ag);
  m.def("tc_linear_error", &ax::tc_linear_error);
  m.def("tc_stream_linear", &ax::tc_stream_linear, py::arg("x"), py::arg("w"), py::arg("residual") = py::none());
  m.def("tc_stream_error", &ax::tc_stream_error);
  m.def("stream_cluster_fit", &ax::stream_cluster_fit, "resident clusters of 1..16 CTAs of the cluster streaming GEMM for ntok rows");
  m.def("decode_tma_error", &ax::decode_tma_error);
  m.def("tc_linear_dgrad", &ax::tc_linear_dgrad);
  m.def("adamw_p2p_step", &ax::adamw_p2p_step);
  m.def("tc_linear_wgrad_acc", &ax::tc_linear_wgrad_acc);
}

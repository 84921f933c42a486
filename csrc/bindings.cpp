// Python bindings of the sm_100a kernels (module saint_llm_b200._C).
#include <torch/extension.h>

namespace sv4 {
// gemm.cu
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn, bool accumulate,
          double alpha, torch::Tensor err, bool symmetric);
void grouped_gemm(int64_t mode, torch::Tensor a, torch::Tensor b0, torch::Tensor b1, torch::Tensor out,
                  torch::Tensor aux, torch::Tensor rowscale, torch::Tensor probs, torch::Tensor total_tiles,
                  int64_t n_probs, double gate_max, double lin_lo, double lin_hi, int64_t ksplit,
                  bool accumulate, torch::Tensor err);
void build_moe_problems(torch::Tensor seg_start, torch::Tensor seg_rows, int64_t mode, int64_t D, int64_t I,
                        torch::Tensor probs, torch::Tensor total);
int64_t problem_bytes();
void gemm_axpby(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor out, bool a_mn, bool b_mn,
                double alpha, double beta, torch::Tensor err, bool symmetric);
// gemm_fp8.cu
void fp8_quant_rows(torch::Tensor x, torch::Tensor q, torch::Tensor sf, c10::optional<torch::Tensor> scale);
void fp8_gather_quant_rows(torch::Tensor h, torch::Tensor row_token, torch::Tensor q, torch::Tensor sf,
                           torch::Tensor err);
void fp8_quant_blocks_gu(torch::Tensor wg, torch::Tensor wu, torch::Tensor q, torch::Tensor sf);
void fake_quant_fp4(torch::Tensor x, torch::Tensor out);
int64_t gemm_peer_push(torch::Tensor x, torch::Tensor w, torch::Tensor out, std::vector<int64_t> peer_slots,
                       std::vector<int64_t> peer_cnts, torch::Tensor err);
int64_t tp_push(torch::Tensor x, std::vector<int64_t> peer_slots, std::vector<int64_t> peer_cnts);
void tp_reduce(torch::Tensor x, torch::Tensor recv_parity, int64_t slot_elems, torch::Tensor counters,
               std::vector<int64_t> expect, int64_t rank, int64_t timeout_ns, torch::Tensor err);
void zero_signal(std::vector<int64_t> flag_ptrs, int64_t slot, int64_t rank, int64_t epoch);
void zero_pull_reduce(torch::Tensor chunks, std::vector<int64_t> grad_ptrs, int64_t rank, double scale,
                      torch::Tensor my_flags, int64_t slot, int64_t epoch, int64_t timeout_ns, int64_t blocks,
                      torch::Tensor err);
void zero_pull_params(torch::Tensor chunks, std::vector<int64_t> param_ptrs, int64_t rank, torch::Tensor my_flags,
                      int64_t slot, int64_t epoch, int64_t timeout_ns, int64_t blocks, torch::Tensor err);
void compress_pool_fwd(torch::Tensor c, torch::Tensor z, torch::Tensor bias, int64_t m, torch::Tensor out);
void compress_pool_bwd(torch::Tensor c, torch::Tensor z, torch::Tensor bias, int64_t m, torch::Tensor out,
                       torch::Tensor dout, torch::Tensor dc, torch::Tensor dz, torch::Tensor dz_f32);
void fp8_quant_blocks(torch::Tensor w, torch::Tensor q, torch::Tensor sf, c10::optional<torch::Tensor> scale);
void gemm_fp8(torch::Tensor a, torch::Tensor sfa, torch::Tensor b, torch::Tensor sfb, torch::Tensor out,
              torch::Tensor err);
int64_t fp8_sf_bytes(int64_t rows, int64_t k);
void grouped_gemm_fp8(int64_t mode, torch::Tensor a, torch::Tensor sfa, torch::Tensor b, torch::Tensor sfb,
                      torch::Tensor out, c10::optional<torch::Tensor> pre, torch::Tensor probs, torch::Tensor total,
                      int64_t n_probs, int64_t b_rows, double gmax, double lo, double hi, torch::Tensor err);
// decode_attn.cu
void decode_attention(torch::Tensor q, torch::Tensor k_win, torch::Tensor v_win, torch::Tensor pos,
                      c10::optional<torch::Tensor> sink_sw, double softcap, int64_t mode,
                      c10::optional<torch::Tensor> comp, c10::optional<torch::Tensor> norm_w, double eps, int64_t m,
                      c10::optional<torch::Tensor> top, c10::optional<torch::Tensor> sink_c, double scale,
                      torch::Tensor out);
void decode_attention_paged(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_table,
                            torch::Tensor k_len, int64_t window, c10::optional<torch::Tensor> sink_sw, double softcap,
                            int64_t mode, c10::optional<torch::Tensor> e_pool, c10::optional<torch::Tensor> e_table,
                            c10::optional<torch::Tensor> e_len, c10::optional<torch::Tensor> norm_w, double eps,
                            int64_t m, c10::optional<torch::Tensor> top, c10::optional<torch::Tensor> sink_c,
                            double scale, int64_t max_rows, torch::Tensor out, torch::Tensor err);
void decode_window_split(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_table,
                         torch::Tensor k_len, int64_t window, double softcap, double scale, int64_t splits,
                         int64_t max_rows, torch::Tensor pm, torch::Tensor pl, torch::Tensor po, torch::Tensor err);
void lse_merge(torch::Tensor m, torch::Tensor l, torch::Tensor o, c10::optional<torch::Tensor> extra,
               torch::Tensor out, c10::optional<torch::Tensor> out_m, c10::optional<torch::Tensor> out_l);
// router.cu
void router_bwd(torch::Tensor z, torch::Tensor aff, torch::Tensor idx, torch::Tensor gate,
                c10::optional<torch::Tensor> d_gate, c10::optional<torch::Tensor> d_aff, int64_t mode,
                torch::Tensor dz);
void router_fwd(torch::Tensor z, int64_t k, int64_t mode, c10::optional<torch::Tensor> bias,
                c10::optional<torch::Tensor> modality_bias, c10::optional<torch::Tensor> is_visual,
                torch::Tensor aff, torch::Tensor idx, torch::Tensor gate);
// optim.cu
void muon_momentum(torch::Tensor m, torch::Tensor g, torch::Tensor sumsq, int64_t slice, double mu);
void muon_normalize(torch::Tensor m, torch::Tensor g, torch::Tensor sumsq, torch::Tensor y, int64_t slice, double mu,
                    double eps);
void muon_apply(torch::Tensor p, torch::Tensor o, double decay, double step);
void adamw_multi(torch::Tensor table, torch::Tensor chunks, double lr, double beta1, double beta2, double eps,
                 double weight_decay, double step);
int64_t adamw_chunk_elems();
void swiglu_dense(torch::Tensor x, torch::Tensor wg, torch::Tensor wu, torch::Tensor act, torch::Tensor pre,
                  double gmax, double lo, double hi, torch::Tensor err);
void swiglu_dense_dgrad(torch::Tensor dpre, torch::Tensor wg, torch::Tensor wu, torch::Tensor dx, torch::Tensor err);
// moe.cu
void moe_route_plan(torch::Tensor idx, int64_t n_experts, int64_t k, torch::Tensor counts, torch::Tensor seg_start,
                    torch::Tensor seg_rows, torch::Tensor total, torch::Tensor pos, torch::Tensor row_token,
                    torch::Tensor err);
void moe_gather(torch::Tensor h, torch::Tensor row_token, torch::Tensor out, torch::Tensor err);
void moe_combine(torch::Tensor y, torch::Tensor pos, c10::optional<torch::Tensor> w, torch::Tensor out,
                 torch::Tensor err);
void moe_combine_bwd(torch::Tensor dout, c10::optional<torch::Tensor> y, torch::Tensor pos, torch::Tensor w,
                     torch::Tensor dy, c10::optional<torch::Tensor> dw, torch::Tensor err);
void swiglu_bwd_gate(torch::Tensor dact, torch::Tensor pre, torch::Tensor dpre, double gmax, double lo, double hi,
                     torch::Tensor act, torch::Tensor row_pair, torch::Tensor gate, torch::Tensor dgate,
                     torch::Tensor err);
void moe_zero_pad_rows(torch::Tensor row_token, torch::Tensor buf);
void swiglu_bwd(torch::Tensor dact, torch::Tensor pre, torch::Tensor dpre, double gmax, double lo, double hi,
                c10::optional<torch::Tensor> act);
// norm.cu
void rmsnorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor rstd, double eps);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dx);
void rope_norm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor cosb, torch::Tensor sinb, torch::Tensor y,
                   torch::Tensor rstd, int64_t heads, int64_t rd, bool norm_first, double eps);
torch::Tensor rope_norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor cosb,
                            torch::Tensor sinb, torch::Tensor rstd, torch::Tensor dx, int64_t heads, int64_t rd,
                            bool norm_first);
void row_sumsq(torch::Tensor X, torch::Tensor ssq);
void mhc_gates_fwd(torch::Tensor p, torch::Tensor ssq, torch::Tensor r, int64_t F, double eps, torch::Tensor alpha,
                   torch::Tensor s_pre, torch::Tensor s_res, torch::Tensor s_post, torch::Tensor a, torch::Tensor b,
                   torch::Tensor c, int64_t n, int64_t iters);
void mhc_gates_bwd(torch::Tensor p, torch::Tensor alpha, torch::Tensor s_pre, torch::Tensor s_res,
                   torch::Tensor s_post, torch::Tensor da, torch::Tensor db, torch::Tensor dc, torch::Tensor dz,
                   int64_t n, int64_t iters);
void mhc_premix(torch::Tensor X, torch::Tensor a, torch::Tensor out, int64_t n);
void mhc_combine(torch::Tensor X, torch::Tensor o, torch::Tensor B, torch::Tensor C, torch::Tensor Y, int64_t n);
void mhc_combine_bwd(torch::Tensor dY, torch::Tensor X, torch::Tensor o, torch::Tensor B, torch::Tensor C,
                     torch::Tensor dX, torch::Tensor dO, torch::Tensor dB, torch::Tensor dC, int64_t n);
void mhc_premix_da(torch::Tensor X, torch::Tensor din, torch::Tensor da, int64_t n);
void mhc_split_bwd(torch::Tensor dX, torch::Tensor X, torch::Tensor din, torch::Tensor a, torch::Tensor dp,
                   torch::Tensor p, torch::Tensor r, torch::Tensor W, int64_t n);
// attention.cu
void attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor kv, torch::Tensor sel, int64_t mode,
              int64_t m, int64_t window, torch::Tensor sink, double softcap, double scale, torch::Tensor o_sw,
              torch::Tensor o_c, torch::Tensor out, torch::Tensor lse, torch::Tensor max_logit, torch::Tensor err);
void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor kv, torch::Tensor sel, int64_t mode,
              int64_t m, int64_t window, torch::Tensor sink, double softcap, double scale, torch::Tensor o_sw,
              torch::Tensor o_c, torch::Tensor lse, torch::Tensor dout, torch::Tensor dq, torch::Tensor dk,
              torch::Tensor dv, torch::Tensor dkv, torch::Tensor dsink, torch::Tensor err);
void csa_select_mask(torch::Tensor top, int64_t n, torch::Tensor sel, torch::Tensor err);
void indexer_select_mask(torch::Tensor scores, int64_t k, torch::Tensor sel);
// sampling.cu
void sample_tokens(torch::Tensor logits, c10::optional<torch::Tensor> bias, double temperature, int64_t top_k,
                   double top_p, torch::Tensor u, torch::Tensor out, c10::optional<torch::Tensor> thr);
// ce.cu
void ce_fwd(torch::Tensor z, torch::Tensor target, double softcap, torch::Tensor lse, torch::Tensor nll);
void ce_bwd(torch::Tensor z, torch::Tensor target, torch::Tensor lse, double softcap, torch::Tensor scale,
            torch::Tensor dz);
// data.cpp
void bind_data(pybind11::module_& m);
// ep.cu
void ep_signal(std::vector<int64_t> flag_ptrs, int64_t phase, int64_t rank, int64_t epoch);
void ep_post_counts(torch::Tensor counts, std::vector<int64_t> cnt_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                    int64_t slot, int64_t epoch);
void ep_plan(torch::Tensor idx, torch::Tensor pos_local, torch::Tensor seg_start_local, torch::Tensor my_cnt,
             torch::Tensor my_flags, int64_t slot, int64_t epoch, int64_t rank, int64_t ws, int64_t C,
             torch::Tensor gpos, torch::Tensor seg_start_dst, torch::Tensor seg_rows_dst, torch::Tensor seg_pad_dst,
             int64_t timeout_ns, torch::Tensor err);
void ep_dispatch(torch::Tensor h, torch::Tensor gpos, int64_t C, std::vector<int64_t> x_ptrs, torch::Tensor err);
void ep_wait_zero(torch::Tensor my_flags, int64_t phase, int64_t ws, int64_t epoch, torch::Tensor buf,
                  torch::Tensor seg_start, torch::Tensor seg_rows, int64_t timeout_ns, torch::Tensor err);
void ep_combine(std::vector<int64_t> y_ptrs, torch::Tensor gpos, torch::Tensor gate, int64_t C, torch::Tensor out,
                c10::optional<torch::Tensor> ypair, torch::Tensor my_flags, int64_t phase, int64_t ws, int64_t epoch,
                int64_t timeout_ns, torch::Tensor err);
void ep_combine_bwd(torch::Tensor dout, torch::Tensor ypair, torch::Tensor gate, torch::Tensor gpos, int64_t C,
                    std::vector<int64_t> dy_ptrs, torch::Tensor dgate, torch::Tensor err);
void ep_dispatch_bwd(std::vector<int64_t> dx_ptrs, torch::Tensor gpos, int64_t C, torch::Tensor dh,
                     torch::Tensor my_flags, int64_t phase, int64_t ws, int64_t epoch, int64_t timeout_ns,
                     torch::Tensor err);
std::tuple<torch::Tensor, std::string> symm_alloc(int64_t nbytes, int64_t device);
// indexer.cu
void indexer_scores(torch::Tensor q, torch::Tensor keys, torch::Tensor w, c10::optional<torch::Tensor> vis,
                    int64_t m, int64_t q_start, torch::Tensor out, torch::Tensor err);
int64_t symm_open(const std::string& handle, int64_t device);
void symm_close(int64_t ptr, int64_t device);
void symm_free(int64_t ptr, int64_t device);
}  // namespace sv4

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "saint_llm_b200 sm_100a kernels";
  sv4::bind_data(m);
  m.def("attn_fwd", &sv4::attn_fwd);
  m.def("attn_bwd", &sv4::attn_bwd);
  m.def("csa_select_mask", &sv4::csa_select_mask);
  m.def("indexer_select_mask", &sv4::indexer_select_mask);
  m.def("sample_tokens", &sv4::sample_tokens);
  m.def("ce_fwd", &sv4::ce_fwd);
  m.def("ce_bwd", &sv4::ce_bwd);
  m.def("gemm", &sv4::gemm);
  m.def("grouped_gemm", &sv4::grouped_gemm);
  m.def("build_moe_problems", &sv4::build_moe_problems);
  m.def("problem_bytes", &sv4::problem_bytes);
  m.def("gemm_axpby", &sv4::gemm_axpby);
  m.def("fp8_quant_rows", &sv4::fp8_quant_rows);
  m.def("fp8_gather_quant_rows", &sv4::fp8_gather_quant_rows);
  m.def("fp8_quant_blocks_gu", &sv4::fp8_quant_blocks_gu);
  m.def("fake_quant_fp4", &sv4::fake_quant_fp4);
  m.def("compress_pool_fwd", &sv4::compress_pool_fwd);
  m.def("gemm_peer_push", &sv4::gemm_peer_push);
  m.def("tp_push", &sv4::tp_push);
  m.def("tp_reduce", &sv4::tp_reduce);
  m.def("zero_signal", &sv4::zero_signal);
  m.def("zero_pull_reduce", &sv4::zero_pull_reduce);
  m.def("zero_pull_params", &sv4::zero_pull_params);
  m.def("compress_pool_bwd", &sv4::compress_pool_bwd);
  m.def("fp8_quant_blocks", &sv4::fp8_quant_blocks);
  m.def("gemm_fp8", &sv4::gemm_fp8);
  m.def("decode_attention", &sv4::decode_attention);
  m.def("decode_attention_paged", &sv4::decode_attention_paged);
  m.def("decode_window_split", &sv4::decode_window_split);
  m.def("lse_merge", &sv4::lse_merge);
  m.def("router_fwd", &sv4::router_fwd);
  m.def("router_bwd", &sv4::router_bwd);
  m.def("fp8_sf_bytes", &sv4::fp8_sf_bytes);
  m.def("grouped_gemm_fp8", &sv4::grouped_gemm_fp8);
  m.def("muon_momentum", &sv4::muon_momentum);
  m.def("muon_normalize", &sv4::muon_normalize);
  m.def("muon_apply", &sv4::muon_apply);
  m.def("adamw_multi", &sv4::adamw_multi);
  m.def("adamw_chunk_elems", &sv4::adamw_chunk_elems);
  m.def("swiglu_dense", &sv4::swiglu_dense);
  m.def("swiglu_dense_dgrad", &sv4::swiglu_dense_dgrad);
  m.def("moe_route_plan", &sv4::moe_route_plan);
  m.def("moe_gather", &sv4::moe_gather);
  m.def("moe_combine", &sv4::moe_combine);
  m.def("moe_combine_bwd", &sv4::moe_combine_bwd);
  m.def("moe_zero_pad_rows", &sv4::moe_zero_pad_rows);
  m.def("swiglu_bwd", &sv4::swiglu_bwd);
  m.def("swiglu_bwd_gate", &sv4::swiglu_bwd_gate);
  m.def("rmsnorm_fwd", &sv4::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &sv4::rmsnorm_bwd);
  m.def("rope_norm_fwd", &sv4::rope_norm_fwd);
  m.def("rope_norm_bwd", &sv4::rope_norm_bwd);
  m.def("row_sumsq", &sv4::row_sumsq);
  m.def("indexer_scores", &sv4::indexer_scores);
  m.def("ep_signal", &sv4::ep_signal);
  m.def("ep_post_counts", &sv4::ep_post_counts);
  m.def("ep_plan", &sv4::ep_plan);
  m.def("ep_dispatch", &sv4::ep_dispatch);
  m.def("ep_wait_zero", &sv4::ep_wait_zero);
  m.def("ep_combine", &sv4::ep_combine);
  m.def("ep_combine_bwd", &sv4::ep_combine_bwd);
  m.def("ep_dispatch_bwd", &sv4::ep_dispatch_bwd);
  m.def("symm_alloc", [](int64_t n, int64_t dev) {
    auto r = sv4::symm_alloc(n, dev);
    return pybind11::make_tuple(std::get<0>(r), pybind11::bytes(std::get<1>(r)));
  });
  m.def("symm_open", [](pybind11::bytes h, int64_t dev) { return sv4::symm_open(std::string(h), dev); });
  m.def("symm_close", &sv4::symm_close);
  m.def("symm_free", &sv4::symm_free);
  m.def("mhc_gates_fwd", &sv4::mhc_gates_fwd);
  m.def("mhc_gates_bwd", &sv4::mhc_gates_bwd);
  m.def("mhc_premix", &sv4::mhc_premix);
  m.def("mhc_combine", &sv4::mhc_combine);
  m.def("mhc_combine_bwd", &sv4::mhc_combine_bwd);
  m.def("mhc_premix_da", &sv4::mhc_premix_da);
  m.def("mhc_split_bwd", &sv4::mhc_split_bwd);
}

// torch.library registrations for the sm_100a kernel library (namespace torch.ops.r9k).
// Every op mutates preallocated outputs and returns nothing, so all of them are safe inside CUDA
// graph capture (no allocation, no host sync). Reference counterpart: the `r9700` op namespace
// registered in r9700_vllm/ops.py:125-136.
#include <torch/extension.h>
#include <torch/library.h>

namespace r9k {
// gemm_tc.cu
void gemm_mx(torch::Tensor w, torch::Tensor w_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf, torch::Tensor out,
             c10::optional<torch::Tensor> residual, double alpha, torch::Tensor status,
             c10::optional<torch::Tensor> workspace);
void gemm_mx_swiglu(torch::Tensor wg, torch::Tensor wg_sf, torch::Tensor wu, torch::Tensor wu_sf, bool w_fp4,
                    torch::Tensor x, torch::Tensor x_sf, torch::Tensor out_q, torch::Tensor out_sf, torch::Tensor status,
                    c10::optional<torch::Tensor> workspace);
void gemm_bf16(torch::Tensor w, torch::Tensor x, torch::Tensor out, c10::optional<torch::Tensor> residual, double alpha,
               torch::Tensor status, c10::optional<torch::Tensor> workspace);
void gemm_mx_push(torch::Tensor w, torch::Tensor w_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf, int64_t N,
                  torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call, torch::Tensor step,
                  int64_t calls_per_step, torch::Tensor status, c10::optional<torch::Tensor> workspace, int64_t ll);
void gemm_mx_grouped(torch::Tensor w, torch::Tensor w_sf, c10::optional<torch::Tensor> w2,
                     c10::optional<torch::Tensor> w2_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf,
                     torch::Tensor work, torch::Tensor work_count, int64_t N, int64_t E, int64_t BN, torch::Tensor out,
                     c10::optional<torch::Tensor> out_sf, torch::Tensor status);
void gemm_bf16_swiglu(torch::Tensor wg, torch::Tensor wu, torch::Tensor x, torch::Tensor out, torch::Tensor status,
                      c10::optional<torch::Tensor> workspace);
void gemm_trace(c10::optional<torch::Tensor> buf);
void gdn_chunk_trace(c10::optional<torch::Tensor> buf);
// moe.cu
void moe_route(torch::Tensor logits, int64_t k, int64_t mode, c10::optional<torch::Tensor> bias, int64_t n_group,
               int64_t topk_group, double scale, bool renorm, torch::Tensor ids, torch::Tensor w);
void moe_align(torch::Tensor ids, int64_t e0, int64_t E_local, int64_t BN, torch::Tensor perm_row,
               torch::Tensor seg_start, torch::Tensor work, torch::Tensor work_count);
void moe_gather(torch::Tensor q, torch::Tensor sf, int64_t k, torch::Tensor perm_row, torch::Tensor oq,
                torch::Tensor osf);
void moe_combine(torch::Tensor y, torch::Tensor perm_row, torch::Tensor w, int64_t k,
                 c10::optional<torch::Tensor> shared, c10::optional<torch::Tensor> shared_gate, torch::Tensor out);
// comm.cu
int64_t symm_alloc(int64_t nbytes);
void symm_free(int64_t ptr);
torch::Tensor symm_ipc_handle(int64_t ptr);
int64_t symm_open(torch::Tensor handle);
void symm_close(int64_t ptr);
torch::Tensor symm_view(int64_t ptr, int64_t offset_bytes, int64_t rows, int64_t cols, int64_t device);
void symm_step_begin(torch::Tensor step);
torch::Tensor p2p_probe(torch::Tensor peers, int64_t rank, int64_t peer_rank, int64_t off, int64_t kind, int64_t mode,
                        int64_t iters, torch::Tensor status, double timeout_s);
void push_partial(torch::Tensor x, torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems,
                  int64_t call, torch::Tensor step, int64_t calls_per_step);
void ar_rmsnorm(torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call, torch::Tensor step,
                int64_t calls_per_step, int64_t T, c10::optional<torch::Tensor> res_in,
                c10::optional<torch::Tensor> res_out, torch::Tensor w, double eps, bool plus_one,
                c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf,
                torch::Tensor status, double timeout_s);
void ar_pull_rmsnorm(torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call,
                     torch::Tensor step, int64_t calls_per_step, int64_t T, c10::optional<torch::Tensor> res_in,
                     c10::optional<torch::Tensor> res_out, torch::Tensor w, double eps, bool plus_one,
                     c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf,
                     torch::Tensor status, double timeout_s);
void ar_ll_rmsnorm(torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call,
                   torch::Tensor step, int64_t calls_per_step, int64_t T, c10::optional<torch::Tensor> res_in,
                   c10::optional<torch::Tensor> res_out, torch::Tensor w, double eps, bool plus_one,
                   c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf,
                   torch::Tensor status, double timeout_s);
void ll_push(torch::Tensor x, torch::Tensor peers, int64_t rank, int64_t world, int64_t slot_elems, int64_t call,
             torch::Tensor step, int64_t calls_per_step);
// quant.cu
void rmsnorm_quant(torch::Tensor x, c10::optional<torch::Tensor> res_in, c10::optional<torch::Tensor> res_out,
                   torch::Tensor w, double eps, bool plus_one, c10::optional<torch::Tensor> y,
                   c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf);
void swiglu_quant_mxfp8(torch::Tensor g, torch::Tensor u, torch::Tensor q, torch::Tensor sf);
void quant_act_mxfp8(torch::Tensor x, torch::Tensor q, torch::Tensor sf);
void quant_weight_mxfp4(torch::Tensor w, torch::Tensor packed, torch::Tensor sf, bool search);
void quant_weight_mxfp8(torch::Tensor w, torch::Tensor q, torch::Tensor sf);
void quant_weight_nvfp4(torch::Tensor w, double global_scale, torch::Tensor packed, torch::Tensor s16);
void nvfp4_to_mxfp4(torch::Tensor packed_in, torch::Tensor s16, double global_scale, torch::Tensor packed_out,
                    torch::Tensor sf, bool search);
void dequant_mx(torch::Tensor q, torch::Tensor sf, bool fp4, torch::Tensor out);
// attention.cu
void qk_norm_rope_cache(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t q_off, int64_t k_off, int64_t v_off,
                        torch::Tensor qw, torch::Tensor kw, double eps, bool plus_one, torch::Tensor positions,
                        torch::Tensor cos_sin, int64_t rot, torch::Tensor slots, torch::Tensor q_out,
                        torch::Tensor k_cache, torch::Tensor v_cache, double k_scale, double v_scale);
void nvls_all_reduce(c10::optional<torch::Tensor> x, torch::Tensor out, int64_t mc, int64_t local, int64_t cap_bytes,
                     torch::Tensor sig_ptrs, int64_t sig_slots, int64_t rank, int64_t world, torch::Tensor seq,
                     torch::Tensor status, double timeout_s);
void nvls_all_gather(torch::Tensor x, torch::Tensor out, int64_t mc, int64_t local, int64_t cap_bytes,
                     torch::Tensor sig_ptrs, int64_t sig_slots, int64_t rank, int64_t world, torch::Tensor seq,
                     torch::Tensor status, double timeout_s);
void gemm_nvf4(torch::Tensor wq, torch::Tensor ws, double alpha, c10::optional<torch::Tensor> wq2,
               c10::optional<torch::Tensor> ws2, double alpha2, torch::Tensor x, torch::Tensor out, torch::Tensor status);
void kv_cache_write(torch::Tensor k, torch::Tensor v, torch::Tensor slots, torch::Tensor k_cache,
                    torch::Tensor v_cache, double k_scale, double v_scale);
void paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                     torch::Tensor tok_seq, torch::Tensor tok_ctx, double sm_scale, double k_scale, double v_scale,
                     c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> out,
                     c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf, int64_t window);
// attention_tc.cu
void attn_tc_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                    torch::Tensor tok_ctx, torch::Tensor seq_start, torch::Tensor seq_len, double sm_scale,
                    double k_scale, double v_scale, torch::Tensor part_o, torch::Tensor part_ml,
                    c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> out,
                    c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf, torch::Tensor status, int64_t max_rows);
void attn_tc_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                     torch::Tensor tok_ctx, torch::Tensor tile_tab, int64_t ntiles, double sm_scale, double k_scale,
                     double v_scale, c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> out,
                     c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf, torch::Tensor status);
// gdn.cu
void gdn_conv_prep(torch::Tensor proj, int64_t Hk, int64_t Hv, int64_t dk, int64_t dv, int64_t b_off, int64_t a_off,
                   torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor tok_slot, torch::Tensor tok_pos,
                   torch::Tensor tok_has_state, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor q_out,
                   torch::Tensor k_out, torch::Tensor v_out, torch::Tensor g_out, torch::Tensor beta_out,
                   c10::optional<torch::Tensor> qkv_bf16);
void gdn_conv_state_update(torch::Tensor proj, torch::Tensor conv_state, torch::Tensor seq_slot,
                           torch::Tensor seq_start, torch::Tensor seq_len, torch::Tensor seq_has_state);
void gdn_spec_commit(torch::Tensor table, int64_t Hk, int64_t Hv, int64_t dv, int64_t C, int64_t W, int64_t ld,
                     bool state_f32, torch::Tensor seq_slot, torch::Tensor seq_start, torch::Tensor acc_len,
                     torch::Tensor seq_has_state);
void spec_accept(torch::Tensor input_ids, torch::Tensor target, torch::Tensor seq_start, torch::Tensor seq_len,
                 torch::Tensor acc_len);
void dspark_markov_step(torch::Tensor base, int64_t j, torch::Tensor embed, torch::Tensor head, torch::Tensor hrows,
                        torch::Tensor conf_w, double min_conf, torch::Tensor prev, torch::Tensor run,
                        torch::Tensor lengths, torch::Tensor drafts, torch::Tensor part, torch::Tensor counter);
void mhc_seam(torch::Tensor R, c10::optional<torch::Tensor> so, c10::optional<torch::Tensor> post_in,
              c10::optional<torch::Tensor> comb_in, torch::Tensor fn, torch::Tensor scale, torch::Tensor base,
              double rms_eps, double pre_eps, double sk_eps, double post_mult, int64_t sk_repeat, torch::Tensor R_out,
              torch::Tensor post_out, torch::Tensor comb_out, torch::Tensor li, torch::Tensor part);
void exl3_dequant(torch::Tensor trellis, torch::Tensor suh, torch::Tensor svh, int64_t K, int64_t cb, torch::Tensor out);
void exl3_gemv(torch::Tensor trellis, torch::Tensor suh, int64_t K, int64_t cb, torch::Tensor x, int64_t M,
               c10::optional<torch::Tensor> work, c10::optional<torch::Tensor> work_count, int64_t nz, int64_t ksplit,
               torch::Tensor part);
void exl3_finish(torch::Tensor part, c10::optional<torch::Tensor> part_up, torch::Tensor svh,
                 c10::optional<torch::Tensor> svh_up, int64_t ksplit, int64_t nz, int64_t M, int64_t n_out,
                 c10::optional<torch::Tensor> work, c10::optional<torch::Tensor> work_count, torch::Tensor out);
void mla_cache_write(torch::Tensor kv, torch::Tensor kv_w, c10::optional<torch::Tensor> ik,
                     c10::optional<torch::Tensor> ik_w, double eps, torch::Tensor positions, torch::Tensor cos_sin,
                     torch::Tensor slots, torch::Tensor lat_cache, c10::optional<torch::Tensor> idx_cache);
void rope_heads(torch::Tensor x, int64_t H, int64_t off, torch::Tensor positions, torch::Tensor cos_sin);
void indexer_score(torch::Tensor q, torch::Tensor w, torch::Tensor idx_cache, torch::Tensor block_table,
                   torch::Tensor tok_seq, torch::Tensor tok_ctx, int64_t max_ctx, torch::Tensor scores,
                   c10::optional<torch::Tensor> status);
void topk_select(torch::Tensor scores, torch::Tensor tok_ctx, int64_t k, torch::Tensor out, torch::Tensor count);
void sparse_mla_decode(torch::Tensor q, torch::Tensor lat_cache, torch::Tensor block_table, torch::Tensor tok_seq,
                       torch::Tensor sel, torch::Tensor sel_count, double scale, torch::Tensor part_o,
                       torch::Tensor part_ml, torch::Tensor out);
void sparse_mla_decode_tc(torch::Tensor q, torch::Tensor lat_cache, torch::Tensor block_table, torch::Tensor tok_seq,
                          torch::Tensor sel, torch::Tensor sel_count, double scale, torch::Tensor part_o,
                          torch::Tensor part_ml, torch::Tensor out, torch::Tensor status);
void head_gemv(torch::Tensor x, torch::Tensor W, torch::Tensor out);
void host_gather(torch::Tensor table, torch::Tensor ids, int64_t fmt, int64_t dim, torch::Tensor out);
void moe_gather_bf16(torch::Tensor x, int64_t k, torch::Tensor perm_row, torch::Tensor out);
void ngram_ids(torch::Tensor ids, torch::Tensor seq_start, torch::Tensor seq_len, torch::Tensor seq_slot,
               torch::Tensor seq_has_state, torch::Tensor hist, int64_t n_orders, int64_t rows, bool write_state,
               torch::Tensor out);
void symm_collective(int64_t mode, torch::Tensor x, torch::Tensor out, torch::Tensor peers, int64_t rank,
                     int64_t world, int64_t slot_bytes, torch::Tensor seq, torch::Tensor status, double timeout_s);
int64_t symm_collective_region_bytes(int64_t slot_bytes);
void qsa_key_write(torch::Tensor ik, torch::Tensor slots, torch::Tensor ktok);
void qsa_compress(torch::Tensor ktok, torch::Tensor block_table, torch::Tensor tok_seq, torch::Tensor tok_ctx,
                  torch::Tensor ckey);
void qsa_attention(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor block_table,
                   torch::Tensor tok_seq, torch::Tensor tok_ctx, torch::Tensor sel, torch::Tensor count,
                   double sm_scale, double k_scale, double v_scale, int64_t nsplit, torch::Tensor part_o,
                   torch::Tensor part_ml, c10::optional<torch::Tensor> gate, torch::Tensor out);
void hc_gate_mix(torch::Tensor x, torch::Tensor g, int64_t HC, torch::Tensor y);
void hc_combine_norm(torch::Tensor res, c10::optional<torch::Tensor> block, c10::optional<torch::Tensor> l,
                     torch::Tensor w, int64_t HC, double eps, torch::Tensor y);
void trace_stamp(torch::Tensor buf, int64_t slot);
void hc_point(torch::Tensor res, c10::optional<torch::Tensor> y, torch::Tensor wl, torch::Tensor w, torch::Tensor g,
              int64_t HC, double eps, torch::Tensor out);
void symm_ar_wht(torch::Tensor x, torch::Tensor out, torch::Tensor peers, int64_t rank, int64_t world,
                 int64_t slot_bytes, torch::Tensor seq, torch::Tensor status, double timeout_s, int64_t bits,
                 int64_t phase);
void lru_route(torch::Tensor ids, int64_t e0, int64_t E, int64_t S, torch::Tensor slot_of, torch::Tensor expert_of,
               torch::Tensor stamp, torch::Tensor clock, torch::Tensor miss_e, torch::Tensor miss_s,
               torch::Tensor miss_count, torch::Tensor counters, torch::Tensor slot_ids, torch::Tensor status);
void expert_copy(std::vector<torch::Tensor> srcs, std::vector<torch::Tensor> dsts, std::vector<int64_t> bytes,
                 torch::Tensor miss_e, torch::Tensor miss_s, torch::Tensor miss_count, int64_t max_misses);
void gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                   torch::Tensor state, torch::Tensor seq_slot, torch::Tensor seq_start, torch::Tensor seq_len,
                   torch::Tensor seq_has_state, bool write_state, c10::optional<torch::Tensor> o);
void gdn_out_norm_quant(torch::Tensor o, torch::Tensor proj, int64_t z_off, torch::Tensor w, double eps,
                        c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> out_q,
                        c10::optional<torch::Tensor> out_sf);
void gdn_state_prefetch(torch::Tensor state, c10::optional<torch::Tensor> conv_state, torch::Tensor seq_slot);
// gdn_chunk.cu
void gdn_chunked(torch::Tensor qkv, torch::Tensor g, torch::Tensor beta, torch::Tensor state, torch::Tensor ctab,
                 torch::Tensor seq_chunk0, torch::Tensor seq_slot, torch::Tensor seq_has_state, bool write_state,
                 int64_t Hk, int64_t Hv, torch::Tensor w, torch::Tensor qg, torch::Tensor kh, torch::Tensor p,
                 torch::Tensor uT, torch::Tensor gC, torch::Tensor o, torch::Tensor status);
void gdn_decode_fused(torch::Tensor proj, int64_t Hk, int64_t Hv, int64_t z_off, int64_t b_off, int64_t a_off,
                      torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor state, torch::Tensor seq_slot,
                      torch::Tensor seq_has_state, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w,
                      double eps, c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_sf,
                      c10::optional<torch::Tensor> out_bf16);
}  // namespace r9k

TORCH_LIBRARY(r9k, m) {
  m.def("gemm_mx(Tensor w, Tensor w_sf, bool w_fp4, Tensor x, Tensor x_sf, Tensor(a!) out, Tensor? residual, "
        "float alpha, Tensor(b!) status, Tensor(c!)? workspace=None) -> ()");
  m.def("gemm_mx_swiglu(Tensor wg, Tensor wg_sf, Tensor wu, Tensor wu_sf, bool w_fp4, Tensor x, Tensor x_sf, "
        "Tensor(a!) out_q, Tensor(b!) out_sf, Tensor(c!) status, Tensor(d!)? workspace=None) -> ()");
  m.def("gemm_bf16(Tensor w, Tensor x, Tensor(a!) out, Tensor? residual, float alpha, Tensor(b!) status, "
        "Tensor(c!)? workspace=None) -> ()");
  m.def("gemm_mx_push(Tensor w, Tensor w_sf, bool w_fp4, Tensor x, Tensor x_sf, int N, Tensor peers, int rank, "
        "int world, int slot_elems, int call, Tensor step, int calls_per_step, Tensor(a!) status, "
        "Tensor(b!)? workspace=None, int ll=0) -> ()");
  m.def("gemm_mx_grouped(Tensor w, Tensor w_sf, Tensor? w2, Tensor? w2_sf, bool w_fp4, Tensor x, Tensor x_sf, "
        "Tensor work, Tensor work_count, int N, int E, int BN, Tensor(a!) out, Tensor(b!)? out_sf, "
        "Tensor(c!) status) -> ()");
  m.def("gemm_bf16_swiglu(Tensor wg, Tensor wu, Tensor x, Tensor(a!) out, Tensor(b!) status, "
        "Tensor(c!)? workspace=None) -> ()");
  m.def("moe_route(Tensor logits, int k, int mode, Tensor? bias, int n_group, int topk_group, float scale, "
        "bool renorm, Tensor(a!) ids, Tensor(b!) w) -> ()");
  m.def("moe_align(Tensor ids, int e0, int E_local, int BN, Tensor(a!) perm_row, Tensor(b!) seg_start, "
        "Tensor(c!) work, Tensor(d!) work_count) -> ()");
  m.def("moe_gather(Tensor q, Tensor sf, int k, Tensor perm_row, Tensor(a!) oq, Tensor(b!) osf) -> ()");
  m.def("moe_combine(Tensor y, Tensor perm_row, Tensor w, int k, Tensor? shared, Tensor? shared_gate, "
        "Tensor(a!) out) -> ()");
  m.def("symm_step_begin(Tensor(a!) step) -> ()");
  m.def("push_partial(Tensor x, Tensor peers, int rank, int world, int slot_elems, int call, Tensor step, "
        "int calls_per_step) -> ()");
  m.def("ar_rmsnorm(Tensor peers, int rank, int world, int slot_elems, int call, Tensor step, int calls_per_step, "
        "int T, Tensor? res_in, Tensor(a!)? res_out, Tensor w, float eps, bool plus_one, Tensor(b!)? y, "
        "Tensor(c!)? q, Tensor(d!)? sf, Tensor(e!) status, float timeout_s) -> ()");
  m.def("ar_pull_rmsnorm(Tensor peers, int rank, int world, int slot_elems, int call, Tensor step, "
        "int calls_per_step, int T, Tensor? res_in, Tensor(a!)? res_out, Tensor w, float eps, bool plus_one, "
        "Tensor(b!)? y, Tensor(c!)? q, Tensor(d!)? sf, Tensor(e!) status, float timeout_s) -> ()");
  m.def("ar_ll_rmsnorm(Tensor peers, int rank, int world, int slot_elems, int call, Tensor step, "
        "int calls_per_step, int T, Tensor? res_in, Tensor(a!)? res_out, Tensor w, float eps, bool plus_one, "
        "Tensor(b!)? y, Tensor(c!)? q, Tensor(d!)? sf, Tensor(e!) status, float timeout_s) -> ()");
  m.def("ll_push(Tensor x, Tensor peers, int rank, int world, int slot_elems, int call, Tensor step, "
        "int calls_per_step) -> ()");
  m.def("rmsnorm_quant(Tensor x, Tensor? res_in, Tensor(a!)? res_out, Tensor w, float eps, bool plus_one, "
        "Tensor(b!)? y, Tensor(c!)? q, Tensor(d!)? sf) -> ()");
  m.def("swiglu_quant_mxfp8(Tensor g, Tensor u, Tensor(a!) q, Tensor(b!) sf) -> ()");
  m.def("quant_act_mxfp8(Tensor x, Tensor(a!) q, Tensor(b!) sf) -> ()");
  m.def("quant_weight_mxfp4(Tensor w, Tensor(a!) packed, Tensor(b!) sf, bool search) -> ()");
  m.def("quant_weight_mxfp8(Tensor w, Tensor(a!) q, Tensor(b!) sf) -> ()");
  m.def("quant_weight_nvfp4(Tensor w, float global_scale, Tensor(a!) packed, Tensor(b!) s16) -> ()");
  m.def("nvfp4_to_mxfp4(Tensor packed_in, Tensor s16, float global_scale, Tensor(a!) packed_out, Tensor(b!) sf, "
        "bool search) -> ()");
  m.def("dequant_mx(Tensor q, Tensor sf, bool fp4, Tensor(a!) out) -> ()");
  m.def("qk_norm_rope_cache(Tensor qkv, int Hq, int Hkv, int q_off, int k_off, int v_off, Tensor qw, Tensor kw, "
        "float eps, bool plus_one, Tensor positions, Tensor cos_sin, int rot, Tensor slots, Tensor(a!) q_out, "
        "Tensor(b!) k_cache, Tensor(c!) v_cache, float k_scale, float v_scale) -> ()");
  m.def("nvls_all_reduce(Tensor? x, Tensor(a!) out, int mc, int local, int cap_bytes, Tensor sig_ptrs, "
        "int sig_slots, int rank, int world, Tensor(b!) seq, Tensor(c!) status, float timeout_s) -> ()");
  m.def("nvls_all_gather(Tensor x, Tensor(a!) out, int mc, int local, int cap_bytes, Tensor sig_ptrs, "
        "int sig_slots, int rank, int world, Tensor(b!) seq, Tensor(c!) status, float timeout_s) -> ()");
  m.def("gemm_nvf4(Tensor wq, Tensor ws, float alpha, Tensor? wq2, Tensor? ws2, float alpha2, Tensor x, "
        "Tensor(a!) out, Tensor(b!) status) -> ()");
  m.def("kv_cache_write(Tensor k, Tensor v, Tensor slots, Tensor(a!) k_cache, Tensor(b!) v_cache, float k_scale, "
        "float v_scale) -> ()");
  m.def("paged_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor tok_seq, "
        "Tensor tok_ctx, float sm_scale, float k_scale, float v_scale, Tensor? gate, Tensor(a!)? out, "
        "Tensor(b!)? out_q, Tensor(c!)? out_sf, int window) -> ()");
  m.def("attn_tc_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor tok_ctx, "
        "Tensor seq_start, Tensor seq_len, float sm_scale, float k_scale, float v_scale, Tensor(a!) part_o, "
        "Tensor(b!) part_ml, Tensor? gate, Tensor(c!)? out, Tensor(d!)? out_q, Tensor(e!)? out_sf, "
        "Tensor(f!) status, int max_rows=0) -> ()");
  m.def("attn_tc_prefill(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor tok_ctx, "
        "Tensor tile_tab, int ntiles, float sm_scale, float k_scale, float v_scale, Tensor? gate, "
        "Tensor(a!)? out, Tensor(b!)? out_q, Tensor(c!)? out_sf, Tensor(d!) status) -> ()");
  m.def("gdn_conv_prep(Tensor proj, int Hk, int Hv, int dk, int dv, int b_off, int a_off, Tensor conv_w, "
        "Tensor conv_state, Tensor tok_slot, Tensor tok_pos, Tensor tok_has_state, Tensor A_log, Tensor dt_bias, "
        "Tensor(a!) q_out, Tensor(b!) k_out, Tensor(c!) v_out, Tensor(d!) g_out, Tensor(e!) beta_out, "
        "Tensor(f!)? qkv_bf16=None) -> ()");
  m.def("gdn_conv_state_update(Tensor proj, Tensor(a!) conv_state, Tensor seq_slot, Tensor seq_start, "
        "Tensor seq_len, Tensor seq_has_state) -> ()");
  m.def("gdn_spec_commit(Tensor table, int Hk, int Hv, int dv, int C, int W, int ld, bool state_f32, "
        "Tensor seq_slot, Tensor seq_start, Tensor acc_len, Tensor seq_has_state) -> ()");
  m.def("spec_accept(Tensor input_ids, Tensor target, Tensor seq_start, Tensor seq_len, Tensor(a!) acc_len) -> ()");
  m.def("dspark_markov_step(Tensor base, int j, Tensor embed, Tensor head, Tensor hrows, Tensor conf_w, float min_conf, "
        "Tensor(a!) prev, Tensor(b!) run, Tensor(c!) lengths, Tensor(d!) drafts, Tensor(e!) part, Tensor(f!) counter) -> ()");
  m.def("mhc_seam(Tensor R, Tensor? so, Tensor? post_in, Tensor? comb_in, Tensor fn, Tensor scale, Tensor base, "
        "float rms_eps, float pre_eps, float sk_eps, float post_mult, int sk_repeat, Tensor(a!) R_out, "
        "Tensor(b!) post_out, Tensor(c!) comb_out, Tensor(d!) li, Tensor(e!) part) -> ()");
  m.def("exl3_dequant(Tensor trellis, Tensor suh, Tensor svh, int K, int cb, Tensor(a!) out) -> ()");
  m.def("exl3_gemv(Tensor trellis, Tensor suh, int K, int cb, Tensor x, int M, Tensor? work, Tensor? work_count, "
        "int nz, int ksplit, Tensor(a!) part) -> ()");
  m.def("exl3_finish(Tensor part, Tensor? part_up, Tensor svh, Tensor? svh_up, int ksplit, int nz, int M, int n_out, "
        "Tensor? work, Tensor? work_count, Tensor(a!) out) -> ()");
  m.def("mla_cache_write(Tensor kv, Tensor kv_w, Tensor? ik, Tensor? ik_w, float eps, Tensor positions, "
        "Tensor cos_sin, Tensor slots, Tensor(a!) lat_cache, Tensor(b!)? idx_cache) -> ()");
  m.def("rope_heads(Tensor(a!) x, int H, int off, Tensor positions, Tensor cos_sin) -> ()");
  m.def("indexer_score(Tensor q, Tensor w, Tensor idx_cache, Tensor block_table, Tensor tok_seq, Tensor tok_ctx, "
        "int max_ctx, Tensor(a!) scores, Tensor(b!)? status=None) -> ()");
  m.def("topk_select(Tensor scores, Tensor tok_ctx, int k, Tensor(a!) out, Tensor(b!) count) -> ()");
  m.def("sparse_mla_decode(Tensor q, Tensor lat_cache, Tensor block_table, Tensor tok_seq, Tensor sel, "
        "Tensor sel_count, float scale, Tensor(a!) part_o, Tensor(b!) part_ml, Tensor(c!) out) -> ()");
  m.def("sparse_mla_decode_tc(Tensor q, Tensor lat_cache, Tensor block_table, Tensor tok_seq, Tensor sel, "
        "Tensor sel_count, float scale, Tensor(a!) part_o, Tensor(b!) part_ml, Tensor(c!) out, Tensor(d!) status) -> ()");
  m.def("head_gemv(Tensor x, Tensor W, Tensor(a!) out) -> ()");
  m.def("host_gather(Tensor table, Tensor ids, int fmt, int dim, Tensor(a!) out) -> ()");
  m.def("moe_gather_bf16(Tensor x, int k, Tensor perm_row, Tensor(a!) out) -> ()");
  m.def("ngram_ids(Tensor ids, Tensor seq_start, Tensor seq_len, Tensor seq_slot, Tensor seq_has_state, "
        "Tensor(a!) hist, int n_orders, int rows, bool write_state, Tensor(b!) out) -> ()");
  m.def("symm_collective(int mode, Tensor x, Tensor(a!) out, Tensor peers, int rank, int world, int slot_bytes, "
        "Tensor(b!) seq, Tensor(c!) status, float timeout_s) -> ()");
  m.def("qsa_key_write(Tensor ik, Tensor slots, Tensor(a!) ktok) -> ()");
  m.def("qsa_compress(Tensor ktok, Tensor block_table, Tensor tok_seq, Tensor tok_ctx, Tensor(a!) ckey) -> ()");
  m.def("qsa_attention(Tensor q, Tensor kc, Tensor vc, Tensor block_table, Tensor tok_seq, Tensor tok_ctx, "
        "Tensor sel, Tensor count, float sm_scale, float k_scale, float v_scale, int nsplit, Tensor(a!) part_o, "
        "Tensor(b!) part_ml, Tensor? gate, Tensor(c!) out) -> ()");
  m.def("hc_gate_mix(Tensor x, Tensor g, int HC, Tensor(a!) y) -> ()");
  m.def("hc_combine_norm(Tensor(a!) res, Tensor? block, Tensor? l, Tensor w, int HC, float eps, Tensor(b!) y) -> ()");
  m.def("trace_stamp(Tensor(a!) buf, int slot) -> ()");
  m.def("hc_point(Tensor(a!) res, Tensor? y, Tensor wl, Tensor w, Tensor g, int HC, float eps, Tensor(b!) out) -> ()");
  m.def("symm_ar_wht(Tensor x, Tensor(a!) out, Tensor peers, int rank, int world, int slot_bytes, "
        "Tensor(b!) seq, Tensor(c!) status, float timeout_s, int bits, int phase) -> ()");
  m.def("lru_route(Tensor ids, int e0, int E, int S, Tensor(a!) slot_of, Tensor(b!) expert_of, Tensor(c!) stamp, "
        "Tensor(d!) clock, Tensor(e!) miss_e, Tensor(f!) miss_s, Tensor(g!) miss_count, Tensor(h!) counters, "
        "Tensor(i!) slot_ids, Tensor(j!) status) -> ()");
  m.def("expert_copy(Tensor[] srcs, Tensor(a!)[] dsts, int[] bytes, Tensor miss_e, Tensor miss_s, Tensor miss_count, "
        "int max_misses) -> ()");
  m.def("gdn_recurrent(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor(a!) state, Tensor seq_slot, "
        "Tensor seq_start, Tensor seq_len, Tensor seq_has_state, bool write_state, Tensor(b!)? o) -> ()");
  m.def("gdn_state_prefetch(Tensor state, Tensor? conv_state, Tensor seq_slot) -> ()");
  m.def("gdn_chunked(Tensor qkv, Tensor g, Tensor beta, Tensor(a!) state, Tensor ctab, Tensor seq_chunk0, "
        "Tensor seq_slot, Tensor seq_has_state, bool write_state, int Hk, int Hv, Tensor(b!) w, Tensor(c!) qg, "
        "Tensor(d!) kh, Tensor(e!) p, Tensor(f!) uT, Tensor(g!) gC, Tensor(h!) o, Tensor(i!) status) -> ()");
  m.def("gdn_decode_fused(Tensor proj, int Hk, int Hv, int z_off, int b_off, int a_off, Tensor conv_w, "
        "Tensor(a!) conv_state, Tensor(b!) state, Tensor seq_slot, Tensor seq_has_state, Tensor A_log, "
        "Tensor dt_bias, Tensor norm_w, float eps, Tensor(c!)? out_q, Tensor(d!)? out_sf, Tensor(e!)? out_bf16) -> ()");
  m.def("gdn_out_norm_quant(Tensor o, Tensor proj, int z_off, Tensor w, float eps, Tensor(a!)? y, "
        "Tensor(b!)? out_q, Tensor(c!)? out_sf) -> ()");
}

TORCH_LIBRARY_IMPL(r9k, CUDA, m) {
  m.impl("gemm_mx", &r9k::gemm_mx);
  m.impl("host_gather", &r9k::host_gather);
  m.impl("gemm_mx_swiglu", &r9k::gemm_mx_swiglu);
  m.impl("gemm_bf16", &r9k::gemm_bf16);
  m.impl("rmsnorm_quant", &r9k::rmsnorm_quant);
  m.impl("gemm_mx_push", &r9k::gemm_mx_push);
  m.impl("symm_step_begin", &r9k::symm_step_begin);
  m.impl("gemm_mx_grouped", &r9k::gemm_mx_grouped);
  m.impl("gemm_bf16_swiglu", &r9k::gemm_bf16_swiglu);
  m.impl("moe_route", &r9k::moe_route);
  m.impl("moe_align", &r9k::moe_align);
  m.impl("moe_gather", &r9k::moe_gather);
  m.impl("moe_combine", &r9k::moe_combine);
  m.impl("push_partial", &r9k::push_partial);
  m.impl("ar_rmsnorm", &r9k::ar_rmsnorm);
  m.impl("ar_pull_rmsnorm", &r9k::ar_pull_rmsnorm);
  m.impl("ar_ll_rmsnorm", &r9k::ar_ll_rmsnorm);
  m.impl("ll_push", &r9k::ll_push);
  m.impl("swiglu_quant_mxfp8", &r9k::swiglu_quant_mxfp8);
  m.impl("quant_act_mxfp8", &r9k::quant_act_mxfp8);
  m.impl("quant_weight_mxfp4", &r9k::quant_weight_mxfp4);
  m.impl("quant_weight_mxfp8", &r9k::quant_weight_mxfp8);
  m.impl("quant_weight_nvfp4", &r9k::quant_weight_nvfp4);
  m.impl("nvfp4_to_mxfp4", &r9k::nvfp4_to_mxfp4);
  m.impl("dequant_mx", &r9k::dequant_mx);
  m.impl("qk_norm_rope_cache", &r9k::qk_norm_rope_cache);
  m.impl("paged_attention", &r9k::paged_attention);
  m.impl("kv_cache_write", &r9k::kv_cache_write);
  m.impl("nvls_all_reduce", &r9k::nvls_all_reduce);
  m.impl("nvls_all_gather", &r9k::nvls_all_gather);
  m.impl("gemm_nvf4", &r9k::gemm_nvf4);
  m.impl("attn_tc_decode", &r9k::attn_tc_decode);
  m.impl("attn_tc_prefill", &r9k::attn_tc_prefill);
  m.impl("gdn_conv_prep", &r9k::gdn_conv_prep);
  m.impl("gdn_conv_state_update", &r9k::gdn_conv_state_update);
  m.impl("gdn_spec_commit", &r9k::gdn_spec_commit);
  m.impl("spec_accept", &r9k::spec_accept);
  m.impl("dspark_markov_step", &r9k::dspark_markov_step);
  m.impl("mhc_seam", &r9k::mhc_seam);
  m.impl("exl3_dequant", &r9k::exl3_dequant);
  m.impl("exl3_gemv", &r9k::exl3_gemv);
  m.impl("exl3_finish", &r9k::exl3_finish);
  m.impl("mla_cache_write", &r9k::mla_cache_write);
  m.impl("rope_heads", &r9k::rope_heads);
  m.impl("indexer_score", &r9k::indexer_score);
  m.impl("topk_select", &r9k::topk_select);
  m.impl("sparse_mla_decode", &r9k::sparse_mla_decode);
  m.impl("sparse_mla_decode_tc", &r9k::sparse_mla_decode_tc);
  m.impl("head_gemv", &r9k::head_gemv);
  m.impl("moe_gather_bf16", &r9k::moe_gather_bf16);
  m.impl("ngram_ids", &r9k::ngram_ids);
  m.impl("symm_collective", &r9k::symm_collective);
  m.impl("symm_ar_wht", &r9k::symm_ar_wht);
  m.impl("trace_stamp", &r9k::trace_stamp);
  m.impl("hc_point", &r9k::hc_point);
  m.impl("hc_gate_mix", &r9k::hc_gate_mix);
  m.impl("hc_combine_norm", &r9k::hc_combine_norm);
  m.impl("qsa_key_write", &r9k::qsa_key_write);
  m.impl("qsa_compress", &r9k::qsa_compress);
  m.impl("qsa_attention", &r9k::qsa_attention);
  m.impl("lru_route", &r9k::lru_route);
  m.impl("expert_copy", &r9k::expert_copy);
  m.impl("gdn_recurrent", &r9k::gdn_recurrent);
  m.impl("gdn_out_norm_quant", &r9k::gdn_out_norm_quant);
  m.impl("gdn_decode_fused", &r9k::gdn_decode_fused);
  m.impl("gdn_state_prefetch", &r9k::gdn_state_prefetch);
  m.impl("gdn_chunked", &r9k::gdn_chunked);
}

// host-only helpers of the symmetric-memory runtime (no tensors on the device side of the call)
TORCH_LIBRARY_FRAGMENT(r9k, m) {
  m.def("symm_alloc(int nbytes) -> int", &r9k::symm_alloc);
  m.def("symm_free(int ptr) -> ()", &r9k::symm_free);
  m.def("symm_ipc_handle(int ptr) -> Tensor", &r9k::symm_ipc_handle);
  m.def("symm_open(Tensor handle) -> int", &r9k::symm_open);
  m.def("symm_close(int ptr) -> ()", &r9k::symm_close);
  m.def("symm_collective_region_bytes(int slot_bytes) -> int", &r9k::symm_collective_region_bytes);
  m.def("symm_view(int ptr, int offset_bytes, int rows, int cols, int device) -> Tensor", &r9k::symm_view);
  m.def("p2p_probe(Tensor peers, int rank, int peer_rank, int off, int kind, int mode, int iters, Tensor status, "
        "float timeout_s) -> Tensor", &r9k::p2p_probe);
  // tuning: per-CTA timestamps of the tiled GEMM into an int64 buffer (None switches them off)
  m.def("gemm_trace(Tensor? buf) -> ()", &r9k::gemm_trace);
  m.def("gdn_chunk_trace(Tensor? buf) -> ()", &r9k::gdn_chunk_trace);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) { m.doc() = "r9700_stack_b200 sm_100a kernel library"; }

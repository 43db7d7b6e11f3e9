// Declarations and schemas of every op in the `_C` extension.
#pragma once
#include <torch/extension.h>

namespace b200 {

// torch_ops.cpp (kernels in the .cu files named beside each)
void gemm_bf16_out(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                   const at::Tensor& status, int64_t splits);                       // gemm_bf16.cu
void rms_norm_out(at::Tensor& out, const at::Tensor& x, const at::Tensor& w, double eps);  // norm.cu
void fused_add_rms_norm_(at::Tensor& x, at::Tensor& residual, const at::Tensor& w, double eps);  // norm.cu
void silu_mul_op(at::Tensor& out, const at::Tensor& x, double limit);  // norm.cu

void moe_topk_op(const at::Tensor& logits, int64_t k, int64_t mode, const c10::optional<at::Tensor>& bias,
                 double scale, bool renorm, at::Tensor& ids, at::Tensor& weights);  // router.cu
void moe_build_assignments_op(const at::Tensor& ids, const at::Tensor& weights,
                              const c10::optional<at::Tensor>& expert_map, int64_t E_local, int64_t tile_rows,
                              at::Tensor& sorted_token, at::Tensor& sorted_weight, at::Tensor& slot_of,
                              at::Tensor& items, at::Tensor& num_items, at::Tensor& expert_offsets);  // router.cu
void exl3_input_rotate_op(const at::Tensor& x, int64_t in_features, const c10::optional<at::Tensor>& sorted_token,
                          const c10::optional<at::Tensor>& expert_offsets, int64_t E_local, const at::Tensor& suh0,
                          const c10::optional<at::Tensor>& suh1, at::Tensor& out0,
                          const c10::optional<at::Tensor>& out1, int64_t rows,
                          const c10::optional<at::Tensor>& sum0, const c10::optional<at::Tensor>& sum1);  // exl3.cu
void exl3_gemm_op(int64_t nmat, const at::Tensor& trellis0, const c10::optional<at::Tensor>& trellis1,
                  const at::Tensor& svh0, const c10::optional<at::Tensor>& svh1,
                  const c10::optional<at::Tensor>& suh_next, int64_t bits_x2, int64_t codebook, const at::Tensor& b0,
                  const c10::optional<at::Tensor>& b1, int64_t tile_rows, const at::Tensor& items,
                  const at::Tensor& num_items, int64_t max_work, at::Tensor& out, int64_t out_mode,
                  double swiglu_limit, const at::Tensor& status, const c10::optional<at::Tensor>& sx0,
                  const c10::optional<at::Tensor>& sx1, int64_t sx_parts,
                  const c10::optional<at::Tensor>& hsum);  // exl3.cu
void moe_combine_op(const at::Tensor& y, const at::Tensor& slot_of, const at::Tensor& sorted_weight, int64_t k,
                    const c10::optional<at::Tensor>& add, at::Tensor& out);  // exl3.cu

void gqa_prep_op(const at::Tensor& proj, int64_t nh, int64_t nkv, const at::Tensor& q_norm_w,
                 const at::Tensor& k_norm_w, double eps, const at::Tensor& positions, const at::Tensor& cos_sin,
                 const at::Tensor& slots, at::Tensor& q_out, at::Tensor& cache);
void gqa_attention_op(const at::Tensor& q, const at::Tensor& cache, const at::Tensor& ctx_lens,
                      const at::Tensor& token_seq, const at::Tensor& block_table, int64_t kv_heads, double sm_scale,
                      int64_t splits, at::Tensor& out, const at::Tensor& status);
void gqa_gate_op(const at::Tensor& attn, const at::Tensor& proj, int64_t nh, at::Tensor& out);
void dsv4_index_scores_op(const at::Tensor& q, const at::Tensor& w, const at::Tensor& keys,
                          const at::Tensor& block_table, const at::Tensor& seq, const at::Tensor& n_vis,
                          int64_t heads_per_group, at::Tensor& scores);
void dsv4_rot_qdq_op(const at::Tensor& x, at::Tensor& out, const at::Tensor& positions, int64_t heads,
                     const at::Tensor& freqs, bool inverse, const c10::optional<at::Tensor>& norm_w, double eps,
                     int64_t mode);
void engram_gate_op(const at::Tensor& h, const at::Tensor& kv, const at::Tensor& wh, const at::Tensor& wk, double eps,
                    at::Tensor& out);
void kda_forward_op(const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& state_idx,
                    const c10::optional<at::Tensor>& has_init, const at::Tensor& qkv, const at::Tensor& g_raw,
                    const at::Tensor& beta_raw, const c10::optional<at::Tensor>& g2, at::Tensor& conv_state,
                    const c10::optional<at::Tensor>& conv_w, const c10::optional<at::Tensor>& conv_b,
                    const at::Tensor& a_log, const c10::optional<at::Tensor>& g_bias, double lower_bound,
                    const c10::optional<at::Tensor>& norm_w, double eps, double l2_eps, double q_scale, bool l2norm,
                    at::Tensor& state, at::Tensor& out, const c10::optional<at::Tensor>& verify,
                    const c10::optional<at::Tensor>& rec, int64_t chunk_min_len,
                    const c10::optional<at::Tensor>& chunk_scratch, const c10::optional<at::Tensor>& status,
                    int64_t gate_mode);
void mhc_post_pre_op(const c10::optional<at::Tensor>& x, const at::Tensor& H, const c10::optional<at::Tensor>& post,
                     const c10::optional<at::Tensor>& comb, const at::Tensor& fn, const at::Tensor& scale,
                     const at::Tensor& base, const at::Tensor& norm_w, const c10::optional<at::Tensor>& pre_mix,
                     double rms_eps, double eps, double post_mult, int64_t iters, double norm_eps, int64_t mode,
                     at::Tensor& H_out, at::Tensor& y, at::Tensor& post_out, at::Tensor& comb_out, at::Tensor& pre_out);
void kda_recover_op(const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& state_idx, const at::Tensor& keep,
                    const at::Tensor& rec, at::Tensor& state, const at::Tensor& qkv,
                    const c10::optional<at::Tensor>& conv_state);  // kda.cu
void kda_core_op(const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& state_idx,
                 const c10::optional<at::Tensor>& has_init, const at::Tensor& q, const at::Tensor& k,
                 const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta, at::Tensor& state,
                 at::Tensor& out);  // kda.cu

void rope_op(at::Tensor& x, const at::Tensor& positions, const at::Tensor& cos_sin, int64_t offset, int64_t rot_dim,
             bool interleaved, const c10::optional<at::Tensor>& out, int64_t out_offset);  // mla_prep.cu
void mla_latent_cache_write_op(const at::Tensor& kv, const at::Tensor& norm_w, double eps, const at::Tensor& positions,
                               const at::Tensor& cos_sin, bool interleaved, const at::Tensor& slots,
                               at::Tensor& cache);  // mla_prep.cu
void mla_index_k_write_op(const at::Tensor& k, const c10::optional<at::Tensor>& ln_w,
                          const c10::optional<at::Tensor>& ln_b, double eps, const at::Tensor& positions,
                          const at::Tensor& cos_sin, bool interleaved, const at::Tensor& slots, at::Tensor& cache,
                          at::Tensor& cache_scale);  // mla_prep.cu
void mla_index_q_prep_op(const at::Tensor& q, const at::Tensor& positions, const at::Tensor& cos_sin, bool interleaved,
                         const at::Tensor& w, double wscale, at::Tensor& q8, at::Tensor& w_out);  // mla_prep.cu
void mla_indexer_scores_op(const at::Tensor& q8, const at::Tensor& w, const at::Tensor& k_cache,
                           const at::Tensor& k_scale, const at::Tensor& ctx_lens,
                           const c10::optional<at::Tensor>& token_seq, const at::Tensor& block_table,
                           int64_t max_ctx, at::Tensor& scores, const at::Tensor& status);  // mla_attn.cu
void mla_topk_op(const at::Tensor& scores, const at::Tensor& ctx_lens, int64_t k,
                 const c10::optional<at::Tensor>& token_seq, const at::Tensor& block_table, int64_t block_size,
                 at::Tensor& out_idx, at::Tensor& out_count);  // mla_prep.cu
void mla_sparse_attention_op(const at::Tensor& q, const at::Tensor& cache, const at::Tensor& indices,
                             const at::Tensor& counts, double sm_scale, int64_t splits, at::Tensor& out,
                             const c10::optional<at::Tensor>& lse, const at::Tensor& status,
                             const c10::optional<at::Tensor>& sink, int64_t only_half);  // mla_attn.cu

void sample_rows_op(const at::Tensor& logits, const c10::optional<at::Tensor>& temperature, int64_t seed,
                    const c10::optional<at::Tensor>& step, int64_t vocab_offset, at::Tensor& out_val,
                    at::Tensor& out_idx, const c10::optional<at::Tensor>& bans);  // sampling.cu
void sample_combine_op(const at::Tensor& vals, const at::Tensor& idx, at::Tensor& out);  // sampling.cu

void symm_all_reduce_op(const at::Tensor& in, at::Tensor& out, const at::Tensor& peers, int64_t rank, int64_t world,
                        int64_t data_off, int64_t half_bytes, at::Tensor& epochs, const at::Tensor& status,
                        double timeout_s);  // comm.cu

void gemm_allreduce_op(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                       const at::Tensor& peers, int64_t rank, int64_t world, int64_t flag_off, int64_t data_off,
                       int64_t tile_bytes_cap, int64_t max_ctas, at::Tensor& epochs, const at::Tensor& status,
                       double timeout_s);  // gemm_bf16.cu
void combine_allreduce_op(const at::Tensor& y, const at::Tensor& slot_of, const at::Tensor& sorted_weight, int64_t k,
                          const c10::optional<at::Tensor>& add, at::Tensor& out, const at::Tensor& peers,
                          int64_t rank, int64_t world, int64_t flag_off, int64_t data_off, int64_t slot_bytes,
                          at::Tensor& epochs, const at::Tensor& status, double timeout_s);  // fused_comm.cu

void dequant_rows_op(const at::Tensor& rows, int64_t D, const c10::optional<at::Tensor>& failed,
                     at::Tensor& out);  // rows.cu
void ple_decode_op(const at::Tensor& rows, const at::Tensor& ids, const at::Tensor& head_bias,
                   const at::Tensor& head_offsets, const at::Tensor& head_vocab, int64_t owner_lo, int64_t owner_hi,
                   int64_t bits, const c10::optional<at::Tensor>& failed, at::Tensor& out);  // rows.cu
void timing_stamp_op(at::Tensor& ring, const at::Tensor& cursor, int64_t col);             // timing.cu
void timing_open_row_op(at::Tensor& ring, at::Tensor& cursor, at::Tensor& step_counter);  // timing.cu

void dequant_gemm_op(int64_t format, int64_t nmat, const at::Tensor& w0, const c10::optional<at::Tensor>& w1,
                     const at::Tensor& s0, const c10::optional<at::Tensor>& s1, const at::Tensor& b0,
                     const c10::optional<at::Tensor>& b1, int64_t tile_rows, const at::Tensor& items,
                     const at::Tensor& num_items, int64_t max_work, at::Tensor& out, int64_t out_mode,
                     double swiglu_limit, const at::Tensor& status);  // dequant_gemm.cu
void gather_rows_op(const at::Tensor& x, const c10::optional<at::Tensor>& src, at::Tensor& out,
                    int64_t rows);  // dequant_gemm.cu

// sp_ops.cpp: sequence-parallel collectives (state = int32 [16] call counters, peers = int64 [world])
void sp_residual_norm_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status,
                         double timeout_s, int64_t src, const c10::optional<at::Tensor>& x,
                         const c10::optional<at::Tensor>& add, const c10::optional<at::Tensor>& dmask,
                         int64_t rs_off, int64_t comb_off, int64_t ag_off, at::Tensor& residual, const at::Tensor& w,
                         double eps, const c10::optional<at::Tensor>& out, bool ag);
void sp_route_dispatch_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status,
                          double timeout_s, const at::Tensor& logits, const at::Tensor& h, int64_t k, int64_t mode,
                          const c10::optional<at::Tensor>& bias, double scale, bool renorm, int64_t e_per_rank,
                          int64_t rows_off, int64_t ids_off, int64_t w_off, at::Tensor& dmask,
                          const c10::optional<at::Tensor>& ids_local, const c10::optional<at::Tensor>& w_local);
void sp_combine_push_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status, double timeout_s,
                        const at::Tensor& y, const at::Tensor& slot_of, const at::Tensor& sorted_weight, int64_t k,
                        int64_t comb_off, int64_t Tr, int64_t H, int64_t channel);
void sp_wait_op(const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status, double timeout_s,
                int64_t channel);
void gemm_sp_op(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& out, at::Tensor& status,
                int64_t splits, const at::Tensor& peers, int64_t rank, at::Tensor& state, double timeout_s, int64_t mode,
                int64_t rs_off, int64_t rows_per_rank);
void moe_build_assignments_sp_op(const at::Tensor& ids, const at::Tensor& weights,
                                 const c10::optional<at::Tensor>& expert_map, int64_t E_local, int64_t tile_rows,
                                 at::Tensor& sorted_token, at::Tensor& sorted_weight, at::Tensor& slot_of,
                                 at::Tensor& items, at::Tensor& num_items, at::Tensor& expert_offsets,
                                 const at::Tensor& peers, int64_t rank, at::Tensor& state, at::Tensor& status,
                                 double timeout_s);

void gemm_batched_op(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const at::Tensor& status);

// Host (non-op) bindings: C++ runtime pieces exposed through pybind11.
void register_host_bindings(pybind11::module_& m);

}  // namespace b200

// Schema list: one line per op.
#define B200_OP_SCHEMAS(X)                                                                               \
  X("gemm_bf16_out(Tensor x, Tensor w, Tensor? bias, Tensor(a!) out, Tensor(b!) status, int splits) -> ()") \
  X("rms_norm_out(Tensor(a!) out, Tensor x, Tensor w, float eps) -> ()")                                 \
  X("fused_add_rms_norm(Tensor(a!) x, Tensor(b!) residual, Tensor w, float eps) -> ()")                 \
  X("silu_mul(Tensor(a!) out, Tensor x, float limit) -> ()")                                           \
  X("moe_topk(Tensor logits, int k, int mode, Tensor? bias, float scale, bool renorm, Tensor(a!) ids, "     \
    "Tensor(b!) weights) -> ()")                                                                         \
  X("moe_build_assignments(Tensor ids, Tensor weights, Tensor? expert_map, int E_local, int tile_rows, "   \
    "Tensor(a!) sorted_token, Tensor(b!) sorted_weight, Tensor(c!) slot_of, Tensor(d!) items, "            \
    "Tensor(e!) num_items, Tensor(f!) expert_offsets) -> ()")                                           \
  X("exl3_input_rotate(Tensor x, int in_features, Tensor? sorted_token, Tensor? expert_offsets, "          \
    "int E_local, Tensor suh0, Tensor? suh1, Tensor(a!) out0, Tensor(b!)? out1, int rows, "                \
    "Tensor(c!)? sum0=None, Tensor(d!)? sum1=None) -> ()")                                                 \
  X("exl3_gemm(int nmat, Tensor trellis0, Tensor? trellis1, Tensor svh0, Tensor? svh1, Tensor? suh_next, " \
    "int bits_x2, int codebook, Tensor b0, Tensor? b1, int tile_rows, Tensor items, Tensor num_items, "     \
    "int max_work, Tensor(a!) out, int out_mode, float swiglu_limit, Tensor(b!) status, "                 \
    "Tensor? sx0=None, Tensor? sx1=None, int sx_parts=1, Tensor(c!)? hsum=None) -> ()")                    \
  X("moe_combine(Tensor y, Tensor slot_of, Tensor sorted_weight, int k, Tensor? add, Tensor(a!) out) -> ()") \
  X("kda_forward(Tensor cu_seqlens, Tensor? state_idx, Tensor? has_init, Tensor qkv, Tensor g_raw, "        \
    "Tensor beta_raw, Tensor? g2, Tensor(a!) conv_state, Tensor? conv_w, Tensor? conv_b, Tensor a_log, "   \
    "Tensor? g_bias, float lower_bound, Tensor? norm_w, float eps, float l2_eps, float q_scale, "            \
    "bool l2norm, Tensor(b!) state, Tensor(c!) out, Tensor? verify=None, Tensor(d!)? rec=None, "            \
    "int chunk_min_len=0, Tensor(e!)? chunk_scratch=None, Tensor(f!)? status=None, int gate_mode=0) -> ()")                  \
  X("mhc_post_pre(Tensor? x, Tensor H, Tensor? post, Tensor? comb, Tensor fn, Tensor scale, Tensor base, "   \
    "Tensor norm_w, Tensor? pre_mix, float rms_eps, float eps, float post_mult, int iters, float norm_eps, "  \
    "int mode, Tensor(a!) H_out, Tensor(b!) y, Tensor(c!) post_out, Tensor(d!) comb_out, Tensor(e!) pre_out) -> ()") \
  X("kda_recover(Tensor cu_seqlens, Tensor? state_idx, Tensor keep, Tensor rec, Tensor(a!) state, "         \
    "Tensor qkv, Tensor(b!)? conv_state) -> ()")                                                          \
  X("kda_core(Tensor cu_seqlens, Tensor? state_idx, Tensor? has_init, Tensor q, Tensor k, Tensor v, "      \
    "Tensor g, Tensor beta, Tensor(a!) state, Tensor(b!) out) -> ()")                                     \
  X("rope(Tensor(a!) x, Tensor positions, Tensor cos_sin, int offset, int rot_dim, bool interleaved, "        \
    "Tensor(b!)? out=None, int out_offset=0) -> ()")                                                      \
  X("mla_latent_cache_write(Tensor kv, Tensor norm_w, float eps, Tensor positions, Tensor cos_sin, "        \
    "bool interleaved, Tensor slots, Tensor(a!) cache) -> ()")                                            \
  X("mla_index_k_write(Tensor k, Tensor? ln_w, Tensor? ln_b, float eps, Tensor positions, Tensor cos_sin, " \
    "bool interleaved, Tensor slots, Tensor(a!) cache, Tensor(b!) cache_scale) -> ()")                    \
  X("mla_index_q_prep(Tensor q, Tensor positions, Tensor cos_sin, bool interleaved, Tensor w, float wscale, " \
    "Tensor(a!) q8, Tensor(b!) w_out) -> ()")                                                             \
  X("mla_indexer_scores(Tensor q8, Tensor w, Tensor k_cache, Tensor k_scale, Tensor ctx_lens, "           \
    "Tensor? token_seq, Tensor block_table, int max_ctx, Tensor(a!) scores, Tensor(b!) status) -> ()")    \
  X("mla_topk(Tensor scores, Tensor ctx_lens, int k, Tensor? token_seq, Tensor block_table, int block_size, " \
    "Tensor(a!) out_idx, Tensor(b!) out_count) -> ()")                                                    \
  X("mla_sparse_attention(Tensor q, Tensor cache, Tensor indices, Tensor counts, float sm_scale, int splits, " \
    "Tensor(a!) out, Tensor(b!)? lse, Tensor(c!) status, Tensor? sink=None, int only_half=-1) -> ()")                      \
  X("sample_rows(Tensor logits, Tensor? temperature, int seed, Tensor? step, int vocab_offset, "          \
    "Tensor(a!) out_val, Tensor(b!) out_idx, Tensor? bans=None) -> ()")                                  \
  X("sample_combine(Tensor vals, Tensor idx, Tensor(a!) out) -> ()")                                     \
  X("symm_all_reduce(Tensor input, Tensor(a!) out, Tensor peers, int rank, int world, int data_off, "     \
    "int half_bytes, Tensor(b!) epochs, Tensor(c!) status, float timeout_s) -> ()")                       \
  X("dequant_gemm(int format, int nmat, Tensor w0, Tensor? w1, Tensor s0, Tensor? s1, Tensor b0, Tensor? b1, " \
    "int tile_rows, Tensor items, Tensor num_items, int max_work, Tensor(a!) out, int out_mode, "             \
    "float swiglu_limit, Tensor(b!) status) -> ()")                                                       \
  X("gather_rows(Tensor x, Tensor? src, Tensor(a!) out, int rows) -> ()")                               \
  X("gemm_allreduce(Tensor x, Tensor w, Tensor? bias, Tensor(a!) out, Tensor peers, int rank, int world, "  \
    "int flag_off, int data_off, int tile_bytes_cap, int max_ctas, Tensor(b!) epochs, Tensor(c!) status, " \
    "float timeout_s) -> ()")                                                                            \
  X("dequant_rows(Tensor rows, int D, Tensor? failed, Tensor(a!) out) -> ()")                           \
  X("ple_decode(Tensor rows, Tensor ids, Tensor head_bias, Tensor head_offsets, Tensor head_vocab, "     \
    "int owner_lo, int owner_hi, int bits, Tensor? failed, Tensor(a!) out) -> ()")                      \
  X("timing_stamp(Tensor(a!) ring, Tensor cursor, int col) -> ()")                                      \
  X("timing_open_row(Tensor(a!) ring, Tensor(b!) cursor, Tensor(c!) step_counter) -> ()")               \
  X("combine_allreduce(Tensor y, Tensor slot_of, Tensor sorted_weight, int k, Tensor? add, Tensor(a!) out, " \
    "Tensor peers, int rank, int world, int flag_off, int data_off, int slot_bytes, Tensor(b!) epochs, "    \
    "Tensor(c!) status, float timeout_s) -> ()")                                                           \
  X("sp_residual_norm(Tensor peers, int rank, Tensor(a!) state, Tensor(b!) status, float timeout_s, int src, " \
    "Tensor? x, Tensor? add, Tensor? dmask, int rs_off, int comb_off, int ag_off, Tensor(c!) residual, "     \
    "Tensor w, float eps, Tensor(d!)? out, bool ag) -> ()")                                                \
  X("sp_route_dispatch(Tensor peers, int rank, Tensor(a!) state, Tensor(b!) status, float timeout_s, "      \
    "Tensor logits, Tensor h, int k, int mode, Tensor? bias, float scale, bool renorm, int e_per_rank, "     \
    "int rows_off, int ids_off, int w_off, Tensor(c!) dmask, Tensor(d!)? ids_local, Tensor(e!)? w_local) -> ()") \
  X("sp_combine_push(Tensor peers, int rank, Tensor(a!) state, Tensor(b!) status, float timeout_s, Tensor y, " \
    "Tensor slot_of, Tensor sorted_weight, int k, int comb_off, int Tr, int H, int channel=3) -> ()")                      \
  X("sp_wait(Tensor peers, int rank, Tensor(a!) state, Tensor(b!) status, float timeout_s, int channel) -> ()") \
  X("gemm_sp(Tensor x, Tensor w, Tensor(a!)? out, Tensor(b!) status, int splits, Tensor peers, int rank, "  \
    "Tensor(c!) state, float timeout_s, int mode, int rs_off, int rows_per_rank) -> ()")                   \
  X("moe_build_assignments_sp(Tensor ids, Tensor weights, Tensor? expert_map, int E_local, int tile_rows, " \
    "Tensor(a!) sorted_token, Tensor(b!) sorted_weight, Tensor(c!) slot_of, Tensor(d!) items, "             \
    "Tensor(e!) num_items, Tensor(f!) expert_offsets, Tensor peers, int rank, Tensor(g!) state, "           \
    "Tensor(h!) status, float timeout_s) -> ()")                                                      \
  X("gemm_batched(Tensor x, Tensor w, Tensor(a!) out, Tensor(b!) status) -> ()")                       \
  X("gqa_prep(Tensor proj, int nh, int nkv, Tensor q_norm_w, Tensor k_norm_w, float eps, Tensor positions, " \
    "Tensor cos_sin, Tensor slots, Tensor(a!) q_out, Tensor(b!) cache) -> ()")                             \
  X("gqa_attention(Tensor q, Tensor cache, Tensor ctx_lens, Tensor token_seq, Tensor block_table, "         \
    "int kv_heads, float sm_scale, int splits, Tensor(a!) out, Tensor(b!) status) -> ()")                  \
  X("gqa_gate(Tensor attn, Tensor proj, int nh, Tensor(a!) out) -> ()")                                   \
  X("engram_gate(Tensor h, Tensor kv, Tensor wh, Tensor wk, float eps, Tensor(a!) out) -> ()")              \
  X("dsv4_index_scores(Tensor q, Tensor w, Tensor keys, Tensor block_table, Tensor seq, Tensor n_vis, "     \
    "int heads_per_group, Tensor(a!) scores) -> ()")                                                        \
  X("dsv4_rot_qdq(Tensor x, Tensor(a!) out, Tensor positions, int heads, Tensor freqs, bool inverse, "     \
    "Tensor? norm_w, float eps, int mode) -> ()")

#define B200_OP_IMPLS(X)                   \
  X("gemm_bf16_out", b200::gemm_bf16_out)  \
  X("rms_norm_out", b200::rms_norm_out)    \
  X("fused_add_rms_norm", b200::fused_add_rms_norm_) \
  X("silu_mul", b200::silu_mul_op)                    \
  X("moe_topk", b200::moe_topk_op)                    \
  X("moe_build_assignments", b200::moe_build_assignments_op) \
  X("exl3_input_rotate", b200::exl3_input_rotate_op)  \
  X("exl3_gemm", b200::exl3_gemm_op)                  \
  X("moe_combine", b200::moe_combine_op)              \
  X("kda_forward", b200::kda_forward_op)              \
  X("kda_core", b200::kda_core_op)                    \
  X("kda_recover", b200::kda_recover_op)              \
  X("mhc_post_pre", b200::mhc_post_pre_op)            \
  X("rope", b200::rope_op)                            \
  X("mla_latent_cache_write", b200::mla_latent_cache_write_op) \
  X("mla_index_k_write", b200::mla_index_k_write_op)  \
  X("mla_index_q_prep", b200::mla_index_q_prep_op)    \
  X("mla_indexer_scores", b200::mla_indexer_scores_op) \
  X("mla_topk", b200::mla_topk_op)                    \
  X("mla_sparse_attention", b200::mla_sparse_attention_op) \
  X("sample_rows", b200::sample_rows_op)              \
  X("sample_combine", b200::sample_combine_op)        \
  X("symm_all_reduce", b200::symm_all_reduce_op)      \
  X("dequant_gemm", b200::dequant_gemm_op)            \
  X("gather_rows", b200::gather_rows_op)              \
  X("gemm_allreduce", b200::gemm_allreduce_op)        \
  X("combine_allreduce", b200::combine_allreduce_op) \
  X("timing_stamp", b200::timing_stamp_op)            \
  X("dequant_rows", b200::dequant_rows_op)            \
  X("ple_decode", b200::ple_decode_op)                \
  X("timing_open_row", b200::timing_open_row_op)      \
  X("sp_residual_norm", b200::sp_residual_norm_op)    \
  X("sp_route_dispatch", b200::sp_route_dispatch_op)  \
  X("sp_combine_push", b200::sp_combine_push_op)      \
  X("sp_wait", b200::sp_wait_op)                      \
  X("gemm_sp", b200::gemm_sp_op)                      \
  X("moe_build_assignments_sp", b200::moe_build_assignments_sp_op) \
  X("gemm_batched", b200::gemm_batched_op)            \
  X("gqa_prep", b200::gqa_prep_op)                    \
  X("gqa_attention", b200::gqa_attention_op)          \
  X("gqa_gate", b200::gqa_gate_op)                    \
  X("engram_gate", b200::engram_gate_op)              \
  X("dsv4_index_scores", b200::dsv4_index_scores_op)  \
  X("dsv4_rot_qdq", b200::dsv4_rot_qdq_op)

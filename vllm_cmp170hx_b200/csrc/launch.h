// Plain C++ interface between the torch glue (*.cpp, compiled by the host
// compiler) and the kernel translation units (*.cu).  Nothing here includes
// torch, so the .cu files compile in seconds.  Launchers take raw device
// pointers and a stream and return a cudaError_t; the glue turns errors into
// exceptions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

int device_sm_count();

// ---------------------------------------------------------------- sequence-parallel collectives
// Flag protocol: sp_sync.cuh.  Channels of the symmetric buffer's flag area flags[channel][src].
enum SpChannel : int { kSpAllGather = 0, kSpReduceScatter = 1, kSpDispatch = 2, kSpCombine = 3, kSpChannels = 4 };
constexpr int kSpMaxRanks = 32;
constexpr int64_t kSpFlagBytes = 4096;  // flags[kSpChannels][kSpMaxRanks] uint32, padded

struct SpSync {
  const uint64_t* peers;  // [world] base address of every rank's symmetric buffer (this rank's included)
  int rank, world;
  uint32_t* state;        // [kSpChannels * 4] local: pushes, push arrivals, receives, receive arrivals
  uint32_t* status;       // error word (kErrPeerTimeout)
  uint64_t timeout_ns;
};

// sp_comm.cu.  Receive areas (byte offsets into every rank's symmetric buffer; row r of a [world * Tr]
// area is token r % Tr of source rank r / Tr):
//   all-gather [world * Tr, H] bf16, reduce-scatter [world * Tr, H] bf16, dispatch rows [world * Tr, H]
//   bf16 + ids [world * Tr, k] int32 + weights [world * Tr, k] fp32, combine [world * Tr, H] bf16.
struct SpNormArgs {
  SpSync s;
  int src;                       // 0: rows x (the residual starts as x), 1: reduce-scatter area, 2: combine area,
                                 // 3: rows x computed on this rank (added to the residual)
  const __nv_bfloat16* x;        // src 0: [Tr, ld_x]
  int64_t ld_x;
  const __nv_bfloat16* add;      // src 2: added to the combined rows (shared expert output [Tr, H]) or null
  const uint32_t* dmask;         // src 2: [Tr] ranks that pushed a combine row for the token (bit per rank)
  int64_t rs_off, comb_off, ag_off;
  __nv_bfloat16* residual;       // [Tr, H]: src 0 writes x, else residual += reduced rows
  const __nv_bfloat16* w;        // RMSNorm weight [H]
  float eps;
  __nv_bfloat16* out;            // normalised rows [Tr, ld_out] or null
  int64_t ld_out;
  int ag;                        // 1: push the normalised rows into every rank's all-gather area
  int Tr, H;
};
cudaError_t sp_residual_norm(const SpNormArgs& a, cudaStream_t stream);

struct SpDispatchArgs {
  SpSync s;
  const float* logits;           // [Tr, E] router logits
  const __nv_bfloat16* h;        // [Tr, ld_h] the MoE input rows
  int64_t ld_h;
  int E, k, mode, renorm;
  const float* bias;
  float scale;
  int e_per_rank;                // experts [d * e_per_rank, (d + 1) * e_per_rank) live on rank d
  int64_t rows_off, ids_off, w_off;
  uint32_t* dmask;               // [Tr] out: ranks this rank pushed each token to
  int* ids_local;                // [Tr, k] out (optional): the picks, for diagnostics and tests
  float* w_local;
  int Tr, H;
};
cudaError_t sp_route_dispatch(const SpDispatchArgs& a, cudaStream_t stream);

struct SpCombineArgs {
  SpSync s;
  const float* y;                // [assignments, ld_y] expert outputs
  int64_t ld_y;
  const int* slot_of;            // [world * Tr, k] assignment row of (received row, j), -1: none here
  const float* sorted_weight;    // [assignments]
  int k;
  int64_t comb_off;              // area the rows go to (the combine area, or the reduce-scatter area)
  int Tr, H;
  int channel;                   // kSpCombine, or kSpReduceScatter for a row-parallel output already computed
};
cudaError_t sp_combine_push(const SpCombineArgs& a, cudaStream_t stream);

// Waits for every source's latest push on `channel` (for consumers that are not a fused kernel).
cudaError_t sp_wait(const SpSync& s, int channel, cudaStream_t stream);

// ---------------------------------------------------------------- gemm_bf16.cu
// C[M, N] = X[M, K] . W[N, K]^T (+ bias[N]); bf16 in/out, fp32 accumulate.
// `partial` (fp32, >= splits * M * N elements) is required when splits > 1;
// pass splits = 0 to let the launcher choose (then `partial_cap` elements are
// available).  Returns the number of splits used through *splits_used.
struct GemmArgs {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  const void* bias;
  void* c;
  int64_t ldc;
  int out_f32;  // 1: c is fp32
  int M, N, K;
  int splits;
  float* partial;
  int64_t partial_cap;
  uint32_t* status;
};
int gemm_bf16_splits(int M, int N, int K, int splits_req);
// Whether a launch with this many splits needs the fp32 partial scratch (cluster-reduced splits do not).
bool gemm_bf16_uses_partial(int M, int splits);
cudaError_t gemm_bf16(const GemmArgs& a, cudaStream_t stream);

// Batched: C[b] = X[b] . W[b]^T for b < batch (strides in elements; per-head projections such as the
// MLA absorb / up-projection), bf16 out, no split-K.
struct GemmBatchedArgs {
  const void* x;
  int64_t ldx, x_bstride;
  const void* w;
  int64_t ldw, w_bstride;
  void* c;
  int64_t ldc, c_bstride;
  int M, N, K, batch;
  uint32_t* status;
};
cudaError_t gemm_bf16_batched(const GemmBatchedArgs& a, cudaStream_t stream);

// The same GEMM fused with a sequence-parallel collective (gemm_bf16.cu):
//   mode 1 (reduce-scatter): row t of the output (a token) is pushed into rank t / rows_per_rank's
//          reduce-scatter area at row (this rank, t % rows_per_rank); C is not written;
//   mode 2 (all-gather): x is this rank's all-gather area; the kernel streams its first weight tiles
//          while it waits for every rank's push, then reads x.
struct GemmSpArgs {
  GemmArgs g;
  int mode;
  SpSync sp;
  int64_t rs_off;
  int rows_per_rank;
};
cudaError_t gemm_bf16_sp(const GemmSpArgs& a, cudaStream_t stream);

// GEMM fused with the tensor-parallel all-reduce over symmetric peer buffers (gemm_bf16.cu).
struct GemmArArgs {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  const void* bias;
  void* c;  // bf16 [M, N] (ldc), the all-reduced result
  int64_t ldc;
  int M, N, K;
  const uint64_t* peers;  // [world] symmetric buffer base of each rank
  int rank, world;
  int64_t flag_off, data_off;
  int64_t tile_bytes_cap;  // bytes reserved per (cta, parity, src) slot
  int max_ctas;            // CTAs the flag / slot areas are sized for
  uint32_t* epochs;        // [max_ctas] per-CTA call counters
  uint32_t* status;
  uint64_t timeout_ns;
};
cudaError_t gemm_bf16_allreduce(const GemmArArgs& a, cudaStream_t stream);

// MoE combine fused with the tensor-parallel all-reduce (fused_comm.cu).
struct CombineArArgs {
  const float* y;  // [assignments, ld_y] fp32 expert outputs
  int64_t ld_y;
  const int* slot_of;         // [T, k] assignment row of (token, j), -1 none
  const float* sorted_weight;  // [assignments] router weight
  int k;
  const __nv_bfloat16* add;  // [T, H] shared-expert output or null
  __nv_bfloat16* out;        // [T, H]
  int T, H;
  const uint64_t* peers;
  int rank, world;
  int64_t flag_off, data_off, slot_bytes;
  uint32_t* epochs;  // [blocks]
  uint32_t* status;
  uint64_t timeout_ns;
};
cudaError_t combine_allreduce(const CombineArArgs& a, int blocks, cudaStream_t stream);

// ---------------------------------------------------------------- rows.cu
cudaError_t dequant_rows_e4m3(const void* rows, int64_t row_bytes, int D, const uint8_t* failed, void* out, int n,
                              cudaStream_t stream);
cudaError_t ple_decode_rows(const void* rows, int64_t words, const int64_t* ids, const void* bias,
                            const int64_t* head_off, const int64_t* head_vocab, int heads, int dim, int bits,
                            int64_t owner_lo, int64_t owner_hi, const uint8_t* failed, void* out, int n,
                            cudaStream_t stream);

// ---------------------------------------------------------------- timing.cu
cudaError_t timing_stamp(int64_t* ring, const int* cursor, int width, int col, cudaStream_t stream);
cudaError_t timing_open_row(int64_t* ring, int* cursor, int rows, int width, int64_t* step_counter,
                            cudaStream_t stream);
int gemm_bf16_allreduce_fits(int M, int N, int max_ctas, int64_t tile_bytes_cap);

// ---------------------------------------------------------------- norm.cu
cudaError_t rms_norm(void* out, int64_t ld_out, const void* x, int64_t ld_x, const void* w, int T, int H, float eps,
                     cudaStream_t stream);
cudaError_t fused_add_rms_norm(void* x, int64_t ld_x, void* residual, int64_t ld_res, const void* w, int T, int H,
                               float eps, cudaStream_t stream);
// out[t, i] = silu(min(x[t, i], L)) * clamp(x[t, I + i], -L, L)  (L <= 0: no clamp), bf16
cudaError_t silu_mul(void* out, int64_t ld_out, const void* x, int64_t ld_x, int T, int I, float limit,
                     cudaStream_t stream);

// ---------------------------------------------------------------- router.cu
// mode 0 softmax+renorm, 1 sigmoid(+bias select), 2 sqrt(softplus)(+bias select)
cudaError_t moe_topk(const float* logits, int T, int E, int k, int mode, const float* bias, float scale, int renorm,
                     int* ids, float* weights, cudaStream_t stream);
cudaError_t moe_build_assignments(const int* ids, const float* weights, int T, int k, const int* expert_map,
                                  int E_map, int E_local, int tile_rows, int* sorted_token, float* sorted_weight, int* slot_of,
                                  int4* items, int* num_items, int* expert_offsets, int max_items,
                                  cudaStream_t stream, const SpSync* sp = nullptr);

// ---------------------------------------------------------------- exl3.cu
struct Exl3GemmArgs {
  int nmat;                 // 2: gate/up pass, 1: down / dense
  const void* trellis[2];   // int16 [E, K/16, N/16, 8*bits_x2]
  int64_t trellis_estride;  // elements between experts (contiguous [E, K/16, N/16, 8*bits_x2])
  int num_experts;
  const void* svh[2];       // fp16 [E, N]
  int64_t svh_estride;
  const void* suh_next;     // fp16 [E, N] (gate/up pass only): suh of the down matrix
  int64_t suh_next_estride;
  int K, N, bits_x2, codebook;
  const void* b0;           // fp16 [b_rows, K] rotated activations (matrix 0)
  const void* b1;           // fp16 [b_rows, K] (matrix 1, gate/up pass)
  int64_t b_rows;
  int tile_rows;            // rows per work item (<= 128 gate/up, <= 256 down)
  const int* items;         // int4 [max_items] {expert, row0, rows, 0}
  const int* num_items;
  int max_work;             // upper bound of items * (N / 128) (grid size)
  void* out;
  int64_t ld_out;
  int out_mode;             // 0 fp16, 1 fp32, 2 bf16
  float swiglu_limit;
  // codebook 2: per-row sums of the activation rows b0 / b1, [b_rows][sx_parts] partials each
  // (the input rotation writes them with sx_parts = 1; the gate/up pass writes the down pass's)
  const float* sx0;
  const float* sx1;
  int sx_parts;
  float* hsum;              // gate/up pass: [b_rows][N / 128] partial row sums of the intermediate
  uint32_t* status;
};
cudaError_t exl3_gemm(const Exl3GemmArgs& a, cudaStream_t stream);
// Also writes sum0 / sum1 [rows]: each output row's sum of its fp16 values (nullable).
cudaError_t exl3_input_rotate(const void* x, int64_t ld_x, int in_features, int K, const int* sorted_token,
                              const int* expert_offsets, int E_local, const void* suh0, const void* suh1,
                              int64_t suh_estride, void* out0, void* out1, float* sum0, float* sum1, int rows,
                              cudaStream_t stream);
cudaError_t moe_combine(const float* y, int64_t ld_y, const int* slot_of, const float* sorted_weight, int T, int k,
                        int H, const void* add, void* out, int64_t ld_out, float* out_f32, cudaStream_t stream);

// ---------------------------------------------------------------- kda.cu
struct KdaArgs {
  int full;  // 1: GLM layer semantics (bf16 inputs, conv, gates, gated norm); 0: core recurrence (fp32)
  int H, D, num_seqs;
  const int* cu_seqlens;  // [num_seqs + 1] token ranges
  const int* state_idx;   // [num_seqs] state slot per sequence (nullptr: identity)
  const int* has_init;    // [num_seqs] 0 = fresh sequence (zero state/conv window); nullptr: all 1
  // full mode inputs
  const __nv_bfloat16* qkv;  // [T, 3*H*D] pre-conv q | k | v
  int64_t ld_qkv;
  const __nv_bfloat16* g_raw;  // [T, H*D] decay gate input
  int64_t ld_g;
  const __nv_bfloat16* beta_raw;  // [T, H] pre-sigmoid
  int64_t ld_beta;
  const __nv_bfloat16* g2;  // [T, H*D] output gate (pre-sigmoid), nullable
  int64_t ld_g2;
  __nv_bfloat16* conv_state;     // [slots, 3*H*D, 3]
  const __nv_bfloat16* conv_w;   // [3*H*D, 4] (nullable: no conv)
  const __nv_bfloat16* conv_b;   // [3*H*D] nullable
  const float* a_log;            // [H]
  const float* g_bias;           // [H*D] nullable
  float lower_bound;
  const __nv_bfloat16* norm_w;   // [D] nullable: no gated norm
  float eps, l2_eps, q_scale;
  int l2norm;
  // core mode inputs (fp32, [T, H, D] / [T, H])
  const float *q_f32, *k_f32, *v_f32, *g_f32, *beta_f32;
  // state and outputs
  float* state;  // [slots, H, D(v), D(k)]
  __nv_bfloat16* out;  // [T, H*D] (ld_out)
  int64_t ld_out;
  float* out_f32;  // core mode [T, H, D]
  // speculative verify: for sequences with verify[s] != 0 the state and conv window are left as they
  // were and every token's update is recorded instead, rec [T, H, 3, D] = (u, k, decay); kda_recover
  // then applies the accepted prefix
  const int* verify;  // [num_seqs] nullable
  float* rec;
  int skip_long;  // > 0: sequences of at least this many tokens are left to the chunked kernel
  // 0: KDA gates (per-channel decay exp(lb * sigmoid(exp(A_log) * (g + bias))), output gate sigmoid(g2));
  // 1: gated delta net (one decay per head exp(-exp(A_log) * softplus(a + dt_bias)) with g_raw [T, H] and
  //    g_bias = dt_bias [H], output gate silu(g2))
  int gate_mode;
};
cudaError_t kda_recurrent(const KdaArgs& a, cudaStream_t stream);

// Chunked prefill (kda_chunk.cu): the sequences of at least `min_len` tokens run in chunks of 64 on the
// tensor cores (the recurrence skips them when its `skip_long` is the same length).  `scratch` holds the
// per-token prep outputs (kda_chunk_scratch_bytes); the fields after it are filled by the launcher.
struct KdaChunkArgs {
  KdaArgs k;
  int T;
  int min_len;
  void* scratch;
  size_t scratch_bytes;
  uint32_t* status;
  __nv_bfloat16 *qn, *kn, *vv;  // [T, H, 128]
  float *gl, *beta;             // [T, H, 128] log2 decay, [T, H]
};
size_t kda_chunk_scratch_bytes(int T, int H);
cudaError_t kda_chunked(const KdaChunkArgs& a, cudaStream_t stream);

// Applies the first keep[s] recorded tokens of each verified sequence to its state, and moves its conv
// window past them (the window is rebuilt from the step's pre-conv inputs).
struct KdaRecoverArgs {
  int H, num_seqs;
  const int* cu_seqlens;
  const int* state_idx;
  const int* keep;  // [num_seqs] tokens to apply (0: sequence untouched)
  const float* rec;  // [T, H, 3, 128]
  float* state;      // [slots, H, 128, 128]
  const __nv_bfloat16* qkv;  // [T, 3*H*128] pre-conv inputs of the step
  int64_t ld_qkv;
  __nv_bfloat16* conv_state;  // [slots, 3*H*128, 3] (nullable)
};
cudaError_t kda_recover(const KdaRecoverArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- mhc.cu
// One mHC sublayer boundary per token: post of x into the streams (x nullable), coefficients of the
// new streams (pre / post / Sinkhorn comb), and the next sublayer input RMSNorm(collapse).
// mode 0: collapse with the fresh pre; 1: with pre_mix (carried); 2: stream 0.
struct MhcArgs {
  const __nv_bfloat16* x;      // [T, d] or nullptr
  const __nv_bfloat16* H;      // [T, hc, d]
  const float* post;           // [T, hc] (with x)
  const float* comb;           // [T, hc, hc] (with x)
  const float* fn;             // [2 hc + hc^2, hc d]
  const float* scale;          // [3]
  const float* base;           // [2 hc + hc^2]
  const __nv_bfloat16* norm_w; // [d]
  const float* pre_mix;        // [T, hc] (mode 1)
  float rms_eps, eps, post_mult, norm_eps;
  int iters, mode, T, hc, d;
  __nv_bfloat16* H_out;  // may equal H
  __nv_bfloat16* y;      // [T, d]
  float* post_out;       // [T, hc]
  float* comb_out;       // [T, hc, hc]
  float* pre_out;        // [T, hc]
};
cudaError_t mhc_post_pre(const MhcArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- mla_prep.cu / mla_attn.cu
cudaError_t rope_apply(void* x, int64_t ld_tok, int64_t ld_head, int nheads, int offset, int rot_dim,
                       const int* positions, const float* cos_sin, int interleaved, int T, cudaStream_t stream,
                       void* y = nullptr, int64_t y_ld_tok = 0, int64_t y_ld_head = 0, int y_offset = 0);
cudaError_t mla_latent_cache_write(const void* kv, int64_t ld_kv, const void* norm_w, float eps, const int* positions,
                                   const float* cos_sin, int interleaved, const int64_t* slots, void* cache, int T,
                                   cudaStream_t stream);
cudaError_t mla_index_k_write(const void* k, int64_t ld_k, const void* ln_w, const void* ln_b, float eps,
                              const int* positions, const float* cos_sin, int rope_dim, int interleaved,
                              const int64_t* slots, void* cache, float* cache_scale, int T, cudaStream_t stream);
cudaError_t mla_index_q_prep(const void* q, int64_t ld_tok, int nheads, const int* positions, const float* cos_sin,
                             int rope_dim, int interleaved, const void* w, int64_t ld_w, float wscale, void* q8,
                             float* w_out, int T, cudaStream_t stream);
cudaError_t mla_topk(const float* scores, int64_t ld_scores, const int* ctx_lens, int k, const int* token_seq,
                     const int* block_table, int64_t ld_bt, int block_size, int* out_idx, int* out_count, int T,
                     cudaStream_t stream);
cudaError_t mla_indexer_scores(const void* q8, const float* w, int T, const void* k_cache, int64_t num_slots,
                               const float* k_scale, const int* ctx_lens, const int* token_seq, const int* block_table,
                               int64_t ld_bt, float* scores, int64_t ld_scores, int max_ctx, uint32_t* status,
                               cudaStream_t stream);
// q [T, nh, dim] (dim 576: MLA latent + RoPE; 512: DeepSeek-V4.1 rows), cache rows of dim; V = the
// first 512 dims.  sink: per-head logits added to the softmax denominator (null: none).
// DeepSeek-V4.1 indexer scores (dsv4_index.cu): q [T, H, 128], w [T, H] bf16, keys [rows, 128] bf16 paged by
// the block table; scores [T, N] fp32 (-inf past n_vis).  H in {4, 8, 16, 32, 64}.
cudaError_t dsv4_index_scores(const void* q, const void* w, const void* keys, const int* block_table, int64_t ld_bt,
                              const int* seq, const int* n_vis, int T, int H, int heads_per_group, float* scores,
                              int64_t ld_scores, int N, cudaStream_t stream);

// DeepSeek-V4.1 row transforms (dsv4_rot.cu): optional RMSNorm, RoPE turn of the last 2 n_pairs dims at
// positions[row / heads] (inverse: the opposite turn), then mode 0 (none), 1 (FP8 per 32), 2 (FP4, E4M3 scales
// per 16) or 3 (FP4, power-of-two scales per 32); rows of D <= 512 bf16 values, D a multiple of 32.
cudaError_t dsv4_rot_qdq(const void* x, int64_t ld_x, void* out, int64_t ld_out, int rows, int D,
                         const int64_t* positions, int heads, const float* freqs, int n_pairs, int inverse,
                         const void* norm_w, float eps, int mode, cudaStream_t stream);

// Engram gate (engram.cu): out[t] += sigmoid(<rmsnorm(h_t) w_h, rmsnorm(k_t) w_k> / sqrt(H)) v_t, kv = [k | v].
cudaError_t engram_gate(const void* h, int64_t ld_h, const void* kv, int64_t ld_kv, const void* wh, const void* wk,
                        float eps, int T, int H, void* out, int64_t ld_out, cudaStream_t stream);

// Gated grouped-query attention (gqa.cu); head_dim 256.
struct GqaPrepArgs {
  const __nv_bfloat16* proj;  // [T, ld_proj]: nh x [q | gate] (512 each), nkv x k (256), nkv x v (256)
  int64_t ld_proj;
  int nh, nkv, group;         // this rank's query heads, key-value heads, query heads per key-value head
  const __nv_bfloat16* q_norm_w;  // [256]
  const __nv_bfloat16* k_norm_w;  // [256]
  float eps;
  const int* positions;       // [T]
  const float* cos_sin;       // [max_pos, rot_dim] fp32 (cos | sin)
  int rot_dim;                // NeoX RoPE on the first rot_dim dims
  const int64_t* slots;       // [T] cache position of each token (< 0: none)
  __nv_bfloat16* q_out;       // [T * nkv, group, 512] query rows [q' | 0]
  __nv_bfloat16* cache;       // [positions * nkv, 512] rows [k' | v]
};
cudaError_t gqa_prep(const GqaPrepArgs& a, int T, cudaStream_t stream);
cudaError_t gqa_gate(const void* attn, const void* proj, int64_t ld_proj, int T, int nh, void* out, int64_t ld_out,
                     cudaStream_t stream);
// Dense causal attention of the query rows [Tq = T * kv_heads, group, 512] over the paged [K | V] rows
// (mla_attn.cu's block kernel in its dense mode): out [Tq, group, 512], value half [256, 512) written.
cudaError_t gqa_dense_attention(const void* q, int Tq, int group, const void* cache, const int* ctx_lens,
                                const int* token_seq, const int* block_table, int64_t ld_bt, int kv_heads,
                                float sm_scale, int splits, void* out, float* part_o, float* part_ml,
                                uint32_t* status, cudaStream_t stream);

cudaError_t mla_sparse_attention(const void* q, int T, int nh, int dim, const void* cache, const int* indices,
                                 const int* counts, int topk, float sm_scale, int splits, void* out, float* part_o,
                                 float* part_ml, float* lse, const float* sink, uint32_t* status,
                                 cudaStream_t stream, int only_half = -1);

// ---------------------------------------------------------------- sampling.cu
cudaError_t sample_rows(const void* logits, int dtype, int64_t ld, int rows, int V, const float* temperature,
                        uint64_t seed, const int64_t* step, int vocab_offset, const int* bans, int nbans,
                        float* out_val, int* out_idx, cudaStream_t stream);
cudaError_t sample_combine(const float* vals, const int* idx, int R, int rows, int64_t* out, cudaStream_t stream);

// ---------------------------------------------------------------- comm.cu
cudaError_t symm_all_reduce(const void* in, void* out, int64_t n, const uint64_t* peers, int rank, int world,
                            int64_t data_off, int64_t half_bytes, uint32_t* epochs, int blocks, uint32_t* status,
                            uint64_t timeout_ns, cudaStream_t stream);

// ---------------------------------------------------------------- dequant_gemm.cu
struct DequantGemmArgs {
  int format;            // 0 Marlin int4 g128, 1 fp8 e4m3 128x128 block
  int nmat;              // 2: gate/up pass (SwiGLU), 1: down / dense
  const void* w[2];      // Marlin int32 [E, K/16, 2N]; fp8 uint8 [E, N, K]
  const void* scale[2];  // Marlin bf16 [E, K/128, N] (stored order); fp8 fp32 [E, N/128, K/128]
  int E, K, N;
  const void* b0;        // activations [b_rows, K] (bf16 Marlin, fp16 fp8)
  const void* b1;
  int64_t b_rows;
  int tile_rows;
  const int* items;
  const int* num_items;
  int max_work;
  void* out;
  int64_t ld_out;
  int out_mode;          // 0 operand type, 1 fp32, 2 bf16
  float swiglu_limit;
  uint32_t* status;
};
cudaError_t dequant_gemm(const DequantGemmArgs& a, cudaStream_t stream);
cudaError_t gather_rows(const void* x, int64_t ld_x, int K, const int* src, void* out, int to_f16, int rows,
                        cudaStream_t stream);

}  // namespace b200

// Sparse-MLA tensor-core kernels: indexer logits (fp8, kind::f8f6f4) and
// latent attention over the selected cache rows (bf16, kind::f16).
//
// Reference contracts: `fp8_paged_mqa_logits` / `fp8_mqa_logits`
// (vllm_sm80/kernels/attention/triton_mqa_logits.py:1-25, 591: per query
// token, score(s) = sum_h w_h * relu(q_h . k_s) over a paged uint8 cache) and
// `sparse_mla_fwd(q, kv, indices, sm_scale, d_v=512) -> (out, max_logits,
// lse)` (vllm_sm80/kernels/attention/sparse_prefill_mla_pp.py:15-25;
// decode kernel triton_mla_sparse.py:473).
//
// Indexer (one CTA per (token, position split)): the query token's 64 fp8
// head vectors stay resident (TMA, 8 KiB); 128-position key tiles of the
// paged cache (block 64 -> two TMA boxes per tile) stream through a 4-stage
// ring; one thread issues D[128 pos x 64 heads] = K . Q^T (4 x K=32 fp8 MMAs)
// into one of two TMEM buffers; the epilogue thread of each position reduces
// its TMEM row: sum_h w_h relu(d_h) * k_scale.
//
// Attention: see the block-form kernel below (blocks of 128 positions, K chunks
// retained as V, P in tensor memory); splits are merged by merge_kernel.
#include "common.cuh"
#include "launch.h"
#include "tma_host.h"

namespace b200 {
namespace mla {

B200_DEVICE void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ============================================================================= indexer logits
namespace idx {
constexpr int kThreads = 192;
constexpr int STAGES = 4;
constexpr int A_BYTES = 128 * 128;  // 128 positions x 128 fp8
constexpr int B_BYTES = 64 * 128;   // 64 heads x 128 fp8
constexpr int SMEM = 1024 + STAGES * A_BYTES + B_BYTES + 64 * 4 + 256;

struct Params {
  const float* w;        // [T, 64] head weights (q scale folded in)
  const float* k_scale;  // [slots]
  const int* ctx_lens;   // [T]
  const int* token_seq;  // [T] -> block-table row
  const int* block_table;
  int64_t ld_bt;
  float* scores;  // [T, ld_scores]
  int64_t ld_scores;
  uint32_t* status;
};

__global__ void __launch_bounds__(kThreads, 1)
    indexer_kernel(const __grid_constant__ CUtensorMap tma_k, const __grid_constant__ CUtensorMap tma_q, Params p) {
  pdl_prologue();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;
  float* sw = reinterpret_cast<float*>(sb + B_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sw + 64);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* qbar = bars + 2 * STAGES + 4;
  uint64_t* drain = bars + 2 * STAGES + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ctx = p.ctx_lens[t];
  const int ntiles = (ctx + 127) / 128;
  const int nblocks = (ctx + 63) / 64;
  const int* bt = p.block_table + (int64_t)(p.token_seq ? p.token_seq[t] : t) * p.ld_bt;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(qbar, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 64) sw[threadIdx.x] = p.w[(int64_t)t * 64 + threadIdx.x];
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(qbar, B_BYTES);
      tma_load_2d(sb, &tma_q, qbar, 0, t * 64);
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      bool ok = true;
      for (int tile = blockIdx.y; tile < ntiles && ok; tile += gridDim.y) {
        if (!mbar_wait_or_abort(&empty[stage], phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        const int b0 = bt[tile * 2];
        const int b1 = tile * 2 + 1 < nblocks ? bt[tile * 2 + 1] : b0;
        mbar_arrive_expect_tx(&full[stage], A_BYTES);
        tma_load_2d(sa + stage * A_BYTES, &tma_k, &full[stage], 0, b0 * 64);
        tma_load_2d(sa + stage * A_BYTES + 64 * 128, &tma_k, &full[stage], 0, b1 * 64);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        const uint32_t n = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t k = issued - 1 - i;
          mbar_wait(&full[k % STAGES], (k / STAGES) & 1, nullptr);
        }
      }
      mbar_wait(qbar, 0, nullptr);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_e4m3(128, 64);
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = mbar_wait_or_abort(qbar, 0, p.status, abort_flag);
      tc_fence_after();
      for (int tile = blockIdx.y; tile < ntiles && ok; tile += gridDim.y, ++local) {
        const int acc = local & 1;
        if (!mbar_wait_or_abort(&tempty[acc], ((local >> 1) & 1) ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        if (!mbar_wait_or_abort(&full[stage], phase, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = desc_kmajor_sw128(sa + stage * A_BYTES);
        const uint64_t db = desc_kmajor_sw128(sb);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f8(tmem_base + acc * 64, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
        umma_commit(&empty[stage]);
        umma_commit(&tfull[acc]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.y; tile < ntiles; tile += gridDim.y, ++local) {
      const int acc = local & 1;
      const bool got = mbar_wait_or_abort(&tfull[acc], (local >> 1) & 1, p.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;  // TMEM loads are warp-collective
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * 64;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) s += sw[c + i] * fmaxf(__uint_as_float(r[i]), 0.f);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      const int pos = tile * 128 + q * 32 + lane;
      if (pos < ctx) {
        const int64_t slot = (int64_t)bt[pos >> 6] * 64 + (pos & 63);
        p.scores[(int64_t)t * p.ld_scores + pos] = s * p.k_scale[slot];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 128);
  }
}
}  // namespace idx

// ============================================================================= split merge
namespace attn {
constexpr float kLog2e = 1.4426950408889634f;

// merge split partials: out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s
__global__ void merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits, int T,
                             int nh, __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                             const float* __restrict__ sink, int c_lo, int c_hi) {
  pdl_prologue();
  const int th = blockIdx.x;  // t * nh + h
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[((int64_t)s * T * nh + th) * 2]);
  float L = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_ml[((int64_t)s * T * nh + th) * 2];
    if (m != -INFINITY) L += exp2f(m - M) * part_ml[((int64_t)s * T * nh + th) * 2 + 1];
  }
  if (threadIdx.x == 0 && lse) lse[th] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
  // a sink adds exp(sink) to the denominator only (not to the returned log-sum-exp)
  if (sink != nullptr && M != -INFINITY) L += exp2f(sink[th % nh] * kLog2e - M);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int c = c_lo + threadIdx.x; c < c_hi; c += blockDim.x) {  // the output dims the splits computed
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float m = part_ml[((int64_t)s * T * nh + th) * 2];
      if (m != -INFINITY) acc += exp2f(m - M) * part_o[((int64_t)s * T * nh + th) * 512 + c];
    }
    out[(int64_t)th * 512 + c] = __float2bfloat16(acc * inv);
  }
}
}  // namespace attn


// ============================================================================= sparse attention, block form
// One CTA per (token, head group of 128, latent half, split); the split's
// positions are processed in blocks of 128.
//   QK   S[128 heads x 128 pos] = sum over the 9 dim chunks of Q_c K_c^T.
//        A K chunk (128 gathered rows x 64 dims) is copied with cp.async
//        into the 128-byte-swizzled layout: the 8 lanes of a row write one
//        128-byte line (coalesced, bank-conflict free).  That layout is at
//        once the K-major B operand of Q K^T (rows = positions) and the
//        MN-major B operand of P V (64-dim atoms, 8 positions per 1024-byte
//        row group), so the 4 chunks holding this CTA's latent half are
//        RETAINED (double-buffered across blocks) and serve as V: no second
//        gather.  The other 5 chunks stream through a 3-stage ring.  Copies
//        complete on mbarriers (cp.async.mbarrier.arrive), so up to 11
//        chunks are in flight per SM.
//   softmax  one head row per thread: exact max / exp over the block, a lazy
//        rescale of the O accumulator across blocks; P is converted to bf16
//        in place in TMEM (over its S columns).
//   PV   O[128 x 256 latent dims of this half] += P V, A = P from TMEM.
// The MMA thread interleaves Q K^T of block b with P V of block b - 1, so the
// softmax of one block overlaps the next block's Q K^T.
// TMEM columns: S/P 0 [0, 128), S/P 1 [128, 256), O [256, 512).
namespace attn4 {
constexpr int kThreads = 320;  // w0 Q TMA, w1-4 gather, w5 MMA, w6-9 softmax + epilogue
constexpr int BP = 128;        // positions per block
// Row width D (template): 576 = MLA latent 512 + RoPE 64 (V = the latent), or 512 = DeepSeek-V4.1
// rows (RoPE tail inside; V = the whole row).  Either way V is 512 dims, 256 per latent half.
constexpr int NRET = 4;                 // retained chunks = this half's 256 V dims
template <int D>
struct Geo {
  static constexpr int NCH = D / 64;             // dim chunks: 9 or 8
  static constexpr int NSTREAM = NCH - NRET;     // chunks outside this half's V dims: 5 or 4
};
constexpr int CH_BYTES = BP * 128;      // 16 KiB: 128 positions x 64 dims
constexpr int Q_BYTES = 128 * 128;      // 16 KiB: 128 head rows x 64 dims
constexpr int NQ = 3, NKS = 3;          // Q ring, streamed-K ring
constexpr int R_BYTES = NRET * CH_BYTES;  // 64 KiB per retained buffer (x2)
constexpr int OFF_Q = 0;
constexpr int OFF_KS = OFF_Q + NQ * Q_BYTES;
constexpr int OFF_R = OFF_KS + NKS * CH_BYTES;
constexpr int OFF_BAR = OFF_R + 2 * R_BYTES;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.f;

struct Params {
  const int* indices;
  const int* counts;
  int topk;
  int nh;
  const __nv_bfloat16* cache;
  float sm_scale_log2;
  int splits;
  int q_box_rows;
  __nv_bfloat16* out;
  float* part_o;
  float* part_ml;
  float* lse;
  const float* sink;  // per-head softmax sink logit (natural-log units, already scaled), or null
  int T;
  uint32_t* status;
  // -1: both latent halves (grid z = 2 x splits); 0 or 1: only that half of the output dims (grid z = splits)
  int only_half;
  // dense causal mode (grouped-query attention over paged [K | V] rows): when dense_ctx is set, query row
  // t is (token t / kv_heads, key-value head t % kv_heads); it attends positions [0, dense_ctx[token]) of
  // its sequence, whose rows are (block_table[seq][pos / 64] * 64 + pos % 64) * kv_heads + head
  const int* dense_ctx;
  const int* dense_seq;
  const int* dense_bt;
  int64_t dense_ld_bt;
  int dense_kv_heads;
};

// byte offset of (row r, 16-byte chunk c) in a 128-byte-swizzled tile of 128-byte rows
B200_DEVICE uint32_t sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

// dim chunk processed i-th in a block: first the chunks outside this half's V dims (the other
// half's, then the RoPE chunk 8 when D = 576), then this half's 4 (retained as V)
template <int D>
B200_DEVICE int chunk_at(int i, int half) {
  if (i >= Geo<D>::NSTREAM) return half * 4 + (i - Geo<D>::NSTREAM);
  return half == 0 ? 4 + i : (i < 4 ? i : i + 4);
}

B200_DEVICE void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

// arrive on `bar` once all of this thread's earlier cp.async copies have landed (the barrier's
// expected count includes this arrival)
B200_DEVICE void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_attn_block_kernel(const __grid_constant__ CUtensorMap tma_q, Params p) {
  constexpr int NCH = Geo<D>::NCH, NSTREAM = Geo<D>::NSTREAM;
  pdl_prologue();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sq = smem + OFF_Q;
  uint8_t* sks = smem + OFF_KS;
  uint8_t* sr = smem + OFF_R;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;         // NQ, TMA
  uint64_t* q_empty = bars + 3;    // NQ, MMA commit
  uint64_t* ks_full = bars + 6;    // NKS, 128 gather threads
  uint64_t* ks_empty = bars + 9;   // NKS, MMA commit
  uint64_t* r_full = bars + 12;    // [2][NRET], 128 gather threads, one phase per use
  uint64_t* r_empty = bars + 20;   // 2, MMA commit after P V
  uint64_t* s_full = bars + 22;    // 2, MMA commit after Q K^T
  uint64_t* p_full = bars + 24;    // 2, 128 softmax threads
  uint64_t* pv_done = bars + 26;   // 2, MMA commit after P V
  uint64_t* o_full = bars + 28;
  uint64_t* drain = bars + 29;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 30);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = blockIdx.x;
  const int hg = blockIdx.y;
  const int half = p.only_half >= 0 ? p.only_half : (int)(blockIdx.z & 1);
  const int split = p.only_half >= 0 ? (int)blockIdx.z : (int)(blockIdx.z >> 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool dense = p.dense_ctx != nullptr;
  const int count = dense ? p.dense_ctx[t / p.dense_kv_heads] : min(p.counts[t], p.topk);
  const int nblk_all = (count + BP - 1) / BP;
  const int per = (nblk_all + p.splits - 1) / p.splits;
  const int blk0 = split * per;
  const int nb = max(0, min(nblk_all, blk0 + per) - blk0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NQ; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < NKS; ++i) {
      mbar_init(&ks_full[i], 128);
      mbar_init(&ks_empty[i], 1);
    }
    for (int i = 0; i < 2 * NRET; ++i) mbar_init(&r_full[i], 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&r_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Q rows past the group's real heads are never loaded: keep them zero
  for (int i = threadIdx.x; i < NQ * Q_BYTES / 16; i += kThreads) reinterpret_cast<uint4*>(sq)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tO = tmem_base + 256;

  if (warp == 0) {
    // ------------------------------------------------------------------ Q chunks (TMA), in MMA order
    if (elect_one()) {
      const int row0 = t * p.nh + hg * 128;
      const uint32_t q_bytes = (uint32_t)p.q_box_rows * 128;
      uint32_t issued = 0;
      bool ok = true;
      for (int b = 0; b < nb && ok; ++b) {
        for (int i = 0; i < NCH; ++i) {
          const uint32_t st = issued % NQ, ph = (issued / NQ) & 1;
          if (!mbar_wait_or_abort(&q_empty[st], ph ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[st], q_bytes);
          tma_load_2d(sq + st * Q_BYTES, &tma_q, &q_full[st], chunk_at<D>(i, half) * 64, row0);
          ++issued;
        }
      }
      if (!ok) {  // let the loads in flight land before the CTA exits
        const uint32_t n = issued < (uint32_t)NQ ? issued : (uint32_t)NQ;
        for (uint32_t j = 0; j < n; ++j) {
          const uint32_t k = issued - 1 - j;
          mbar_wait(&q_full[k % NQ], (k / NQ) & 1, nullptr);
        }
      }
    }
  } else if (warp >= 1 && warp <= 4) {
    // ------------------------------------------------------------------ row gathers (128 threads)
    // A warp instruction copies 4 rows x 128 bytes; warp gw copies the rows r with r % 4 == gw,
    // and lane l holds the cache row index of block row 4 l + gw.
    const int gw = warp - 1;
    const int sub = lane >> 3, ch = lane & 7;
    const int* idx_g = dense ? nullptr : p.indices + (int64_t)t * p.topk;
    const int* bt_g = dense ? p.dense_bt + (int64_t)p.dense_seq[t / p.dense_kv_heads] * p.dense_ld_bt : nullptr;
    const int kvh = dense ? t % p.dense_kv_heads : 0;
    auto fetch_idx = [&](int b) -> int {
      const int pos = (blk0 + b) * BP + lane * 4 + gw;
      if (pos >= count) return -1;
      return dense ? (bt_g[pos >> 6] * 64 + (pos & 63)) * p.dense_kv_heads + kvh : idx_g[pos];
    };
    int cur = nb > 0 ? fetch_idx(0) : -1;
    uint32_t ns = 0;
    bool ok = true;
    for (int b = 0; b < nb && ok; ++b) {
      const int nxt = b + 1 < nb ? fetch_idx(b + 1) : -1;  // in flight while this block's copies issue
      const int rb = b & 1;
      for (int i = 0; i < NCH; ++i) {
        const int c = chunk_at<D>(i, half);
        uint32_t dst;
        uint64_t* bar;
        if (i < NSTREAM) {
          const uint32_t st = ns % NKS, ph = (ns / NKS) & 1;
          // warp-uniform outcome: the copy loop below shuffles across all lanes
          if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&ks_empty[st], ph ^ 1, p.status, abort_flag))) {
            ok = false;
            break;
          }
          dst = smem_u32(sks + st * CH_BYTES);
          bar = &ks_full[st];
          ++ns;
        } else {
          // retained buffer rb was V of block b - 2: wait until its P V has run
          if (i == NSTREAM && b >= 2 &&
              !__all_sync(0xffffffffu, mbar_wait_or_abort(&r_empty[rb], ((b >> 1) - 1) & 1, p.status, abort_flag))) {
            ok = false;
            break;
          }
          dst = smem_u32(sr + rb * R_BYTES + (i - NSTREAM) * CH_BYTES);
          bar = &r_full[rb * NRET + (i - NSTREAM)];
        }
#pragma unroll
        for (int it = 0; it < BP / 16; ++it) {
          const int r = it * 16 + sub * 4 + gw;
          const int slot = __shfl_sync(0xffffffffu, cur, it * 4 + sub);
          const void* src = slot >= 0 ? reinterpret_cast<const void*>(p.cache + (int64_t)slot * D + c * 64 + ch * 8)
                                      : reinterpret_cast<const void*>(p.cache);
          cp_async16(dst + sw128(r, ch), src, slot >= 0 ? 16u : 0u);
        }
        cp_async_arrive(bar);
      }
      cur = nxt;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = make_idesc_f16(128, BP, 1);
      constexpr uint32_t idesc_pv = make_idesc_f16(128, 256, 1, false, true);
      uint32_t nq = 0, nk = 0;
      bool ok = true;
      auto qk_block = [&](int b) -> bool {
        const int sb = b & 1;
        // S/P buffer sb last held P of block b - 2: its P V must have read it
        if (b >= 2 && !mbar_wait_or_abort(&pv_done[sb], ((b >> 1) - 1) & 1, p.status, abort_flag)) return false;
        const uint32_t ts = tmem_base + (uint32_t)sb * BP;
        for (int i = 0; i < NCH; ++i) {
          const uint32_t qs = nq % NQ, qph = (nq / NQ) & 1;
          if (!mbar_wait_or_abort(&q_full[qs], qph, p.status, abort_flag)) return false;
          uint32_t kbase;
          uint32_t kst = 0;
          if (i < NSTREAM) {
            kst = nk % NKS;
            if (!mbar_wait_or_abort(&ks_full[kst], (nk / NKS) & 1, p.status, abort_flag)) return false;
            kbase = smem_u32(sks + kst * CH_BYTES);
          } else {
            if (!mbar_wait_or_abort(&r_full[sb * NRET + (i - NSTREAM)], (b >> 1) & 1, p.status, abort_flag))
              return false;
            kbase = smem_u32(sr + sb * R_BYTES + (i - NSTREAM) * CH_BYTES);
          }
          fence_proxy_async_smem();  // the rows were written by cp.async (generic proxy)
          tc_fence_after();
          const uint64_t dq = desc_kmajor_sw128(sq + qs * Q_BYTES);
          const uint64_t dk = make_smem_desc(kbase, 16, 1024, kSwizzle128B);
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16(ts, dq + 2 * k, dk + 2 * k, idesc_qk, (i > 0 || k > 0) ? 1u : 0u);
          umma_commit(&q_empty[qs]);
          ++nq;
          if (i < NSTREAM) {
            umma_commit(&ks_empty[kst]);
            ++nk;
          }
        }
        umma_commit(&s_full[sb]);
        return true;
      };
      auto pv_block = [&](int b) -> bool {
        const int sb = b & 1;
        if (!mbar_wait_or_abort(&p_full[sb], (b >> 1) & 1, p.status, abort_flag)) return false;
        tc_fence_after();
        const uint32_t pa = tmem_base + (uint32_t)sb * BP;  // P: 128 positions = 64 columns of bf16 pairs
        const uint32_t rbase = smem_u32(sr + sb * R_BYTES);
#pragma unroll
        for (int kk = 0; kk < BP / 16; ++kk) {
          // V: 16 positions = two 1024-byte row groups; the next 64 latent dims = the next retained chunk
          const uint64_t dv = make_smem_desc(rbase + kk * 2048, CH_BYTES /*LBO*/, 1024 /*SBO*/, kSwizzle128B);
          umma_f16_ts(tO, pa + kk * 8, dv, idesc_pv, (b > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&r_empty[sb]);
        umma_commit(&pv_done[sb]);
        return true;
      };
      for (int b = 0; b <= nb && ok; ++b) {
        if (b < nb) ok = qk_block(b);
        if (ok && b >= 1) ok = pv_block(b - 1);
      }
      if (ok && nb > 0) umma_commit(o_full);
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 6..9)
    const int q = warp & 3;
    const int h = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int b = 0; b < nb; ++b) {
      const int sb = b & 1;
      if (!mbar_wait_or_abort(&s_full[sb], (b >> 1) & 1, p.status, abort_flag)) ok = false;
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = tmem_base + lane_off + (uint32_t)sb * BP;
      const int valid = min(BP, count - (blk0 + b) * BP);
      float mt = -INFINITY;
      for (int c = 0; c < BP; c += 16) {
        uint32_t r[16];
        tmem_ld16(ts + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c + j < valid) mt = fmaxf(mt, __uint_as_float(r[j]) * p.sm_scale_log2);
      }
      const bool need = (mt > m_run + kRescaleThreshold) || (m_run == -INFINITY);
      const float m_new = need ? fmaxf(mt, m_run) : m_run;
      const bool need_o = need && b > 0 && m_run != -INFINITY;
      if (__any_sync(0xffffffffu, need_o)) {
        // O holds every earlier P V only once block b - 1's has completed
        if (!mbar_wait_or_abort(&pv_done[(b - 1) & 1], ((b - 1) >> 1) & 1, p.status, abort_flag)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = need_o ? exp2f(m_run - m_new) : 1.f;
        for (int c = 0; c < 256; c += 16) {
          uint32_t r[16];
          tmem_ld16(tO + lane_off + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * f);
          tmem_st16(tO + lane_off + c, r);
        }
        tmem_wait_st();
        l_run *= f;
      }
      m_run = m_new;
      // P in place: positions c..c+15 (S columns c..c+15, already read) -> bf16 pair columns c/2..c/2+7
      for (int c = 0; c < BP; c += 16) {
        uint32_t r[16];
        tmem_ld16(ts + c, r);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float e0 = (c + 2 * j < valid) ? exp2f(__uint_as_float(r[2 * j]) * p.sm_scale_log2 - m_run) : 0.f;
          const float e1 = (c + 2 * j + 1 < valid) ? exp2f(__uint_as_float(r[2 * j + 1]) * p.sm_scale_log2 - m_run)
                                                   : 0.f;
          l_run += e0 + e1;
          pk[j] = pack_bf16x2(e0, e1);
        }
        tmem_st8(ts + c / 2, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    // ---------------------------------------------------------------- epilogue
    const int head = hg * 128 + h;
    bool o_ok = ok && nb > 0;
    if (o_ok) o_ok = mbar_wait_or_abort(o_full, 0, p.status, abort_flag);
    if (__all_sync(0xffffffffu, o_ok)) {
      tc_fence_after();
      float l_tot = l_run;
      if (p.sink != nullptr && p.splits == 1 && head < p.nh) l_tot += exp2f(p.sink[head] * kLog2e - m_run);
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      for (int c = 0; c < 256; c += 16) {
        uint32_t r[16];
        tmem_ld16(tO + lane_off + c, r);
        tmem_wait_ld();
        if (head < p.nh) {
          const int64_t base = ((int64_t)t * p.nh + head) * 512 + half * 256 + c;
          if (p.splits == 1) {
            uint4 v0, v1;
            v0.x = pack_bf16x2(__uint_as_float(r[0]) * inv, __uint_as_float(r[1]) * inv);
            v0.y = pack_bf16x2(__uint_as_float(r[2]) * inv, __uint_as_float(r[3]) * inv);
            v0.z = pack_bf16x2(__uint_as_float(r[4]) * inv, __uint_as_float(r[5]) * inv);
            v0.w = pack_bf16x2(__uint_as_float(r[6]) * inv, __uint_as_float(r[7]) * inv);
            v1.x = pack_bf16x2(__uint_as_float(r[8]) * inv, __uint_as_float(r[9]) * inv);
            v1.y = pack_bf16x2(__uint_as_float(r[10]) * inv, __uint_as_float(r[11]) * inv);
            v1.z = pack_bf16x2(__uint_as_float(r[12]) * inv, __uint_as_float(r[13]) * inv);
            v1.w = pack_bf16x2(__uint_as_float(r[14]) * inv, __uint_as_float(r[15]) * inv);
            reinterpret_cast<uint4*>(p.out + base)[0] = v0;
            reinterpret_cast<uint4*>(p.out + base)[1] = v1;
          } else {
            float* dst = p.part_o + (int64_t)split * p.T * p.nh * 512 + base;
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          }
        }
      }
    } else if (head < p.nh && nb == 0) {
      if (p.splits == 1) {
        for (int c = 0; c < 256; ++c) p.out[((int64_t)t * p.nh + head) * 512 + half * 256 + c] = __float2bfloat16(0.f);
      } else {
        float* dst = p.part_o + (int64_t)split * p.T * p.nh * 512 + ((int64_t)t * p.nh + head) * 512 + half * 256;
        for (int c = 0; c < 256; ++c) dst[c] = 0.f;
      }
    }
    if (head < p.nh && half == (p.only_half >= 0 ? p.only_half : 0)) {
      if (p.splits > 1) {
        float* ml = p.part_ml + (((int64_t)split * p.T + t) * p.nh + head) * 2;
        ml[0] = nb > 0 ? m_run : -INFINITY;
        ml[1] = nb > 0 ? l_run : 0.f;
      } else if (p.lse) {
        p.lse[(int64_t)t * p.nh + head] = l_run > 0.f ? (m_run + log2f(l_run)) / kLog2e : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}
}  // namespace attn4

}  // namespace mla

cudaError_t mla_indexer_scores(const void* q8, const float* w, int T, const void* k_cache, int64_t num_slots,
                               const float* k_scale, const int* ctx_lens, const int* token_seq, const int* block_table,
                               int64_t ld_bt, float* scores, int64_t ld_scores, int max_ctx, uint32_t* status,
                               cudaStream_t stream) {
  using namespace mla::idx;
  if (T == 0) return cudaSuccess;
  CUtensorMap tk = make_tma_2d(k_cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, num_slots, 128, 128, 64, 128,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tq = make_tma_2d(q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)T * 64, 128, 128, 64, 128,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  Params p{w, k_scale, ctx_lens, token_seq, block_table, ld_bt, scores, ld_scores, status};
  cudaError_t e = cudaFuncSetAttribute(indexer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return e;
  const int tiles = (max_ctx + 127) / 128;
  const int sms = device_sm_count();
  int ysplit = std::max(1, std::min(tiles, (2 * sms + T - 1) / T));
  dim3 grid(T, ysplit);
  launch_pdl(indexer_kernel, dim3(grid), dim3(kThreads), SMEM, stream, tk, tq, p);
  return cudaGetLastError();
}

namespace {
template <int D>
cudaError_t launch_sparse_attention(const CUtensorMap& tq, const mla::attn4::Params& p, int T, int nh, int splits,
                                    cudaStream_t stream) {
  using namespace mla::attn4;
  cudaError_t e = cudaFuncSetAttribute(sparse_attn_block_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(T, (nh + 127) / 128, (p.only_half >= 0 ? 1 : 2) * splits);
  launch_pdl(sparse_attn_block_kernel<D>, dim3(grid), dim3(kThreads), SMEM, stream, tq, p);
  return cudaGetLastError();
}
}  // namespace

cudaError_t mla_sparse_attention(const void* q, int T, int nh, int dim, const void* cache, const int* indices,
                                 const int* counts, int topk, float sm_scale, int splits, void* out, float* part_o,
                                 float* part_ml, float* lse, const float* sink, uint32_t* status,
                                 cudaStream_t stream, int only_half) {
  using namespace mla::attn4;
  if (T == 0) return cudaSuccess;
  if (dim != 512 && dim != 576) return cudaErrorInvalidValue;
  if (only_half < -1 || only_half > 1) return cudaErrorInvalidValue;
  const int DIM = dim;
  const int box_rows = nh >= 128 ? 128 : (nh + 7) / 8 * 8;
  CUtensorMap tq = make_tma_2d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)T * nh, DIM, DIM, box_rows, 64,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  Params p{};
  p.q_box_rows = box_rows;
  p.indices = indices;
  p.counts = counts;
  p.topk = topk;
  p.nh = nh;
  p.cache = reinterpret_cast<const __nv_bfloat16*>(cache);
  p.sm_scale_log2 = sm_scale * kLog2e;
  p.splits = splits;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.lse = lse;
  p.sink = sink;
  p.T = T;
  p.status = status;
  p.only_half = only_half;
  cudaError_t e = dim == 512 ? launch_sparse_attention<512>(tq, p, T, nh, splits, stream)
                             : launch_sparse_attention<576>(tq, p, T, nh, splits, stream);
  if (e != cudaSuccess || splits == 1) return e;
  const int c_lo = only_half == 1 ? 256 : 0, c_hi = only_half == 0 ? 256 : 512;
  launch_pdl(mla::attn::merge_kernel, dim3(T * nh), dim3(128), 0, stream, part_o, part_ml, splits, T, nh,
             reinterpret_cast<__nv_bfloat16*>(out), lse, sink, c_lo, c_hi);
  return cudaGetLastError();
}

cudaError_t gqa_dense_attention(const void* q, int Tq, int group, const void* cache, const int* ctx_lens,
                                const int* token_seq, const int* block_table, int64_t ld_bt, int kv_heads,
                                float sm_scale, int splits, void* out, float* part_o, float* part_ml,
                                uint32_t* status, cudaStream_t stream) {
  using namespace mla::attn4;
  if (Tq == 0) return cudaSuccess;
  if (group < 1 || group > 128 || kv_heads < 1) return cudaErrorInvalidValue;
  const int box_rows = (group + 7) / 8 * 8;
  CUtensorMap tq = make_tma_2d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)Tq * group, 512, 512, box_rows, 64,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  Params p{};
  p.q_box_rows = box_rows;
  p.topk = 1 << 30;
  p.nh = group;
  p.cache = reinterpret_cast<const __nv_bfloat16*>(cache);
  p.sm_scale_log2 = sm_scale * kLog2e;
  p.splits = splits;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.T = Tq;
  p.status = status;
  p.only_half = 1;  // rows are [K (256) | V (256)]: the value dims are the upper half
  p.dense_ctx = ctx_lens;
  p.dense_seq = token_seq;
  p.dense_bt = block_table;
  p.dense_ld_bt = ld_bt;
  p.dense_kv_heads = kv_heads;
  cudaError_t e = launch_sparse_attention<512>(tq, p, Tq, group, splits, stream);
  if (e != cudaSuccess || splits == 1) return e;
  launch_pdl(mla::attn::merge_kernel, dim3(Tq * group), dim3(128), 0, stream, part_o, part_ml, splits, Tq, group,
             reinterpret_cast<__nv_bfloat16*>(out), static_cast<float*>(nullptr), static_cast<const float*>(nullptr),
             256, 512);
  return cudaGetLastError();
}

}  // namespace b200

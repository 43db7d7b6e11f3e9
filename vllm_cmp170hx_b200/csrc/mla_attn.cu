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
// Attention (one CTA per (token, head group of 128, latent half, split)):
//   * Q (heads x 576) streams in 64-dim chunks through TMA (128-byte swizzle);
//   * 4 gather warps copy the 64 selected latent rows of a tile
//     (64 x 1152 B) into shared memory as 8x16-byte core matrices, a layout
//     that is at once the K-major B operand of S = Q K^T (N = positions) and
//     the MN-major B operand of O += P V (N = latent dims);
//   * S (heads x 64 positions, fp32) double-buffers in TMEM; the softmax warps
//     (one head row per thread, no cross-thread reductions) keep a running
//     max with lazy rescaling of the TMEM accumulator, write P (bf16) into
//     shared memory as the A operand of P V;
//   * O (heads x 256 latent dims of this CTA's half) accumulates in TMEM.
//   The 576-dim QK^T is recomputed by the two latent halves: TMEM (512 fp32
//   columns per lane) cannot hold the full 128 x 512 O next to S.
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

// ============================================================================= sparse attention
namespace attn {
constexpr int kThreads = 320;           // 10 warps
constexpr int PT = 64;                  // positions per tile
constexpr int DIM = 576;                // latent 512 + rope 64
constexpr int KV_BYTES = PT * DIM * 2;  // 73728
constexpr int Q_BYTES = 128 * 64 * 2;   // one 64-dim chunk of 128 head rows
constexpr int QST = 3;
constexpr int P_BYTES = 128 * PT * 2;   // 16384
constexpr int SMEM = 1024 + 2 * KV_BYTES + QST * Q_BYTES + 2 * P_BYTES + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.f;  // log2 units

struct Params {
  const int* indices;  // [T, topk] cache rows (-1 = none)
  const int* counts;   // [T]
  int topk;
  int nh;              // heads of the token
  const __nv_bfloat16* cache;  // [slots, 576]
  float sm_scale_log2;
  int splits;
  int q_box_rows;      // rows of Q loaded per chunk (real heads of the group, <= 128)
  __nv_bfloat16* out;  // [T, nh, 512] (splits == 1)
  float* part_o;       // [splits, T, nh, 512] (splits > 1)
  float* part_ml;      // [splits, T, nh, 2] (max, sum) log2 domain
  float* lse;          // [T, nh] natural log (splits == 1, optional)
  int T;
  uint32_t* status;
};

// core-matrix layout of a KV tile: (dim group di, pos group pi) at (di*8 + pi)*128, row r at +16r
B200_DEVICE uint32_t kv_off(int pos, int chunk) { return (uint32_t)((chunk * 8 + (pos >> 3)) * 128 + (pos & 7) * 16); }

__global__ void __launch_bounds__(kThreads, 1)
    sparse_attn_kernel(const __grid_constant__ CUtensorMap tma_q, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* skv = smem;                          // [2][KV_BYTES]
  uint8_t* sq = smem + 2 * KV_BYTES;            // [QST][Q_BYTES]
  uint8_t* sp = sq + QST * Q_BYTES;             // [2][P_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * P_BYTES);
  uint64_t* kv_full = bars;        // 2, count 4 (gather warps)
  uint64_t* kv_empty = bars + 2;   // 2, MMA commit
  uint64_t* q_full = bars + 4;     // QST (<= 4)
  uint64_t* q_empty = bars + 8;    // QST
  uint64_t* s_full = bars + 12;    // 2
  uint64_t* p_full = bars + 14;    // 2, count 128
  uint64_t* p_empty = bars + 16;   // 2
  uint64_t* o_full = bars + 18;
  uint64_t* drain = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = blockIdx.x;
  const int hg = blockIdx.y;        // head group of 128
  const int half = blockIdx.z % 2;  // latent half
  const int split = blockIdx.z / 2;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int count = p.counts[t];
  const int ntiles_all = (count + PT - 1) / PT;
  const int per = (ntiles_all + p.splits - 1) / p.splits;
  const int tile0 = split * per;
  const int tile1 = min(ntiles_all, tile0 + per);
  const int nt = max(0, tile1 - tile0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < QST; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 4);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tS = tmem_base;        // 2 x 64 columns
  const uint32_t tO = tmem_base + 256;  // 256 columns

  if (warp == 0) {
    // ------------------------------------------------------------------ Q chunk producer
    if (elect_one()) {
      int qs = 0;
      uint32_t qph = 0, issued = 0;
      bool ok = true;
      const int row0 = t * p.nh + hg * 128;
      // only this group's real head rows are loaded; the MMA's other rows
      // read stale shared memory and their TMEM rows are never used
      const uint32_t q_bytes = (uint32_t)p.q_box_rows * 128;
      for (int i = 0; i < nt && ok; ++i) {
        for (int c = 0; c < DIM / 64; ++c) {
          if (!mbar_wait_or_abort(&q_empty[qs], qph ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[qs], q_bytes);
          tma_load_2d(sq + qs * Q_BYTES, &tma_q, &q_full[qs], c * 64, row0);
          ++issued;
          if (++qs == QST) {
            qs = 0;
            qph ^= 1;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        const uint32_t n = issued < (uint32_t)QST ? issued : (uint32_t)QST;
        for (uint32_t j = 0; j < n; ++j) {
          const uint32_t k = issued - 1 - j;
          mbar_wait(&q_full[k % QST], (k / QST) & 1, nullptr);
        }
      }
    }
  } else if (warp >= 1 && warp <= 4) {
    // ------------------------------------------------------------------ KV gather (128 threads)
    const int gw = warp - 1;
    const int* idx = p.indices + (int64_t)t * p.topk;
    for (int i = 0; i < nt; ++i) {
      const int b = i & 1;
      if (!mbar_wait_or_abort(&kv_empty[b], ((i >> 1) & 1) ^ 1, p.status, abort_flag)) break;
      uint8_t* dst = skv + b * KV_BYTES;
      const int pbase = (tile0 + i) * PT;
      // warp iteration: 8 rows x 4 chunks; 8 row groups x 18 chunk groups =
      // 144 iterations over 4 warps.  Every copy is issued before any wait
      // (cp.async, 16 B, zero-filled for positions without a row).
      for (int it = gw; it < 144; it += 4) {
        const int rg = it / 18, cgp = it % 18;
        const int pos = rg * 8 + (lane & 7);
        const int chunk = cgp * 4 + (lane >> 3);
        const int gp = pbase + pos;
        const int slot = gp < count ? idx[gp] : -1;
        const void* src = slot >= 0 ? reinterpret_cast<const void*>(reinterpret_cast<const uint4*>(p.cache +
                                                                     (int64_t)slot * DIM) + chunk)
                                    : reinterpret_cast<const void*>(p.cache);
        const uint32_t sz = slot >= 0 ? 16u : 0u;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst + kv_off(pos, chunk))),
                     "l"(src), "r"(sz)
                     : "memory");
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_full[b]);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = make_idesc_f16(128, PT, 1);
      constexpr uint32_t idesc_pv = make_idesc_f16(128, 256, 1, false, true);
      int qs = 0;
      uint32_t qph = 0;
      bool ok = true;
      auto issue_qk = [&](int i) -> bool {
        const int b = i & 1;
        if (!mbar_wait_or_abort(&kv_full[b], (i >> 1) & 1, p.status, abort_flag)) return false;
        tc_fence_after();
        const uint32_t kv_base = smem_u32(skv + b * KV_BYTES);
        for (int c = 0; c < DIM / 64; ++c) {
          if (!mbar_wait_or_abort(&q_full[qs], qph, p.status, abort_flag)) return false;
          tc_fence_after();
          const uint64_t dq = desc_kmajor_sw128(sq + qs * Q_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int di0 = c * 8 + 2 * k;  // 16 dims = 2 dim groups
            const uint64_t dk = make_smem_desc(kv_base + di0 * 8 * 128, 8 * 128 /*LBO: next dim group*/,
                                               128 /*SBO: next pos group*/, kSwizzleNone);
            umma_f16(tS + b * 64, dq + 2 * k, dk, idesc_qk, (c > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&q_empty[qs]);
          if (++qs == QST) {
            qs = 0;
            qph ^= 1;
          }
        }
        umma_commit(&s_full[b]);
        return true;
      };
      if (nt > 0) ok = issue_qk(0);
      for (int i = 0; i < nt && ok; ++i) {
        const int b = i & 1;
        if (i + 1 < nt) {
          ok = issue_qk(i + 1);
          if (!ok) break;
        }
        if (!mbar_wait_or_abort(&p_full[b], (i >> 1) & 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t p_base = smem_u32(sp + b * P_BYTES);
        const uint32_t kv_base = smem_u32(skv + b * KV_BYTES);
#pragma unroll
        for (int k = 0; k < PT / 16; ++k) {
          const uint64_t dp = make_smem_desc(p_base + 2 * k * 2048, 2048, 128, kSwizzleNone);
          // V (MN-major): latent dims of this half = dim groups [32*half, 32*half + 32); K = positions 16k..
          const uint64_t dv = make_smem_desc(kv_base + ((half * 32) * 8 + 2 * k) * 128, 128 /*LBO: next pos group*/,
                                             8 * 128 /*SBO: next dim group*/, kSwizzleNone);
          umma_f16(tO, dp, dv, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[b]);
        umma_commit(&p_empty[b]);
      }
      if (ok) umma_commit(o_full);
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 6..9)
    const int q = warp & 3;  // TMEM lane quarter: head row = 32q + lane
    const int h = q * 32 + lane;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int i = 0; i < nt; ++i) {
      const int b = i & 1;
      if (!mbar_wait_or_abort(&s_full[b], (i >> 1) & 1, p.status, abort_flag)) ok = false;
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[PT];
      const uint32_t ta = tS + ((uint32_t)(q * 32) << 16) + b * 64;
#pragma unroll
      for (int c = 0; c < PT; c += 16) {
        uint32_t r[16];
        tmem_ld16(ta + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) s[c + j] = __uint_as_float(r[j]) * p.sm_scale_log2;
      }
      const int pbase = (tile0 + i) * PT;
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < PT; ++j) {
        if (pbase + j >= count) s[j] = -INFINITY;
        mt = fmaxf(mt, s[j]);
      }
      // Lazy rescale: a row moves its reference max only when the tile's max
      // exceeds it by more than 2^8.  TMEM loads/stores are warp-collective,
      // so the warp rescales together when any of its rows needs it (factor 1
      // for the others).
      const bool need = (mt > m_run + kRescaleThreshold) || (m_run == -INFINITY);
      const float m_new = need ? fmaxf(mt, m_run) : m_run;
      const bool need_o = need && i > 0 && m_run != -INFINITY;
      if (__any_sync(0xffffffffu, need_o)) {
        // O must hold every earlier PV before it is rescaled
        const int pb = (i - 1) & 1;
        if (!mbar_wait_or_abort(&p_empty[pb], ((i - 1) >> 1) & 1, p.status, abort_flag)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = need_o ? exp2f(m_run - m_new) : 1.f;
        const uint32_t to = tO + ((uint32_t)(q * 32) << 16);
        for (int c = 0; c < 256; c += 16) {
          uint32_t r[16];
          tmem_ld16(to + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * f);
          tmem_st16(to + c, r);
        }
        tmem_wait_st();
        l_run *= f;
      }
      m_run = m_new;
      // P buffer b is free once PV(i - 2) completed
      if (i >= 2 && !mbar_wait_or_abort(&p_empty[b], ((i - 2) >> 1) & 1, p.status, abort_flag)) {
        ok = false;
        break;
      }
      uint8_t* pb = sp + b * P_BYTES;
#pragma unroll
      for (int kg = 0; kg < PT / 8; ++kg) {
        float e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          e[j] = m_run == -INFINITY ? 0.f : exp2f(s[kg * 8 + j] - m_run);
          l_run += e[j];
        }
        uint4 v;
        v.x = pack_bf16x2(e[0], e[1]);
        v.y = pack_bf16x2(e[2], e[3]);
        v.z = pack_bf16x2(e[4], e[5]);
        v.w = pack_bf16x2(e[6], e[7]);
        // A operand (heads x positions, K-major core matrices): (kg, head group) at kg*2048 + (h/8)*128 + (h%8)*16
        *reinterpret_cast<uint4*>(pb + kg * 2048 + (h >> 3) * 128 + (h & 7) * 16) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
    }
    // ---------------------------------------------------------------- epilogue
    const int head = hg * 128 + h;
    bool o_ok = ok && nt > 0;
    if (o_ok) o_ok = mbar_wait_or_abort(o_full, 0, p.status, abort_flag);
    if (__all_sync(0xffffffffu, o_ok)) {
      tc_fence_after();
      const uint32_t to = tO + ((uint32_t)(q * 32) << 16);
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      for (int c = 0; c < 256; c += 16) {
        uint32_t r[16];
        tmem_ld16(to + c, r);
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
    } else if (head < p.nh && nt == 0) {
      // no positions in this split
      if (p.splits == 1) {
        for (int c = 0; c < 256; ++c) p.out[((int64_t)t * p.nh + head) * 512 + half * 256 + c] = __float2bfloat16(0.f);
      } else {
        float* dst = p.part_o + (int64_t)split * p.T * p.nh * 512 + ((int64_t)t * p.nh + head) * 512 + half * 256;
        for (int c = 0; c < 256; ++c) dst[c] = 0.f;
      }
    }
    if (head < p.nh && half == 0) {
      if (p.splits > 1) {
        float* ml = p.part_ml + (((int64_t)split * p.T + t) * p.nh + head) * 2;
        ml[0] = m_run;
        ml[1] = l_run;
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

// merge split partials: out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s
__global__ void merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits, int T,
                             int nh, __nv_bfloat16* __restrict__ out, float* __restrict__ lse) {
  const int th = blockIdx.x;  // t * nh + h
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[((int64_t)s * T * nh + th) * 2]);
  float L = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_ml[((int64_t)s * T * nh + th) * 2];
    if (m != -INFINITY) L += exp2f(m - M) * part_ml[((int64_t)s * T * nh + th) * 2 + 1];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int c = threadIdx.x; c < 512; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float m = part_ml[((int64_t)s * T * nh + th) * 2];
      if (m != -INFINITY) acc += exp2f(m - M) * part_o[((int64_t)s * T * nh + th) * 512 + c];
    }
    out[(int64_t)th * 512 + c] = __float2bfloat16(acc * inv);
  }
  if (threadIdx.x == 0 && lse) lse[th] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
}
}  // namespace attn

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
  indexer_kernel<<<grid, kThreads, SMEM, stream>>>(tk, tq, p);
  return cudaGetLastError();
}

cudaError_t mla_sparse_attention(const void* q, int T, int nh, const void* cache, const int* indices, const int* counts,
                                 int topk, float sm_scale, int splits, void* out, float* part_o, float* part_ml,
                                 float* lse, uint32_t* status, cudaStream_t stream) {
  using namespace mla::attn;
  if (T == 0) return cudaSuccess;
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
  p.T = T;
  p.status = status;
  cudaError_t e = cudaFuncSetAttribute(sparse_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(T, (nh + 127) / 128, 2 * splits);
  sparse_attn_kernel<<<grid, kThreads, SMEM, stream>>>(tq, p);
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  merge_kernel<<<T * nh, 128, 0, stream>>>(part_o, part_ml, splits, T, nh, reinterpret_cast<__nv_bfloat16*>(out), lse);
  return cudaGetLastError();
}

}  // namespace b200

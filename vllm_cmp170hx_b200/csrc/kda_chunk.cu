// KDA prefill in chunks of 64 tokens on tcgen05 (the chunk-parallel form of the gated delta rule with
// per-channel decay).
//
// Reference behaviour: vllm_sm80/models/glm5next/ops/kda_prefill.py:1064 (`chunk_kda_with_fused_gate`:
// gate + chunk-local cumsum, A = beta k k^T and Aqk = q k^T with the decay folded into the operands,
// (I + A)^-1 from 16x16 diagonal inverses, w / u, the sequential state pass, o = qg h^T + Aqk v_new).
// The token recurrence it evaluates is S <- S diag(e_t); u_t = beta_t (v_t - S k_t); S += u_t k_t^T;
// o_t = S q_t.  Within a chunk of C tokens from state S0, with G_t the cumulative log2-decay (per key
// channel) up to and including token t:
//
//   u   = T^-1 diag(beta) (V - (K*2^G) S0^T),   T = I + diag(beta) L,  L[t,s] = sum_k k_tk k_sk 2^(G_tk-G_sk), s < t
//   o_t = S0 (q_t*2^G_t) + sum_{s<=t} M[t,s] u_s,  M[t,s] = sum_k q_tk k_sk 2^(G_tk-G_sk)
//   S_C = S0 diag(2^G_C) + sum_s u_s (k_s*2^(G_C-G_s))^T
//
// Every exponent above is of a non-positive number except in L and M, which are formed per 16-row
// block b with the block's first cumulative decay R_b as reference: the row operand k_t 2^(G_t - R_b)
// (<= 1) against the column operand k_s 2^(R_b - G_s), which is <= 1 for earlier blocks and at most
// 2^(15 |lower bound| log2 e) inside the block (finite in bf16 for |lower bound| < 5.8; the host falls
// back to the recurrence otherwise); columns after the block are zero, never formed.
//
// B200 layout: a persistent CTA of 16 warps per (sequence, head) item, the fp32 state resident in TMEM
// for the whole sequence (128 lanes = value rows, 128 columns = key channels).  Per chunk, one thread
// issues five tcgen05 MMA groups (bf16 operands in 128-byte-swizzled shared memory, fp32 accumulate):
//   P   = [K 2^(G-R) ; Q 2^(G-R)] [K 2^(R-G)]_b^T           -> L and M (four blocks, N = 16 .. 64; hi/lo
//                                                           passes: three for L, two for M)
//   D2  = [Q 2^G ; K 2^G] S0^T                              (S0 as bf16 hi + lo: two passes)
//   U   = T^-1 R,  R = diag(beta) (V - K 2^G S0^T)          (T^-1 hi + lo, R hi + lo: three passes)
//   D2 += M U                                               (M hi + lo, U hi + lo: three passes)
//   S  += U^T (K 2^(G_C - G))                               (three hi/lo passes)
// The key-key products (L: the delta rule's correction can cancel, so its errors are amplified), the
// state and the value-side operands keep about 16 mantissa bits through the hi/lo splits; the decayed
// queries and the keys of the state products are bf16.  T^-1 (unit lower triangular) comes from the four 16x16 diagonal
// inverses by forward substitution and the off-diagonal blocks by block products, on the CUDA cores in
// fp32.  A prep kernel computes the per-token inputs in parallel first (conv1d + SiLU, L2 norms, the
// log2 decay, beta); the gated RMSNorm of the output runs in the chunk's epilogue.
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace kdac {

constexpr int D = 128;
constexpr int C = 64;
constexpr int kThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;

// shared memory (byte offsets from a 1024-aligned base).  Region X is reused three times per chunk:
// the operands of the first MMA group, then S0 (hi / lo) for the second, then the phase-2 tiles.
constexpr int OFF_A1H = 0;        // [K 2^(G-R) ; Q 2^(G-R)] hi: 128 rows x 128 K, two 64-wide K chunks of 16 KiB
constexpr int OFF_A1L = 32768;    // lo of the K rows; rows 64..127 zero (M needs no lo part)
constexpr int OFF_B1H = 65536;    // [K 2^(R_b - G)] hi for b = 0..3: 16 (b + 1) rows each, two K chunks
constexpr int OFF_B1L = 106496;   // lo
constexpr int REGION_X = 147456;
constexpr int OFF_B2H = 0;        // (after the first group) S0 hi: 128 value rows x 128 key K
constexpr int OFF_B2L = 32768;    // S0 lo
constexpr int OFF_A2 = REGION_X;  // [Q 2^G ; K 2^G]: 128 rows x 128 K
constexpr int OFF_KEH = OFF_A2 + 32768;   // K 2^(G_C - G) hi, MN-major: [64 tokens][128 keys] as two 64-key chunks
constexpr int OFF_KEL = OFF_KEH + 16384;  // lo
constexpr int OFF_SMALL = OFF_KEL + 16384;
constexpr int OFF_GC = OFF_SMALL;               // [128] f32 chunk-end decay (log2)
constexpr int OFF_BETA = OFF_GC + 512;          // [64] f32
constexpr int OFF_NSQ = OFF_BETA + 256;         // [4][64] f32 partial sums of squares of the output rows
constexpr int OFF_W = OFF_NSQ + 1024;           // [3][16][16] f32 block-product scratch
constexpr int OFF_NW = OFF_W + 3 * 1024;        // [128] bf16 output norm weights
constexpr int OFF_BAR = OFF_NW + 256;           // mbarrier + tmem slot + flags
constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;  // + alignment slack
// phase-2 tiles in region X (after the second group).  The rows 64.. of the 128-row A operands are read
// by the MMAs but never used: they hold stale, finite data of the earlier phases.
constexpr int OFF_TM = 0;                 // T fp32 [64][64]
constexpr int OFF_TI = 16384;             // T^-1 fp32 [64][64]
constexpr int OFF_A3 = 32768;             // M hi, K-major [128 rows][64]
constexpr int OFF_A3L = 49152;            // M lo
constexpr int OFF_A5H = 65536;            // T^-1 hi, K-major [128 rows][64]
constexpr int OFF_A5L = 81920;            // T^-1 lo
constexpr int OFF_RH = 98304;             // R hi, MN-major [64 rows][128 values]
constexpr int OFF_RL = 114688;            // R lo
constexpr int OFF_UH = 131072;            // U hi, MN-major [64 rows][128 values]
constexpr int OFF_UL = OFF_A2;            // U lo (the second group's A operand is free by then)
// B1 block b: rows 16 (b + 1), chunk stride rows * 128
__host__ __device__ constexpr int b1_off(int b) { return b == 0 ? 0 : b == 1 ? 4096 : b == 2 ? 12288 : 24576; }

// TMEM columns
constexpr uint32_t COL_S = 0, COL_P = 128, COL_U = 128, COL_D2 = 384;
__host__ __device__ constexpr uint32_t p_col(int b) { return COL_P + (b == 0 ? 0 : b == 1 ? 16 : b == 2 ? 48 : 96); }

// byte offset of (row r, 16-byte unit u) in a 128-byte-swizzled tile of 128-byte rows
B200_DEVICE uint32_t swz(int r, int u) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((u ^ (r & 7)) << 4)); }

// 2^x by the hardware's ex2.approx (relative error about 2^-22; flushes denormal results to zero, which
// only affects factors below 2^-126 that multiply unit-size operands)
B200_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bring `bytes` (multiple of 16) at a 16-byte aligned global address into L2 ahead of use
B200_DEVICE void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

B200_DEVICE uint4 pack8(const float (&x)[8]) {
  uint4 v;
  v.x = pack_bf16x2(x[0], x[1]);
  v.y = pack_bf16x2(x[2], x[3]);
  v.z = pack_bf16x2(x[4], x[5]);
  v.w = pack_bf16x2(x[6], x[7]);
  return v;
}
// hi = bf16(x), lo = bf16(x - hi)
B200_DEVICE void pack8_hilo(const float (&x)[8], uint4& hi, uint4& lo) {
  float h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[i] = __bfloat162float(__float2bfloat16(x[i]));
    l[i] = x[i] - h[i];
  }
  hi = pack8(h);
  lo = pack8(l);
}
B200_DEVICE void sts128(uint8_t* base, uint32_t off, uint4 v) { *reinterpret_cast<uint4*>(base + off) = v; }
B200_DEVICE void bf16x8_to_f32(uint4 v, float (&x)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// ----------------------------------------------------------------------------------- prep
// One warp per (token, head) of the sequences run in chunks: lane l owns channels 4l..4l+3 of q, k, v
// and of the gate.  Writes q (L2-normalised, scaled), k (L2-normalised), v (post conv + SiLU, bf16
// rounded like the recurrence), the log2 decay and beta.
__global__ void __launch_bounds__(256) kda_prep_kernel(KdaChunkArgs a) {
  pdl_prologue();
  const KdaArgs& p = a.k;
  const int wg = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (wg >= a.T * p.H) return;
  const int t = wg / p.H, h = wg % p.H;
  int lo = 0, hi = p.num_seqs;  // the sequence holding token t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.cu_seqlens[mid] <= t) lo = mid; else hi = mid;
  }
  const int t0 = p.cu_seqlens[lo], t1 = p.cu_seqlens[lo + 1];
  if (t1 - t0 < a.min_len) return;  // the recurrence runs this sequence
  const int i = t - t0;
  const int slot = p.state_idx ? p.state_idx[lo] : lo;
  const bool init = p.has_init ? p.has_init[lo] != 0 : true;
  const int HD = p.H * D;
  float y[3][4];
#pragma unroll
  for (int w = 0; w < 3; ++w) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t g = (int64_t)w * HD + h * D + lane * 4 + j;
      float x = __bfloat162float(p.qkv[(int64_t)t * p.ld_qkv + g]);
      if (p.conv_w) {
        float acc = (p.conv_b ? __bfloat162float(p.conv_b[g]) : 0.f) + __bfloat162float(p.conv_w[g * 4 + 3]) * x;
#pragma unroll
        for (int m = 1; m <= 3; ++m) {
          const int idx = i - m;
          float xm = 0.f;
          if (idx >= 0) xm = __bfloat162float(p.qkv[(int64_t)(t0 + idx) * p.ld_qkv + g]);
          else if (init) xm = __bfloat162float(p.conv_state[((int64_t)slot * 3 * HD + g) * 3 + 3 + idx]);
          acc += __bfloat162float(p.conv_w[g * 4 + 3 - m]) * xm;
        }
        x = __bfloat162float(__float2bfloat16(siluf_(acc)));
      }
      y[w][j] = x;
    }
  }
  float qn = p.q_scale, kn = 1.f;
  if (p.l2norm) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sq += y[0][j] * y[0][j];
      sk += y[1][j] * y[1][j];
    }
    qn *= rsqrtf(warp_sum(sq) + p.l2_eps);
    kn = rsqrtf(warp_sum(sk) + p.l2_eps);
  }
  const int64_t row = ((int64_t)h * a.T + t) * D + lane * 4;  // head-major: a chunk's rows are contiguous
  uint2 vq, vk, vv;
  vq.x = pack_bf16x2(y[0][0] * qn, y[0][1] * qn);
  vq.y = pack_bf16x2(y[0][2] * qn, y[0][3] * qn);
  vk.x = pack_bf16x2(y[1][0] * kn, y[1][1] * kn);
  vk.y = pack_bf16x2(y[1][2] * kn, y[1][3] * kn);
  vv.x = pack_bf16x2(y[2][0], y[2][1]);
  vv.y = pack_bf16x2(y[2][2], y[2][3]);
  *reinterpret_cast<uint2*>(a.qn + row) = vq;
  *reinterpret_cast<uint2*>(a.kn + row) = vk;
  *reinterpret_cast<uint2*>(a.vv + row) = vv;
  const float ah = __expf(p.a_log[h]);
  float gv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = h * D + lane * 4 + j;
    const float x = __bfloat162float(p.g_raw[(int64_t)t * p.ld_g + c]) + (p.g_bias ? p.g_bias[c] : 0.f);
    gv[j] = p.lower_bound * sigmoidf_(ah * x) * kLog2e;
  }
  *reinterpret_cast<float4*>(a.gl + row) = make_float4(gv[0], gv[1], gv[2], gv[3]);
  if (lane == 0) a.beta[(int64_t)h * a.T + t] = sigmoidf_(__bfloat162float(p.beta_raw[(int64_t)t * p.ld_beta + h]));
}

// ----------------------------------------------------------------------------------- chunk kernel
B200_DEVICE uint64_t kdesc(uint32_t addr) { return make_smem_desc(addr, 16, 1024, kSwizzle128B); }
// MN-major operand: rows of 128 bytes = 64 elements of the M/N dimension, K rows; chunks of 64 M/N
// elements `chunk` bytes apart
B200_DEVICE uint64_t mdesc(uint32_t addr, uint32_t chunk) { return make_smem_desc(addr, chunk, 1024, kSwizzle128B); }

__global__ void __launch_bounds__(kThreads, 1) kda_chunk_kernel(KdaChunkArgs a) {
  pdl_prologue();
  const KdaArgs& p = a.k;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  float* s_gc = reinterpret_cast<float*>(sm + OFF_GC);
  float* s_beta = reinterpret_cast<float*>(sm + OFF_BETA);
  float* s_nsq = reinterpret_cast<float*>(sm + OFF_NSQ);
  float* s_w = reinterpret_cast<float*>(sm + OFF_W);
  float* s_t = reinterpret_cast<float*>(sm + OFF_TM);
  float* s_ti = reinterpret_cast<float*>(sm + OFF_TI);
  __nv_bfloat16* s_nw = reinterpret_cast<__nv_bfloat16*>(sm + OFF_NW);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + OFF_BAR + 12);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3;          // TMEM lanes [32 quarter, 32 quarter + 32) of this warp
  const int cgrp = warp >> 2;            // column group of the TMEM passes
  const int HD = p.H * D;
  if (tid == 0) {
    mbar_init(bar, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (tid < D) s_nw[tid] = p.norm_w ? p.norm_w[tid] : __float2bfloat16(1.f);
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tl = tbase + ((uint32_t)(quarter * 32) << 16);  // this warp's lane quarter
  const uint32_t sbase = smem_u32(sm);
  uint32_t mma_phase = 0;

  // one MMA group issued by thread 0 and waited on by everyone, for at most two seconds (a group takes
  // microseconds); on time-out the error is recorded and the CTA leaves its items
  auto mma_wait = [&]() -> bool {
    const uint64_t t_start = globaltimer();
    bool ok = true;
    while (!mbar_try_wait(bar, mma_phase)) {
      if (globaltimer() - t_start > 2000000000ull) {
        record_error(a.status, kErrMbarTimeout);
        ok = false;
        break;
      }
    }
    mma_phase ^= 1;
    if (!ok) *s_abort = 1;
    tc_fence_after();
    return ok;
  };
  auto sync_for_mma = [&]() {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };

  const int items = p.num_seqs * p.H;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int seq = item / p.H, h = item % p.H;
    const int t0 = p.cu_seqlens[seq], t1 = p.cu_seqlens[seq + 1];
    if (t1 - t0 < a.min_len) continue;  // uniform over the CTA
    const int slot = p.state_idx ? p.state_idx[seq] : seq;
    const bool init = p.has_init ? p.has_init[seq] != 0 : true;
    float* S = p.state + ((int64_t)slot * p.H + h) * D * D;

    // ---- the state into TMEM: warp (quarter, cgrp) moves rows 32 quarter + lane, columns 32 cgrp..
    {
      const int v = quarter * 32 + lane;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint32_t r[8];
        const int col = cgrp * 32 + c8 * 8;
        if (init) {
          const float4 x0 = *reinterpret_cast<const float4*>(S + v * D + col);
          const float4 x1 = *reinterpret_cast<const float4*>(S + v * D + col + 4);
          r[0] = __float_as_uint(x0.x); r[1] = __float_as_uint(x0.y); r[2] = __float_as_uint(x0.z);
          r[3] = __float_as_uint(x0.w); r[4] = __float_as_uint(x1.x); r[5] = __float_as_uint(x1.y);
          r[6] = __float_as_uint(x1.z); r[7] = __float_as_uint(x1.w);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) r[i] = 0u;
        }
        tmem_st8(tl + COL_S + col, r);
      }
      tmem_wait_st();
    }

    // the chunk's per-token inputs into L2 one chunk ahead (head-major rows are contiguous)
    auto prefetch_chunk = [&](int r) {
      if (tid == 0 && r < t1) {
        const int m = min(C, t1 - r);
        const int64_t row = (int64_t)h * a.T + r;
        prefetch_l2(a.kn + row * D, (uint32_t)m * D * 2);
        prefetch_l2(a.qn + row * D, (uint32_t)m * D * 2);
        prefetch_l2(a.vv + row * D, (uint32_t)m * D * 2);
        prefetch_l2(a.gl + row * D, (uint32_t)m * D * 4);
      }
      if (p.g2 && tid >= 32 && tid < 32 + C && r + tid - 32 < t1)  // the output gate rows (256 B each)
        prefetch_l2(p.g2 + (int64_t)(r + tid - 32) * p.ld_g2 + h * D, D * 2);
    };
    prefetch_chunk(t0);
    for (int r0 = t0; r0 < t1 && !*s_abort; r0 += C) {
      const int n = min(C, t1 - r0);
      prefetch_chunk(r0 + C);
      // ============================================================== P0: chunk operands
      // warp w: key channels 8w..8w+7; lane: rows lane and 32 + lane
      {
        const int c0 = warp * 8;
        float G[2][8], kx[2][8], qx[2][8];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int t = hf * 32 + lane;
          const bool valid = t < n;
          const int64_t row = ((int64_t)h * a.T + r0 + t) * D + c0;
          if (valid) {
            const float4 g0 = *reinterpret_cast<const float4*>(a.gl + row);
            const float4 g1 = *reinterpret_cast<const float4*>(a.gl + row + 4);
            G[hf][0] = g0.x; G[hf][1] = g0.y; G[hf][2] = g0.z; G[hf][3] = g0.w;
            G[hf][4] = g1.x; G[hf][5] = g1.y; G[hf][6] = g1.z; G[hf][7] = g1.w;
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.kn + row), kx[hf]);
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.qn + row), qx[hf]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) G[hf][j] = kx[hf][j] = qx[hf][j] = 0.f;
          }
          // inclusive scan over the 32 rows of this half
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float y = __shfl_up_sync(0xffffffffu, G[hf][j], o);
              if (lane >= o) G[hf][j] += y;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) G[1][j] += __shfl_sync(0xffffffffu, G[0][j], 31);
        float R[4][8], GCv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          R[0][j] = __shfl_sync(0xffffffffu, G[0][j], 0);
          R[1][j] = __shfl_sync(0xffffffffu, G[0][j], 16);
          R[2][j] = __shfl_sync(0xffffffffu, G[1][j], 0);
          R[3][j] = __shfl_sync(0xffffffffu, G[1][j], 16);
          GCv[j] = __shfl_sync(0xffffffffu, G[1][j], 31);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (lane == j) s_gc[c0 + j] = GCv[j];
        const int kc = warp >> 3, u = warp & 7;  // K chunk and 16-byte unit of these 8 channels
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int t = hf * 32 + lane;
          const int b = t >> 4;  // 2 hf + (lane >> 4)
          float x[8], y[8], Rb[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) Rb[j] = (lane >> 4) ? R[2 * hf + 1][j] : R[2 * hf][j];
          // row operands (<= 1): K 2^(G - R_b), Q 2^(G - R_b)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float e = ex2(G[hf][j] - Rb[j]);
            x[j] = kx[hf][j] * e;
            y[j] = qx[hf][j] * e;
          }
          {
            uint4 vh, vl;
            pack8_hilo(x, vh, vl);
            sts128(sm, OFF_A1H + kc * 16384 + swz(t, u), vh);
            sts128(sm, OFF_A1L + kc * 16384 + swz(t, u), vl);
            sts128(sm, OFF_A1H + kc * 16384 + swz(64 + t, u), pack8(y));
            sts128(sm, OFF_A1L + kc * 16384 + swz(64 + t, u), make_uint4(0, 0, 0, 0));
          }
          // Q 2^G, K 2^G
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float e = ex2(G[hf][j]);
            x[j] = qx[hf][j] * e;
            y[j] = kx[hf][j] * e;
          }
          sts128(sm, OFF_A2 + kc * 16384 + swz(t, u), pack8(x));
          sts128(sm, OFF_A2 + kc * 16384 + swz(64 + t, u), pack8(y));
          // column operands K 2^(R_b' - G) of the blocks b' >= b (row t of each)
#pragma unroll
          for (int bb = 2 * hf; bb < 4; ++bb) {
            if (bb < b) continue;
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = kx[hf][j] * ex2(R[bb][j] - G[hf][j]);
            uint4 vh, vl;
            pack8_hilo(x, vh, vl);
            sts128(sm, OFF_B1H + b1_off(bb) + kc * (16 * (bb + 1) * 128) + swz(t, u), vh);
            sts128(sm, OFF_B1L + b1_off(bb) + kc * (16 * (bb + 1) * 128) + swz(t, u), vl);
          }
          // K 2^(G_C - G), MN-major [token][key], hi / lo
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] = kx[hf][j] * ex2(GCv[j] - G[hf][j]);
          uint4 vh, vl;
          pack8_hilo(x, vh, vl);
          sts128(sm, OFF_KEH + kc * 8192 + swz(t, u), vh);
          sts128(sm, OFF_KEL + kc * 8192 + swz(t, u), vl);
        }
        if (warp == 0) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int t = hf * 32 + lane;
            s_beta[t] = t < n ? a.beta[(int64_t)h * a.T + r0 + t] : 0.f;
          }
        }
      }
      sync_for_mma();  // the operands of the first group (and s_gc) are written
      if (tid == 0) {
        // P_b = [K 2^(G-R) ; Q 2^(G-R)] (K 2^(R_b - G))^T, b = 0..3: (hi, hi), (hi, lo), (lo, hi); the
        // lo part of A holds only the key rows, so the M rows get two passes
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t idesc = make_idesc_f16(128, 16 * (b + 1), 1);
#pragma unroll
          for (int pass = 0; pass < 3; ++pass) {
            const int ao = pass == 2 ? OFF_A1L : OFF_A1H;
            const int bo = (pass == 1 ? OFF_B1L : OFF_B1H) + b1_off(b);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t da = kdesc(sbase + ao + (kk >> 2) * 16384 + (kk & 3) * 32);
              const uint64_t db = kdesc(sbase + bo + (kk >> 2) * (16 * (b + 1) * 128) + (kk & 3) * 32);
              umma_f16(tbase + p_col(b), da, db, idesc, (pass > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        umma_commit(bar);
      }
      if (!mma_wait()) break;
      // ---- S0 hi / lo as the K-major B operand (row v, K = keys) over the first group's operands,
      // then S *= 2^G_C in TMEM
      {
        const int v = quarter * 32 + lane;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t r[16];
          const int col = cgrp * 32 + half * 16;
          tmem_ld16(tl + COL_S + col, r);
          tmem_wait_ld();
          float x[2][8];
#pragma unroll
          for (int i = 0; i < 16; ++i) x[i >> 3][i & 7] = __uint_as_float(r[i]);
#pragma unroll
          for (int g8 = 0; g8 < 2; ++g8) {
            const int k0 = col + g8 * 8;
            uint4 vh, vl;
            pack8_hilo(x[g8], vh, vl);
            sts128(sm, OFF_B2H + (k0 >> 6) * 16384 + swz(v, (k0 & 63) >> 3), vh);
            sts128(sm, OFF_B2L + (k0 >> 6) * 16384 + swz(v, (k0 & 63) >> 3), vl);
          }
          uint32_t w8[2][8];
#pragma unroll
          for (int i = 0; i < 16; ++i) w8[i >> 3][i & 7] = __float_as_uint(x[i >> 3][i & 7] * ex2(s_gc[col + i]));
          tmem_st8(tl + COL_S + col, w8[0]);
          tmem_st8(tl + COL_S + col + 8, w8[1]);
        }
        tmem_wait_st();
      }
      sync_for_mma();
      if (tid == 0) {
        // D2 = [Q 2^G ; K 2^G] S0^T, S0 = hi + lo
        const uint32_t idesc2 = make_idesc_f16(128, 128, 1);
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = kdesc(sbase + OFF_A2 + (kk >> 2) * 16384 + (kk & 3) * 32);
            const uint64_t db = kdesc(sbase + (pass ? OFF_B2L : OFF_B2H) + (kk >> 2) * 16384 + (kk & 3) * 32);
            umma_f16(tbase + COL_D2, da, db, idesc2, (pass > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(bar);
      }
      if (!mma_wait()) break;
      // ============================================================== P1: T, M and R
      // A warp's 32 rows span two 16-row blocks (lanes 0..15: block bA, 16..31: bA + 1).  tcgen05.ld is
      // warp-collective, so the warp loads the columns of both blocks (each when it has them) and every
      // lane keeps its own block's.
      float pb[16];
      {
        const int bA = 2 * (quarter & 1), bB = bA + 1;
        uint32_t rA[16], rB[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) rA[i] = rB[i] = 0u;
        if (cgrp <= bA) tmem_ld16(tl + p_col(bA) + cgrp * 16, rA);
        if (cgrp <= bB) tmem_ld16(tl + p_col(bB) + cgrp * 16, rB);
        tmem_wait_ld();
        const bool upper = lane >= 16;
        const bool have = cgrp <= (upper ? bB : bA);
#pragma unroll
        for (int i = 0; i < 16; ++i) pb[i] = have ? __uint_as_float(upper ? rB[i] : rA[i]) : 0.f;
      }
      if (quarter < 2) {
        // rows t of L (lanes 0..63): T[t][s] = 1 (s = t), beta_t L[t][s] (s < t), 0 (s > t); columns
        // 16 cgrp .. 16 cgrp + 15 come from block b's P columns when cgrp <= b
        const int t = quarter * 32 + lane;
        const float bt = s_beta[t];
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = pb[i];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int s = cgrp * 16 + i;
          x[i] = s < t ? bt * x[i] : (s == t ? 1.f : 0.f);
        }
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(s_t + t * 64 + cgrp * 16 + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
      } else {
        // rows t of M (lanes 64..127): M[t][s] for s <= t, as the K-major A operand (K = s)
        const int t = (quarter - 2) * 32 + lane;
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = (cgrp * 16 + i <= t) ? pb[i] : 0.f;
        float y[8];
#pragma unroll
        for (int g8 = 0; g8 < 2; ++g8) {
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = x[g8 * 8 + i];
          uint4 vh, vl;
          pack8_hilo(y, vh, vl);
          sts128(sm, OFF_A3 + swz(t, cgrp * 2 + g8), vh);
          sts128(sm, OFF_A3L + swz(t, cgrp * 2 + g8), vl);
        }
        // R[s][v] = beta_s (v_s - (K 2^G S0^T)[s][v]) for values 32 cgrp .. + 31, MN-major hi / lo
        const int s = t;
        const float bs = s_beta[s];
        const bool valid = s < n;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int v0 = cgrp * 32 + half * 16;
          uint32_t r[16];
          tmem_ld16(tl + COL_D2 + v0, r);
          tmem_wait_ld();
          float vin[16];
          if (valid) {
            const __nv_bfloat16* src = a.vv + ((int64_t)h * a.T + r0 + s) * D + v0;
            float f8[8];
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(src), f8);
#pragma unroll
            for (int i = 0; i < 8; ++i) vin[i] = f8[i];
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(src + 8), f8);
#pragma unroll
            for (int i = 0; i < 8; ++i) vin[8 + i] = f8[i];
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) vin[i] = 0.f;
          }
#pragma unroll
          for (int g8 = 0; g8 < 2; ++g8) {
            float z[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) z[i] = bs * (vin[g8 * 8 + i] - __uint_as_float(r[g8 * 8 + i]));
            uint4 vh, vl;
            pack8_hilo(z, vh, vl);
            const int vv0 = v0 + g8 * 8;
            sts128(sm, OFF_RH + (vv0 >> 6) * 8192 + swz(s, (vv0 & 63) >> 3), vh);
            sts128(sm, OFF_RL + (vv0 >> 6) * 8192 + swz(s, (vv0 & 63) >> 3), vl);
          }
        }
      }
      __syncthreads();
      // ============================================================== P2: T^-1 (unit lower triangular)
      // diagonal 16x16 blocks by forward substitution: thread (block b, column j)
      if (tid < 64) {
        const int b = tid >> 4, j = tid & 15;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float acc = (r == j) ? 1.f : 0.f;
#pragma unroll
          for (int k = 0; k < 16; ++k)
            if (k < r && k >= j) acc -= s_t[(16 * b + r) * 64 + 16 * b + k] * x[k];
          x[r] = (r < j) ? 0.f : acc;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) s_ti[(16 * b + r) * 64 + 16 * b + j] = x[r];
      }
      // the blocks above the diagonal are zero
      for (int e = tid; e < 64 * 64; e += kThreads) {
        const int r = e >> 6, c = e & 63;
        if ((c >> 4) > (r >> 4)) s_ti[e] = 0.f;
      }
      __syncthreads();
      // off-diagonal blocks by distance d: T^-1_ij = -T^-1_ii sum_{k=j}^{i-1} T_ik T^-1_kj
      for (int d = 1; d < 4; ++d) {
        const int nb = 4 - d;
        for (int e = tid; e < nb * 256; e += kThreads) {
          const int blk = e >> 8, r = (e >> 4) & 15, c = e & 15;
          const int i = blk + d, j = blk;
          float acc = 0.f;
          for (int k = 16 * j; k < 16 * i; ++k) acc += s_t[(16 * i + r) * 64 + k] * s_ti[k * 64 + 16 * j + c];
          s_w[blk * 256 + r * 16 + c] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nb * 256; e += kThreads) {
          const int blk = e >> 8, r = (e >> 4) & 15, c = e & 15;
          const int i = blk + d, j = blk;
          float acc = 0.f;
#pragma unroll
          for (int m = 0; m < 16; ++m) acc += s_ti[(16 * i + r) * 64 + 16 * i + m] * s_w[blk * 256 + m * 16 + c];
          s_ti[(16 * i + r) * 64 + 16 * j + c] = -acc;
        }
        __syncthreads();
      }
      // T^-1 hi / lo as the K-major A operand: thread (row t, unit u)
      {
        const int t = tid >> 3, u = tid & 7;
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = s_ti[t * 64 + u * 8 + i];
        uint4 vh, vl;
        pack8_hilo(x, vh, vl);
        sts128(sm, OFF_A5H + swz(t, u), vh);
        sts128(sm, OFF_A5L + swz(t, u), vl);
      }
      sync_for_mma();
      if (tid == 0) {
        // U = T^-1 R: (hi, hi), (hi, lo), (lo, hi)
        const uint32_t idesc = make_idesc_f16(128, 128, 1, false, true);
#pragma unroll
        for (int pass = 0; pass < 3; ++pass) {
          const int ao = pass == 2 ? OFF_A5L : OFF_A5H;
          const int bo = pass == 1 ? OFF_RL : OFF_RH;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tbase + COL_U, kdesc(sbase + ao + kk * 32), mdesc(sbase + bo + kk * 2048, 8192), idesc,
                     (pass > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar);
      }
      if (!mma_wait()) break;
      // ============================================================== P3: U hi / lo, MN-major [s][v]
      if (quarter < 2) {
        const int s = quarter * 32 + lane;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int v0 = cgrp * 32 + half * 16;
          uint32_t r[16];
          tmem_ld16(tl + COL_U + v0, r);
          tmem_wait_ld();
#pragma unroll
          for (int g8 = 0; g8 < 2; ++g8) {
            float z[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) z[i] = __uint_as_float(r[g8 * 8 + i]);
            uint4 vh, vl;
            pack8_hilo(z, vh, vl);
            const int vv0 = v0 + g8 * 8;
            sts128(sm, OFF_UH + (vv0 >> 6) * 8192 + swz(s, (vv0 & 63) >> 3), vh);
            sts128(sm, OFF_UL + (vv0 >> 6) * 8192 + swz(s, (vv0 & 63) >> 3), vl);
          }
        }
      }
      sync_for_mma();
      if (tid == 0) {
        // D2 += M U: (hi, hi), (hi, lo), (lo, hi)
        const uint32_t idesc3 = make_idesc_f16(128, 128, 1, false, true);
#pragma unroll
        for (int pass = 0; pass < 3; ++pass)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tbase + COL_D2, kdesc(sbase + (pass == 2 ? OFF_A3L : OFF_A3) + kk * 32),
                     mdesc(sbase + (pass == 1 ? OFF_UL : OFF_UH) + kk * 2048, 8192), idesc3, 1u);
        // S += U^T (K 2^(G_C - G)): (hi, hi), (hi, lo), (lo, hi); A = U MN-major, B MN-major
        const uint32_t idesc4 = make_idesc_f16(128, 128, 1, true, true);
#pragma unroll
        for (int pass = 0; pass < 3; ++pass) {
          const int ao = pass == 2 ? OFF_UL : OFF_UH;
          const int bo = pass == 1 ? OFF_KEL : OFF_KEH;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tbase + COL_S, mdesc(sbase + ao + kk * 2048, 8192), mdesc(sbase + bo + kk * 2048, 8192), idesc4,
                     1u);
        }
        umma_commit(bar);
      }
      if (!mma_wait()) break;
      // ============================================================== P4: output rows, gated RMSNorm
      const int t = quarter * 32 + lane;  // rows 0..63 in quarters 0, 1
      if (quarter < 2) {
        float ss = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t r[16];
          tmem_ld16(tl + COL_D2 + cgrp * 32 + half * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) ss += __uint_as_float(r[i]) * __uint_as_float(r[i]);
        }
        s_nsq[cgrp * 64 + t] = ss;
      }
      __syncthreads();
      if (quarter < 2) {  // warp-uniform: the TMEM reads are warp-collective; rows past n are not stored
        const int64_t tok = r0 + t;
        float scale = 1.f;
        if (p.norm_w) scale = rsqrtf((s_nsq[t] + s_nsq[64 + t] + s_nsq[128 + t] + s_nsq[192 + t]) / D + p.eps);
        __nv_bfloat16* dst = p.out + tok * p.ld_out + h * D + cgrp * 32;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t r[16];
          tmem_ld16(tl + COL_D2 + cgrp * 32 + half * 16, r);
          tmem_wait_ld();
          if (t < n) {
#pragma unroll
            for (int g8 = 0; g8 < 2; ++g8) {
              const int c8 = half * 16 + g8 * 8;  // first of these 8 values within the 32
              float y[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(r[g8 * 8 + i]);
              if (p.norm_w) {
                float nw[8], gg[8];
                bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_nw + cgrp * 32 + c8), nw);
                if (p.g2)  // the chunk's gate rows were prefetched into L2 at its start
                  bf16x8_to_f32(*reinterpret_cast<const uint4*>(p.g2 + tok * p.ld_g2 + h * D + cgrp * 32 + c8), gg);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  y[i] *= scale * nw[i];
                  if (p.g2) y[i] *= sigmoidf_(gg[i]);
                }
              }
              *reinterpret_cast<uint4*>(dst + c8) = pack8(y);
            }
          }
        }
      }
      // the next chunk's first barrier orders these TMEM reads before its MMAs
    }
    // ---- final state and conv window
    __syncthreads();
    tc_fence_after();
    if (!*s_abort) {
      const int v = quarter * 32 + lane;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[16];
        const int col = cgrp * 32 + half * 16;
        tmem_ld16(tl + COL_S + col, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(S + v * D + col + i) = make_float4(
              __uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
      }
      if (p.conv_w && tid < 3 * D) {
        const int which = tid / D, c = tid % D;
        const int64_t g = (int64_t)which * HD + h * D + c;
        __nv_bfloat16* cs = p.conv_state + ((int64_t)slot * 3 * HD + g) * 3;
        const int len = t1 - t0;
        float w[3];
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          const int idx = len - 3 + m;
          w[m] = idx >= 0 ? __bfloat162float(p.qkv[(int64_t)(t0 + idx) * p.ld_qkv + g])
                          : (init ? __bfloat162float(cs[3 + idx]) : 0.f);
        }
#pragma unroll
        for (int m = 0; m < 3; ++m) cs[m] = __float2bfloat16(w[m]);
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (*s_abort) break;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace kdac

size_t kda_chunk_scratch_bytes(int T, int H) {
  const size_t n = (size_t)T * H * kdac::D;
  return n * 2 * 3 + n * 4 + (size_t)T * H * 4 + 256 * 5;
}

cudaError_t kda_chunked(const KdaChunkArgs& a_in, cudaStream_t stream) {
  using namespace kdac;
  KdaChunkArgs a = a_in;
  const KdaArgs& p = a.k;
  if (p.num_seqs == 0 || a.T == 0) return cudaSuccess;
  if (p.D != D || !p.full || p.verify != nullptr || a.min_len < 1) return cudaErrorInvalidValue;
  if (!(p.lower_bound >= -5.8f)) return cudaErrorInvalidValue;  // block-local exponents must stay finite in bf16
  if (a.scratch == nullptr) return cudaErrorInvalidValue;
  // scratch: qn, kn, vv bf16 [T, H, D]; gl fp32 [T, H, D]; beta fp32 [T, H] (256-byte aligned pieces)
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t n = (size_t)a.T * p.H * D;
  uint8_t* s = reinterpret_cast<uint8_t*>(a.scratch);
  size_t off = 0;
  a.qn = reinterpret_cast<__nv_bfloat16*>(s + off);
  off += up(n * 2);
  a.kn = reinterpret_cast<__nv_bfloat16*>(s + off);
  off += up(n * 2);
  a.vv = reinterpret_cast<__nv_bfloat16*>(s + off);
  off += up(n * 2);
  a.gl = reinterpret_cast<float*>(s + off);
  off += up(n * 4);
  a.beta = reinterpret_cast<float*>(s + off);
  off += up((size_t)a.T * p.H * 4);
  if (off > a.scratch_bytes) return cudaErrorInvalidValue;
  const int warps = a.T * p.H;
  launch_pdl(kda_prep_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kda_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int grid = std::min(p.num_seqs * p.H, device_sm_count());
  launch_pdl(kda_chunk_kernel, dim3(grid), dim3(kThreads), SMEM_BYTES, stream, a);
  return cudaGetLastError();
}

}  // namespace b200

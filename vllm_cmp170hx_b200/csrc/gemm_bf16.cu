// Dense bf16 GEMM on tcgen05:  C[M, N] = A[M, K] . B[N, K]^T  (fp32 accumulate).
//
// This is the dense projection engine of the package (the role cuBLAS plays
// for upstream vLLM's `F.linear`; the reference's thin-M BF16 GEMM family,
// vllm_sm80/kernels/thin_gemm/thin_gemm_v74.py:616, solves the same problem
// on sm_80 with split-K mma.sync).  B200 design:
//
//   * persistent grid, one CTA per SM, 6 warps:
//       warp 0      TMA producer (A and B tiles, 128-byte swizzle, K step 64)
//       warp 1      TMEM owner + single-thread tcgen05.mma issuer
//       warps 2..5  epilogue: tcgen05.ld 32x32b, convert, store
//   * two TMEM accumulators (2 x BN fp32 columns) so the epilogue of tile i
//     overlaps the MMAs of tile i+1;
//   * split-K over the grid for decode shapes (few output tiles): each split
//     writes fp32 partials, a second kernel sums them in a fixed order
//     (deterministic);
//   * "swap" mode for small M: the host passes the weight as A (its output
//     features fill the 128-row MMA M dimension) and the activations as B, and
//     the epilogue writes the transposed tile (coalesced along the lanes).
//
// Every wait is bounded (common.cuh); a timed-out wait records an error bit
// in `status` and the CTA unwinds after draining its own in-flight copies.
#include "common.cuh"
#include <algorithm>

#include "launch.h"
#include "sp_sync.cuh"
#include "tma_host.h"

namespace b200 {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // transposed (swap-mode) output tile staged in shared memory: BN token rows x 128 features, bf16
  static constexpr int OUT_BYTES = BN <= 128 ? BN * BM * 2 : 0;
  static constexpr int STAGE_BUDGET = 224 * 1024 - OUT_BYTES - 1024 - 256;
  static constexpr int STAGES = STAGE_BUDGET / STAGE_BYTES > 8 ? 8 : STAGE_BUDGET / STAGE_BYTES;
  static constexpr int TMEM_COLS = (2 * BN) < 32 ? 32 : 2 * BN;  // power of two for BN in {16..256}
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
};

struct Params {
  int M, N, K;
  int ldc;            // row stride of C (elements)
  int transpose_out;  // 1: tile (m, n) is stored at C[n * ldc + m]
  int splits;         // K splits; >1 writes fp32 partials to `partial`
  int k_blocks_per_split;
  int m_tiles, n_tiles;
  __nv_bfloat16* C;
  float* Cf;        // fp32 output instead of C (router logits)
  float* partial;  // [splits, M, N] (in the output's orientation) when splits > 1
  const __nv_bfloat16* bias;  // optional [N] (out features), added in the epilogue when splits == 1
  uint32_t* status;
  // Fused all-reduce over the tensor-parallel group (ar = 1; one tile per CTA, splits == 1).
  // Symmetric buffer of every rank: flags[cta][quarter][src] (uint32 epochs) at flag_off, tile slots
  // [cta][epoch parity][src][128][BN] bf16 at data_off.  Each CTA pushes its bf16 tile into slot
  // `rank` of every rank, publishes a flag per TMEM lane quarter, then sums its tile over the
  // ranks' slots (pushed to it) in rank order and writes C.
  int ar;
  const uint64_t* peers;
  int rank, world;
  int64_t flag_off, data_off, tile_bytes;
  uint32_t* epochs;  // [gridDim.x] per-CTA call counters (this rank)
  uint64_t timeout_ns;
  // Sequence-parallel collectives (sp_sync.cuh): 1 = reduce-scatter, every output token row pushed to
  // its owner rank (token / sp_rows) at row (rank, token % sp_rows) of the area at sp_rs_off, C unused;
  // 2 = all-gather, the activation operand (B when act_is_b, else A) is read only after every rank's
  // all-gather flag arrived; the weight tiles of the first stages stream meanwhile.
  int sp_mode;
  SpSync sp;
  int64_t sp_rs_off;
  int sp_rows;
  int act_is_b;
  // Batched GEMM (batch > 1, splits == 1): tile t covers matrix t / (m_tiles * n_tiles); the operand
  // maps are 3-D (K, rows, batch) and C of matrix b starts c_bstride elements after matrix b - 1's.
  int batch;
  int64_t c_bstride;
};

// Destination of output row `tok` (a token), columns from `feat`, in the reduce-scatter mode.
__device__ __forceinline__ __nv_bfloat16* rs_dst(const Params& p, int tok, int feat, int feats) {
  const int owner = tok / p.sp_rows;
  const int lt = tok - owner * p.sp_rows;
  return reinterpret_cast<__nv_bfloat16*>(p.sp.peers[owner] + p.sp_rs_off) +
         (size_t)(p.sp.rank * p.sp_rows + lt) * feats + feat;
}

// All-gather mode of the producer: loads of the activation operand of the first stages wait here until
// every rank's flag arrived.  `pend` holds (stage, k block, m tile, n tile) of deferred loads.
struct AgGate {
  bool open;
  uint32_t e;
  int n;
  int pend[8][4];
};

__device__ __forceinline__ void ag_release(AgGate& g, const Params& p, const CUtensorMap* act_map, uint8_t* smem_act,
                                           int act_bytes, uint64_t* full, int act_rows) {
  if (!g.open) return;
  for (int src = 0; src < p.sp.world; ++src) sp_wait_flag(p.sp, kSpAllGather, g.e, src);
  asm volatile("fence.proxy.async.global;" ::: "memory");  // peer stores (generic) -> TMA reads (async)
  for (int i = 0; i < g.n; ++i) {
    const int st = g.pend[i][0], kb = g.pend[i][1];
    const int row0 = p.act_is_b ? g.pend[i][3] * act_rows : g.pend[i][2] * act_rows;
    tma_load_2d(smem_act + st * act_bytes, act_map, &full[st], kb * BK, row0);
  }
  g.n = 0;
  g.open = false;
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_cg_u4(const void* ptr) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(ptr));
  return v;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                        Params p) {
  using C_ = Cfg<BN>;
  constexpr int S = C_::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * C_::A_BYTES;
  uint8_t* smem_out = smem + S * C_::STAGE_BYTES;  // OUT_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_out + C_::OUT_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint64_t* staged = bars + 2 * S + 5;   // 128 epilogue threads: the output tile is in smem_out
  uint64_t* written = bars + 2 * S + 6;  // 128 epilogue threads: smem_out may be refilled
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* s_epoch = tmem_slot + 2;
  uint32_t* s_ag_epoch = tmem_slot + 3;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    mbar_init(staged, 128);
    mbar_init(written, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  pdl_prologue();  // setup above overlaps the previous kernel's tail
  if (p.ar) {  // this CTA's call counter (written by the previous call of this kernel)
    if (threadIdx.x == 0) *s_epoch = p.epochs[blockIdx.x] + 1;
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // bf16 output, transposed: staged in smem, written as 16-byte runs of features (a token's row)
  const bool rs = p.sp_mode == 1;
  const bool staged_out = C_::OUT_BYTES > 0 && p.transpose_out && !p.ar && p.splits == 1 && p.Cf == nullptr &&
                          (rs || ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0 && (p.ldc & 7) == 0));

  const int tiles_mn = p.m_tiles * p.n_tiles;
  const bool batched = p.batch > 1;
  const int total = tiles_mn * (batched ? p.batch : p.splits);
  const int kb_total = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      // the call number is read after the programmatic-launch wait (the previous kernel has completed);
      // thread 0 reads it back from shared memory for the arrival at the end of the kernel
      AgGate gate;
      gate.open = p.sp_mode == 2;
      gate.e = gate.open ? sp_recv_epoch(p.sp, kSpAllGather) : 0u;
      gate.n = 0;
      if (gate.open) *s_ag_epoch = gate.e;
      const CUtensorMap* act_map = p.act_is_b ? &tma_b : &tma_a;
      uint8_t* act_smem = p.act_is_b ? smem_b : smem_a;
      const int act_bytes = p.act_is_b ? C_::B_BYTES : C_::A_BYTES;
      const int act_rows = p.act_is_b ? BN : BM;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int split = batched ? 0 : t / tiles_mn;
        const int bz = batched ? t / tiles_mn : 0;
        const int mn = t % tiles_mn;
        const int mt = mn % p.m_tiles;
        const int nt = mn / p.m_tiles;
        const int kb0 = split * p.k_blocks_per_split;
        const int kb1 = min(kb_total, kb0 + p.k_blocks_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_or_abort(&empty[stage], phase ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C_::STAGE_BYTES);
          if (batched) {
            tma_load_3d(smem_a + stage * C_::A_BYTES, &tma_a, &full[stage], kb * BK, mt * BM, bz);
            tma_load_3d(smem_b + stage * C_::B_BYTES, &tma_b, &full[stage], kb * BK, nt * BN, bz);
          } else if (gate.open) {
            // weights now, the activation tile once the all-gather landed
            if (p.act_is_b)
              tma_load_2d(smem_a + stage * C_::A_BYTES, &tma_a, &full[stage], kb * BK, mt * BM);
            else
              tma_load_2d(smem_b + stage * C_::B_BYTES, &tma_b, &full[stage], kb * BK, nt * BN);
            gate.pend[gate.n][0] = stage;
            gate.pend[gate.n][1] = kb;
            gate.pend[gate.n][2] = mt;
            gate.pend[gate.n][3] = nt;
            if (++gate.n == S || gate.n == 8) ag_release(gate, p, act_map, act_smem, act_bytes, full, act_rows);
          } else {
            tma_load_2d(smem_a + stage * C_::A_BYTES, &tma_a, &full[stage], kb * BK, mt * BM);
            tma_load_2d(smem_b + stage * C_::B_BYTES, &tma_b, &full[stage], kb * BK, nt * BN);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      ag_release(gate, p, act_map, act_smem, act_bytes, full, act_rows);  // fewer k blocks than stages
      if (!ok) {
        *abort_flag = 1;
        // Drain: the most recent load of every stage must land before exit.
        const uint32_t n = issued < (uint32_t)S ? issued : (uint32_t)S;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t k = issued - 1 - i;
          mbar_wait(&full[k % S], (k / S) & 1, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, 1 /*bf16*/);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
        const int split = batched ? 0 : t / tiles_mn;
        const int kb0 = split * p.k_blocks_per_split;
        const int kb1 = min(kb_total, kb0 + p.k_blocks_per_split);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_or_abort(&tempty[acc], acc_phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_or_abort(&full[stage], phase, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = desc_kmajor_sw128(smem_a + stage * C_::A_BYTES);
          const uint64_t db = desc_kmajor_sw128(smem_b + stage * C_::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle row.
            umma_f16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) *abort_flag = 1;
      // Every MMA this thread issued has completed once `drain` flips.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      const int split = batched ? 0 : t / tiles_mn;
      __nv_bfloat16* const Cb = batched ? p.C + (size_t)(t / tiles_mn) * p.c_bstride : p.C;
      const int mn = t % tiles_mn;
      const int mt = mn % p.m_tiles;
      const int nt = mn / p.m_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // TMEM loads are warp-collective: leave together
      const bool got = mbar_wait_or_abort(&tfull[acc], acc_phase, p.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;  // A row == TMEM lane
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (staged_out) {
        // this thread's feature row of the tile -> column (q * 32 + lane) of the [token][feature]
        // staging tile (a warp's 32 lanes fill 64 contiguous bytes per token: no bank conflicts)
        const float bias = (p.bias && row < p.M) ? __bfloat162float(p.bias[row]) : 0.f;
        const uint32_t so = smem_u32(smem_out) + (uint32_t)(q * 32 + lane) * 2;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const __nv_bfloat16 h = __float2bfloat16(__uint_as_float(r[j]) + bias);
            asm volatile("st.shared.b16 [%0], %1;" ::"r"(so + (uint32_t)(c + j) * (BM * 2)),
                         "h"(*reinterpret_cast<const unsigned short*>(&h))
                         : "memory");
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);  // the accumulator is free once read
        mbar_arrive(staged);
        const bool st_ok = mbar_wait_or_abort(staged, local & 1, p.status, abort_flag);
        if (st_ok) {
          // 16-byte runs: token row n of the tile, features 8 g .. 8 g + 7
          const int et = (warp - 2) * 32 + lane;
          for (int i = et; i < BN * (BM / 8); i += 128) {
            const int n = i / (BM / 8), g = i % (BM / 8);
            const int col = nt * BN + n, f0 = mt * BM + g * 8;
            if (col >= p.N || f0 >= p.M) continue;
            const uint8_t* src = smem_out + n * (BM * 2) + g * 16;
            __nv_bfloat16* dst = rs ? rs_dst(p, col, f0, p.M) : Cb + (size_t)col * p.ldc + f0;
            if (f0 + 8 <= p.M) {
              *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
            } else {
              for (int k = 0; k < p.M - f0; ++k) dst[k] = reinterpret_cast<const __nv_bfloat16*>(src)[k];
            }
          }
        }
        mbar_arrive(written);
        if (!mbar_wait_or_abort(written, local & 1, p.status, abort_flag) || !st_ok) break;
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_wait_ld();
        const int col0 = nt * BN + c;
        if (p.ar) {
          // bf16 tile row (this lane), columns c..c+15, into slot `rank` of every rank
          uint4 v0, v1;
          v0.x = pack_bf16x2(__uint_as_float(r[0]), __uint_as_float(r[1]));
          v0.y = pack_bf16x2(__uint_as_float(r[2]), __uint_as_float(r[3]));
          v0.z = pack_bf16x2(__uint_as_float(r[4]), __uint_as_float(r[5]));
          v0.w = pack_bf16x2(__uint_as_float(r[6]), __uint_as_float(r[7]));
          v1.x = pack_bf16x2(__uint_as_float(r[8]), __uint_as_float(r[9]));
          v1.y = pack_bf16x2(__uint_as_float(r[10]), __uint_as_float(r[11]));
          v1.z = pack_bf16x2(__uint_as_float(r[12]), __uint_as_float(r[13]));
          v1.w = pack_bf16x2(__uint_as_float(r[14]), __uint_as_float(r[15]));
          const uint32_t e = *s_epoch;
          const int64_t slot = ((int64_t)(blockIdx.x * 2 + (e & 1)) * p.world + p.rank) * p.tile_bytes +
                               ((int64_t)(q * 32 + lane) * BN + c) * 2;
          for (int dst = 0; dst < p.world; ++dst) {
            uint4* d = reinterpret_cast<uint4*>(p.peers[dst] + p.data_off + slot);
            d[0] = v0;
            d[1] = v1;
          }
          continue;
        }
        if (row < p.M) {
          if (p.splits > 1) {
            // fp32 partials in output orientation
            float* dst = p.partial + (size_t)split * p.M * p.N;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = col0 + j;
              if (col < p.N) {
                const size_t off = p.transpose_out ? (size_t)col * p.M + row : (size_t)row * p.N + col;
                dst[off] = __uint_as_float(r[j]);
              }
            }
          } else if (p.Cf != nullptr) {
            const float bias = p.bias ? __bfloat162float(p.bias[p.transpose_out ? row : 0]) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = col0 + j;
              if (col < p.N) {
                const float b = p.bias ? (p.transpose_out ? bias : __bfloat162float(p.bias[col])) : 0.f;
                const size_t off = p.transpose_out ? (size_t)col * p.ldc + row : (size_t)row * p.ldc + col;
                p.Cf[off] = __uint_as_float(r[j]) + b;
              }
            }
          } else if (p.transpose_out) {
            const float bias = p.bias ? __bfloat162float(p.bias[row]) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = col0 + j;
              if (col < p.N) Cb[(size_t)col * p.ldc + row] = __float2bfloat16(__uint_as_float(r[j]) + bias);
            }
          } else {
            __nv_bfloat16* dst = rs ? rs_dst(p, row, col0, p.N) : Cb + (size_t)row * p.ldc + col0;
            if (col0 + 16 <= p.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) && p.bias == nullptr) {
              uint4 v0, v1;
              v0.x = pack_bf16x2(__uint_as_float(r[0]), __uint_as_float(r[1]));
              v0.y = pack_bf16x2(__uint_as_float(r[2]), __uint_as_float(r[3]));
              v0.z = pack_bf16x2(__uint_as_float(r[4]), __uint_as_float(r[5]));
              v0.w = pack_bf16x2(__uint_as_float(r[6]), __uint_as_float(r[7]));
              v1.x = pack_bf16x2(__uint_as_float(r[8]), __uint_as_float(r[9]));
              v1.y = pack_bf16x2(__uint_as_float(r[10]), __uint_as_float(r[11]));
              v1.z = pack_bf16x2(__uint_as_float(r[12]), __uint_as_float(r[13]));
              v1.w = pack_bf16x2(__uint_as_float(r[14]), __uint_as_float(r[15]));
              reinterpret_cast<uint4*>(dst)[0] = v0;
              reinterpret_cast<uint4*>(dst)[1] = v1;
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int col = col0 + j;
                if (col < p.N) {
                  const float bias = p.bias ? __bfloat162float(p.bias[col]) : 0.f;
                  dst[j] = __float2bfloat16(__uint_as_float(r[j]) + bias);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (p.ar) {
        // this quarter's rows reached every rank: publish (stores before the flag, system scope)
        __threadfence_system();
        __syncwarp();
        if (lane < p.world) {
          uint32_t* f = reinterpret_cast<uint32_t*>(p.peers[lane] + p.flag_off) +
                        ((int64_t)blockIdx.x * 4 + q) * p.world + p.rank;
          st_release_sys_u32(f, *s_epoch);
        }
      }
    }
    if (p.ar && local == 1 && !*abort_flag) {
      // ---------------------------------------------------------- all-reduce of this CTA's tile
      const uint32_t e = *s_epoch;
      const int mt = blockIdx.x % p.m_tiles, nt = blockIdx.x / p.m_tiles;
      bool ok = true;
      if (lane < p.world) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(p.peers[p.rank] + p.flag_off) +
                            ((int64_t)blockIdx.x * 4 + q) * p.world + lane;
        const uint64_t t0 = globaltimer();
        while ((int32_t)(ld_acquire_sys_u32(f) - e) < 0) {
          if (globaltimer() - t0 > p.timeout_ns) {
            record_error(p.status, kErrPeerTimeout);
            ok = false;
            break;
          }
        }
      }
      if (__all_sync(0xffffffffu, ok)) {
        const int row = mt * BM + q * 32 + lane;  // A row of this lane
        const uint8_t* base = reinterpret_cast<const uint8_t*>(p.peers[p.rank] + p.data_off) +
                              (int64_t)(blockIdx.x * 2 + (e & 1)) * p.world * p.tile_bytes +
                              (int64_t)(q * 32 + lane) * BN * 2;
        const float bias = (p.bias && p.transpose_out && row < p.M) ? __bfloat162float(p.bias[row]) : 0.f;
#pragma unroll 1
        for (int c = 0; c < BN; c += 8) {
          float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int src = 0; src < p.world; ++src) {
            const uint4 v = ld_cg_u4(base + (int64_t)src * p.tile_bytes + c * 2);
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc8[i] += __bfloat162float(h[i]);
          }
          if (row >= p.M) continue;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int col = nt * BN + c + i;
            if (col >= p.N) break;
            if (p.transpose_out) {
              p.C[(size_t)col * p.ldc + row] = __float2bfloat16(acc8[i] + bias);
            } else {
              const float b = p.bias ? __bfloat162float(p.bias[col]) : 0.f;
              p.C[(size_t)row * p.ldc + col] = __float2bfloat16(acc8[i] + b);
            }
          }
        }
      }
    }
  }

  if (rs) __threadfence_system();  // this CTA's pushed rows before the arrival below
  tc_fence_before();
  __syncthreads();
  if (p.ar && threadIdx.x == 0) p.epochs[blockIdx.x] = *s_epoch;
  if (threadIdx.x == 0) {
    if (rs) sp_push_arrive(p.sp, kSpReduceScatter, gridDim.x);
    if (p.sp_mode == 2) sp_recv_arrive(p.sp, kSpAllGather, gridDim.x, *s_ag_epoch);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- cluster split-K
// Decode-shaped GEMMs (few output tiles, long K).  The K range of one 128 x BN output tile is split
// over the `splits` CTAs of a thread-block cluster (splits <= 8).  Each CTA accumulates its share in
// TMEM and parks the fp32 partial in its own shared memory, grouped by the CTA that will reduce
// each row range; one thread then bulk-copies every group into its reducer's receive slot
// (cp.async.bulk shared::cta -> shared::cluster, completion as transaction bytes on the reducer's
// mbarrier).  CTA r sums the `splits` slots of rows [r R, (r + 1) R) in split order (deterministic),
// adds the bias and writes C in 16-byte runs.  No fp32 partials go through global memory, there is
// no second kernel, and the only cluster-wide barrier is the one after the mbarrier initialisation.
// Shared memory of the cluster kernel: the operand stages (at most 4: a CTA holds a few K blocks),
// over which the parked groups are written once its own MMAs are done, then the receive slots in a
// region of their own (peers copy into them while this CTA may still be streaming its operands),
// then the barriers.
template <int BN>
struct CskPlan {
  static constexpr int S = Cfg<BN>::STAGES < 4 ? Cfg<BN>::STAGES : 4;
  static constexpr int MAX_ROWS = 144;  // max of splits x R over splits = 2..8 (R = ceil(128 / splits), to 4)
  static constexpr int GROUPS_BYTES = MAX_ROWS * BN * 4;
  static constexpr int STAGE_REGION = S * Cfg<BN>::STAGE_BYTES > GROUPS_BYTES ? S * Cfg<BN>::STAGE_BYTES : GROUPS_BYTES;
  static constexpr int SLOTS_OFF = STAGE_REGION;
  static constexpr int BARS_OFF = SLOTS_OFF + GROUPS_BYTES;
  static constexpr int SMEM_BYTES = BARS_OFF + 256 + 1024;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_csk_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                         Params p) {
  using C_ = Cfg<BN>;
  using P_ = CskPlan<BN>;
  constexpr int S = P_::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * C_::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_::BARS_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* parked = bars + 2 * S + 1;  // 128 epilogue threads: the partial groups are in smem
  uint64_t* recv = bars + 2 * S + 2;    // every CTA's group for this CTA's rows has landed
  uint64_t* drain = bars + 2 * S + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* s_ag_epoch = tmem_slot + 2;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int splits = p.splits;
  const bool rs = p.sp_mode == 1;
  const uint32_t rank = cluster_ctarank();
  const int mn = blockIdx.x / splits;
  const int mt = mn % p.m_tiles, nt = mn / p.m_tiles;
  const int kb_total = (p.K + BK - 1) / BK;
  const int kb0 = (int)rank * p.k_blocks_per_split;
  const int kb1 = min(kb_total, kb0 + p.k_blocks_per_split);
  // rows of the tile reduced by CTA j: [j R, j R + R), R a multiple of 4 (16-byte groups)
  const int R = ((BM + splits - 1) / splits + 3) / 4 * 4;
  const int GROUP = BN * R;  // floats of one group: [BN columns][R rows]
  // parked groups [splits][BN][R] over the drained stages; receive slots [splits][BN][R] apart
  float* park = reinterpret_cast<float*>(smem);
  float* slots = reinterpret_cast<float*>(smem + P_::SLOTS_OFF);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(parked, 128);
    mbar_init(recv, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  // peers copy into this CTA's slots and signal its barrier: all initialised first
  cluster_sync_all();
  pdl_prologue();  // setup above overlaps the previous kernel's tail
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      bool ok = true;
      // the call number is read after the programmatic-launch wait (the previous kernel has completed);
      // thread 0 reads it back from shared memory for the arrival at the end of the kernel
      AgGate gate;
      gate.open = p.sp_mode == 2;
      gate.e = gate.open ? sp_recv_epoch(p.sp, kSpAllGather) : 0u;
      gate.n = 0;
      if (gate.open) *s_ag_epoch = gate.e;
      const CUtensorMap* act_map = p.act_is_b ? &tma_b : &tma_a;
      uint8_t* act_smem = p.act_is_b ? smem_b : smem_a;
      const int act_bytes = p.act_is_b ? C_::B_BYTES : C_::A_BYTES;
      const int act_rows = p.act_is_b ? BN : BM;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_or_abort(&empty[stage], phase ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], C_::STAGE_BYTES);
        if (gate.open) {
          if (p.act_is_b)
            tma_load_2d(smem_a + stage * C_::A_BYTES, &tma_a, &full[stage], kb * BK, mt * BM);
          else
            tma_load_2d(smem_b + stage * C_::B_BYTES, &tma_b, &full[stage], kb * BK, nt * BN);
          gate.pend[gate.n][0] = stage;
          gate.pend[gate.n][1] = kb;
          gate.pend[gate.n][2] = mt;
          gate.pend[gate.n][3] = nt;
          if (++gate.n == S) ag_release(gate, p, act_map, act_smem, act_bytes, full, act_rows);
        } else {
          tma_load_2d(smem_a + stage * C_::A_BYTES, &tma_a, &full[stage], kb * BK, mt * BM);
          tma_load_2d(smem_b + stage * C_::B_BYTES, &tma_b, &full[stage], kb * BK, nt * BN);
        }
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      ag_release(gate, p, act_map, act_smem, act_bytes, full, act_rows);
      if (!ok) {
        *abort_flag = 1;
        const uint32_t n = issued < (uint32_t)S ? issued : (uint32_t)S;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t k = issued - 1 - i;
          mbar_wait(&full[k % S], (k / S) & 1, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, 1 /*bf16*/);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_or_abort(&full[stage], phase, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = desc_kmajor_sw128(smem_a + stage * C_::A_BYTES);
        const uint64_t db = desc_kmajor_sw128(smem_b + stage * C_::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) umma_f16(tmem_base, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) umma_commit(tfull);
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue: park, exchange, reduce
    const int q = warp & 3;
    const int et = threadIdx.x - 64;  // 0..127
    const int row = q * 32 + lane;    // tile row == TMEM lane
    const int dst = row / R, rl = row % R;
    if (et == 0) mbar_arrive_expect_tx(recv, (uint32_t)(splits * GROUP * 4));
    bool ok = mbar_wait_or_abort(tfull, 0, p.status, abort_flag);
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16);
      float* pg = park + dst * GROUP + rl;  // column c at pg[c * R]
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) pg[(c + j) * R] = __uint_as_float(r[j]);
      }
    } else {
      ok = false;
    }
    fence_proxy_async_smem();  // the parked groups are read by the bulk-copy engine
    mbar_arrive(parked);
    if (et == 0) {
      // every group is written (or abandoned: its reducer still gets bytes and does not wait out)
      if (!mbar_wait(parked, 0, p.status)) *abort_flag = 1;
      for (int j = 0; j < splits; ++j)
        bulk_copy_to_cta(smem_u32(slots + rank * GROUP), park + j * GROUP, (uint32_t)(GROUP * 4), recv, (uint32_t)j);
      bulk_commit_group();
    }
    ok = mbar_wait_or_abort(recv, 0, p.status, abort_flag) && ok;
    const int r0 = (int)rank * R, r1 = min(BM, r0 + R);
    if (ok && r1 > r0) {
      // runs of 4 rows of one column: thread et takes (column n, rows r0 + 4 g ..)
      const int ng = (r1 - r0 + 3) / 4;
      for (int i = et; i < BN * ng; i += 128) {
        const int n = i / ng, g = i % ng;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < splits; ++j) {
          const float4 v = *reinterpret_cast<const float4*>(slots + j * GROUP + n * R + g * 4);
          acc[0] += v.x;
          acc[1] += v.y;
          acc[2] += v.z;
          acc[3] += v.w;
        }
        const int col = nt * BN + n;
        const int grow0 = mt * BM + r0 + g * 4;
        if (col >= p.N || grow0 >= p.M) continue;
        const int nrow = min(4, min(r1 - (r0 + g * 4), p.M - grow0));
        if (p.bias)
          for (int k = 0; k < nrow; ++k) acc[k] += __bfloat162float(p.transpose_out ? p.bias[grow0 + k] : p.bias[col]);
        if (rs && p.transpose_out) {
          // token `col`, features grow0.. of its owner's reduce-scatter row (p.M features)
          __nv_bfloat16* d = rs_dst(p, col, grow0, p.M);
          if (nrow == 4) {
            uint2 v;
            v.x = pack_bf16x2(acc[0], acc[1]);
            v.y = pack_bf16x2(acc[2], acc[3]);
            *reinterpret_cast<uint2*>(d) = v;
          } else {
            for (int k = 0; k < nrow; ++k) d[k] = __float2bfloat16(acc[k]);
          }
        } else if (rs) {
          for (int k = 0; k < nrow; ++k) *rs_dst(p, grow0 + k, col, p.N) = __float2bfloat16(acc[k]);
        } else if (p.transpose_out && p.Cf == nullptr && nrow == 4 && ((reinterpret_cast<uintptr_t>(p.C) & 7) == 0) &&
            (p.ldc & 3) == 0) {
          uint2 v;
          v.x = pack_bf16x2(acc[0], acc[1]);
          v.y = pack_bf16x2(acc[2], acc[3]);
          *reinterpret_cast<uint2*>(p.C + (size_t)col * p.ldc + grow0) = v;
        } else {
          for (int k = 0; k < nrow; ++k) {
            const size_t off = p.transpose_out ? (size_t)col * p.ldc + grow0 + k : (size_t)(grow0 + k) * p.ldc + col;
            if (p.Cf != nullptr)
              p.Cf[off] = acc[k];
            else
              p.C[off] = __float2bfloat16(acc[k]);
          }
        }
      }
    }
    // this CTA's parked groups must be read out before its shared memory goes away
    if (et == 0) bulk_wait_read_all();
    if (rs) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (rs) sp_push_arrive(p.sp, kSpReduceScatter, gridDim.x);
    if (p.sp_mode == 2) sp_recv_arrive(p.sp, kSpAllGather, gridDim.x, *s_ag_epoch);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
}

// Sum of split-K partials in split order, plus optional bias, to bf16.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, __nv_bfloat16* __restrict__ C,
                                     float* __restrict__ Cf, int rows, int cols, int ldc, int splits,
                                     const __nv_bfloat16* __restrict__ bias, int bias_on_rows) {
  pdl_prologue();
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += partial[(size_t)k * n + i];
    const int r = i / cols, c = i % cols;
    if (bias) s += __bfloat162float(bias[bias_on_rows ? r : c]);
    if (Cf)
      Cf[(size_t)r * ldc + c] = s;
    else
      C[(size_t)r * ldc + c] = __float2bfloat16(s);
  }
}

template <int BN>
cudaError_t launch(const void* A, int64_t lda, int rows_a, const void* B, int64_t ldb, int rows_b, int K,
                   const Params& p, cudaStream_t stream, int grid) {
  using C_ = Cfg<BN>;
  CUtensorMap ta = make_tma_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_a, K, lda, BM, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tma_2d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_b, K, ldb, BN, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  auto kern = gemm_bf16_tn_kernel<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  launch_pdl(kern, dim3(grid), dim3(kThreads), C_::SMEM_BYTES, stream, ta, tb, p);
  return cudaGetLastError();
}

template <int BN>
cudaError_t launch_batched(const void* A, int64_t lda, int64_t a_bs, int rows_a, const void* B, int64_t ldb,
                           int64_t b_bs, int rows_b, int K, const Params& p, cudaStream_t stream, int grid) {
  using C_ = Cfg<BN>;
  if (p.batch < 2) return cudaErrorInvalidValue;  // the kernel loads through the 3-D maps only for batch > 1
  CUtensorMap ta = make_tma_3d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_a, K, p.batch, lda, a_bs, BM, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tma_3d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_b, K, p.batch, ldb, b_bs, BN, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  auto kern = gemm_bf16_tn_kernel<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  launch_pdl(kern, dim3(grid), dim3(kThreads), C_::SMEM_BYTES, stream, ta, tb, p);
  return cudaGetLastError();
}

template <int BN>
cudaError_t launch_csk(const void* A, int64_t lda, int rows_a, const void* B, int64_t ldb, int rows_b, int K,
                       const Params& p, cudaStream_t stream) {
  using C_ = Cfg<BN>;
  CUtensorMap ta = make_tma_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_a, K, lda, BM, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tma_2d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows_b, K, ldb, BN, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  using P_ = CskPlan<BN>;
  const int R = ((BM + p.splits - 1) / p.splits + 3) / 4 * 4;
  if (p.splits * R > P_::MAX_ROWS) return cudaErrorInvalidValue;
  auto kern = gemm_bf16_csk_kernel<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.m_tiles * p.n_tiles * p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P_::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace gemm

int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Splits up to this many run as one thread-block cluster per tile, reduced in distributed shared
// memory (gemm_bf16_csk_kernel); more go through fp32 partials and a reduce kernel.
constexpr int kMaxClusterSplits = 8;

bool gemm_bf16_uses_partial(int M, int splits) { return splits > kMaxClusterSplits || (splits > 1 && M > 128); }

// How many clusters of `s` CTAs of the cluster kernel can be resident at once (one wave), cached.
static int csk_max_active(int bn, int s) {
  using namespace gemm;
  static int cache[5][kMaxClusterSplits + 1] = {};
  const int bi = bn <= 16 ? 0 : bn <= 32 ? 1 : bn <= 64 ? 2 : 3;
  int& c = cache[bi][s];
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = s;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(s * 64);
    cfg.blockDim = dim3(kThreads);
    int n = 0;
    cudaError_t e = cudaErrorInvalidValue;
    switch (bi) {
#define B200_CSK_OCC(BN_)                                                                                       \
  {                                                                                                            \
    cfg.dynamicSmemBytes = CskPlan<BN_>::SMEM_BYTES;                                                            \
    cudaFuncSetAttribute(gemm_bf16_csk_kernel<BN_>, cudaFuncAttributeMaxDynamicSharedMemorySize,               \
                         CskPlan<BN_>::SMEM_BYTES);                                                             \
    e = cudaOccupancyMaxActiveClusters(&n, gemm_bf16_csk_kernel<BN_>, &cfg);                                   \
    break;                                                                                                     \
  }
      case 0: B200_CSK_OCC(16)
      case 1: B200_CSK_OCC(32)
      case 2: B200_CSK_OCC(64)
      default: B200_CSK_OCC(128)
#undef B200_CSK_OCC
    }
    c = (e == cudaSuccess && n > 0) ? n : std::max(1, device_sm_count() / s);
  }
  return c;
}

// Number of K splits the launcher uses for this shape (splits_req > 0 forces it).
int gemm_bf16_splits(int M, int N, int K, int splits_req) {
  using namespace gemm;
  const bool swap = M <= 128;
  const int Ma = swap ? N : M;
  const int Nb = swap ? M : N;
  const int bn = swap ? (Nb <= 16 ? 16 : Nb <= 32 ? 32 : Nb <= 64 ? 64 : 128) : 256;
  const int tiles = ((Ma + BM - 1) / BM) * ((Nb + bn - 1) / bn);
  const int kb_total = (K + BK - 1) / BK;
  const int sms = device_sm_count();
  int splits = 1;
  if (splits_req > 0) {
    splits = splits_req;
  } else if (tiles < sms) {
    // K split over a cluster of at most 8 CTAs per tile, at least 2 K blocks each, and no more
    // splits than leave every tile's cluster resident in one wave
    splits = std::max(1, std::min(std::min(kMaxClusterSplits, sms / tiles), kb_total / 2));
    if (M <= 128 && bn <= 128)
      while (splits > 1 && csk_max_active(bn, splits) < tiles) --splits;
  }
  splits = std::max(1, std::min(splits, kb_total));
  const int per = (kb_total + splits - 1) / splits;
  return (kb_total + per - 1) / per;
}

static cudaError_t gemm_bf16_impl(const GemmArgs& a, const GemmSpArgs* sp, cudaStream_t stream) {
  using namespace gemm;
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.K % 8 != 0) return cudaErrorInvalidValue;
  const int sms = device_sm_count();
  // Small M: weights fill the 128-row MMA dimension, tokens the N dimension.
  const bool swap = a.M <= 128;
  const void* A = swap ? a.w : a.x;
  const void* B = swap ? a.x : a.w;
  const int64_t lda = swap ? a.ldw : a.ldx;
  const int64_t ldb = swap ? a.ldx : a.ldw;
  const int Ma = swap ? a.N : a.M;
  const int Nb = swap ? a.M : a.N;
  const int bn = swap ? (Nb <= 16 ? 16 : Nb <= 32 ? 32 : Nb <= 64 ? 64 : 128) : 256;
  Params p{};
  p.M = Ma;
  p.N = Nb;
  p.K = a.K;
  p.ldc = (int)a.ldc;
  p.transpose_out = swap ? 1 : 0;
  p.m_tiles = (Ma + BM - 1) / BM;
  p.n_tiles = (Nb + bn - 1) / bn;
  const int kb_total = (a.K + BK - 1) / BK;
  int splits = gemm_bf16_splits(a.M, a.N, a.K, a.splits);
  if (sp != nullptr) {
    // the reduce-scatter pushes finished output rows: no fp32 partial pass (cluster split-K is fine)
    if (sp->mode == 1 && (splits > kMaxClusterSplits || (splits > 1 && (bn > 128 || a.M > 128)))) splits = 1;
    p.sp_mode = sp->mode;
    p.sp = sp->sp;
    p.sp_rs_off = sp->rs_off;
    p.sp_rows = sp->rows_per_rank;
    p.act_is_b = swap ? 1 : 0;
  }
  p.k_blocks_per_split = (kb_total + splits - 1) / splits;
  p.splits = splits;
  p.C = a.out_f32 ? nullptr : reinterpret_cast<__nv_bfloat16*>(a.c);
  p.Cf = a.out_f32 ? reinterpret_cast<float*>(a.c) : nullptr;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.status = a.status;
  if (splits > 1 && splits <= kMaxClusterSplits && bn <= 128) {
    switch (bn) {
      case 16: return launch_csk<16>(A, lda, Ma, B, ldb, Nb, a.K, p, stream);
      case 32: return launch_csk<32>(A, lda, Ma, B, ldb, Nb, a.K, p, stream);
      case 64: return launch_csk<64>(A, lda, Ma, B, ldb, Nb, a.K, p, stream);
      default: return launch_csk<128>(A, lda, Ma, B, ldb, Nb, a.K, p, stream);
    }
  }
  if (splits > 1) {
    if (a.partial == nullptr || a.partial_cap < (int64_t)splits * a.M * a.N) return cudaErrorInvalidValue;
    p.partial = a.partial;
    p.bias = nullptr;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = std::min(tiles * splits, sms);
  cudaError_t e;
  switch (bn) {
    case 16: e = launch<16>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid); break;
    case 32: e = launch<32>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid); break;
    case 64: e = launch<64>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid); break;
    case 128: e = launch<128>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid); break;
    default: e = launch<256>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid); break;
  }
  if (e != cudaSuccess || splits == 1) return e;
  // partial is [splits, M, N] in output orientation (never in the reduce-scatter mode).
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>(((int64_t)a.M * a.N + threads - 1) / threads, (int64_t)sms * 8);
  launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(threads), 0, stream, p.partial, p.C, p.Cf, a.M, a.N, (int)a.ldc, splits,
                                                       reinterpret_cast<const __nv_bfloat16*>(a.bias), 0);
  return cudaGetLastError();
}

cudaError_t gemm_bf16(const GemmArgs& a, cudaStream_t stream) { return gemm_bf16_impl(a, nullptr, stream); }

cudaError_t gemm_bf16_batched(const GemmBatchedArgs& a, cudaStream_t stream) {
  using namespace gemm;
  if (a.M == 0 || a.N == 0 || a.batch == 0) return cudaSuccess;
  if (a.K % 8 != 0 || a.batch < 1) return cudaErrorInvalidValue;
  const bool swap = a.M <= 128;
  const void* A = swap ? a.w : a.x;
  const void* B = swap ? a.x : a.w;
  const int64_t lda = swap ? a.ldw : a.ldx, a_bs = swap ? a.w_bstride : a.x_bstride;
  const int64_t ldb = swap ? a.ldx : a.ldw, b_bs = swap ? a.x_bstride : a.w_bstride;
  const int Ma = swap ? a.N : a.M;
  const int Nb = swap ? a.M : a.N;
  const int bn = swap ? (Nb <= 16 ? 16 : Nb <= 32 ? 32 : Nb <= 64 ? 64 : 128) : 256;
  Params p{};
  p.M = Ma;
  p.N = Nb;
  p.K = a.K;
  p.ldc = (int)a.ldc;
  p.transpose_out = swap ? 1 : 0;
  p.m_tiles = (Ma + BM - 1) / BM;
  p.n_tiles = (Nb + bn - 1) / bn;
  p.k_blocks_per_split = (a.K + BK - 1) / BK;
  p.splits = 1;
  p.C = reinterpret_cast<__nv_bfloat16*>(a.c);
  p.status = a.status;
  p.batch = a.batch;
  p.c_bstride = a.c_bstride;
  const int grid = std::min(p.m_tiles * p.n_tiles * a.batch, device_sm_count());
  if (a.batch == 1) {
    // one matrix: the plain kernel path with 2-D maps (the kernel issues 3-D loads only for batch > 1,
    // and a 2-D load through a 3-D map is an illegal instruction)
    switch (bn) {
      case 16: return launch<16>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid);
      case 32: return launch<32>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid);
      case 64: return launch<64>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid);
      case 128: return launch<128>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid);
      default: return launch<256>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, grid);
    }
  }
  switch (bn) {
    case 16: return launch_batched<16>(A, lda, a_bs, Ma, B, ldb, b_bs, Nb, a.K, p, stream, grid);
    case 32: return launch_batched<32>(A, lda, a_bs, Ma, B, ldb, b_bs, Nb, a.K, p, stream, grid);
    case 64: return launch_batched<64>(A, lda, a_bs, Ma, B, ldb, b_bs, Nb, a.K, p, stream, grid);
    case 128: return launch_batched<128>(A, lda, a_bs, Ma, B, ldb, b_bs, Nb, a.K, p, stream, grid);
    default: return launch_batched<256>(A, lda, a_bs, Ma, B, ldb, b_bs, Nb, a.K, p, stream, grid);
  }
}

cudaError_t gemm_bf16_sp(const GemmSpArgs& a, cudaStream_t stream) {
  const SpSync& s = a.sp;
  if (a.mode < 1 || a.mode > 2 || s.peers == nullptr || s.state == nullptr || s.world < 1 || s.world > kSpMaxRanks ||
      (a.mode == 1 && (a.rows_per_rank < 1 || a.g.M != a.rows_per_rank * s.world || a.g.bias != nullptr ||
                       a.g.out_f32 || a.g.N % 8)))
    return cudaErrorInvalidValue;
  return gemm_bf16_impl(a.g, &a, stream);
}

cudaError_t gemm_bf16_allreduce(const GemmArArgs& a, cudaStream_t stream) {
  using namespace gemm;
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.K % 8 != 0 || a.world < 1 || a.world > 8) return cudaErrorInvalidValue;
  const int sms = device_sm_count();
  const bool swap = a.M <= 128;
  const void* A = swap ? a.w : a.x;
  const void* B = swap ? a.x : a.w;
  const int64_t lda = swap ? a.ldw : a.ldx;
  const int64_t ldb = swap ? a.ldx : a.ldw;
  const int Ma = swap ? a.N : a.M;
  const int Nb = swap ? a.M : a.N;
  const int bn = swap ? (Nb <= 16 ? 16 : Nb <= 32 ? 32 : Nb <= 64 ? 64 : 128) : 256;
  Params p{};
  p.M = Ma;
  p.N = Nb;
  p.K = a.K;
  p.ldc = (int)a.ldc;
  p.transpose_out = swap ? 1 : 0;
  p.m_tiles = (Ma + BM - 1) / BM;
  p.n_tiles = (Nb + bn - 1) / bn;
  const int kb_total = (a.K + BK - 1) / BK;
  p.k_blocks_per_split = kb_total;
  p.splits = 1;
  p.C = reinterpret_cast<__nv_bfloat16*>(a.c);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.status = a.status;
  p.ar = 1;
  p.peers = a.peers;
  p.rank = a.rank;
  p.world = a.world;
  p.flag_off = a.flag_off;
  p.data_off = a.data_off;
  p.tile_bytes = (int64_t)BM * bn * 2;
  p.epochs = a.epochs;
  p.timeout_ns = a.timeout_ns;
  const int tiles = p.m_tiles * p.n_tiles;
  // one tile per CTA, every CTA resident: the fused reduction waits on peers
  if (tiles > sms || tiles > a.max_ctas || p.tile_bytes > a.tile_bytes_cap) return cudaErrorInvalidValue;
  switch (bn) {
    case 16: return launch<16>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, tiles);
    case 32: return launch<32>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, tiles);
    case 64: return launch<64>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, tiles);
    case 128: return launch<128>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, tiles);
    default: return launch<256>(A, lda, Ma, B, ldb, Nb, a.K, p, stream, tiles);
  }
}

// Whether gemm_bf16_allreduce takes this shape (one output tile per CTA within the CTA and slot caps).
int gemm_bf16_allreduce_fits(int M, int N, int max_ctas, int64_t tile_bytes_cap) {
  using namespace gemm;
  const bool swap = M <= 128;
  const int Ma = swap ? N : M;
  const int Nb = swap ? M : N;
  const int bn = swap ? (Nb <= 16 ? 16 : Nb <= 32 ? 32 : Nb <= 64 ? 64 : 128) : 256;
  const int tiles = ((Ma + BM - 1) / BM) * ((Nb + bn - 1) / bn);
  return tiles <= device_sm_count() && tiles <= max_ctas && (int64_t)BM * bn * 2 <= tile_bytes_cap;
}

}  // namespace b200

// ============================================================================
// Allocation-free entry point (declared and documented in noalloc.h; it has
// no counterpart in the reference).  The split-K scratch and the status word
// are file-scope device arrays; their device addresses are looked up once
// per device and passed to the same kernel the ordinary op launches.
// ============================================================================
#include <mutex>

#include "noalloc.h"

namespace b200 {
namespace noalloc {

static __device__ __align__(256) float g_scratch[B200_NOALLOC_SCRATCH_FLOATS];
static __device__ __align__(256) uint32_t g_status[64];

struct DeviceScratch {
  float* partial = nullptr;
  uint32_t* status = nullptr;
};
constexpr int kMaxDevices = 64;
static DeviceScratch g_dev[kMaxDevices];
static std::mutex g_mu;

// Device addresses of this device's copy of the scratch arrays (looked up on
// the first call made with that device current).
static cudaError_t scratch_for_current_device(DeviceScratch* out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_dev[dev].partial == nullptr) {
    void* p = nullptr;
    void* s = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    e = cudaGetSymbolAddress(&s, g_status);
    if (e != cudaSuccess) return e;
    g_dev[dev].partial = static_cast<float*>(p);
    g_dev[dev].status = static_cast<uint32_t*>(s);
  }
  *out = g_dev[dev];
  return cudaSuccess;
}

}  // namespace noalloc
}  // namespace b200

extern "C" int b200_gemm_bf16_noalloc(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc,
                                      int M, int N, int K, int splits, cudaStream_t stream) {
  using namespace b200;
  if (x == nullptr || w == nullptr || c == nullptr || M <= 0 || N <= 0 || K <= 0 || K % 8 != 0 || splits < 0 ||
      ldx < K || ldw < K || ldc < N)
    return B200_NOALLOC_BAD_ARGS;
  noalloc::DeviceScratch s;
  cudaError_t e = noalloc::scratch_for_current_device(&s);
  if (e != cudaSuccess) return (int)e;
  const int used = gemm_bf16_splits(M, N, K, splits);
  if (gemm_bf16_uses_partial(M, used) && (uint64_t)used * (uint64_t)M * (uint64_t)N > (uint64_t)B200_NOALLOC_SCRATCH_FLOATS)
    return B200_NOALLOC_TOO_LARGE;
  // The status word must start at zero for this call; the partial sums need
  // no clearing (every split writes its whole [M, N] slice).
  e = cudaMemsetAsync(s.status, 0, sizeof(uint32_t), stream);
  if (e != cudaSuccess) return (int)e;
  GemmArgs a{};
  a.x = x;
  a.ldx = ldx;
  a.w = w;
  a.ldw = ldw;
  a.bias = nullptr;
  a.c = c;
  a.ldc = ldc;
  a.out_f32 = 0;
  a.M = M;
  a.N = N;
  a.K = K;
  a.splits = used;
  a.partial = s.partial;
  a.partial_cap = B200_NOALLOC_SCRATCH_FLOATS;
  a.status = s.status;
  try {
    e = gemm_bf16(a, stream);
  } catch (...) {  // tensor-map encoding rejected the operands (alignment)
    return B200_NOALLOC_BAD_ARGS;
  }
  return (int)e;
}

extern "C" int b200_gemm_bf16_noalloc_status(uint32_t* out, cudaStream_t stream) {
  using namespace b200;
  if (out == nullptr) return B200_NOALLOC_BAD_ARGS;
  noalloc::DeviceScratch s;
  cudaError_t e = noalloc::scratch_for_current_device(&s);
  if (e != cudaSuccess) return (int)e;
  uint32_t v = 0;
  e = cudaMemcpyAsync(&v, s.status, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return (int)e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return (int)e;
  *out = v;
  return 0;
}

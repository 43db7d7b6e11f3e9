// Dequantizing grouped GEMM on tcgen05 for Marlin int4 (group 128, bf16
// scales) and fp8 e4m3 128x128 block-scaled weights: routed MoE experts
// (gate/up pass with SwiGLU, down pass) and dense linears (one "expert").
//
// Reference behaviour: the Marlin W4A16 MoE decode/prefill GEMMs
// (csrc/ampere_marlin/decode_v2.cu:121, marlin_moe_ops.cuh:437: (q - 8) * s,
// SwiGLU with clamp between the passes) and DeepSeek's fp8 block-scaled
// projections (models/deepseek_v41/ops/sm80_wo_a_grouped.py).  Same B200
// pipeline as the EXL3 kernel (exl3.cu):
//   * a TMA warp streams each 128-output x 64-K chunk of packed weights (and,
//     for Marlin, the chunk's 128 scales) into a raw ring;
//   * 16 decoder warps dequantize into the 128-byte-swizzled K-major operand
//     tile: Marlin nibbles become bf16 (q - 8) * s exactly (one rounding),
//     fp8 becomes fp16 scaled by the block scale;
//   * a second TMA warp streams the activation rows (bf16 for Marlin, fp16 for
//     fp8) in their own ring; one thread issues tcgen05.mma into TMEM;
//   * epilogue from TMEM: SwiGLU (gate/up) or a plain store (down / dense).
#include <algorithm>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "tma_host.h"

namespace b200 {
namespace dq {

constexpr int kDecodeWarps = 16;
constexpr int BK = 64;
constexpr int A_BYTES = 128 * BK * 2;
constexpr int kRawWarp = kDecodeWarps, kBWarp = kDecodeWarps + 1, kMmaWarp = kDecodeWarps + 2;
constexpr int kThreads = (kDecodeWarps + 3) * 32;
constexpr int kGroups = kDecodeWarps / 4;

enum Fmt : int { kMarlin = 0, kFp8Block = 1 };

struct Params {
  const void* w[2];        // Marlin: int32 [E, K/16, 2N]; fp8: uint8 [E, N, K]
  const void* scale[2];    // Marlin: bf16 [E, K/128, N] (stored order); fp8: fp32 [E, N/128, K/128]
  int K, N;
  int tile_rows;
  const int4* items;
  const int* num_items;
  void* out;
  int64_t ld_out;
  int out_mode;            // 0: operand type (gate/up intermediate), 1: fp32, 2: bf16
  float swiglu_limit;
  uint32_t* status;
};

struct Plan {
  int a_stages, b_stages, raw_stages, a_bytes, b_bytes, raw_bytes, smem;
};

template <int FMT>
__host__ __device__ constexpr int raw_mat_bytes() {
  return FMT == kMarlin ? 4096 + 256 : 128 * 64;  // Marlin: 4 k16 rows x 2 tiles x 512 B + 128 scales
}

inline Plan make_plan(int fmt, int nmat, int tile_rows) {
  Plan pl{};
  pl.a_bytes = nmat * A_BYTES;
  pl.b_bytes = nmat * tile_rows * 128;
  pl.raw_bytes = nmat * (fmt == kMarlin ? raw_mat_bytes<kMarlin>() : raw_mat_bytes<kFp8Block>());
  pl.raw_bytes = (pl.raw_bytes + 1023) / 1024 * 1024;
  const int budget = 210 * 1024;
  pl.a_stages = 3;
  pl.raw_stages = 4;
  pl.b_stages = std::min(8, (budget - pl.a_stages * pl.a_bytes - pl.raw_stages * pl.raw_bytes) / pl.b_bytes);
  if (pl.b_stages < 2) {
    pl.a_stages = 2;
    pl.b_stages = std::min(8, (budget - pl.a_stages * pl.a_bytes - pl.raw_stages * pl.raw_bytes) / pl.b_bytes);
  }
  pl.raw_stages = std::min(8, (budget - pl.a_stages * pl.a_bytes - pl.b_stages * pl.b_bytes) / pl.raw_bytes);
  pl.smem = 1024 + pl.a_stages * pl.a_bytes + pl.b_stages * pl.b_bytes + pl.raw_stages * pl.raw_bytes + 512;
  return pl;
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// bf16x2 of two nibbles (q_lo, q_hi) at bits [0,4) and [16,20) of v:
// (q | 0x4300) is bf16(128 + q); minus 136 is q - 8 exactly; times the
// column's scale pair rounds once.
__device__ __forceinline__ uint32_t marlin_pair(uint32_t v, uint32_t s2) {
  uint32_t x, r;
  asm("lop3.b32 %0, %1, 0x000f000f, 0x43004300, 0xea;" : "=r"(x) : "r"(v));
  asm("{\n\t.reg .b32 t;\n\t"
      "fma.rn.bf16x2 t, %1, %3, %4;\n\t"
      "mul.rn.bf16x2 %0, t, %2;\n\t}"
      : "=r"(r)
      : "r"(x), "r"(s2), "r"(0x3f803f80u), "r"(0xc308c308u));
  return r;
}

// Operand tile offset (128-byte swizzle, K-major, 2-byte elements).
__device__ __forceinline__ uint32_t sw_off(uint32_t m, uint32_t k) {
  return (m >> 3) * 1024 + (m & 7) * 128 + ((((k >> 3) ^ (m & 7)) & 7) << 4) + (k & 7) * 2;
}

template <int NMAT, int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    dequant_gemm_kernel(const __grid_constant__ CUtensorMap tma_b0, const __grid_constant__ CUtensorMap tma_b1,
                        const __grid_constant__ CUtensorMap tma_w0, const __grid_constant__ CUtensorMap tma_w1,
                        const __grid_constant__ CUtensorMap tma_s0, const __grid_constant__ CUtensorMap tma_s1,
                        Params p, Plan pl) {
  pdl_prologue();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int tile_rows = p.tile_rows;
  const int b_bytes = tile_rows * 128;
  const int stages = pl.a_stages, bstages = pl.b_stages, rstages = pl.raw_stages;
  uint8_t* sa = smem;
  uint8_t* sbb = sa + stages * pl.a_bytes;
  uint8_t* raw = sbb + bstages * pl.b_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + rstages * pl.raw_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + 4;
  uint64_t* raw_full = bars + 8;
  uint64_t* raw_empty = bars + 16;
  uint64_t* b_full = bars + 24;
  uint64_t* b_empty = bars + 32;
  uint64_t* tfull = bars + 40;
  uint64_t* drain = bars + 41;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 42);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr int kMatRaw = raw_mat_bytes<FMT>();

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ncols = NMAT * tile_rows;
  const uint32_t tmem_cols = ncols <= 32 ? 32 : ncols <= 64 ? 64 : ncols <= 128 ? 128 : ncols <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], kDecodeWarps);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < bstages; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < rstages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDecodeWarps);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = p.N / 128;
  const int n_items = *p.num_items;
  const int total = n_items * n_tiles;
  const int kchunks = p.K / BK;

  if (warp < kDecodeWarps) {
    // =================================================================== decoders + epilogue
    int stage = 0, rs = 0;
    uint32_t phase = 0, rphase = 0;
    int local = 0;
    const int g = warp / 4, q = warp % 4;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++local) {
      const int4 it = p.items[u / n_tiles];
      const int tile = u % n_tiles;
      const int e = it.x;
      bool ok = true;
      for (int kc = 0; kc < kchunks; ++kc) {
        bool got = mbar_wait_or_abort(&raw_full[rs], rphase, p.status, abort_flag);
        got = got && mbar_wait_or_abort(&empty[stage], phase ^ 1, p.status, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t rb = smem_u32(raw + rs * pl.raw_bytes);
        const uint32_t ab = smem_u32(sa + stage * pl.a_bytes);
        if constexpr (FMT == kMarlin) {
          // warp -> (k16 row r, 64-col tile tt, words j0, j0+1); lane (c, gg)
          const int r = warp >> 2, tt = (warp >> 1) & 1, j0 = (warp & 1) * 2;
          const uint32_t c = lane & 3, gg = lane >> 2;
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const uint32_t mb = rb + m * kMatRaw;
            uint32_t w0, w1;
            asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];"
                         : "=r"(w0), "=r"(w1)
                         : "r"(mb + (uint32_t)(((r * 2 + tt) * 128 + lane * 4 + j0) * 4)));
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int j = j0 + jj;
              const uint32_t w = jj ? w1 : w0;
              uint32_t s2;  // (s[col 16j + gg], s[col 16j + gg + 8]) of this tile
              asm volatile("ld.shared.b32 %0, [%1];" : "=r"(s2) : "r"(mb + 4096 + (tt * 64 + 8 * gg + 2 * j) * 2));
              const uint32_t s_lo = __byte_perm(s2, s2, 0x1010), s_hi = __byte_perm(s2, s2, 0x3232);
              const uint32_t mrow = tt * 64 + 16 * j + gg;
              const uint32_t kk = r * 16 + 2 * c;
              const uint32_t a_m = ab + m * A_BYTES;
              sts32(a_m + sw_off(mrow, kk), marlin_pair(w, s_lo));             // nib0/nib4
              sts32(a_m + sw_off(mrow, kk + 8), marlin_pair(w >> 4, s_lo));    // nib1/nib5
              sts32(a_m + sw_off(mrow + 8, kk), marlin_pair(w >> 8, s_hi));    // nib2/nib6
              sts32(a_m + sw_off(mrow + 8, kk + 8), marlin_pair(w >> 12, s_hi));  // nib3/nib7
            }
          }
        } else {
          // fp8 rows (out features) of 64 K bytes; warp w converts rows 8w..8w+7
          const int row = warp * 8 + (lane >> 2);
          const int kq = (lane & 3) * 16;
          const float* sc = reinterpret_cast<const float*>(p.scale[0]);
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const float* scm = reinterpret_cast<const float*>(p.scale[m]);
            const float s = scm[((int64_t)e * (p.N / 128) + tile) * (p.K / 128) + (kc >> 1)];
            (void)sc;
            const __half2 s2 = __float2half2_rn(s);
            uint4 v;
            asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"(rb + m * kMatRaw + row * 64 + kq));
            uint32_t h[8];
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t lo, hi;
              asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"((unsigned short)(wv[i] & 0xffff)));
              asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"((unsigned short)(wv[i] >> 16)));
              __half2 a = __hmul2(*reinterpret_cast<__half2*>(&lo), s2);
              __half2 b = __hmul2(*reinterpret_cast<__half2*>(&hi), s2);
              h[2 * i] = *reinterpret_cast<uint32_t*>(&a);
              h[2 * i + 1] = *reinterpret_cast<uint32_t*>(&b);
            }
            const uint32_t a_m = ab + m * A_BYTES;
            sts128(a_m + sw_off(row, kq), make_uint4(h[0], h[1], h[2], h[3]));
            sts128(a_m + sw_off(row, kq + 8), make_uint4(h[4], h[5], h[6], h[7]));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[stage]);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
        if (++rs == rstages) {
          rs = 0;
          rphase ^= 1;
        }
      }
      if (!ok) break;
      // ---------------------------------------------------------------- epilogue
      const bool got = mbar_wait_or_abort(tfull, local & 1, p.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int rows = it.z, row0 = it.y;
      const int feat = tile * 128 + q * 32 + lane;
      const int nchunks = (rows + 15) / 16;
      for (int c = g; c < nchunks; c += kGroups) {
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)c * 16;
        uint32_t ra[16], rb2[16];
        tmem_ld16(taddr, ra);
        if (NMAT == 2) tmem_ld16(taddr + tile_rows, rb2);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int r = c * 16 + i;
          if (r >= rows) continue;
          float v = __uint_as_float(ra[i]);
          if (NMAT == 2) {
            float gg = v, uu = __uint_as_float(rb2[i]);
            if (p.swiglu_limit > 0.f) {
              gg = fminf(gg, p.swiglu_limit);
              uu = fminf(fmaxf(uu, -p.swiglu_limit), p.swiglu_limit);
            }
            v = siluf_(gg) * uu;
          }
          const int64_t o = (int64_t)(row0 + r) * p.ld_out + feat;
          if (p.out_mode == 1)
            reinterpret_cast<float*>(p.out)[o] = v;
          else if (p.out_mode == 2 || FMT == kMarlin)
            reinterpret_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16(v);
          else
            reinterpret_cast<__half*>(p.out)[o] = __float2half_rn(v);
        }
      }
      tc_fence_before();
    }
  } else if (warp == kRawWarp) {
    // =================================================================== weight producer
    if (elect_one()) {
      int rs = 0;
      uint32_t rphase = 0, issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int4 it = p.items[u / n_tiles];
        const int tile = u % n_tiles;
        for (int kc = 0; kc < kchunks; ++kc) {
          if (!mbar_wait_or_abort(&raw_empty[rs], rphase ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* dst = raw + rs * pl.raw_bytes;
          if (FMT == kMarlin) {
            mbar_arrive_expect_tx(&raw_full[rs], NMAT * (4096 + 256));
            const int y = it.x * (p.K / 16) + kc * 4;
            const int ys = it.x * (p.K / 128) + (kc >> 1);
            tma_load_2d(dst, &tma_w0, &raw_full[rs], tile * 256, y);
            tma_load_2d(dst + 4096, &tma_s0, &raw_full[rs], tile * 128, ys);
            if (NMAT == 2) {
              tma_load_2d(dst + kMatRaw, &tma_w1, &raw_full[rs], tile * 256, y);
              tma_load_2d(dst + kMatRaw + 4096, &tma_s1, &raw_full[rs], tile * 128, ys);
            }
          } else {
            mbar_arrive_expect_tx(&raw_full[rs], NMAT * 128 * 64);
            const int y = it.x * p.N + tile * 128;
            tma_load_2d(dst, &tma_w0, &raw_full[rs], kc * 64, y);
            if (NMAT == 2) tma_load_2d(dst + kMatRaw, &tma_w1, &raw_full[rs], kc * 64, y);
          }
          ++issued;
          if (++rs == rstages) {
            rs = 0;
            rphase ^= 1;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        const uint32_t n = issued < (uint32_t)rstages ? issued : (uint32_t)rstages;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t k = issued - 1 - i;
          mbar_wait(&raw_full[k % rstages], (k / rstages) & 1, nullptr);
        }
      }
    }
  } else if (warp == kBWarp) {
    // =================================================================== activation producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int4 it = p.items[u / n_tiles];
        for (int kc = 0; kc < kchunks; ++kc) {
          if (!mbar_wait_or_abort(&b_empty[stage], phase ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[stage], NMAT * b_bytes);
          tma_load_2d(sbb + stage * pl.b_bytes, &tma_b0, &b_full[stage], kc * BK, it.y);
          if (NMAT == 2) tma_load_2d(sbb + stage * pl.b_bytes + b_bytes, &tma_b1, &b_full[stage], kc * BK, it.y);
          ++issued;
          if (++stage == bstages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        const uint32_t n = issued < (uint32_t)bstages ? issued : (uint32_t)bstages;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t k = issued - 1 - i;
          mbar_wait(&b_full[k % bstages], (k / bstages) & 1, nullptr);
        }
      }
    }
  } else {
    // =================================================================== MMA issuer
    if (elect_one()) {
      constexpr uint32_t fmt_bits = FMT == kMarlin ? 1 : 0;  // bf16 : fp16
      int stage = 0, bs = 0;
      uint32_t phase = 0, bphase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int4 it = p.items[u / n_tiles];
        const uint32_t idesc = make_idesc_f16(128, (it.z + 15) / 16 * 16, fmt_bits);
        for (int kc = 0; kc < kchunks; ++kc) {
          const bool ga = mbar_wait_or_abort(&b_full[bs], bphase, p.status, abort_flag) &&
                          mbar_wait_or_abort(&full[stage], phase, p.status, abort_flag);
          if (!ga) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t da = desc_kmajor_sw128(sa + stage * pl.a_bytes + m * A_BYTES) + 2 * k;
              const uint64_t db = desc_kmajor_sw128(sbb + bs * pl.b_bytes + m * b_bytes) + 2 * k;
              umma_f16(tmem_base + m * tile_rows, da, db, idesc, (kc > 0 || k > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[stage]);
          umma_commit(&b_empty[bs]);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
          if (++bs == bstages) {
            bs = 0;
            bphase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// out[r, :] = x[src(r), :] converted to the operand type (bf16 copy or fp16).
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int K,
                                   const int* __restrict__ src, void* out, int to_f16, int rows) {
  pdl_prologue();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int s = src ? src[r] : r;
  const __nv_bfloat16* xr = x + (int64_t)s * ld_x;
  for (int c = threadIdx.x * 8; c < K; c += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    if (to_f16) {
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) ow[i] = pack_half2(__bfloat162float(h[2 * i]), __bfloat162float(h[2 * i + 1]));
      reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out) + (int64_t)r * K + c)[0] = o;
    } else {
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (int64_t)r * K + c)[0] = v;
    }
  }
}

template <int NMAT, int FMT>
cudaError_t launch(const DequantGemmArgs& a, const Params& p, cudaStream_t stream) {
  const Plan pl = make_plan(FMT, NMAT, p.tile_rows);
  if (pl.a_stages < 2 || pl.b_stages < 2 || pl.raw_stages < 2 || pl.smem > 227 * 1024) return cudaErrorInvalidValue;
  const CUtensorMapDataType bt = FMT == kMarlin ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap b0 = make_tma_2d(a.b0, bt, 2, a.b_rows, p.K, p.K, p.tile_rows, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap b1 = NMAT == 2 ? make_tma_2d(a.b1, bt, 2, a.b_rows, p.K, p.K, p.tile_rows, BK, CU_TENSOR_MAP_SWIZZLE_128B)
                             : b0;
  CUtensorMap w0, w1, s0, s1;
  if (FMT == kMarlin) {
    // packed [E*K/16, 2N] int32; scales [E*K/128, N] bf16
    w0 = make_tma_2d(a.w[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)a.E * (p.K / 16), 2 * p.N, 2 * p.N, 4, 256,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    s0 = make_tma_2d(a.scale[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)a.E * (p.K / 128), p.N, p.N, 1, 128,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    w1 = NMAT == 2 ? make_tma_2d(a.w[1], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)a.E * (p.K / 16), 2 * p.N,
                                 2 * p.N, 4, 256, CU_TENSOR_MAP_SWIZZLE_NONE)
                   : w0;
    s1 = NMAT == 2 ? make_tma_2d(a.scale[1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)a.E * (p.K / 128), p.N,
                                 p.N, 1, 128, CU_TENSOR_MAP_SWIZZLE_NONE)
                   : s0;
  } else {
    // fp8 [E*N, K] bytes
    w0 = make_tma_2d(a.w[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E * p.N, p.K, p.K, 128, 64,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    w1 = NMAT == 2 ? make_tma_2d(a.w[1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.E * p.N, p.K, p.K, 128, 64,
                                 CU_TENSOR_MAP_SWIZZLE_NONE)
                   : w0;
    s0 = s1 = w0;
  }
  auto kern = dequant_gemm_kernel<NMAT, FMT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  const int grid = std::max(1, std::min(a.max_work, device_sm_count()));
  launch_pdl(kern, dim3(grid), dim3(kThreads), pl.smem, stream, b0, b1, w0, w1, s0, s1, p, pl);
  return cudaGetLastError();
}

}  // namespace dq

cudaError_t dequant_gemm(const DequantGemmArgs& a, cudaStream_t stream) {
  using namespace dq;
  if (a.K % 128 || a.N % 128 || a.tile_rows % 16 || a.tile_rows < 16 || a.tile_rows > 256) return cudaErrorInvalidValue;
  if (a.nmat == 2 && a.tile_rows > 128) return cudaErrorInvalidValue;
  Params p{};
  for (int m = 0; m < a.nmat; ++m) {
    p.w[m] = a.w[m];
    p.scale[m] = a.scale[m];
  }
  p.K = a.K;
  p.N = a.N;
  p.tile_rows = a.tile_rows;
  p.items = reinterpret_cast<const int4*>(a.items);
  p.num_items = a.num_items;
  p.out = a.out;
  p.ld_out = a.ld_out;
  p.out_mode = a.out_mode;
  p.swiglu_limit = a.swiglu_limit;
  p.status = a.status;
  try {
    if (a.format == kMarlin) return a.nmat == 2 ? launch<2, kMarlin>(a, p, stream) : launch<1, kMarlin>(a, p, stream);
    return a.nmat == 2 ? launch<2, kFp8Block>(a, p, stream) : launch<1, kFp8Block>(a, p, stream);
  } catch (const std::exception&) {
    return cudaErrorInvalidValue;
  }
}

cudaError_t gather_rows(const void* x, int64_t ld_x, int K, const int* src, void* out, int to_f16, int rows,
                        cudaStream_t stream) {
  if (K % 8 || ld_x % 8) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  launch_pdl(dq::gather_rows_kernel, dim3(rows), dim3(128), 0, stream, reinterpret_cast<const __nv_bfloat16*>(x), ld_x, K, src, out, to_f16,
                                                   rows);
  return cudaGetLastError();
}

}  // namespace b200

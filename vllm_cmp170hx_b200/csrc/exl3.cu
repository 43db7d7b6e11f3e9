// EXL3 trellis-quantised linear layers and MoE experts on tcgen05.
//
// Reference behaviour: csrc/exl3/{dense.cu,moe.cu,moe_v2.cu,reference.cu} of
// the reference (y = H128(H128(x*suh) @ W) * svh; routed experts with SwiGLU
// and a weighted combine).  The reference decodes the trellis into mma.sync
// register fragments (dense_mma.cu:249, moe_v2.cu:443); on sm_100 the MMA
// reads its operands from shared memory, so here:
//
//   * a TMA warp streams the trellis words of each 4 x 8-tile chunk into a
//     shared-memory ring; 16 decoder warps decode 8 states per lane and store
//     fp16 pairs into the 128-byte-swizzled K-major operand layout
//     (bank-conflict-free: the swizzle spreads a warp's 8 rows over all banks);
//   * a second TMA warp stages the (Hadamard-rotated, fp16) activation rows of
//     the work item in their own ring (128-byte swizzle);
//   * one thread issues tcgen05.mma (M = 128 output features, N = rows of the
//     item rounded to 16, K = 64 per stage) into TMEM;
//   * four epilogue warps read the result from TMEM: the output H128 is a
//     butterfly across the 128 TMEM lanes (shuffles + one shared exchange),
//     svh scaling, and for the gate/up pass SwiGLU plus the down projection's
//     input rotation, so the intermediate is written once, already in the
//     form the down pass consumes.  Two accumulators alternate between work
//     units, so the decoders start unit u + 1 while unit u is read out.
//
// A work item is (local expert, first row, rows <= tile_rows) of the
// expert-sorted assignment list (router.cu); a dense EXL3 linear is the same
// kernel with one "expert" whose rows are all tokens.
#include "common.cuh"
#include "launch.h"
#include <cstdio>
#include <stdexcept>
#include <string>

#include "tma_host.h"

namespace b200 {
namespace exl3 {

// Decoder warps per CTA (a template parameter DW of the kernel): 16 decode 2 tile rows each of every
// 4-row chunk, 8 decode all 4 rows of their tile column (twice the work per barrier round).
constexpr int kDecodeWarps = 16;

constexpr int BK = 64;                              // K per pipeline stage (4 tile rows)
constexpr int A_BYTES = 128 * BK * 2;               // one 128 x 64 fp16 operand tile
constexpr int A_LBO = 2048;                         // bytes between K-adjacent core matrices
constexpr int A_SBO = 128;                          // bytes between M-adjacent core matrices
constexpr float kH128 = 0.08838834764831845f;       // 1/sqrt(128)

struct GemmParams {
  const uint16_t* trellis[2];
  int64_t trellis_estride[2];  // int16 elements between experts
  const __half* svh[2];
  int64_t svh_estride[2];
  const __half* suh_next;  // gate/up pass: the down matrix's suh (rotation of the intermediate)
  int64_t suh_next_estride;
  int K;        // padded input features (multiple of 128)
  int N;        // padded output features of these matrices (multiple of 128)
  int bits_x2;
  int codebook;
  int tile_rows;  // TMA box rows == max rows per item
  const int4* items;
  const int* num_items;
  void* out;
  int64_t ld_out;
  int out_mode;        // 0: fp16 (gate/up intermediate), 1: fp32, 2: bf16
  float swiglu_limit;  // <= 0: none
  // Codebook 2 keeps the per-weight fp16 affine step out of the decode: the A operand holds
  // half(0x6400 + bytesum) = 1024 + bytesum exactly, and the epilogue forms
  // a * acc + b * sum_k x_k (a, b the codebook's constants) from the activation row sums:
  const float* sx[2];  // per matrix: [rows][sx_parts] partial sums of the activation rows (summed in order)
  int sx_parts;
  float* hsum;         // gate/up pass: [rows][N / 128] partial sums of the intermediate it writes
  uint32_t* status;
};

// Codebook 2's affine constants (fp16 0x1eee and 0xc931 as floats).
__device__ __forceinline__ float cb2_a() { return __half2float(__ushort_as_half((unsigned short)0x1eee)); }
__device__ __forceinline__ float cb2_b() { return __half2float(__ushort_as_half((unsigned short)0xc931)); }

// ----------------------------------------------------------------------------- codebooks
// Two states -> two fp16 weights packed as half2 (inline PTX keeps the
// format constants as immediates).
template <int CB>
__device__ __forceinline__ uint32_t cb_pair(uint32_t s0, uint32_t s1) {
  uint32_t r;
  if constexpr (CB == 2) {
    // t = 0x6400 + bytesum(s * 0x83DCD12D) as fp16 (= 1024 + bytesum, exact); the codebook's
    // w = 0x1eee * t + 0xc931 is applied to the accumulator in the epilogue (kCbA, kCbB)
    asm("{\n\t.reg .b32 p0, p1, t0, t1;\n\t"
        "mul.lo.u32 p0, %1, 0x83DCD12D;\n\t"
        "mul.lo.u32 p1, %2, 0x83DCD12D;\n\t"
        "dp4a.u32.u32 t0, p0, 0x01010101, 0x6400;\n\t"
        "dp4a.u32.u32 t1, p1, 0x01010101, 0x6400;\n\t"
        "prmt.b32 %0, t0, t1, 0x5410;\n\t}"
        : "=r"(r)
        : "r"(s0), "r"(s1));
  } else {
    // p = (s * 0xCBAC1FED) & 0x8fff8fff ^ 0x3b603b60; w = half(p.lo) + half(p.hi)
    asm("{\n\t.reg .b32 p0, p1, lo, hi;\n\t"
        "mul.lo.u32 p0, %1, 0xCBAC1FED;\n\t"
        "mul.lo.u32 p1, %2, 0xCBAC1FED;\n\t"
        "lop3.b32 p0, p0, 0x8fff8fff, 0x3b603b60, 0x6a;\n\t"
        "lop3.b32 p1, p1, 0x8fff8fff, 0x3b603b60, 0x6a;\n\t"
        "prmt.b32 lo, p0, p1, 0x5410;\n\t"
        "prmt.b32 hi, p0, p1, 0x7632;\n\t"
        "add.rn.f16x2 %0, lo, hi;\n\t}"
        : "=r"(r)
        : "r"(s0), "r"(s1));
  }
  return r;
}

// 8 states of lane L in a 16x16 tile at 4 bits per weight (bits_x2 = 8):
// the lane's window is word L-1 (low bits) and word L of the 32-word ring.
// State j is the 64-bit window (w_prev:w_self) shifted right by 28 - 4j and
// masked to 16 bits.  Shifts that are multiples of 8 are byte selections of
// w_self; shifts of 4 mod 8 are byte selections of the window shifted by 4.
__device__ __forceinline__ void states_b8(uint32_t w_prev, uint32_t w_self, uint32_t (&s)[8]) {
  const uint32_t lo4 = __funnelshift_r(w_self, w_prev, 4);  // low word of (window >> 4)
  s[0] = __funnelshift_r(w_self, w_prev, 28) & 0xffffu;
  s[1] = __funnelshift_r(w_self, w_prev, 24) & 0xffffu;
  // __byte_perm(x, 0, sel): result byte i = byte sel_i of x (selector 4 = zero)
  s[2] = __byte_perm(lo4, 0, 0x4432);
  s[3] = __byte_perm(w_self, 0, 0x4432);
  s[4] = __byte_perm(lo4, 0, 0x4421);
  s[5] = __byte_perm(w_self, 0, 0x4421);
  s[6] = __byte_perm(lo4, 0, 0x4410);
  s[7] = __byte_perm(w_self, 0, 0x4410);
}

// Generic bitrate: lane L's state j starts at ring bit (L*4*b + c_j) mod (128 b)
// with c_j = (j+1)*(b/2) + (b odd ? (j+1)/2 : 0) - 16.
__device__ __forceinline__ void states_generic(const uint32_t* __restrict__ words, int b, int lane,
                                               uint32_t (&s)[8]) {
  const int ring = 128 * b;
  const int nwords = 4 * b;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    int c = (j + 1) * (b >> 1) + ((b & 1) ? ((j + 1) >> 1) : 0) - 16;
    int pos = lane * 4 * b + c;
    pos = pos < 0 ? pos + ring : pos;
    pos = pos >= ring ? pos - ring : pos;
    const int lo = pos >> 5;
    const int hi = lo + 1 == nwords ? 0 : lo + 1;
    const uint32_t w0 = words[lo], w1 = words[hi];
    s[j] = __funnelshift_l(w1, w0, pos & 31) >> 16;
  }
}

// Decode one 16x16 tile (trellis tile words `tw`) and store it into the A
// operand stage: tile column `tc` (output features 16*tc..), tile row `tr`
// (K 16*tr..) of the 64-wide stage.
template <int CB, bool FAST>
__device__ __forceinline__ void decode_tile_store(const uint32_t* __restrict__ tw, uint32_t w_self, int b, int lane,
                                                  uint8_t* a_stage, int tc, int tr) {
  uint32_t s[8];
  if constexpr (FAST) {
    const uint32_t w_prev = __shfl_sync(0xffffffffu, w_self, (lane + 31) & 31);
    states_b8(w_prev, w_self, s);
  } else {
    states_generic(tw, b, lane, s);
  }
  const uint32_t v01 = cb_pair<CB>(s[0], s[1]);  // rows 2a, 2a+1   col b
  const uint32_t v23 = cb_pair<CB>(s[2], s[3]);  // rows 2a+8, 2a+9 col b
  const uint32_t v45 = cb_pair<CB>(s[4], s[5]);  // rows 2a, 2a+1   col b+8
  const uint32_t v67 = cb_pair<CB>(s[6], s[7]);  // rows 2a+8, 2a+9 col b+8
  // 128-byte-swizzled K-major tile (128 rows x 64 fp16): element (m, k) at
  // (m / 8) * 1024 + (m % 8) * 128 + ((k / 8) ^ (m % 8)) * 16 + (k % 8) * 2.
  // Lane (a = lane & 3, b = lane >> 2) holds rows m = 16 tc + b (+8) and
  // columns k = 16 tr + 2a (+8); the XOR spreads the 8 rows b over all banks.
  const uint32_t la = lane & 3, lb = lane >> 2;
  const uint32_t row = (uint32_t)tc * 2048 + lb * 128 + la * 4;
  const uint32_t c0 = (((uint32_t)tr * 2) ^ lb) << 4, c1 = (((uint32_t)tr * 2 + 1) ^ lb) << 4;
  *reinterpret_cast<uint32_t*>(a_stage + row + c0) = v01;
  *reinterpret_cast<uint32_t*>(a_stage + row + c1) = v23;
  *reinterpret_cast<uint32_t*>(a_stage + row + 1024 + c0) = v45;
  *reinterpret_cast<uint32_t*>(a_stage + row + 1024 + c1) = v67;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// 4-bit fast path: decode the lane's 8 weights of one tile whose words start
// at shared address `tw` (word `lane` at tw + 4 lane) and store them at the
// four precomputed operand addresses o0..o3 (see decode_tile_store).
template <int CB>
__device__ __forceinline__ void decode_tile_b8(uint32_t tw_lane, int lane, uint32_t o0, uint32_t o1, uint32_t o2,
                                               uint32_t o3) {
  const uint32_t w_self = lds32(tw_lane);
  const uint32_t w_prev = __shfl_sync(0xffffffffu, w_self, (lane + 31) & 31);
  uint32_t st[8];
  states_b8(w_prev, w_self, st);
  sts32(o0, cb_pair<CB>(st[0], st[1]));
  sts32(o1, cb_pair<CB>(st[2], st[3]));
  sts32(o2, cb_pair<CB>(st[4], st[5]));
  sts32(o3, cb_pair<CB>(st[6], st[7]));
}

// In-register butterfly over the 128 features held one per thread of a
// 4-warp group (feature f = 32*q + lane), for NV columns at once.
template <int NV>
__device__ __forceinline__ void h128_group(float (&v)[NV], int lane, int q, float* xbuf, int bar_id) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float o = __shfl_xor_sync(0xffffffffu, v[i], d);
      v[i] = (lane & d) ? (o - v[i]) : (v[i] + o);
    }
  }
  const int f = q * 32 + lane;
#pragma unroll
  for (int qb = 1; qb <= 2; qb <<= 1) {
#pragma unroll
    for (int i = 0; i < NV; ++i) xbuf[i * 128 + f] = v[i];
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id));
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float o = xbuf[i * 128 + (f ^ (qb * 32))];
      v[i] = (q & qb) ? (o - v[i]) : (v[i] + o);
    }
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id));
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] *= kH128;
}

// Sum over the 128 threads of a 4-warp group of each of NV values (fixed order: deterministic).
template <int NV>
__device__ __forceinline__ void group_sum(float (&v)[NV], int lane, int q, float* xbuf, int bar_id) {
#pragma unroll
  for (int i = 0; i < NV; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) xbuf[q * NV + i] = v[i];
  }
  asm volatile("bar.sync %0, 128;" ::"r"(bar_id));
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = (xbuf[i] + xbuf[NV + i]) + (xbuf[2 * NV + i] + xbuf[3 * NV + i]);
  asm volatile("bar.sync %0, 128;" ::"r"(bar_id));
}

// The activation row sum of row `row` for matrix m (0 outside the item's rows).
__device__ __forceinline__ float row_sum(const GemmParams& p, int m, int row, bool valid) {
  if (!valid || p.sx[m] == nullptr) return 0.f;
  float s = 0.f;
  for (int i = 0; i < p.sx_parts; ++i) s += p.sx[m][(int64_t)row * p.sx_parts + i];
  return s;
}

template <int NV>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[NV]) {
  if constexpr (NV == 16) {
    tmem_ld16(taddr, r);
  } else {
    static_assert(NV == 4, "4 or 16 columns");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  }
}

// Epilogue of NV accumulator columns (= rows c0 .. c0+NV-1 of the item) for this thread's output
// feature: H128 across the 128 TMEM lanes, svh, and for the gate/up pass SwiGLU plus the down
// projection's input rotation (suh, H128), written in the form the down pass reads.
template <int NMAT, int NV>
__device__ __forceinline__ void epilogue_block(const GemmParams& p, uint32_t tlane, int tile_rows, int c0, int rows,
                                               int row0, int feat, int tile, float sg, float su, float sn, int lane,
                                               int q, float* xb, int bar_id, const float* pre0 = nullptr,
                                               const float* pre1 = nullptr) {
  const bool fold = p.codebook == 2;
  const float ca = cb2_a(), cbb = cb2_b();
  if constexpr (NMAT == 2) {
    uint32_t rg[NV], ru[NV];
    tmem_ld_cols<NV>(tlane + c0, rg);
    tmem_ld_cols<NV>(tlane + tile_rows + c0, ru);
    tmem_wait_ld();
    float gv[NV], uv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      gv[i] = __uint_as_float(rg[i]);
      uv[i] = __uint_as_float(ru[i]);
      if (fold) {
        const bool ok = c0 + i < rows;
        gv[i] = ca * gv[i] + cbb * (pre0 ? pre0[i] : row_sum(p, 0, row0 + c0 + i, ok));
        uv[i] = ca * uv[i] + cbb * (pre1 ? pre1[i] : row_sum(p, 1, row0 + c0 + i, ok));
      }
    }
    h128_group<NV>(gv, lane, q, xb, bar_id);
    h128_group<NV>(uv, lane, q, xb, bar_id);
    const float L = p.swiglu_limit;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float gg = gv[i] * sg, uu = uv[i] * su;
      if (L > 0.f) {
        gg = fminf(gg, L);
        uu = fminf(fmaxf(uu, -L), L);
      }
      gv[i] = siluf_(gg) * uu * sn;
    }
    h128_group<NV>(gv, lane, q, xb, bar_id);
    __half* out = reinterpret_cast<__half*>(p.out);
    float hs[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int r = c0 + i;
      const __half hv = __float2half_rn(gv[i]);
      hs[i] = r < rows ? __half2float(hv) : 0.f;
      if (r < rows) out[(int64_t)(row0 + r) * p.ld_out + feat] = hv;
    }
    if (p.hsum != nullptr) {  // the down pass's activation row sums, one partial per feature tile
      group_sum<NV>(hs, lane, q, xb, bar_id);
      if (q == 0 && lane == 0) {
        const int parts = p.N / 128;
#pragma unroll
        for (int i = 0; i < NV; ++i)
          if (c0 + i < rows) p.hsum[(int64_t)(row0 + c0 + i) * parts + tile] = hs[i];
      }
    }
  } else {
    uint32_t ra[NV];
    tmem_ld_cols<NV>(tlane + c0, ra);
    tmem_wait_ld();
    float v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      v[i] = __uint_as_float(ra[i]);
      if (fold) v[i] = ca * v[i] + cbb * (pre0 ? pre0[i] : row_sum(p, 0, row0 + c0 + i, c0 + i < rows));
    }
    h128_group<NV>(v, lane, q, xb, bar_id);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int r = c0 + i;
      if (r >= rows) continue;
      const int64_t o = (int64_t)(row0 + r) * p.ld_out + feat;
      if (p.out_mode == 1)
        reinterpret_cast<float*>(p.out)[o] = v[i] * sg;
      else
        reinterpret_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16(v[i] * sg);
    }
  }
}

// Shared-memory plan: `ab` stages of [NMAT decoded A tiles | NMAT B tiles]
// and `raw` stages of NMAT raw trellis chunks (32 tiles each), sized on the
// host so both rings fit next to the epilogue exchange buffers.
struct Plan {
  int a_stages, b_stages, raw_stages;  // decoded-A ring, activation ring, raw trellis ring
  int a_bytes, b_bytes, raw_bytes;     // bytes per stage of each ring
  int smem;
};

constexpr int kEpiWarps = 4;               // dedicated epilogue warps (one group: 128 TMEM lanes)
constexpr int kGroups = 1;                 // epilogue warp groups (named barrier 1, xbuf slice 0)
constexpr int kXbufBytes = 16 * 128 * 4;   // per-group H128 exchange buffer

// Shared-memory plan: three independent rings so that neither the trellis
// nor the activation loads wait for the decoded-operand ring to drain.
inline Plan make_plan(int nmat, int tile_rows, int bits_x2) {
  Plan pl{};
  pl.a_bytes = nmat * A_BYTES;
  pl.b_bytes = nmat * tile_rows * 128;
  pl.raw_bytes = nmat * 32 * 16 * bits_x2;
  const int budget = 210 * 1024 - kGroups * kXbufBytes;
  pl.a_stages = 3;
  pl.raw_stages = 6;
  pl.b_stages = (budget - pl.a_stages * pl.a_bytes - pl.raw_stages * pl.raw_bytes) / pl.b_bytes;
  if (pl.b_stages > 8) pl.b_stages = 8;
  while (pl.b_stages < 2 && pl.a_stages > 2) {
    --pl.a_stages;
    pl.b_stages = (budget - pl.a_stages * pl.a_bytes - pl.raw_stages * pl.raw_bytes) / pl.b_bytes;
  }
  while (pl.b_stages < 2 && pl.raw_stages > 3) {
    --pl.raw_stages;
    pl.b_stages = (budget - pl.a_stages * pl.a_bytes - pl.raw_stages * pl.raw_bytes) / pl.b_bytes;
  }
  if (pl.b_stages > 8) pl.b_stages = 8;
  const int left = budget - pl.a_stages * pl.a_bytes - pl.b_stages * pl.b_bytes;
  pl.raw_stages = left / pl.raw_bytes > 8 ? 8 : left / pl.raw_bytes;
  pl.smem = 1024 + pl.a_stages * pl.a_bytes + pl.b_stages * pl.b_bytes + pl.raw_stages * pl.raw_bytes +
            kGroups * kXbufBytes + 512;
  return pl;
}

// Warp roles for DW decoder warps: decoders [0, DW), epilogue [DW, DW + 4), trellis producer, activation
// producer, TMEM owner + MMA issuer.
template <int DW>
struct Roles {
  static constexpr int kEpiWarp0 = DW;
  static constexpr int kRawWarp = DW + kEpiWarps;
  static constexpr int kBWarp = kRawWarp + 1;
  static constexpr int kMmaWarp = kRawWarp + 2;
  static constexpr int kThreads = (kMmaWarp + 1) * 32;
};

// NMAT = 2: gate/up pass (writes the rotated SwiGLU intermediate), 1: down / dense.
// Trellis chunks (4 tile rows x 8 tile columns per matrix) arrive by TMA in
// a ring `raw_stages` deep, so the decoder warps never wait on global memory.
template <int NMAT, int CB, bool FAST, int DW>
__global__ void __launch_bounds__(Roles<DW>::kThreads, 1)
    exl3_gemm_kernel(const __grid_constant__ CUtensorMap tma_b0, const __grid_constant__ CUtensorMap tma_b1,
                     const __grid_constant__ CUtensorMap tma_t0, const __grid_constant__ CUtensorMap tma_t1,
                     GemmParams p, Plan pl) {
  constexpr int kDecodeWarps = DW;
  constexpr int kEpiWarp0 = Roles<DW>::kEpiWarp0;
  constexpr int kRawWarp = Roles<DW>::kRawWarp;
  constexpr int kBWarp = Roles<DW>::kBWarp;
  constexpr int kMmaWarp = Roles<DW>::kMmaWarp;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int tile_rows = p.tile_rows;
  const int b_bytes = tile_rows * 128;  // one matrix's activation tile
  const int stages = pl.a_stages;
  const int bstages = pl.b_stages;
  const int rstages = pl.raw_stages;
  uint8_t* sa = smem;
  uint8_t* sbb = sa + stages * pl.a_bytes;
  uint8_t* raw = sbb + bstages * pl.b_bytes;
  float* xbuf = reinterpret_cast<float*>(raw + rstages * pl.raw_bytes);  // [kGroups][16][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xbuf + kGroups * 16 * 128);
  uint64_t* full = bars;             // [4]  decoder warps: decoded A stage ready
  uint64_t* empty = bars + 4;        // [4]  MMA commit: A stage free
  uint64_t* raw_full = bars + 8;     // [8]  trellis TMA tx
  uint64_t* raw_empty = bars + 16;   // [8]  decoder warps
  uint64_t* b_full = bars + 24;      // [8]  activation TMA tx
  uint64_t* b_empty = bars + 32;     // [8]  MMA commit
  uint64_t* tfull = bars + 40;       // [2] MMA commit: accumulator ready
  uint64_t* tempty = bars + 42;      // [2] epilogue warps: accumulator read out
  uint64_t* drain = bars + 44;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 45);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int acc_cols = NMAT * tile_rows;  // one accumulator; two alternate between units
  const int tmem_cols_needed = 2 * acc_cols;
  const uint32_t tmem_cols = tmem_cols_needed <= 32 ? 32 : tmem_cols_needed <= 64 ? 64 : tmem_cols_needed <= 128 ? 128
                             : tmem_cols_needed <= 256 ? 256 : 512;
  const int tile_bytes = FAST ? 128 : 16 * p.bits_x2;  // one 16x16 trellis tile
  const int mat_raw = 32 * tile_bytes;     // one matrix's chunk (4 x 8 tiles)

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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps * 32);
    }
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
  pdl_prologue();  // setup above overlaps the previous kernel's tail
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = p.N / 128;
  const int n_items = *p.num_items;
  const int total = n_items * n_tiles;
  const int kchunks = p.K / BK;
  const int kt_rows = p.K / 16;  // trellis tile rows per expert

  auto a_tile = [&](int stage, int m) { return sa + stage * pl.a_bytes + m * A_BYTES; };
  auto b_tile = [&](int stage, int m) { return sbb + stage * pl.b_bytes + m * b_bytes; };

  if (warp < kDecodeWarps) {
    // =================================================================== decoders
    int stage = 0, rs = 0;
    uint32_t phase = 0, rphase = 0;
    const int tc = warp & 7;                          // decoded tile column (16 output features)
    const int tr0 = (warp >> 3) * (4 / (kDecodeWarps / 8));  // first tile row of this warp
    constexpr int kRowsPerWarp = 4 / (kDecodeWarps / 8);
    // per-warp constant addressing of the 4-bit path: this lane's word of tile
    // (tr0 + r, tc) in a raw stage, and its four operand store offsets
    const uint32_t raw_lane_off = (uint32_t)((tr0 * 8 + tc) * 128 + lane * 4);
    uint32_t st_off[kRowsPerWarp][4];
    {
      const uint32_t la = lane & 3, lb = lane >> 2;
      const uint32_t row = (uint32_t)tc * 2048 + lb * 128 + la * 4;
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const uint32_t tr = tr0 + r;
        const uint32_t c0 = ((tr * 2) ^ lb) << 4, c1 = ((tr * 2 + 1) ^ lb) << 4;
        st_off[r][0] = row + c0;
        st_off[r][1] = row + c1;
        st_off[r][2] = row + 1024 + c0;
        st_off[r][3] = row + 1024 + c1;
      }
    }
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      bool ok = true;
      for (int kc = 0; kc < kchunks; ++kc) {
        bool got = mbar_wait_or_abort(&raw_full[rs], rphase, p.status, abort_flag);
        got = got && mbar_wait_or_abort(&empty[stage], phase ^ 1, p.status, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint8_t* rbase = raw + rs * pl.raw_bytes;
        if constexpr (FAST) {
          // all of this warp's tiles of the chunk at once: loads first, then the independent
          // decode chains (plain shared accesses, so the compiler interleaves them)
          // explicit shared-space loads and stores (32-bit shared addresses, no generic-address
          // resolution); the codebook arithmetic between them schedules freely
          constexpr int NT = NMAT * kRowsPerWarp;
          const uint32_t rw = smem_u32(rbase) + raw_lane_off;
          uint32_t w_self[NT], w_prev[NT];
#pragma unroll
          for (int i = 0; i < NT; ++i) w_self[i] = lds32(rw + (i / kRowsPerWarp) * 32 * 128 + (i % kRowsPerWarp) * 8 * 128);
#pragma unroll
          for (int i = 0; i < NT; ++i) w_prev[i] = __shfl_sync(0xffffffffu, w_self[i], (lane + 31) & 31);
          const uint32_t ab = smem_u32(a_tile(stage, 0));
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            const int m = i / kRowsPerWarp, r = i % kRowsPerWarp;
            uint32_t st[8];
            states_b8(w_prev[i], w_self[i], st);
            const uint32_t mo = ab + m * A_BYTES;
            sts32(mo + st_off[r][0], cb_pair<CB>(st[0], st[1]));
            sts32(mo + st_off[r][1], cb_pair<CB>(st[2], st[3]));
            sts32(mo + st_off[r][2], cb_pair<CB>(st[4], st[5]));
            sts32(mo + st_off[r][3], cb_pair<CB>(st[6], st[7]));
          }
        } else {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
#pragma unroll
            for (int r = 0; r < kRowsPerWarp; ++r) {
              const int tr = tr0 + r;
              const uint32_t* tw =
                  reinterpret_cast<const uint32_t*>(rbase + m * mat_raw + (tr * 8 + tc) * tile_bytes);
              decode_tile_store<CB, FAST>(tw, 0u, p.bits_x2, lane, a_tile(stage, m), tc, tr);
            }
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
    }
  } else if (warp < kEpiWarp0 + kEpiWarps) {
    // =================================================================== epilogue warps
    // Read accumulator (local & 1) of every unit this CTA runs while the decoders and the MMA
    // already fill the other one: the decode of unit u + 1 never waits for the epilogue of u.
    const int q = warp % 4;  // TMEM lane quarter
    const int f = q * 32 + lane;
    int local = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++local) {
      const int4 it = p.items[u / n_tiles];
      const int tile = u % n_tiles;
      const int e = it.x;
      const int acc = local & 1;
      const int rows = it.z;
      const int row0 = it.y;
      const int feat = tile * 128 + f;
      // the unit's scales and (short items) activation row sums: loaded while its MMAs still run
      const float sg = __half2float(p.svh[0][(int64_t)e * p.svh_estride[0] + feat]);
      const float su = NMAT == 2 ? __half2float(p.svh[1][(int64_t)e * p.svh_estride[1] + feat]) : 0.f;
      const float sn = NMAT == 2 ? __half2float(p.suh_next[(int64_t)e * p.suh_next_estride + feat]) : 0.f;
      float pre0[4] = {0.f, 0.f, 0.f, 0.f}, pre1[4] = {0.f, 0.f, 0.f, 0.f};
      if (rows <= 4 && p.codebook == 2) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pre0[i] = row_sum(p, 0, row0 + i, i < rows);
          if (NMAT == 2) pre1[i] = row_sum(p, 1, row0 + i, i < rows);
        }
      }
      const bool got = mbar_wait_or_abort(&tfull[acc], (local >> 1) & 1, p.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;  // TMEM loads are warp-collective
      tc_fence_after();
      const int nchunks = (rows + 15) / 16;
      const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * acc_cols);
      if (rows > 4) {
        for (int c = 0; c < nchunks; ++c)
          epilogue_block<NMAT, 16>(p, tlane, tile_rows, c * 16, rows, row0, feat, tile, sg, su, sn, lane, q, xbuf, 1);
      } else {
        epilogue_block<NMAT, 4>(p, tlane, tile_rows, 0, rows, row0, feat, tile, sg, su, sn, lane, q, xbuf, 1, pre0,
                                pre1);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  } else if (warp == kRawWarp) {
    // =================================================================== trellis producer
    if (elect_one()) {
      tma_prefetch_desc(&tma_t0);
      if (NMAT == 2) tma_prefetch_desc(&tma_t1);
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
          mbar_arrive_expect_tx(&raw_full[rs], NMAT * mat_raw);
          uint8_t* dst = raw + rs * pl.raw_bytes;
          const int z = it.x * kt_rows + kc * 4;
          tma_load_3d(dst, &tma_t0, &raw_full[rs], 0, tile * 8, z);
          if (NMAT == 2) tma_load_3d(dst + mat_raw, &tma_t1, &raw_full[rs], 0, tile * 8, z);
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
      tma_prefetch_desc(&tma_b0);
      if (NMAT == 2) tma_prefetch_desc(&tma_b1);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int4 it = p.items[u / n_tiles];
        for (int kc = 0; kc < kchunks; ++kc) {
          if (!mbar_wait_or_abort(&b_empty[stage], phase ^ 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[stage], NMAT * b_bytes);
          tma_load_2d(b_tile(stage, 0), &tma_b0, &b_full[stage], kc * BK, it.y);
          if (NMAT == 2) tma_load_2d(b_tile(stage, 1), &tma_b1, &b_full[stage], kc * BK, it.y);
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
      int stage = 0, bs = 0;
      uint32_t phase = 0, bphase = 0;
      bool ok = true;
      int local = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++local) {
        const int4 it = p.items[u / n_tiles];
        const int n_pad = (it.z + 15) / 16 * 16;
        const uint32_t idesc = make_idesc_f16(128, n_pad, 0 /*f16*/);
        const int acc = local & 1;
        // the epilogue warps have read this accumulator's previous unit
        if (!mbar_wait_or_abort(&tempty[acc], ((local >> 1) & 1) ^ 1, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
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
            const uint32_t d = tmem_base + acc * acc_cols + m * tile_rows;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t da = desc_kmajor_sw128(a_tile(stage, m)) + 2 * k;
              const uint64_t db = desc_kmajor_sw128(b_tile(bs, m)) + 2 * k;
              umma_f16(d, da, db, idesc, (kc > 0 || k > 0) ? 1u : 0u);
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
        umma_commit(&tfull[acc]);
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

// ----------------------------------------------------------------------------- input rotation
// out[r, :] = fp16( H128( x[src_row(r), :] * suh ) ) for each of NMAT suh vectors (per expert), and
// sum[r] = the sum of the row's fp16 outputs (what the MMA reads): the codebook's affine step is
// applied to the accumulator in the epilogue as a * acc + b * sum.  One CTA per row, one warp per
// 128-block (4 values per lane, 2 in-register butterfly stages + 5 shuffle stages); the row sum is
// reduced over the warps in block order (deterministic).
constexpr int kRotMaxWarps = 32;
__global__ void input_rotate_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int in_features, int K,
                                    const int* __restrict__ sorted_token, const int* __restrict__ expert_offsets,
                                    int E_local, const __half* __restrict__ suh0, const __half* __restrict__ suh1,
                                    int64_t suh_estride, __half* __restrict__ out0, __half* __restrict__ out1,
                                    float* __restrict__ sum0, float* __restrict__ sum1, int rows) {
  pdl_prologue();
  __shared__ float part[2][kRotMaxWarps];
  const int r = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nwarps = blockDim.x / 32;
  const int nblk = K / 128;
  // rows past the assigned ones (expert parallel: assignments to other ranks' experts) are unused
  if (r >= rows || (expert_offsets && r >= expert_offsets[E_local])) return;
  int e = 0;
  if (expert_offsets) {  // expert of row r: binary search in offsets
    int lo = 0, hi = E_local;
    while (hi - lo > 1) {
      const int mid = (lo + hi) / 2;
      if (expert_offsets[mid] <= r) lo = mid; else hi = mid;
    }
    e = lo;
  }
  const int tok = sorted_token ? sorted_token[r] : r;
  float acc[2] = {0.f, 0.f};
  for (int blk = warp; blk < nblk; blk += nwarps) {
    const int c0 = blk * 128 + lane * 4;
    float xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + i;
      xv[i] = c < in_features ? __bfloat162float(x[(int64_t)tok * ld_x + c]) : 0.f;
    }
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const __half* suh = m == 0 ? suh0 : suh1;
      __half* out = m == 0 ? out0 : out1;
      if (suh == nullptr) break;
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = xv[i] * __half2float(suh[(int64_t)e * suh_estride + c0 + i]);
      // in-register: features 4*lane + {0,1,2,3}: distances 1, 2
      float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
      v[0] = a0 + a2;
      v[1] = a1 + a3;
      v[2] = a0 - a2;
      v[3] = a1 - a3;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float o = __shfl_xor_sync(0xffffffffu, v[i], d);
          v[i] = (lane & d) ? (o - v[i]) : (v[i] + o);
        }
      }
      __half2 h01 = __floats2half2_rn(v[0] * kH128, v[1] * kH128);
      __half2 h23 = __floats2half2_rn(v[2] * kH128, v[3] * kH128);
      const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
      acc[m] += (f01.x + f01.y) + (f23.x + f23.y);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&h01);
      pk.y = *reinterpret_cast<uint32_t*>(&h23);
      *reinterpret_cast<uint2*>(out + (int64_t)r * K + c0) = pk;
    }
  }
  if (sum0 == nullptr && sum1 == nullptr) return;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    float v = acc[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) part[m][warp] = v;
  }
  __syncthreads();
  if (threadIdx.x < 2) {
    float* sum = threadIdx.x == 0 ? sum0 : sum1;
    if (sum != nullptr) {
      float v = 0.f;
      for (int w = 0; w < nwarps; ++w) v += part[threadIdx.x][w];
      sum[r] = v;
    }
  }
}

// out[t, :] = sum_j w[t, j] * y[slot[t, j], :]  (+ add[t, :]), fp32 math, fixed j order.
// Grid (token, 256-column block), 64 threads: the token's k slots and weights are read once into
// shared memory (one round of loads), then each thread sums its 4 columns over the k rows with the k
// row loads independent of each other (no load waits on another load's result); many small blocks
// keep enough loads in flight per SM for the fp32 rows to stream at memory speed.
constexpr int kCombineMaxK = 32;
constexpr int kCombineThreads = 64;
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const float* __restrict__ y, int64_t ld_y,
                                                      const int* __restrict__ slot_of,
                                                      const float* __restrict__ sorted_weight, int k, int H,
                                                      const __nv_bfloat16* __restrict__ add,
                                                      __nv_bfloat16* __restrict__ out, int64_t ld_out,
                                                      float* __restrict__ out_f32) {
  pdl_prologue();
  __shared__ int s_slot[kCombineMaxK];
  __shared__ float s_w[kCombineMaxK];
  const int t = blockIdx.x;
  if (threadIdx.x < k) {
    const int s = slot_of[(int64_t)t * k + threadIdx.x];
    s_slot[threadIdx.x] = s;
    s_w[threadIdx.x] = s >= 0 ? sorted_weight[s] : 0.f;
  }
  __syncthreads();
  const bool vec = (ld_y % 4 == 0);
  for (int c = (blockIdx.y * blockDim.x + threadIdx.x) * 4; c < H; c += gridDim.y * blockDim.x * 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec && c + 4 <= H) {
      for (int j0 = 0; j0 < k; j0 += 8) {  // 8 independent row loads in flight, then their sums in j order
        float4 v[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int s = j0 + jj < k ? s_slot[j0 + jj] : -1;
          v[jj] = s >= 0 ? *reinterpret_cast<const float4*>(y + (int64_t)s * ld_y + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float w = j0 + jj < k ? s_w[j0 + jj] : 0.f;
          acc[0] += w * v[jj].x;
          acc[1] += w * v[jj].y;
          acc[2] += w * v[jj].z;
          acc[3] += w * v[jj].w;
        }
      }
    } else {
      for (int j = 0; j < k; ++j) {
        const int s = s_slot[j];
        if (s < 0) continue;
        for (int i = 0; i < 4 && c + i < H; ++i) acc[i] += s_w[j] * y[(int64_t)s * ld_y + c + i];
      }
    }
    for (int i = 0; i < 4 && c + i < H; ++i) {
      float a = acc[i];
      if (add) a += __bfloat162float(add[(int64_t)t * ld_out + c + i]);
      if (out_f32)
        out_f32[(int64_t)t * H + c + i] = a;
      else
        out[(int64_t)t * ld_out + c + i] = __float2bfloat16(a);
    }
  }
}

// 3-D view of a trellis [E, K/16, N/16, 8*bits_x2] int16 as uint32 tile words:
// (words of a tile, tile column, tile row over all experts); box = 4 tile rows
// x 8 tile columns = one pipeline chunk of one 128-wide output tile.
inline CUtensorMap make_trellis_map(const void* base, int E, int K, int N, int bits_x2) {
  const uint64_t words = 4ull * bits_x2;
  CUtensorMap map;
  cuuint64_t gdim[3] = {words, (cuuint64_t)(N / 16), (cuuint64_t)E * (K / 16)};
  cuuint64_t gstride[2] = {words * 4, (cuuint64_t)(N / 16) * words * 4};
  cuuint32_t box[3] = {(cuuint32_t)words, 8, 4};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(base), gdim, gstride,
                                    box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("trellis tensor map: " + std::to_string((int)r));
  return map;
}

template <int NMAT, int CB, bool FAST, int DW>
cudaError_t launch_gemm(const GemmParams& p, const void* b0, const void* b1, int64_t b_rows, int E,
                        cudaStream_t stream, int grid) {
  const Plan pl = make_plan(NMAT, p.tile_rows, p.bits_x2);
  if (pl.a_stages < 2 || pl.b_stages < 2 || pl.raw_stages < 2 || pl.a_stages > 4 || pl.b_stages > 8 ||
      pl.raw_stages > 8 || pl.smem > 227 * 1024)
    return cudaErrorInvalidValue;
  CUtensorMap m0 = make_tma_2d(b0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b_rows, p.K, p.K, p.tile_rows, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap m1 = NMAT == 2 ? make_tma_2d(b1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b_rows, p.K, p.K, p.tile_rows,
                                           BK, CU_TENSOR_MAP_SWIZZLE_128B)
                             : m0;
  CUtensorMap t0 = make_trellis_map(p.trellis[0], E, p.K, p.N, p.bits_x2);
  CUtensorMap t1 = NMAT == 2 ? make_trellis_map(p.trellis[1], E, p.K, p.N, p.bits_x2) : t0;
  auto kern = exl3_gemm_kernel<NMAT, CB, FAST, DW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  launch_pdl(kern, dim3(grid), dim3(Roles<DW>::kThreads), pl.smem, stream, m0, m1, t0, t1, p, pl);
  return cudaGetLastError();
}

// Decoder warps per CTA: VLLM_B200_EXL3_DECODERS when set -- "8" or "16" for both passes, or "G,D" for the
// gate/up pass (two matrices) and the down pass (one) apart -- else the pass's default.
struct DecoderChoice {
  int down = 0, gate_up = 0;
  DecoderChoice() {
    const char* v = std::getenv("VLLM_B200_EXL3_DECODERS");
    if (v == nullptr) return;
    int g = 0, d = 0;
    if (std::sscanf(v, "%d,%d", &g, &d) == 2) {
      gate_up = g;
      down = d;
    } else {
      gate_up = down = std::atoi(v);
    }
  }
};

inline int decoder_warps(int nmat) {
  static const DecoderChoice choice;  // read once per process
  const int w = nmat == 2 ? choice.gate_up : choice.down;
  if (w == 8 || w == 16) return w;
  return 16;
}

template <int NMAT>
cudaError_t dispatch(const GemmParams& p, const void* b0, const void* b1, int64_t b_rows, int E, cudaStream_t s,
                     int grid) {
  const bool fast = p.bits_x2 == 8;
  if (fast && decoder_warps(NMAT) == 8) {
    return p.codebook == 1 ? launch_gemm<NMAT, 1, true, 8>(p, b0, b1, b_rows, E, s, grid)
                           : launch_gemm<NMAT, 2, true, 8>(p, b0, b1, b_rows, E, s, grid);
  }
  if (p.codebook == 1) {
    return fast ? launch_gemm<NMAT, 1, true, 16>(p, b0, b1, b_rows, E, s, grid)
                : launch_gemm<NMAT, 1, false, 16>(p, b0, b1, b_rows, E, s, grid);
  }
  return fast ? launch_gemm<NMAT, 2, true, 16>(p, b0, b1, b_rows, E, s, grid)
              : launch_gemm<NMAT, 2, false, 16>(p, b0, b1, b_rows, E, s, grid);
}

}  // namespace exl3

cudaError_t exl3_input_rotate(const void* x, int64_t ld_x, int in_features, int K, const int* sorted_token,
                              const int* expert_offsets, int E_local, const void* suh0, const void* suh1,
                              int64_t suh_estride, void* out0, void* out1, float* sum0, float* sum1, int rows,
                              cudaStream_t stream) {
  if (K % 128) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int threads = 32 * std::min(K / 128, exl3::kRotMaxWarps);
  launch_pdl(exl3::input_rotate_kernel, dim3(rows), dim3(threads), 0, stream,
             reinterpret_cast<const __nv_bfloat16*>(x), ld_x, in_features, K, sorted_token, expert_offsets, E_local,
             reinterpret_cast<const __half*>(suh0), reinterpret_cast<const __half*>(suh1), suh_estride,
             reinterpret_cast<__half*>(out0), reinterpret_cast<__half*>(out1), sum0, sum1, rows);
  return cudaGetLastError();
}

cudaError_t exl3_gemm(const Exl3GemmArgs& a, cudaStream_t stream) {
  using namespace exl3;
  if (a.K % 128 || a.N % 128 || a.tile_rows % 16 || a.tile_rows < 16 || a.tile_rows > 256) return cudaErrorInvalidValue;
  if (a.nmat == 2 && a.tile_rows > 128) return cudaErrorInvalidValue;
  if (a.bits_x2 < 2 || a.bits_x2 > 16) return cudaErrorInvalidValue;
  GemmParams p{};
  for (int m = 0; m < a.nmat; ++m) {
    p.trellis[m] = reinterpret_cast<const uint16_t*>(a.trellis[m]);
    p.trellis_estride[m] = a.trellis_estride;
    p.svh[m] = reinterpret_cast<const __half*>(a.svh[m]);
    p.svh_estride[m] = a.svh_estride;
  }
  p.suh_next = reinterpret_cast<const __half*>(a.suh_next);
  p.suh_next_estride = a.suh_next_estride;
  p.K = a.K;
  p.N = a.N;
  p.bits_x2 = a.bits_x2;
  p.codebook = a.codebook;
  p.tile_rows = a.tile_rows;
  p.items = reinterpret_cast<const int4*>(a.items);
  p.num_items = a.num_items;
  p.out = a.out;
  p.ld_out = a.ld_out;
  p.out_mode = a.out_mode;
  p.swiglu_limit = a.swiglu_limit;
  p.sx[0] = a.sx0;
  p.sx[1] = a.sx1;
  p.sx_parts = a.sx_parts;
  p.hsum = a.hsum;
  p.status = a.status;
  // codebook 2 folds its affine step into the epilogue: it needs the activation row sums
  if (a.codebook == 2 && (a.sx0 == nullptr || (a.nmat == 2 && a.sx1 == nullptr) || a.sx_parts < 1))
    return cudaErrorInvalidValue;
  const int grid = std::max(1, std::min(a.max_work, device_sm_count()));
  if (a.nmat == 2) return dispatch<2>(p, a.b0, a.b1, a.b_rows, a.num_experts, stream, grid);
  return dispatch<1>(p, a.b0, nullptr, a.b_rows, a.num_experts, stream, grid);
}

cudaError_t moe_combine(const float* y, int64_t ld_y, const int* slot_of, const float* sorted_weight, int T, int k,
                        int H, const void* add, void* out, int64_t ld_out, float* out_f32, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (k > exl3::kCombineMaxK) return cudaErrorInvalidValue;
  const int cblocks = (H + 4 * exl3::kCombineThreads - 1) / (4 * exl3::kCombineThreads);
  launch_pdl(exl3::combine_kernel, dim3(T, cblocks), dim3(exl3::kCombineThreads), 0, stream, y, ld_y, slot_of,
             sorted_weight, k, H,
                                              reinterpret_cast<const __nv_bfloat16*>(add),
                                              reinterpret_cast<__nv_bfloat16*>(out), ld_out, out_f32);
  return cudaGetLastError();
}

}  // namespace b200

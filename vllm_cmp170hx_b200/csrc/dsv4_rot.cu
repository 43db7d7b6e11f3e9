// DeepSeek-V4.1 row transforms: an optional RMSNorm, the RoPE turn of the row's tail and a quantise-
// dequantise onto the FP8 / FP4 grids, in one pass (one CTA per row, one thread per element).
//
// The definitions (the oracle's statement of the model's rounding contract, the reference's
// models/deepseek_v41/ops/sm80_attn_core.py rotate / act_quant):
//   * RMSNorm: x * 1 / sqrt(mean(x^2) + eps) * w in fp32, rounded to bf16;
//   * turn: dims (2i, 2i + 1) of the last 2n dims rotate by the fp32 angle pos * freq_i, with the fp32
//     cos / sin of that angle, the rotation evaluated in fp64 and rounded once to bf16 (inverse: -sin);
//   * FP8 qdq (mode 1): per 32 values s = 2^ceil(log2(max(amax, 1e-4) / 448)), v = e4m3(v / s) * s;
//     FP4 qdq with E4M3 scales (mode 2): per 16, s = e4m3(max(amax, 6 * 2^-9) / 6),
//     v = e2m1(clamp(v / s, -6, 6)) * s; FP4 with power-of-two scales (mode 3): per 32,
//     s = 2^ceil(log2(max(amax, 6 * 2^-126) / 6)); results rounded to bf16.
// E2M1 rounds to the nearest of {0, .5, 1, 1.5, 2, 3, 4, 6}, ties to the even code.
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace dsv4rot {

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// 2^ceil(log2 a) for positive normal a, from frexp (a = m 2^e, m in [0.5, 1); a power of two when m == 0.5)
__device__ __forceinline__ float pow2_ceil(float a) {
  int e;
  const float m = frexpf(a, &e);
  return ldexpf(1.f, m == 0.5f ? e - 1 : e);
}

__device__ __forceinline__ float e4m3_round(float v) {
  const __nv_fp8_e4m3 q(fminf(fmaxf(v, -448.f), 448.f));
  return float(q);
}

__device__ __forceinline__ float e2m1_round(float v) {
  const float a = fabsf(v);
  // steps between neighbouring magnitudes; a threshold itself goes to the even code
  float m = 0.f;
  m += (a > 0.25f) ? 0.5f : 0.f;
  m += (a >= 0.75f) ? 0.5f : 0.f;
  m += (a > 1.25f) ? 0.5f : 0.f;
  m += (a >= 1.75f) ? 0.5f : 0.f;
  m += (a > 2.5f) ? 1.f : 0.f;
  m += (a >= 3.5f) ? 1.f : 0.f;
  m += (a > 5.f) ? 2.f : 0.f;
  return v < 0.f ? -m : m;
}

__global__ void rot_qdq_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, __nv_bfloat16* __restrict__ out,
                               int64_t ld_out, int D, const int64_t* __restrict__ positions, int heads,
                               const float* __restrict__ freqs, int n_pairs, int inverse,
                               const __nv_bfloat16* __restrict__ norm_w, float eps, int mode) {
  pdl_prologue();
  __shared__ float red[16];
  const int row = blockIdx.x, i = threadIdx.x;
  const int warp = i / 32, lane = i % 32;
  float v = __bfloat162float(x[(int64_t)row * ld_x + i]);
  if (norm_w != nullptr) {
    float ss = warp_sum(v * v);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (D + 31) / 32; ++w) tot += red[w];
    const float inv = 1.f / sqrtf(tot / (float)D + eps);
    v = bf16_round(v * inv * __bfloat162float(norm_w[i]));
  }
  const int tail0 = D - 2 * n_pairs;
  if (n_pairs > 0) {
    const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
    if (i >= tail0) {
      const int p = (i - tail0) >> 1;
      const bool re_lane = ((i - tail0) & 1) == 0;
      const float ang = (float)positions[row / heads] * freqs[p];  // the fp32 product
      const double c = (double)(float)cos((double)ang);
      double s = (double)(float)sin((double)ang);
      if (inverse) s = -s;
      const double re = re_lane ? (double)v : (double)partner;
      const double im = re_lane ? (double)partner : (double)v;
      const double r = re_lane ? __dsub_rn(__dmul_rn(re, c), __dmul_rn(im, s))
                               : __dadd_rn(__dmul_rn(re, s), __dmul_rn(im, c));
      v = __bfloat162float(__double2bfloat16(r));
    }
  }
  if (mode != 0) {
    const int B = mode == 2 ? 16 : 32;
    float amax = fabsf(v);
    for (int o = B / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float s;
    if (mode == 1) {
      s = pow2_ceil(fmaxf(amax, 1e-4f) * (1.f / 448.f));
      v = e4m3_round(v / s) * s;
    } else if (mode == 2) {
      s = e4m3_round(fmaxf(amax, 6.f * 0.001953125f) / 6.f);
      v = e2m1_round(fminf(fmaxf(v / s, -6.f), 6.f)) * s;
    } else {
      s = pow2_ceil(fmaxf(amax, 6.f * 1.1754944e-38f) * (1.f / 6.f));
      v = e2m1_round(fminf(fmaxf(v / s, -6.f), 6.f)) * s;
    }
  }
  out[(int64_t)row * ld_out + i] = __float2bfloat16_rn(v);
}

}  // namespace dsv4rot

cudaError_t dsv4_rot_qdq(const void* x, int64_t ld_x, void* out, int64_t ld_out, int rows, int D,
                         const int64_t* positions, int heads, const float* freqs, int n_pairs, int inverse,
                         const void* norm_w, float eps, int mode, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (D % 32 || D > 512 || 2 * n_pairs > D || mode < 0 || mode > 3 || heads < 1) return cudaErrorInvalidValue;
  launch_pdl(dsv4rot::rot_qdq_kernel, dim3(rows), dim3(D), 0, stream, reinterpret_cast<const __nv_bfloat16*>(x),
             ld_x, reinterpret_cast<__nv_bfloat16*>(out), ld_out, D, positions, heads, freqs, n_pairs, inverse,
             reinterpret_cast<const __nv_bfloat16*>(norm_w), eps, mode);
  return cudaGetLastError();
}

}  // namespace b200

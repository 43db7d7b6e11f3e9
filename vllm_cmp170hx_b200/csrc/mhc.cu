// Manifold-constrained hyper-connections (mHC): one fused kernel per sublayer boundary.
//
// One CTA per token.  With the residual widened to HC streams H [T, HC, d] (bf16):
//   1. post of the previous sublayer output x (skipped without x):
//        H'_k = bf16(post_k x + sum_j comb[j][k] H_j), written over H and kept in shared memory;
//   2. coefficients of H': N = 2 HC + HC^2 dot products of the flattened streams (HC d values,
//      promoted to fp32) with the rows of fn, scaled by rsqrt(mean square + rms_eps); then
//      pre = sigmoid(.) + eps, post = post_mult sigmoid(.), comb = row softmax + eps, column
//      normalisation and iters - 1 Sinkhorn row/column passes (one thread: HC^2 <= 64 values);
//   3. the next sublayer's input: RMSNorm(bf16(sum_k mix_k H'_k)) with mix = the fresh pre, the
//      carried pre of the previous boundary (delayed form), or stream 0.
// The reference runs this contract as Triton / TileLang kernels (vllm_sm80/kernels/mhc/decode.py:865,
// vllm_sm80/models/deepseek_v41/ops/sm80_mhc_fused.py); the formulas here follow the fp32 oracle
// in oracle/mhc.py.  fn (N x HC d fp32) is read once per token from L2.
#include <cfloat>

#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace mhc {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

template <int HC>
__global__ void __launch_bounds__(kThreads) post_pre_kernel(MhcArgs a) {
  pdl_prologue();
  constexpr int N = 2 * HC + HC * HC;
  extern __shared__ uint8_t smem_raw[];
  const int d = a.d;
  const int nd = HC * d;
  __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(smem_raw);          // [HC][d] H'
  __nv_bfloat16* cs = hs + nd;                                             // [d] collapsed input
  float* red = reinterpret_cast<float*>(cs + ((d + 7) / 8) * 8);           // [kWarps][N + 1]
  float* coef = red + kWarps * (N + 1);                                    // pre[HC] post[HC] comb[HC*HC] mix[HC] misc
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const __nv_bfloat16* H = a.H + (int64_t)t * nd;
  __nv_bfloat16* Ho = a.H_out + (int64_t)t * nd;

  // ---------------------------------------------------------------- 1. post
  if (a.x != nullptr && tid < HC * HC + HC) {
    // stage this token's post / comb in shared memory
    coef[tid] = tid < HC ? a.post[(int64_t)t * HC + tid] : a.comb[(int64_t)t * HC * HC + tid - HC];
  }
  __syncthreads();
  for (int i = tid; i < d; i += kThreads) {
    float h[HC];
#pragma unroll
    for (int j = 0; j < HC; ++j) h[j] = __bfloat162float(H[j * d + i]);
    if (a.x != nullptr) {
      const float xv = __bfloat162float(a.x[(int64_t)t * d + i]);
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < HC; ++j) v += coef[HC + j * HC + k] * h[j];
        const __nv_bfloat16 o = __float2bfloat16(coef[k] * xv + v);
        hs[k * d + i] = o;
        Ho[k * d + i] = o;
      }
    } else {
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        const __nv_bfloat16 o = __float2bfloat16(h[k]);
        hs[k * d + i] = o;
        if (Ho != H) Ho[k * d + i] = o;
      }
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- 2. coefficients
  float acc[N + 1];
#pragma unroll
  for (int r = 0; r <= N; ++r) acc[r] = 0.f;
  for (int e = tid; e < nd; e += kThreads) {
    const float v = __bfloat162float(hs[e]);
    acc[N] += v * v;
#pragma unroll
    for (int r = 0; r < N; ++r) acc[r] += v * a.fn[(int64_t)r * nd + e];
  }
#pragma unroll
  for (int r = 0; r <= N; ++r) {
    float v = acc[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * (N + 1) + r] = v;
  }
  __syncthreads();
  if (tid == 0) {
    float m[N + 1];
#pragma unroll
    for (int r = 0; r <= N; ++r) {
      float v = 0.f;
      for (int w = 0; w < kWarps; ++w) v += red[w * (N + 1) + r];  // fixed order: deterministic
      m[r] = v;
    }
    const float rs = rsqrtf(m[N] / (float)nd + a.rms_eps);
    const float s0 = a.scale[0], s1 = a.scale[1], s2 = a.scale[2];
    float pre[HC], post[HC], c[HC][HC];
#pragma unroll
    for (int k = 0; k < HC; ++k) {
      pre[k] = 1.f / (1.f + __expf(-(m[k] * rs * s0 + a.base[k]))) + a.eps;
      post[k] = a.post_mult / (1.f + __expf(-(m[HC + k] * rs * s1 + a.base[HC + k])));
    }
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      float mx = -FLT_MAX;
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        c[j][k] = m[2 * HC + j * HC + k] * rs * s2 + a.base[2 * HC + j * HC + k];
        mx = fmaxf(mx, c[j][k]);
      }
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        c[j][k] = __expf(c[j][k] - mx);
        s += c[j][k];
      }
#pragma unroll
      for (int k = 0; k < HC; ++k) c[j][k] = c[j][k] / s + a.eps;
    }
    auto col_norm = [&]() {
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < HC; ++j) s += c[j][k];
        const float inv = 1.f / (s + a.eps);
#pragma unroll
        for (int j = 0; j < HC; ++j) c[j][k] *= inv;
      }
    };
    col_norm();
    for (int it = 1; it < a.iters; ++it) {
#pragma unroll
      for (int j = 0; j < HC; ++j) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < HC; ++k) s += c[j][k];
        const float inv = 1.f / (s + a.eps);
#pragma unroll
        for (int k = 0; k < HC; ++k) c[j][k] *= inv;
      }
      col_norm();
    }
#pragma unroll
    for (int k = 0; k < HC; ++k) {
      a.pre_out[(int64_t)t * HC + k] = pre[k];
      a.post_out[(int64_t)t * HC + k] = post[k];
#pragma unroll
      for (int j = 0; j < HC; ++j) a.comb_out[((int64_t)t * HC + j) * HC + k] = c[j][k];
      // collapse weights: the fresh pre, the carried pre (delayed), or stream 0
      coef[k] = a.mode == 0 ? pre[k] : a.mode == 1 ? a.pre_mix[(int64_t)t * HC + k] : (k == 0 ? 1.f : 0.f);
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- 3. collapse + RMSNorm
  float ss = 0.f;
  for (int i = tid; i < d; i += kThreads) {
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < HC; ++k) v += coef[k] * __bfloat162float(hs[k * d + i]);
    const __nv_bfloat16 cb = __float2bfloat16(v);
    cs[i] = cb;
    const float cf = __bfloat162float(cb);
    ss += cf * cf;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (tid == 0) {
    float v = 0.f;
    for (int w = 0; w < kWarps; ++w) v += red[w];
    coef[HC] = rsqrtf(v / (float)d + a.norm_eps);
  }
  __syncthreads();
  const float r = coef[HC];
  for (int i = tid; i < d; i += kThreads)
    a.y[(int64_t)t * d + i] = __float2bfloat16(__bfloat162float(a.norm_w[i]) * (__bfloat162float(cs[i]) * r));
}

}  // namespace mhc

cudaError_t mhc_post_pre(const MhcArgs& a, cudaStream_t stream) {
  using namespace mhc;
  if (a.T == 0) return cudaSuccess;
  const int N = 2 * a.hc + a.hc * a.hc;
  const size_t smem = (size_t)a.hc * a.d * 2 + ((a.d + 7) / 8) * 8 * 2 + (size_t)kWarps * (N + 1) * 4 +
                      (size_t)(N + 2 * a.hc + 8) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  switch (a.hc) {
#define B200_MHC_CASE(HC)                                                                                      \
  case HC: {                                                                                                  \
    cudaError_t e = cudaFuncSetAttribute(post_pre_kernel<HC>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         (int)smem);                                                        \
    if (e != cudaSuccess) return e;                                                                          \
    launch_pdl(post_pre_kernel<HC>, dim3(a.T), dim3(kThreads), smem, stream, a);                                                 \
    break;                                                                                                    \
  }
    B200_MHC_CASE(2)
    B200_MHC_CASE(4)
    B200_MHC_CASE(8)
#undef B200_MHC_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace b200

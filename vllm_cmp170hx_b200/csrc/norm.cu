// RMSNorm family (the upstream RMSNorm custom op the reference's models call,
// vllm_sm80/models/glm5next/sm80_model.py:264 path; fused residual add as in
// vLLM's fused_add_rms_norm).
//
// One CTA of 256 threads per row, 16-byte vector loads, the row held in
// registers between the reduction and the scaled store, fp32 accumulation.
// Rows may be strided (e.g. the first 512 columns of a [T, 576] latent).
#include "common.cuh"
#include <algorithm>

#include "launch.h"

namespace b200 {
namespace {

constexpr int kNormThreads = 256;
constexpr int kMaxVec = 8;  // rows up to 256 threads * 8 vectors * 8 elems = 16384

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = (l < blockDim.x / 32) ? red[l] : 0.f;
  s = warp_sum(s);
  __syncthreads();
  return s;
}

// mode 0: out = norm(x) * w
// mode 1: r = x + residual; residual = r; out(x) = norm(r) * w   (in place on x)
template <int MODE>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(__nv_bfloat16* out, int ld_out,
                                                                const __nv_bfloat16* x, int ld_x,
                                                                __nv_bfloat16* __restrict__ residual, int ld_res,
                                                                const __nv_bfloat16* __restrict__ w, int H,
                                                                float eps) {
  pdl_prologue();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  const __nv_bfloat16* xr = x + (size_t)row * ld_x;
  float vals[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      uint4 raw = reinterpret_cast<const uint4*>(xr)[v];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
      if (MODE == 1) {
        __nv_bfloat16* rr = residual + (size_t)row * ld_res;
        uint4 rraw = reinterpret_cast<const uint4*>(rr)[v];
        const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rraw);
        uint4 outv;
        __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&outv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          oe[j] = __float2bfloat16(__bfloat162float(e[j]) + __bfloat162float(re[j]));
          vals[i][j] = __bfloat162float(oe[j]);
        }
        reinterpret_cast<uint4*>(rr)[v] = outv;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) vals[i][j] = __bfloat162float(e[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  __nv_bfloat16* orow = out + (size_t)row * ld_out;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nvec) {
      uint4 wraw = reinterpret_cast<const uint4*>(w)[v];
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wraw);
      uint4 o;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(vals[i][j] * inv * __bfloat162float(we[j]));
      reinterpret_cast<uint4*>(orow)[v] = o;
    }
  }
}

__global__ void silu_mul_kernel(__nv_bfloat16* __restrict__ out, int64_t ld_out, const __nv_bfloat16* __restrict__ x,
                                int64_t ld_x, int T, int I, float limit) {
  pdl_prologue();
  const int64_t total = (int64_t)T * (I / 2);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = i / (I / 2);
    const int c = (i % (I / 2)) * 2;
    const __nv_bfloat162 g2 = *reinterpret_cast<const __nv_bfloat162*>(x + t * ld_x + c);
    const __nv_bfloat162 u2 = *reinterpret_cast<const __nv_bfloat162*>(x + t * ld_x + I + c);
    float g0 = __bfloat162float(g2.x), g1 = __bfloat162float(g2.y);
    float u0 = __bfloat162float(u2.x), u1 = __bfloat162float(u2.y);
    if (limit > 0.f) {
      g0 = fminf(g0, limit);
      g1 = fminf(g1, limit);
      u0 = fminf(fmaxf(u0, -limit), limit);
      u1 = fminf(fmaxf(u1, -limit), limit);
    }
    *reinterpret_cast<__nv_bfloat162*>(out + t * ld_out + c) = __floats2bfloat162_rn(siluf_(g0) * u0, siluf_(g1) * u1);
  }
}

}  // namespace

cudaError_t silu_mul(void* out, int64_t ld_out, const void* x, int64_t ld_x, int T, int I, float limit,
                     cudaStream_t stream) {
  if (I % 2 || ld_x % 2 || ld_out % 2) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  const int64_t total = (int64_t)T * (I / 2);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, stream, reinterpret_cast<__nv_bfloat16*>(out), ld_out,
                                              reinterpret_cast<const __nv_bfloat16*>(x), ld_x, T, I, limit);
  return cudaGetLastError();
}

cudaError_t rms_norm(void* out, int64_t ld_out, const void* x, int64_t ld_x, const void* w, int T, int H, float eps,
                     cudaStream_t stream) {
  if (H % 8 != 0 || H > kNormThreads * kMaxVec * 8 || ld_x % 8 != 0 || ld_out % 8 != 0) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  launch_pdl(rms_norm_kernel<0>, dim3(T), dim3(kNormThreads), 0, stream, 
      reinterpret_cast<__nv_bfloat16*>(out), (int)ld_out, reinterpret_cast<const __nv_bfloat16*>(x), (int)ld_x,
      nullptr, 0, reinterpret_cast<const __nv_bfloat16*>(w), H, eps);
  return cudaGetLastError();
}

cudaError_t fused_add_rms_norm(void* x, int64_t ld_x, void* residual, int64_t ld_res, const void* w, int T, int H,
                               float eps, cudaStream_t stream) {
  if (H % 8 != 0 || H > kNormThreads * kMaxVec * 8 || ld_x % 8 != 0 || ld_res % 8 != 0) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  launch_pdl(rms_norm_kernel<1>, dim3(T), dim3(kNormThreads), 0, stream, 
      reinterpret_cast<__nv_bfloat16*>(x), (int)ld_x, reinterpret_cast<const __nv_bfloat16*>(x), (int)ld_x,
      reinterpret_cast<__nv_bfloat16*>(residual), (int)ld_res, reinterpret_cast<const __nv_bfloat16*>(w), H, eps);
  return cudaGetLastError();
}

}  // namespace b200

// Engram gate of the DeepSeek-V4.1-style model: the context-aware gate that mixes a token's n-gram
// memory rows into its hidden state.
//
// For token t with the layer's normalised input h_t and the memory projections k_t, v_t (one GEMM of the
// token's retrieved rows):
//   alpha_t = sigmoid( <rmsnorm(h_t) * w_h, rmsnorm(k_t) * w_k> / sqrt(H) )
//   out_t  += alpha_t * v_t
// (the reference's Engram embedding, vllm_sm80/models/deepseek_v41/sm80_engram.py:879, feeds the upstream
// gated memory block it subclasses; this is that block's gate).  The dot product of the two normalised
// vectors is formed from three sums of one pass, sum h^2, sum k^2 and sum h k w_h w_k, so a token's
// vectors are read once for the gate and v once for the update.  A NaN row (a failed storage read)
// makes alpha and the update NaN for that token only.
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace engram {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) engram_gate_kernel(const __nv_bfloat16* __restrict__ h, int64_t ld_h,
                                                                 const __nv_bfloat16* __restrict__ kv, int64_t ld_kv,
                                                                 const __nv_bfloat16* __restrict__ wh,
                                                                 const __nv_bfloat16* __restrict__ wk, float eps,
                                                                 int H, __nv_bfloat16* __restrict__ out,
                                                                 int64_t ld_out) {
  pdl_prologue();
  __shared__ float red[3][kThreads / 32];
  const int t = blockIdx.x;
  const __nv_bfloat16* ht = h + (int64_t)t * ld_h;
  const __nv_bfloat16* kt = kv + (int64_t)t * ld_kv;
  const __nv_bfloat16* vt = kt + H;
  float shh = 0.f, skk = 0.f, shk = 0.f;
  for (int c = threadIdx.x * 8; c < H; c += kThreads * 8) {
    const uint4 hv = *reinterpret_cast<const uint4*>(ht + c);
    const uint4 kv4 = *reinterpret_cast<const uint4*>(kt + c);
    const uint4 w1 = *reinterpret_cast<const uint4*>(wh + c);
    const uint4 w2 = *reinterpret_cast<const uint4*>(wk + c);
    const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&hv);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&kv4);
    const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&w1);
    const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&w2);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 af = __bfloat1622float2(a[i]), bf = __bfloat1622float2(b[i]);
      const float2 xf = __bfloat1622float2(x[i]), yf = __bfloat1622float2(y[i]);
      shh = fmaf(af.x, af.x, fmaf(af.y, af.y, shh));
      skk = fmaf(bf.x, bf.x, fmaf(bf.y, bf.y, skk));
      shk = fmaf(af.x * xf.x, bf.x * yf.x, fmaf(af.y * xf.y, bf.y * yf.y, shk));
    }
  }
  shh = warp_sum(shh);
  skk = warp_sum(skk);
  shk = warp_sum(shk);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    red[0][warp] = shh;
    red[1][warp] = skk;
    red[2][warp] = shk;
  }
  __syncthreads();
  shh = skk = shk = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) {
    shh += red[0][i];
    skk += red[1][i];
    shk += red[2][i];
  }
  const float dot = shk * rsqrtf(shh / H + eps) * rsqrtf(skk / H + eps);
  const float alpha = sigmoidf_(dot * rsqrtf((float)H));
  __nv_bfloat16* ot = out + (int64_t)t * ld_out;
  for (int c = threadIdx.x * 8; c < H; c += kThreads * 8) {
    const uint4 vv = *reinterpret_cast<const uint4*>(vt + c);
    uint4 ov = *reinterpret_cast<const uint4*>(ot + c);
    const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vv);
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 vf = __bfloat1622float2(v2[i]), of = __bfloat1622float2(o2[i]);
      o2[i] = __floats2bfloat162_rn(fmaf(alpha, vf.x, of.x), fmaf(alpha, vf.y, of.y));
    }
    *reinterpret_cast<uint4*>(ot + c) = ov;
  }
}

}  // namespace engram

cudaError_t engram_gate(const void* h, int64_t ld_h, const void* kv, int64_t ld_kv, const void* wh, const void* wk,
                        float eps, int T, int H, void* out, int64_t ld_out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (H % 8 || ld_h % 8 || ld_kv % 8 || ld_out % 8) return cudaErrorInvalidValue;
  launch_pdl(engram::engram_gate_kernel, dim3(T), dim3(engram::kThreads), 0, stream,
             reinterpret_cast<const __nv_bfloat16*>(h), ld_h, reinterpret_cast<const __nv_bfloat16*>(kv), ld_kv,
             reinterpret_cast<const __nv_bfloat16*>(wh), reinterpret_cast<const __nv_bfloat16*>(wk), eps, H,
             reinterpret_cast<__nv_bfloat16*>(out), ld_out);
  return cudaGetLastError();
}

}  // namespace b200

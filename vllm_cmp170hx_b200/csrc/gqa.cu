// Gated grouped-query attention (the full-attention layers of the Qwen3-Next-style linear/full
// hybrid): the per-head prep before the attention and the output gate after it.
//
// Layer semantics (Qwen3-Next gated attention; the reference serves it through the upstream
// Qwen4Exp model it subclasses, vllm_sm80/models/qwen4_exp/sm80_model.py:1-60): per query head
// q_proj gives [q | gate] (head_dim each); q and k get a per-head RMSNorm and NeoX RoPE on their
// first rot_dim dims; o = softmax(q k^T / sqrt(head_dim)) v over the causal prefix, then
// o * sigmoid(gate) -> o_proj.
//
// B200 layout: the attention itself runs on the block-sparse tcgen05 attention kernel in its dense
// causal mode (mla_attn.cu, `gqa_dense_attention`): a paged cache row is [K (256) | V (256)] of one
// key-value head, a query row is [q (256) | 0 (256)], so Q K^T over the 512-wide row is q.k and the
// upper half of P [K | V] is P V; only that half's CTAs run.  The query rows of one key-value head
// (its `group` query heads) share one CTA's 128-row tile.  This file holds the two kernels around it:
//
//   gqa_prep_kernel   one CTA per (token, head row): RMSNorm + RoPE of q into the padded query rows,
//                     of k (with v alongside) into the token's cache row;
//   gqa_gate_kernel   o * sigmoid(gate) from the attention's value half into the o_proj input.
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace gqa {

constexpr int HD = 256;  // head dim (the [K | V] rows are 512 wide)
constexpr int kThreads = HD;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) s += red[i];
  __syncthreads();
  return s;
}

// proj [T, ld_proj]: nh query heads x [q | gate] (512 each), then nkv x k (256), then nkv x v (256).
// Head row y < nh: query head y = j * group + g -> q_out row (t * nkv + j) * group + g, [q' | 0].
// Head row y >= nh: key-value head j = y - nh -> cache row slot[t] * nkv + j, [k' | v] (slot < 0: none).
__global__ void __launch_bounds__(kThreads) gqa_prep_kernel(GqaPrepArgs a) {
  pdl_prologue();
  __shared__ float xs[HD];
  __shared__ float red[kThreads / 32];
  const int t = blockIdx.x, y = blockIdx.y, c = threadIdx.x;
  const bool is_q = y < a.nh;
  const int j = is_q ? y / a.group : y - a.nh;
  const __nv_bfloat16* row = a.proj + (int64_t)t * a.ld_proj;
  int64_t slot = -1;
  if (!is_q) {
    slot = a.slots[t];
    if (slot < 0) return;  // a padding token: no cache row
  }
  const float x = __bfloat162float(is_q ? row[(int64_t)y * 2 * HD + c] : row[(int64_t)a.nh * 2 * HD + j * HD + c]);
  const float ss = block_sum(x * x, red);
  const __nv_bfloat16* w = is_q ? a.q_norm_w : a.k_norm_w;
  // the normalised value is rounded to bf16 before the rotation (the projection's output precision)
  xs[c] = __bfloat162float(__float2bfloat16(x * rsqrtf(ss / HD + a.eps) * __bfloat162float(w[c])));
  __syncthreads();
  float v = xs[c];
  const int half = a.rot_dim / 2;
  if (c < a.rot_dim) {
    const float* cs = a.cos_sin + (int64_t)a.positions[t] * a.rot_dim;
    const int i = c < half ? c : c - half;
    const float co = cs[i], si = cs[half + i];
    v = c < half ? xs[c] * co - xs[c + half] * si : xs[c] * co + xs[c - half] * si;
  }
  if (is_q) {
    __nv_bfloat16* q = a.q_out + (((int64_t)t * a.nkv + j) * a.group + (y - j * a.group)) * 2 * HD;
    q[c] = __float2bfloat16(v);
    q[HD + c] = __float2bfloat16(0.f);
  } else {
    __nv_bfloat16* r = a.cache + (slot * a.nkv + j) * 2 * HD;
    r[c] = __float2bfloat16(v);
    r[HD + c] = row[(int64_t)a.nh * 2 * HD + (int64_t)a.nkv * HD + j * HD + c];
  }
}

// out [T, nh * 256] = o * sigmoid(gate): o the value half of the attention output rows
// [(t * nkv + j) * group + g, 512], gate the second half of query head (j * group + g)'s projection.
// One thread per 8 channels (16-byte loads and stores).
__global__ void gqa_gate_kernel(const __nv_bfloat16* __restrict__ attn, const __nv_bfloat16* __restrict__ proj,
                                int64_t ld_proj, int T, int nh, __nv_bfloat16* __restrict__ out, int64_t ld_out) {
  pdl_prologue();
  const int per_tok = nh * HD / 8;
  const int64_t total = (int64_t)T * per_tok;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = i / per_tok;
    const int r = i % per_tok;
    const int h = r / (HD / 8), c8 = (r % (HD / 8)) * 8;
    // attention rows follow query heads in order: row t * nh + h (heads grouped by key-value head)
    const uint4 ov = *reinterpret_cast<const uint4*>(attn + ((int64_t)t * nh + h) * 2 * HD + HD + c8);
    const uint4 gv = *reinterpret_cast<const uint4*>(proj + (int64_t)t * ld_proj + (int64_t)h * 2 * HD + HD + c8);
    const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
    uint4 res;
    __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&res);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 o = __bfloat1622float2(o2[k]), g = __bfloat1622float2(g2[k]);
      r2[k] = __floats2bfloat162_rn(o.x * sigmoidf_(g.x), o.y * sigmoidf_(g.y));
    }
    *reinterpret_cast<uint4*>(out + (int64_t)t * ld_out + (int64_t)h * HD + c8) = res;
  }
}

}  // namespace gqa

cudaError_t gqa_prep(const GqaPrepArgs& a, int T, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (a.rot_dim < 0 || a.rot_dim > gqa::HD || a.rot_dim % 2 || a.group < 1 || a.nh != a.nkv * a.group)
    return cudaErrorInvalidValue;
  launch_pdl(gqa::gqa_prep_kernel, dim3(T, a.nh + a.nkv), dim3(gqa::kThreads), 0, stream, a);
  return cudaGetLastError();
}

cudaError_t gqa_gate(const void* attn, const void* proj, int64_t ld_proj, int T, int nh, void* out, int64_t ld_out,
                     cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (ld_proj % 8 || ld_out % 8) return cudaErrorInvalidValue;
  const int64_t work = (int64_t)T * nh * gqa::HD / 8;
  const int grid = (int)std::min<int64_t>((work + 255) / 256, 4 * (int64_t)device_sm_count());
  launch_pdl(gqa::gqa_gate_kernel, dim3(grid), dim3(256), 0, stream,
             reinterpret_cast<const __nv_bfloat16*>(attn), reinterpret_cast<const __nv_bfloat16*>(proj), ld_proj,
             T, nh, reinterpret_cast<__nv_bfloat16*>(out), ld_out);
  return cudaGetLastError();
}

}  // namespace b200

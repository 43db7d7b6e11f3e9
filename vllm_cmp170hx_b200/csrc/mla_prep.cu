// Sparse-MLA glue kernels: RoPE, latent KV-cache write, indexer key/query
// preparation and the canonical top-k selection.
//
// Reference behaviour: the DeepSeek-style sparse attention of
// vllm_sm80/models/deepseek_v41/ops/sm80_attn_core.py (RMSNorm + RoPE of the
// latent, indexer keys with LayerNorm + RoPE + Hadamard + fp8, top-k with
// "lowest index wins ties, selection sorted ascending", lines 17-33) and the
// GLM indexer glue (vllm_sm80/models/glm5next/ops/idx_glue.py: FWHT128 + fp8
// quant with weight scale, latent-cache write merged into the index path).
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace mla {

constexpr float kH128 = 0.08838834764831845f;
constexpr float kFp8Max = 448.f;

// rotary pair (x1, x2) -> (x1 c - x2 s, x2 c + x1 s)
__device__ __forceinline__ void rot(float& a, float& b, float c, float s) {
  const float x1 = a, x2 = b;
  a = x1 * c - x2 * s;
  b = x2 * c + x1 * s;
}

// RoPE on rot_dim dims at `offset` of every head of every token, in place or (y != null) into dims
// y_offset.. of y (e.g. the rope tail of the MLA query rows, next to the absorbed part).
// cos_sin: [max_pos, rot_dim] fp32 = [cos(rot_dim/2) | sin(rot_dim/2)].
// interleaved: pairs (2i, 2i+1); else NeoX pairs (i, i + rot_dim/2).
__global__ void rope_kernel(__nv_bfloat16* x, int64_t ld_tok, int64_t ld_head, int nheads, int offset, int rot_dim,
                            const int* __restrict__ positions, const float* __restrict__ cos_sin, int interleaved,
                            int T, __nv_bfloat16* y, int64_t y_ld_tok, int64_t y_ld_head, int y_offset) {
  pdl_prologue();
  const int half = rot_dim / 2;
  const int64_t total = (int64_t)T * nheads * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = i % half;
    const int h = (i / half) % nheads;
    const int t = i / ((int64_t)half * nheads);
    const float* cs = cos_sin + (int64_t)positions[t] * rot_dim;
    const float c = cs[j], s = cs[half + j];
    __nv_bfloat16* p = x + t * ld_tok + h * ld_head + offset;
    const int i1 = interleaved ? 2 * j : j;
    const int i2 = interleaved ? 2 * j + 1 : j + half;
    float a = __bfloat162float(p[i1]), b = __bfloat162float(p[i2]);
    rot(a, b, c, s);
    __nv_bfloat16* o = y ? y + t * y_ld_tok + h * y_ld_head + y_offset : p;
    o[i1] = __float2bfloat16(a);
    o[i2] = __float2bfloat16(b);
  }
}

// Latent cache row = [RMSNorm(kv[:512]) * w | RoPE(kv[512:576])] (one warp per token).
__global__ void latent_cache_write_kernel(const __nv_bfloat16* __restrict__ kv, int64_t ld_kv,
                                          const __nv_bfloat16* __restrict__ norm_w, float eps,
                                          const int* __restrict__ positions, const float* __restrict__ cos_sin,
                                          int interleaved, const int64_t* __restrict__ slots,
                                          __nv_bfloat16* __restrict__ cache, int T) {
  pdl_prologue();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  const __nv_bfloat16* row = kv + (int64_t)t * ld_kv;
  float c[16];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    c[i] = __bfloat162float(row[lane * 16 + i]);
    ss += c[i] * c[i];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / 512.f + eps);
  __nv_bfloat16* dst = cache + slot * 576;
#pragma unroll
  for (int i = 0; i < 16; ++i) dst[lane * 16 + i] = __float2bfloat16(c[i] * inv * __bfloat162float(norm_w[lane * 16 + i]));
  // rope over the 64 rope dims: lane owns pair j = lane
  const float* cs = cos_sin + (int64_t)positions[t] * 64;
  const float cc = cs[lane], sn = cs[32 + lane];
  const int i1 = interleaved ? 2 * lane : lane, i2 = interleaved ? 2 * lane + 1 : lane + 32;
  float a = __bfloat162float(row[512 + i1]), b = __bfloat162float(row[512 + i2]);
  rot(a, b, cc, sn);
  dst[512 + i1] = __float2bfloat16(a);
  dst[512 + i2] = __float2bfloat16(b);
}

// 128-dim vector held 4 per lane (dims 4*lane + i): H128 in place.
__device__ __forceinline__ void h128_warp(float (&v)[4], int lane) {
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
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] *= kH128;
}

// RoPE (first rope_dim dims, pairs held within a lane for interleaved, or
// across lanes for NeoX) on a 4-per-lane 128-vector.
__device__ __forceinline__ void rope_warp(float (&v)[4], int lane, const float* cs, int rope_dim, int interleaved) {
  const int half = rope_dim / 2;
  if (interleaved) {
    // pairs (4l, 4l+1), (4l+2, 4l+3) -> pair ids 2l, 2l+1
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const int j = 2 * lane + pr;
      if (4 * lane + 2 * pr + 1 < rope_dim) rot(v[2 * pr], v[2 * pr + 1], cs[j], cs[half + j]);
    }
  } else {
    // pair (j, j + half): dims 4l+i for 4l+i < half pair with dims 4l+i+half
    const int lanes_half = half / 4;  // partner lane offset
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float other = __shfl_sync(0xffffffffu, v[i], lane < lanes_half ? lane + lanes_half : lane - lanes_half);
      const int d = 4 * lane + i;
      if (d < half) {
        v[i] = v[i] * cs[d] - other * cs[half + d];
      } else if (d < rope_dim) {
        const int j = d - half;
        v[i] = v[i] * cs[j] + other * cs[half + j];
      }
    }
  }
}

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  __nv_fp8x4_e4m3 q(make_float4(a, b, c, d));
  return *reinterpret_cast<uint32_t*>(&q);
}

// Indexer keys: LayerNorm(k) * w + b -> RoPE -> H128 -> e4m3 with a per-token scale.
__global__ void index_k_write_kernel(const __nv_bfloat16* __restrict__ k, int64_t ld_k,
                                     const __nv_bfloat16* __restrict__ ln_w, const __nv_bfloat16* __restrict__ ln_b,
                                     float eps, const int* __restrict__ positions, const float* __restrict__ cos_sin,
                                     int rope_dim, int interleaved, const int64_t* __restrict__ slots,
                                     uint8_t* __restrict__ cache, float* __restrict__ cache_scale, int T) {
  pdl_prologue();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(k[(int64_t)t * ld_k + lane * 4 + i]);
  float mean = warp_sum(v[0] + v[1] + v[2] + v[3]) / 128.f;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) var += (v[i] - mean) * (v[i] - mean);
  var = warp_sum(var) / 128.f;
  const float inv = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane * 4 + i;
    v[i] = (v[i] - mean) * inv * (ln_w ? __bfloat162float(ln_w[d]) : 1.f) + (ln_b ? __bfloat162float(ln_b[d]) : 0.f);
    v[i] = __bfloat162float(__float2bfloat16(v[i]));
  }
  rope_warp(v, lane, cos_sin + (int64_t)positions[t] * rope_dim, rope_dim, interleaved);
  h128_warp(v, lane);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = amax > 0.f ? amax / kFp8Max : 1.f;
  const float rs = 1.f / scale;
  reinterpret_cast<uint32_t*>(cache + slot * 128)[lane] = pack_e4m3x4(v[0] * rs, v[1] * rs, v[2] * rs, v[3] * rs);
  if (lane == 0) cache_scale[slot] = scale;
}

// Indexer queries: per (token, head): RoPE -> H128 -> e4m3 with scale; the
// head weight absorbs the scale: w_out = w * wscale * scale.
__global__ void index_q_prep_kernel(const __nv_bfloat16* __restrict__ q, int64_t ld_tok, int nheads,
                                    const int* __restrict__ positions, const float* __restrict__ cos_sin, int rope_dim,
                                    int interleaved, const __nv_bfloat16* __restrict__ w, int64_t ld_w, float wscale,
                                    uint8_t* __restrict__ q8, float* __restrict__ w_out, int T) {
  pdl_prologue();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= T * nheads) return;
  const int t = gw / nheads, h = gw % nheads;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(q[(int64_t)t * ld_tok + h * 128 + lane * 4 + i]);
  rope_warp(v, lane, cos_sin + (int64_t)positions[t] * rope_dim, rope_dim, interleaved);
  h128_warp(v, lane);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = amax > 0.f ? amax / kFp8Max : 1.f;
  const float rs = 1.f / scale;
  reinterpret_cast<uint32_t*>(q8 + ((int64_t)t * nheads + h) * 128)[lane] =
      pack_e4m3x4(v[0] * rs, v[1] * rs, v[2] * rs, v[3] * rs);
  if (lane == 0) w_out[(int64_t)t * nheads + h] = __bfloat162float(w[(int64_t)t * ld_w + h]) * wscale * scale;
}

// ----------------------------------------------------------------------------- top-k
// Order-preserving uint32 key of a float (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = f == 0.f ? 0u : __float_as_uint(f);  // -0 and +0 are the same score (a tie)
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kTopkThreads = 1024;

// Block-wide exclusive scan of one int per thread; returns the prefix, *total = sum.
__device__ int block_exclusive_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int s = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += t;
  }
  if (lane == 31) tmp[warp] = s;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (int)(blockDim.x / 32) ? tmp[lane] : 0;
    int ws = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) ws += t;
    }
    tmp[32 + lane] = ws - w;
    if (lane == 31) tmp[64] = ws;
  }
  __syncthreads();
  const int r = tmp[32 + warp] + s - v;
  *total = tmp[64];
  __syncthreads();
  return r;
}

// Per token: the `k` largest scores among positions [0, ctx), ties to the
// lowest position, output in ascending position order as cache slot ids
// (block_table[seq][pos / bs] * bs + pos % bs); -1 pads when ctx < k.
//
// One CTA per token.  The row's order-preserving keys are cached in shared
// memory when they fit (otherwise re-read from global memory each pass).
// Range-adaptive radix select: the k-th key is known to lie in [lo, hi];
// each pass histograms (key - lo) >> shift over 2048 bins, with shift chosen
// so the range fills the bins (scores crowd a narrow band of float
// exponents, so fixed top-bit digits would pile onto a few bins); a warp
// whose lanes all hit one bin adds once.  A parallel suffix scan finds the
// bin holding the k-th key, which becomes the next [lo, hi]; two or three
// passes reach a single key.  The output pass walks the row in
// 1024-position chunks, one position per thread, and places a taken
// position at (#greater before it) + min(#equal before it, remaining) from
// warp ballots: ascending order, lowest positions win ties, coalesced.
template <bool CACHED>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const float* __restrict__ scores, int64_t ld_scores,
                                                            const int* __restrict__ ctx_lens, int k,
                                                            const int* __restrict__ token_seq,
                                                            const int* __restrict__ block_table, int64_t ld_bt,
                                                            int block_size, int* __restrict__ out_idx,
                                                            int* __restrict__ out_count) {
  pdl_prologue();
  extern __shared__ uint32_t skeys[];
  constexpr int NBIN = 2048;
  __shared__ int hist[NBIN];
  __shared__ int tmp[80];
  __shared__ int wcnt[2][32];
  __shared__ uint32_t s_lo, s_hi, s_red[2][32];
  __shared__ int s_remaining;
  __shared__ int s_run[2];
  const int t = blockIdx.x;
  const int ctx = ctx_lens[t];
  const int seq = token_seq ? token_seq[t] : t;
  const float* row = scores + (int64_t)t * ld_scores;
  const int* bt = block_table + (int64_t)seq * ld_bt;
  int* out = out_idx + (int64_t)t * k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (ctx <= k) {
    for (int p = tid; p < k; p += blockDim.x) out[p] = p < ctx ? bt[p / block_size] * block_size + p % block_size : -1;
    if (tid == 0) out_count[t] = ctx;
    return;
  }
  auto key_at = [&](int p) -> uint32_t { return CACHED ? skeys[p] : fkey(row[p]); };
  // keys (cached) and their range
  uint32_t kmin = 0xffffffffu, kmax = 0u;
  for (int base = 0; base < ctx; base += 8 * kTopkThreads) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // eight independent loads in flight per thread
      const int p = base + j * kTopkThreads + tid;
      v[j] = p < ctx ? row[p] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int p = base + j * kTopkThreads + tid;
      if (p < ctx) {
        const uint32_t key = fkey(v[j]);
        if (CACHED) skeys[p] = key;
        kmin = min(kmin, key);
        kmax = max(kmax, key);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  }
  if (lane == 0) {
    s_red[0][warp] = kmin;
    s_red[1][warp] = kmax;
  }
  __syncthreads();
  if (warp == 0) {
    kmin = s_red[0][lane];
    kmax = s_red[1][lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
      kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) {
      s_lo = kmin;
      s_hi = kmax;
      s_remaining = k;
    }
  }
  __syncthreads();
  uint32_t lo = s_lo, hi = s_hi;
  int remaining = s_remaining;
#pragma unroll 1
  while (lo < hi) {
    const uint32_t span = hi - lo;  // >= 1
    const int bits = 32 - __clz(span);
    const int shift = bits > 11 ? bits - 11 : 0;
    for (int i = tid; i < NBIN; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < ctx; base += blockDim.x) {
      const int p = base + tid;
      const uint32_t key = p < ctx ? key_at(p) : 0u;
      const bool sel = p < ctx && key >= lo && key <= hi;
      const int bin = sel ? (int)((key - lo) >> shift) : -1;
      const int bin0 = __shfl_sync(0xffffffffu, bin, 0);
      if (__all_sync(0xffffffffu, bin == bin0)) {
        if (lane == 0 && bin0 >= 0) atomicAdd(&hist[bin0], 32);
      } else if (sel) {
        atomicAdd(&hist[bin], 1);
      }
    }
    __syncthreads();
    // suffix scan: thread j owns bins NBIN-1-2j and NBIN-2-2j (counted from the top)
    const int top = NBIN - 1 - 2 * tid;
    const int c0 = top >= 0 ? hist[top] : 0, c1 = top - 1 >= 0 ? hist[top - 1] : 0;
    int tot;
    const int above = block_exclusive_scan(c0 + c1, tmp, &tot);
    if (top >= 0) {
      int bsel = -1, before = 0;
      if (above < remaining && above + c0 >= remaining) {
        bsel = top;
        before = above;
      } else if (top - 1 >= 0 && above + c0 < remaining && above + c0 + c1 >= remaining) {
        bsel = top - 1;
        before = above + c0;
      }
      if (bsel >= 0) {
        const uint32_t nlo = lo + ((uint32_t)bsel << shift);
        const uint32_t w = shift >= 32 ? 0xffffffffu : ((1u << shift) - 1u);
        s_lo = nlo;
        s_hi = (hi - nlo > w) ? nlo + w : hi;
        s_remaining = remaining - before;
      }
    }
    __syncthreads();
    lo = s_lo;
    hi = s_hi;
    remaining = s_remaining;
  }
  const uint32_t kth = lo;  // key of the k-th largest; the first `remaining` positions holding it are taken
  // Output: warp w walks positions [w * span, (w + 1) * span) in 32-position steps.  Sweep 1
  // counts its keys above / equal to kth, a block scan gives each warp its offsets, sweep 2
  // places the taken positions.
  const int span = ((ctx + 31) / 32 + 31) / 32 * 32;
  const int w0 = warp * span, w1 = min(ctx, w0 + span);
  int g_cnt = 0, e_cnt = 0;
  for (int base = w0; base < w1; base += 32) {
    const int p = base + lane;
    const uint32_t key = p < w1 ? key_at(p) : 0u;
    g_cnt += __popc(__ballot_sync(0xffffffffu, p < w1 && key > kth));
    e_cnt += __popc(__ballot_sync(0xffffffffu, p < w1 && key == kth));
  }
  if (lane == 0) {
    wcnt[0][warp] = g_cnt;
    wcnt[1][warp] = e_cnt;
  }
  __syncthreads();
  if (warp == 0) {
    int g = wcnt[0][lane], e = wcnt[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int g2 = __shfl_up_sync(0xffffffffu, g, o), e2 = __shfl_up_sync(0xffffffffu, e, o);
      if (lane >= o) {
        g += g2;
        e += e2;
      }
    }
    wcnt[0][lane] = g - wcnt[0][lane];  // exclusive
    wcnt[1][lane] = e - wcnt[1][lane];
    if (lane == 31) {
      s_run[0] = g;
      s_run[1] = e;
    }
  }
  __syncthreads();
  const uint32_t lt_mask = (1u << lane) - 1u;
  int g_run = wcnt[0][warp], e_run = wcnt[1][warp];
  for (int base = w0; base < w1; base += 32) {
    const int p = base + lane;
    const uint32_t key = p < w1 ? key_at(p) : 0u;
    const bool gt = p < w1 && key > kth;
    const bool eq = p < w1 && key == kth;
    const uint32_t bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
    const int e_before = e_run + __popc(be & lt_mask);
    if (gt || (eq && e_before < remaining)) out[g_run + __popc(bg & lt_mask) + min(e_before, remaining)] =
        bt[p / block_size] * block_size + p % block_size;
    g_run += __popc(bg);
    e_run += __popc(be);
  }
  const int total = s_run[0] + min(s_run[1], remaining);
  for (int p = total + tid; p < k; p += blockDim.x) out[p] = -1;
  if (tid == 0) out_count[t] = total;
}

}  // namespace mla

cudaError_t rope_apply(void* x, int64_t ld_tok, int64_t ld_head, int nheads, int offset, int rot_dim,
                       const int* positions, const float* cos_sin, int interleaved, int T, cudaStream_t stream,
                       void* y, int64_t y_ld_tok, int64_t y_ld_head, int y_offset) {
  if (T == 0) return cudaSuccess;
  const int64_t total = (int64_t)T * nheads * (rot_dim / 2);
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  launch_pdl(mla::rope_kernel, dim3(blocks), dim3(threads), 0, stream, reinterpret_cast<__nv_bfloat16*>(x), ld_tok, ld_head, nheads,
                                                   offset, rot_dim, positions, cos_sin, interleaved, T,
                                                   reinterpret_cast<__nv_bfloat16*>(y), y_ld_tok, y_ld_head, y_offset);
  return cudaGetLastError();
}

cudaError_t mla_latent_cache_write(const void* kv, int64_t ld_kv, const void* norm_w, float eps, const int* positions,
                                   const float* cos_sin, int interleaved, const int64_t* slots, void* cache, int T,
                                   cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  launch_pdl(mla::latent_cache_write_kernel, dim3((T * 32 + 255) / 256), dim3(256), 0, stream, 
      reinterpret_cast<const __nv_bfloat16*>(kv), ld_kv, reinterpret_cast<const __nv_bfloat16*>(norm_w), eps,
      positions, cos_sin, interleaved, slots, reinterpret_cast<__nv_bfloat16*>(cache), T);
  return cudaGetLastError();
}

cudaError_t mla_index_k_write(const void* k, int64_t ld_k, const void* ln_w, const void* ln_b, float eps,
                              const int* positions, const float* cos_sin, int rope_dim, int interleaved,
                              const int64_t* slots, void* cache, float* cache_scale, int T, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  launch_pdl(mla::index_k_write_kernel, dim3((T * 32 + 255) / 256), dim3(256), 0, stream, 
      reinterpret_cast<const __nv_bfloat16*>(k), ld_k, reinterpret_cast<const __nv_bfloat16*>(ln_w),
      reinterpret_cast<const __nv_bfloat16*>(ln_b), eps, positions, cos_sin, rope_dim, interleaved, slots,
      reinterpret_cast<uint8_t*>(cache), cache_scale, T);
  return cudaGetLastError();
}

cudaError_t mla_index_q_prep(const void* q, int64_t ld_tok, int nheads, const int* positions, const float* cos_sin,
                             int rope_dim, int interleaved, const void* w, int64_t ld_w, float wscale, void* q8,
                             float* w_out, int T, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const int warps = T * nheads;
  launch_pdl(mla::index_q_prep_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, stream, 
      reinterpret_cast<const __nv_bfloat16*>(q), ld_tok, nheads, positions, cos_sin, rope_dim, interleaved,
      reinterpret_cast<const __nv_bfloat16*>(w), ld_w, wscale, reinterpret_cast<uint8_t*>(q8), w_out, T);
  return cudaGetLastError();
}

cudaError_t mla_topk(const float* scores, int64_t ld_scores, const int* ctx_lens, int k, const int* token_seq,
                     const int* block_table, int64_t ld_bt, int block_size, int* out_idx, int* out_count, int T,
                     cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  // keys of a whole row cached in shared memory when they fit (the row width bounds every ctx)
  const int64_t cache_bytes = ld_scores * 4;
  if (cache_bytes <= 192 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(mla::topk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)cache_bytes);
    if (e != cudaSuccess) return e;
    launch_pdl(mla::topk_kernel<true>, dim3(T), dim3(mla::kTopkThreads), cache_bytes, stream, 
        scores, ld_scores, ctx_lens, k, token_seq, block_table, ld_bt, block_size, out_idx, out_count);
  } else {
    launch_pdl(mla::topk_kernel<false>, dim3(T), dim3(mla::kTopkThreads), 0, stream, scores, ld_scores, ctx_lens, k, token_seq,
                                                                 block_table, ld_bt, block_size, out_idx, out_count);
  }
  return cudaGetLastError();
}

}  // namespace b200

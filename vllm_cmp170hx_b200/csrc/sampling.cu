// Token sampling over (vocab-sharded) logits.
//
// * argmax: one CTA per row, (value, index) reduction with the lowest index
//   winning ties; with a vocab shard offset so ranks can combine their local
//   winners (the reference's shard argmax, vllm_sm80/spec_decode/shard_argmax.py,
//   picks the global argmax without gathering logits).
// * sample: temperature sampling by the Gumbel-max trick in one pass,
//   argmax_i (logit_i / T - log(-log(u_i))), u_i from a counter-based hash of
//   (seed, step, row, i) so replays and ranks are reproducible; T <= 0 rows
//   fall back to argmax.  Top-k / top-p restriction is applied before this by
//   masking logits to -inf.
// * banned tokens: up to kMaxBans global token ids per row (-1 = none) never
//   win (the decode mask of a request, e.g. a parser's tool-call opener under
//   tool_choice="none"); a graph-captured step reads them from its input buffer.
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxBans = 4;

__device__ __forceinline__ void better(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

// 64-bit mix (splitmix64 finaliser) -> uniform in (0, 1)
__device__ __forceinline__ float uniform01(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x ^= x >> 31;
  return ((float)(x >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(const T* __restrict__ logits, int64_t ld, int V,
                                                          const float* __restrict__ temperature, uint64_t seed,
                                                          const int64_t* __restrict__ step, int vocab_offset,
                                                          const int* __restrict__ bans, int nbans,
                                                          float* __restrict__ out_val, int* __restrict__ out_idx) {
  pdl_prologue();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int row = blockIdx.x;
  int ban[kMaxBans];
#pragma unroll
  for (int b = 0; b < kMaxBans; ++b) ban[b] = (bans != nullptr && b < nbans) ? bans[(int64_t)row * nbans + b] - vocab_offset : -1;
  const T* x = logits + (int64_t)row * ld;
  const float temp = temperature ? temperature[row] : 0.f;
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;
  const uint64_t base = seed * 0x100000001B3ull + (step ? (uint64_t)step[0] : 0ull) * 0x9E3779B1ull +
                        (uint64_t)row * 0x85EBCA77ull;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = to_float<T>(x[i]);
    bool banned = false;
#pragma unroll
    for (int b = 0; b < kMaxBans; ++b) banned |= (ban[b] == i);
    if (banned) continue;
    if (!greedy) {
      const float u = uniform01(base + (uint64_t)(vocab_offset + i) * 0xC2B2AE3D27D4EB4Full);
      v = v * inv_t - __logf(-__logf(u));
    }
    better(best, bi, v, vocab_offset + i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(best, bi, ov, oi);
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    best = l < (int)(blockDim.x / 32) ? sv[l] : -INFINITY;
    bi = l < (int)(blockDim.x / 32) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(best, bi, ov, oi);
    }
    if (l == 0) {
      out_val[row] = best;
      out_idx[row] = bi;
    }
  }
}

// Combine per-rank winners [R, rows] -> token ids [rows] (first max, lowest index).
__global__ void combine_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int R, int rows,
                               int64_t* __restrict__ out) {
  pdl_prologue();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float b = -INFINITY;
  int bi = 0x7fffffff;
  for (int k = 0; k < R; ++k) better(b, bi, vals[(int64_t)k * rows + r], idx[(int64_t)k * rows + r]);
  out[r] = bi;
}

}  // namespace

cudaError_t sample_rows(const void* logits, int dtype /*0 bf16, 1 fp32*/, int64_t ld, int rows, int V,
                        const float* temperature, uint64_t seed, const int64_t* step, int vocab_offset,
                        const int* bans, int nbans, float* out_val, int* out_idx, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (nbans < 0 || nbans > kMaxBans) return cudaErrorInvalidValue;
  if (dtype == 0)
    launch_pdl(sample_kernel<__nv_bfloat16>, dim3(rows), dim3(kThreads), 0, stream, reinterpret_cast<const __nv_bfloat16*>(logits), ld, V,
                                                                temperature, seed, step, vocab_offset, bans, nbans,
                                                                out_val, out_idx);
  else
    launch_pdl(sample_kernel<float>, dim3(rows), dim3(kThreads), 0, stream, reinterpret_cast<const float*>(logits), ld, V, temperature,
                                                        seed, step, vocab_offset, bans, nbans, out_val, out_idx);
  return cudaGetLastError();
}

cudaError_t sample_combine(const float* vals, const int* idx, int R, int rows, int64_t* out, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  launch_pdl(combine_kernel, dim3((rows + 127) / 128), dim3(128), 0, stream, vals, idx, R, rows, out);
  return cudaGetLastError();
}

}  // namespace b200

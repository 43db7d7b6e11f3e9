// DeepSeek-V4.1 indexer scores over each query's compressed groups, with the model's rounding contract.
//
// Score of query t against its sequence's group n (n < n_vis[t]; -inf beyond):
//   d_h     = bf16( q[t, h] . k[row(t, n)] )              (fp32 dot product over 128 dims)
//   term_h  = bf16( relu(d_h) * w[t, h] )
//   acc_g   = sum of term_h over the heads of rank group g, in head order (fp32)
//   score   = bf16 running sum of bf16(acc_g) over the groups, in group order
// with row(t, n) = block_table[seq[t]][n / 64] * 64 + n % 64 (the groups are paged like the token cache).
// This is the rounding chain of the reference's indexer (vllm_sm80/models/deepseek_v41/ops/sm80_attn_core.py:
// combine_head_scores), where each tensor-parallel rank sums its heads and the all-reduce adds the ranks'
// bf16 partials in rank order.
//
// B200 layout: one CTA per (query, 128 groups); the 128 key rows are gathered with 16-byte loads and stored
// transposed in shared memory ([dim][group], so the 128 threads -- one per group -- read consecutive
// addresses), the query's H rows and weights as fp32; each thread keeps its H dot products in registers
// (H a template parameter) and reads four dims of every query row per shared float4 load.
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace dsv4 {

constexpr int D = 128;
constexpr int BN = 128;

template <int H>
__global__ void __launch_bounds__(BN) index_scores_kernel(const __nv_bfloat16* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const __nv_bfloat16* __restrict__ keys,
                                                          const int* __restrict__ block_table, int64_t ld_bt,
                                                          const int* __restrict__ seq, const int* __restrict__ n_vis,
                                                          int heads_per_group, float* __restrict__ scores,
                                                          int64_t ld_scores, int N) {
  pdl_prologue();
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem);          // [D][BN]
  float* qs = reinterpret_cast<float*>(smem + D * BN * 2);             // [H][D]
  float* ws = qs + H * D;                                              // [H]
  const int t = blockIdx.x;
  const int n0 = blockIdx.y * BN;
  const int tid = threadIdx.x;
  const int vis = n_vis[t];
  const int n = n0 + tid;
  for (int i = tid; i < H * D; i += BN) qs[i] = __bfloat162float(q[(int64_t)t * H * D + i]);
  if (tid < H) ws[tid] = __bfloat162float(w[(int64_t)t * H + tid]);
  if (n0 >= vis) {  // no visible group in this tile
    if (n < N) scores[(int64_t)t * ld_scores + n] = -INFINITY;
    return;
  }
  // gather this thread's key row, transposed into shared memory
  if (n < vis) {
    const int* bt = block_table + (int64_t)seq[t] * ld_bt;
    const int64_t row = (int64_t)bt[n >> 6] * 64 + (n & 63);
    const uint4* src = reinterpret_cast<const uint4*>(keys + row * D);
#pragma unroll 4
    for (int c = 0; c < D / 8; ++c) {
      const uint4 v = src[c];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ks[(c * 8 + j) * BN + tid] = e[j];
    }
  }
  __syncthreads();
  if (n >= N) return;
  if (n >= vis) {
    scores[(int64_t)t * ld_scores + n] = -INFINITY;
    return;
  }
  float acc[H];
#pragma unroll
  for (int h = 0; h < H; ++h) acc[h] = 0.f;
  for (int d = 0; d < D; d += 4) {
    const float k0 = __bfloat162float(ks[(d + 0) * BN + tid]), k1 = __bfloat162float(ks[(d + 1) * BN + tid]);
    const float k2 = __bfloat162float(ks[(d + 2) * BN + tid]), k3 = __bfloat162float(ks[(d + 3) * BN + tid]);
#pragma unroll
    for (int h = 0; h < H; ++h) {
      const float4 qv = *reinterpret_cast<const float4*>(qs + h * D + d);  // broadcast
      acc[h] = fmaf(qv.w, k3, fmaf(qv.z, k2, fmaf(qv.y, k1, fmaf(qv.x, k0, acc[h]))));
    }
  }
  auto bf = [](float x) { return __bfloat162float(__float2bfloat16_rn(x)); };
  // heads in order; a rank group's terms summed in fp32, the groups' bf16 partials in a bf16 running sum
  float total = 0.f, part = 0.f;
  int j = 0, g = 0;
#pragma unroll
  for (int h = 0; h < H; ++h) {
    const float d = bf(acc[h]);
    const float r = d != d ? d : fmaxf(d, 0.f);  // relu that keeps NaN
    const float term = bf(r * ws[h]);
    part = j == 0 ? term : part + term;
    if (++j == heads_per_group) {
      total = g == 0 ? bf(part) : bf(total + bf(part));
      j = 0;
      ++g;
    }
  }
  scores[(int64_t)t * ld_scores + n] = total;
}

}  // namespace dsv4

cudaError_t dsv4_index_scores(const void* q, const void* w, const void* keys, const int* block_table, int64_t ld_bt,
                              const int* seq, const int* n_vis, int T, int H, int heads_per_group, float* scores,
                              int64_t ld_scores, int N, cudaStream_t stream) {
  if (T == 0 || N == 0) return cudaSuccess;
  if (heads_per_group < 1 || H % heads_per_group) return cudaErrorInvalidValue;
  const dim3 grid(T, (N + dsv4::BN - 1) / dsv4::BN);
  const size_t smem = (size_t)dsv4::D * dsv4::BN * 2 + (size_t)H * dsv4::D * 4 + (size_t)H * 4 + 16;
  auto run = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    launch_pdl(kern, grid, dim3(dsv4::BN), smem, stream, reinterpret_cast<const __nv_bfloat16*>(q),
               reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<const __nv_bfloat16*>(keys), block_table,
               ld_bt, seq, n_vis, heads_per_group, scores, ld_scores, N);
    return cudaGetLastError();
  };
  switch (H) {
    case 4: return run(dsv4::index_scores_kernel<4>);
    case 8: return run(dsv4::index_scores_kernel<8>);
    case 16: return run(dsv4::index_scores_kernel<16>);
    case 32: return run(dsv4::index_scores_kernel<32>);
    case 64: return run(dsv4::index_scores_kernel<64>);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b200

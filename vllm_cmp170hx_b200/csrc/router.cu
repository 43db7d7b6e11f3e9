// MoE router: scores -> top-k experts and weights, and the expert-sorted
// assignment list the grouped expert GEMMs consume.
//
// Covers the reference's routing families (vllm_sm80/kernels/moe/route.py:994
// `moe_route`, models/deepseek_v41/ops/sm80_route.py):
//   mode 0  softmax over all experts, top-k, renormalise over the k picked
//   mode 1  sigmoid scores, select by score + bias, weights = score / sum (GLM)
//   mode 2  sqrt(softplus(logit)), select by score + bias, weights = s / (sum + 1e-20)
// then every weight is multiplied by `scale`.  Ties pick the lowest expert id.
//
// The assignment list is built deterministically (counting sort in
// (token, slot) order, no atomics on the data path) by one CTA, and chunked
// into work items of at most `tile_rows` rows for the grouped GEMMs.
#include <cfloat>

#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace {

constexpr int kMaxExpertsPerLane = 16;  // E <= 512

__global__ void topk_kernel(const float* __restrict__ logits, int T, int E, int k, int mode,
                            const float* __restrict__ bias, float scale, int renorm, int* __restrict__ ids,
                            float* __restrict__ weights) {
  pdl_prologue();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const float* row = logits + (size_t)warp * E;
  float score[kMaxExpertsPerLane];  // value used for the weight
  float key[kMaxExpertsPerLane];    // value used for selection
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    float l = e < E ? row[e] : -INFINITY;
    score[i] = l;
    mx = fmaxf(mx, l);
  }
  float denom = 1.f;
  if (mode == 0) {
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = lane + 32 * i;
      score[i] = e < E ? __expf(score[i] - mx) : 0.f;
      s += score[i];
    }
    denom = warp_sum(s);
  }
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    if (e >= E) {
      key[i] = -INFINITY;
      continue;
    }
    if (mode == 0) {
      score[i] = score[i] / denom;
      key[i] = score[i];
    } else if (mode == 1) {
      score[i] = sigmoidf_(score[i]);
      key[i] = score[i] + (bias ? bias[e] : 0.f);
    } else {
      const float l = score[i];
      const float sp = l > 20.f ? l : log1pf(__expf(l));
      score[i] = sqrtf(sp);
      key[i] = score[i] + (bias ? bias[e] : 0.f);
    }
    // a NaN key (a failed row) ranks below every real score but stays selectable, so every row
    // gets k distinct valid expert ids (its weights carry the NaN on to the output row)
    if (key[i] != key[i]) key[i] = -FLT_MAX;
  }
  float picked_sum = 0.f;
  float my_w = 0.f;
  int my_id = 0;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
    float best_s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = lane + 32 * i;
      if (key[i] > best || (key[i] == best && e < best_e)) {
        best = key[i];
        best_e = e;
        best_s = score[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      const float os = __shfl_xor_sync(0xffffffffu, best_s, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
        best_s = os;
      }
    }
    // remove the pick
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      if (lane + 32 * i == best_e) key[i] = -INFINITY;
    picked_sum += best_s;
    if (lane == j) {
      my_w = best_s;
      my_id = best_e;
    }
  }
  if (lane < k) {
    float w = my_w;
    if (renorm) w = mode == 2 ? w / (picked_sum + 1e-20f) : w / picked_sum;
    ids[(size_t)warp * k + lane] = my_id;
    weights[(size_t)warp * k + lane] = w * scale;
  }
}

// One CTA.  Inputs: ids [T*k] (global expert ids), expert_map [E_map] ->
// local index or -1 (nullptr: identity over E_map = E_local experts); an id
// outside [0, E_map) counts as another rank's.  Outputs:
//   sorted_token[a], sorted_weight[a]  for assignment rows a in expert order,
//   slot_of[t*k + j] = a (or -1 when the expert is not local),
//   items[i] = {local_expert, row0, rows, 0}, num_items[0] = count,
//   expert_offsets[E_local + 1].
constexpr int kBuildThreads = 1024;

__global__ void __launch_bounds__(kBuildThreads) build_assignments_kernel(
    const int* __restrict__ ids, const float* __restrict__ weights, int TK, int k, const int* __restrict__ expert_map,
    int E_map, int E_local, int tile_rows, int* __restrict__ sorted_token, float* __restrict__ sorted_weight,
    int* __restrict__ slot_of, int4* __restrict__ items, int* __restrict__ num_items, int* __restrict__ expert_offsets,
    int max_items) {
  pdl_prologue();
  extern __shared__ int sm[];
  int* counts = sm;                         // [E_local]
  int* base = sm + E_local;                 // [E_local]  running base during placement
  int* warp_counts = sm + 2 * E_local;      // [32][E_local]
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  for (int e = tid; e < E_local; e += blockDim.x) counts[e] = 0;
  __syncthreads();
  // pass 1: counts
  for (int a = tid; a < TK; a += blockDim.x) {
    int e = ids[a];
    e = (e >= 0 && e < E_map) ? (expert_map ? expert_map[e] : e) : -1;
    if (e >= 0 && e < E_local) atomicAdd(&counts[e], 1);
  }
  __syncthreads();
  // exclusive scan of counts (single warp, E_local <= 32 * 32 handled in chunks)
  if (warp == 0) {
    int carry = 0;
    for (int c0 = 0; c0 < E_local; c0 += 32) {
      const int e = c0 + lane;
      const int v = e < E_local ? counts[e] : 0;
      int s = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += t;
      }
      if (e < E_local) {
        base[e] = carry + s - v;
        expert_offsets[e] = carry + s - v;
      }
      carry += __shfl_sync(0xffffffffu, s, 31);
    }
    if (lane == 0) expert_offsets[E_local] = carry;
  }
  __syncthreads();
  // pass 2: stable placement, chunks of blockDim assignments in order
  for (int c0 = 0; c0 < TK; c0 += blockDim.x) {
    const int a = c0 + tid;
    int e = -1;
    if (a < TK) {
      e = ids[a];
      e = (e >= 0 && e < E_map) ? (expert_map ? expert_map[e] : e) : -1;
      if (e >= E_local) e = -1;
    }
    for (int i = tid; i < 32 * E_local; i += blockDim.x) warp_counts[i] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(same & ((1u << lane) - 1));
    if (e >= 0 && rank_in_warp == 0) warp_counts[warp * E_local + e] = __popc(same);
    __syncthreads();
    if (e >= 0) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += warp_counts[w * E_local + e];
      const int row = base[e] + before + rank_in_warp;
      sorted_token[row] = a / k;
      sorted_weight[row] = weights[a];
      slot_of[a] = row;
    } else if (a < TK) {
      slot_of[a] = -1;
    }
    __syncthreads();
    // advance bases by this chunk's totals
    for (int ee = tid; ee < E_local; ee += blockDim.x) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += warp_counts[w * E_local + ee];
      base[ee] += tot;
    }
    __syncthreads();
  }
  // rows past the assigned ones (assignments to experts of other ranks): token 0, weight 0, so a
  // consumer that walks all T*k rows reads valid memory
  {
    const int total = expert_offsets[E_local];
    for (int r = total + tid; r < TK; r += blockDim.x) {
      sorted_token[r] = 0;
      sorted_weight[r] = 0.f;
    }
  }
  // work items: expert e contributes ceil(count_e / tile_rows) items, placed
  // at the exclusive prefix of those counts (one block-wide scan)
  __syncthreads();
  int* nitems = warp_counts;  // reuse: [E_local] item counts, then prefix
  for (int e = tid; e < E_local; e += blockDim.x)
    nitems[e] = (expert_offsets[e + 1] - expert_offsets[e] + tile_rows - 1) / tile_rows;
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int c0 = 0; c0 < E_local; c0 += 32) {
      const int e = c0 + lane;
      const int v = e < E_local ? nitems[e] : 0;
      int s = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += t;
      }
      if (e < E_local) base[e] = carry + s - v;  // reuse base[] as the item prefix
      carry += __shfl_sync(0xffffffffu, s, 31);
    }
    if (lane == 0) num_items[0] = carry < max_items ? carry : max_items;
  }
  __syncthreads();
  for (int e = tid; e < E_local; e += blockDim.x) {
    const int r0 = expert_offsets[e], r1 = expert_offsets[e + 1];
    int n = base[e];
    for (int r = r0; r < r1 && n < max_items; r += tile_rows) items[n++] = make_int4(e, r, min(tile_rows, r1 - r), 0);
  }
}

}  // namespace

cudaError_t moe_topk(const float* logits, int T, int E, int k, int mode, const float* bias, float scale, int renorm,
                     int* ids, float* weights, cudaStream_t stream) {
  if (E > 32 * kMaxExpertsPerLane || k > 32 || k > E) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  launch_pdl(topk_kernel, dim3(blocks), dim3(threads), 0, stream, logits, T, E, k, mode, bias, scale, renorm, ids, weights);
  return cudaGetLastError();
}

cudaError_t moe_build_assignments(const int* ids, const float* weights, int T, int k, const int* expert_map,
                                  int E_map, int E_local, int tile_rows, int* sorted_token, float* sorted_weight, int* slot_of,
                                  int4* items, int* num_items, int* expert_offsets, int max_items,
                                  cudaStream_t stream) {
  const size_t smem = sizeof(int) * (2 * E_local + 32 * E_local);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(build_assignments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  launch_pdl(build_assignments_kernel, dim3(1), dim3(kBuildThreads), smem, stream, ids, weights, T * k, k, expert_map,
                                                               expert_map ? E_map : E_local, E_local,
                                                               tile_rows, sorted_token, sorted_weight, slot_of, items,
                                                               num_items, expert_offsets, max_items);
  return cudaGetLastError();
}

}  // namespace b200

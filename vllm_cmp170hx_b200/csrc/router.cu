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
#include "route_topk.cuh"
#include "sp_sync.cuh"

namespace b200 {

namespace {

__global__ void topk_kernel(const float* __restrict__ logits, int T, int E, int k, int mode,
                            const float* __restrict__ bias, float scale, int renorm, int* __restrict__ ids,
                            float* __restrict__ weights) {
  pdl_prologue();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  int id;
  float w;
  route_topk_warp(logits + (size_t)warp * E, E, k, mode, bias, scale, renorm, &id, &w);
  if (lane < k) {
    ids[(size_t)warp * k + lane] = id;
    weights[(size_t)warp * k + lane] = w;
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
    int max_items, SpSync sp, int sp_wait) {
  pdl_prologue();
  extern __shared__ int sm[];
  // sequence-parallel dispatch: ids / weights are the receive area the ranks pushed into; wait for
  // every source's push of this call first (loads below bypass L1)
  // (a source that never arrives is recorded in the status word; the stale ids are still in range)
  __shared__ uint32_t s_epoch;
  if (sp_wait) {
    if (threadIdx.x == 0) s_epoch = sp_recv_epoch(sp, kSpDispatch);
    __syncthreads();
    if (threadIdx.x < sp.world) sp_wait_flag(sp, kSpDispatch, s_epoch, threadIdx.x);
    __syncthreads();
  }
  int* counts = sm;                         // [E_local]
  int* base = sm + E_local;                 // [E_local]  running base during placement
  int* warp_counts = sm + 2 * E_local;      // [32][E_local]
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  for (int e = tid; e < E_local; e += blockDim.x) counts[e] = 0;
  __syncthreads();
  // pass 1: counts
  for (int a = tid; a < TK; a += blockDim.x) {
    int e = __ldcg(ids + a);
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
      e = __ldcg(ids + a);
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
      sorted_weight[row] = __ldcg(weights + a);
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
  if (sp_wait && threadIdx.x == 0) sp_recv_arrive(sp, kSpDispatch, 1, s_epoch);
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
                                  cudaStream_t stream, const SpSync* sp) {
  const size_t smem = sizeof(int) * (2 * E_local + 32 * E_local);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(build_assignments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  launch_pdl(build_assignments_kernel, dim3(1), dim3(kBuildThreads), smem, stream, ids, weights, T * k, k, expert_map,
                                                               expert_map ? E_map : E_local, E_local,
                                                               tile_rows, sorted_token, sorted_weight, slot_of, items,
                                                               num_items, expert_offsets, max_items,
                                                               sp ? *sp : SpSync{}, sp ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace b200

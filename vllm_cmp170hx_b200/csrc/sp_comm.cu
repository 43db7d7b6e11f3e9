// Sequence-parallel collectives of expert-parallel decode, each fused with the op beside it.
//
// Layout across the group (world ranks, T tokens of the step, Tr = T / world): rank r owns the
// residual stream of tokens [r Tr, (r + 1) Tr).  Per layer:
//
//   residual_norm_kernel   (combine receive) + residual add + RMSNorm + ALL-GATHER push of the
//                          normalised rows into every rank's all-gather area;
//   GEMM, all-gather mode  the column-parallel input projection streams its weight tiles while it
//                          waits for the all-gather flags, then reads the gathered rows (gemm_bf16.cu);
//   GEMM, reduce-scatter   the row-parallel output projection pushes each token's row to its owner
//                          (gemm_bf16.cu);
//   residual_norm_kernel   REDUCE-SCATTER receive (sum of the world pushed partials, rank order) +
//                          residual add + RMSNorm;
//   route_dispatch_kernel  router top-k per token + DISPATCH: the token's row goes once to every rank
//                          that holds one of its experts, with its (expert, weight) list (the experts of
//                          other ranks masked to -1) to every rank;
//   assignment builder     waits for the dispatch flags, then sorts the received (row, expert) pairs
//                          by expert (router.cu); the grouped expert GEMMs run on the received rows;
//   combine_push_kernel    COMBINE: the weighted sum over this rank's experts of every received row,
//                          pushed back to the token's owner, summed there by the next
//                          residual_norm_kernel (fixed rank order).
//
// The reference moves the same data with an all-gather before the experts and a reduce-scatter after
// them (vllm_sm80/kernels/exl3/quant.py:1913-1934) and reduces the row-parallel projections with an
// all-reduce (vllm_sm80/distributed/communicator.py:545).  Here each rank sends only the rows a peer
// needs (the dispatch sends a token's row once per destination rank, not to all), every byte moves as
// a plain peer store from inside the producing kernel, and no kernel reads another GPU's memory.  Flag
// protocol and buffer reuse: sp_sync.cuh.
#include "common.cuh"
#include "launch.h"
#include "route_topk.cuh"
#include "sp_sync.cuh"

namespace b200 {
namespace spc {

constexpr int kThreads = 256;
constexpr int kMaxVec = 8;  // rows up to 256 threads x 8 vectors x 8 = 16384 values

B200_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = (l < blockDim.x / 32) ? red[l] : 0.f;
  s = warp_sum(s);
  __syncthreads();
  return s;
}

B200_DEVICE void add8(float (&acc)[8], const uint4& v) {
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(h[i]);
}

B200_DEVICE uint4 pack8(const float (&v)[8]) {
  uint4 o;
  o.x = pack_bf16x2(v[0], v[1]);
  o.y = pack_bf16x2(v[2], v[3]);
  o.z = pack_bf16x2(v[4], v[5]);
  o.w = pack_bf16x2(v[6], v[7]);
  return o;
}

// ------------------------------------------------------------------ residual + RMSNorm (+ all-gather)
// One block per local token row.
__global__ void __launch_bounds__(kThreads) residual_norm_kernel(SpNormArgs a) {
  pdl_prologue();
  __shared__ float red[32];
  __shared__ uint32_t s_e;
  const int t = blockIdx.x, tid = threadIdx.x;
  const int nvec = a.H / 8;
  const int ch = a.src == 1 ? kSpReduceScatter : kSpCombine;
  const int world = a.s.world, rank = a.s.rank;
  const bool recv = a.src == 1 || a.src == 2;
  if (recv) {
    if (tid == 0) s_e = sp_recv_epoch(a.s, ch);
    __syncthreads();
    if (tid < world) sp_wait_flag(a.s, ch, s_e, tid);
    __syncthreads();
  }
  const uint32_t dm = a.src == 2 ? a.dmask[t] : 0u;
  const uint8_t* mine = reinterpret_cast<const uint8_t*>(a.s.peers[rank]);
  const int64_t area = a.src == 1 ? a.rs_off : a.comb_off;
  float vals[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = tid + i * kThreads;
    if (v >= nvec) continue;
    uint4* res = reinterpret_cast<uint4*>(a.residual + (int64_t)t * a.H) + v;
    if (a.src == 0) {
      const uint4 x = reinterpret_cast<const uint4*>(a.x + (int64_t)t * a.ld_x)[v];
      *res = x;
#pragma unroll
      for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
      add8(vals[i], x);
    } else {
      uint4 y;
      if (a.src == 3) {  // rows computed on this rank
        y = reinterpret_cast<const uint4*>(a.x + (int64_t)t * a.ld_x)[v];
      } else {
        // the pushed rows of this token, summed in rank order (fp32), rounded like the unfused op's output
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < world; ++r) {
          if (a.src == 2 && !((dm >> r) & 1u)) continue;
          add8(acc, sp_ld_cg_v4(mine + area + ((int64_t)(r * a.Tr + t) * nvec + v) * 16));
        }
        if (a.src == 2 && a.add) add8(acc, reinterpret_cast<const uint4*>(a.add + (int64_t)t * a.H)[v]);
        y = pack8(acc);
      }
      const uint4 r0 = *res;
      float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      add8(sum, y);
      add8(sum, r0);
      const uint4 nr = pack8(sum);
      *res = nr;
#pragma unroll
      for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
      add8(vals[i], nr);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
  }
  const float inv = rsqrtf(block_sum(ss, red) / a.H + a.eps);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int v = tid + i * kThreads;
    if (v >= nvec) continue;
    const uint4 wr = reinterpret_cast<const uint4*>(a.w)[v];
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wr);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = vals[i][j] * inv * __bfloat162float(we[j]);
    const uint4 ov = pack8(o);
    if (a.out) reinterpret_cast<uint4*>(a.out + (int64_t)t * a.ld_out)[v] = ov;
    if (a.ag) {
      const int64_t off = a.ag_off + ((int64_t)(rank * a.Tr + t) * nvec + v) * 16;
      for (int d = 0; d < world; ++d) *reinterpret_cast<uint4*>(a.s.peers[d] + off) = ov;
    }
  }
  if (a.ag) __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    if (a.ag) sp_push_arrive(a.s, kSpAllGather, gridDim.x);
    if (recv) sp_recv_arrive(a.s, ch, gridDim.x, s_e);
  }
}

// ------------------------------------------------------------------ router top-k + dispatch
// One warp per local token.
__global__ void __launch_bounds__(kThreads) route_dispatch_kernel(SpDispatchArgs a) {
  pdl_prologue();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  const int world = a.s.world, rank = a.s.rank;
  if (t < a.Tr) {
    int id;
    float w;
    route_topk_warp(a.logits + (int64_t)t * a.E, a.E, a.k, a.mode, a.bias, a.scale, a.renorm, &id, &w);
    const int dest = id >= 0 ? id / a.e_per_rank : -1;
    const uint32_t m = __reduce_or_sync(0xffffffffu, (dest >= 0 && dest < world) ? (1u << dest) : 0u);
    if (lane == 0) a.dmask[t] = m;
    if (a.ids_local && lane < a.k) {
      a.ids_local[(int64_t)t * a.k + lane] = id;
      a.w_local[(int64_t)t * a.k + lane] = w;
    }
    const int64_t row = (int64_t)rank * a.Tr + t;
    const int nvec = a.H / 8;
    const uint4* src = reinterpret_cast<const uint4*>(a.h + (int64_t)t * a.ld_h);
    for (int d = 0; d < world; ++d) {
      const uint64_t base = a.s.peers[d];
      if (lane < a.k) {
        reinterpret_cast<int*>(base + a.ids_off)[row * a.k + lane] = dest == d ? id : -1;
        reinterpret_cast<float*>(base + a.w_off)[row * a.k + lane] = w;
      }
      if ((m >> d) & 1u) {
        uint4* dst = reinterpret_cast<uint4*>(base + a.rows_off) + row * nvec;
        for (int c = lane; c < nvec; c += 32) dst[c] = src[c];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) sp_push_arrive(a.s, kSpDispatch, gridDim.x);
}

// ------------------------------------------------------------------ combine + push to the owner
// Blocks stride over the received rows (world * Tr); a row without an expert on this rank is skipped
// (its owner does not read this rank's slot for it).  With channel kSpReduceScatter the same kernel
// pushes a row-parallel output that is already computed (rows = the step's tokens, one slot each).
__global__ void __launch_bounds__(kThreads) combine_push_kernel(SpCombineArgs a) {
  pdl_prologue();
  __shared__ int s_slot[32];
  __shared__ float s_w[32];
  __shared__ int s_any;
  const int world = a.s.world, rank = a.s.rank;
  const int R = world * a.Tr, nvec = a.H / 8;
  for (int row = blockIdx.x; row < R; row += gridDim.x) {
    if (threadIdx.x == 0) s_any = 0;
    __syncthreads();
    if (threadIdx.x < a.k) {
      const int s = a.slot_of[(int64_t)row * a.k + threadIdx.x];
      s_slot[threadIdx.x] = s;
      s_w[threadIdx.x] = s >= 0 ? a.sorted_weight[s] : 0.f;
      if (s >= 0) s_any = 1;
    }
    __syncthreads();
    if (s_any) {
      const int src = row / a.Tr, t = row % a.Tr;
      uint4* dst = reinterpret_cast<uint4*>(a.s.peers[src] + a.comb_off) + (int64_t)(rank * a.Tr + t) * nvec;
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j0 = 0; j0 < a.k; j0 += 4) {  // fixed slot order; 4 rows' loads in flight at once
          float4 p[4], q[4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int s = j0 + jj < a.k ? s_slot[j0 + jj] : -1;
            if (s >= 0) {
              const float4* yr = reinterpret_cast<const float4*>(a.y + (int64_t)s * a.ld_y + v * 8);
              p[jj] = yr[0];
              q[jj] = yr[1];
            } else {
              p[jj] = q[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float wt = j0 + jj < a.k ? s_w[j0 + jj] : 0.f;
            acc[0] += wt * p[jj].x;
            acc[1] += wt * p[jj].y;
            acc[2] += wt * p[jj].z;
            acc[3] += wt * p[jj].w;
            acc[4] += wt * q[jj].x;
            acc[5] += wt * q[jj].y;
            acc[6] += wt * q[jj].z;
            acc[7] += wt * q[jj].w;
          }
        }
        dst[v] = pack8(acc);
      }
    }
    __syncthreads();
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) sp_push_arrive(a.s, a.channel, gridDim.x);
}

__global__ void wait_kernel(SpSync s, int ch) {
  pdl_prologue();
  __shared__ uint32_t s_e;
  if (threadIdx.x == 0) s_e = sp_recv_epoch(s, ch);
  __syncthreads();
  if (threadIdx.x < s.world) sp_wait_flag(s, ch, s_e, threadIdx.x);
  __syncthreads();
  if (threadIdx.x == 0) sp_recv_arrive(s, ch, 1, s_e);
}

}  // namespace spc

static bool sp_ok(const SpSync& s) {
  return s.peers != nullptr && s.state != nullptr && s.world >= 1 && s.world <= kSpMaxRanks && s.rank >= 0 &&
         s.rank < s.world;
}

cudaError_t sp_residual_norm(const SpNormArgs& a, cudaStream_t stream) {
  if (!sp_ok(a.s) || a.H % 8 || a.H > spc::kThreads * spc::kMaxVec * 8 || a.Tr < 1 || a.src < 0 || a.src > 3 ||
      ((a.src == 0 || a.src == 3) && a.x == nullptr) || (a.src == 2 && a.dmask == nullptr) || a.residual == nullptr)
    return cudaErrorInvalidValue;
  launch_pdl(spc::residual_norm_kernel, dim3(a.Tr), dim3(spc::kThreads), 0, stream, a);
  return cudaGetLastError();
}

cudaError_t sp_route_dispatch(const SpDispatchArgs& a, cudaStream_t stream) {
  if (!sp_ok(a.s) || a.H % 8 || a.k < 1 || a.k > 32 || a.E > 512 || a.e_per_rank < 1 || a.Tr < 1)
    return cudaErrorInvalidValue;
  const int blocks = (a.Tr * 32 + spc::kThreads - 1) / spc::kThreads;
  launch_pdl(spc::route_dispatch_kernel, dim3(blocks), dim3(spc::kThreads), 0, stream, a);
  return cudaGetLastError();
}

cudaError_t sp_combine_push(const SpCombineArgs& a, cudaStream_t stream) {
  if (!sp_ok(a.s) || a.H % 8 || a.k < 1 || a.k > 32 || (a.ld_y % 4) || a.Tr < 1 ||
      (a.channel != kSpCombine && a.channel != kSpReduceScatter))
    return cudaErrorInvalidValue;
  const int rows = a.s.world * a.Tr;
  const int blocks = rows < 2 * device_sm_count() ? rows : 2 * device_sm_count();
  launch_pdl(spc::combine_push_kernel, dim3(blocks), dim3(spc::kThreads), 0, stream, a);
  return cudaGetLastError();
}

cudaError_t sp_wait(const SpSync& s, int channel, cudaStream_t stream) {
  if (!sp_ok(s) || channel < 0 || channel >= kSpChannels) return cudaErrorInvalidValue;
  launch_pdl(spc::wait_kernel, dim3(1), dim3(32), 0, stream, s, channel);
  return cudaGetLastError();
}

}  // namespace b200

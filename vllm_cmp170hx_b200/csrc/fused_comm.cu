// Compute fused with the tensor-parallel all-reduce over symmetric peer
// buffers (NVLink P2P stores, no NCCL on the path).
//
// combine + all-reduce (the MoE output): the routed experts of every rank
// produce fp32 rows for the (token, slot) assignments it holds; the combine
// sums each token's top-k rows with their router weights (plus the shared
// expert's output) and the TP group sums the ranks' partial outputs.  Here
// one kernel does both: block b owns the same slice of the [T, H] output on
// every rank; it computes its slice of this rank's partial (fp32, fixed slot
// order, rounded to bf16 as a separate combine would), PUSHES it into slot
// `rank` of every rank's buffer (posted peer stores), publishes a per-block
// epoch flag to every rank, waits for every rank's flag, and sums the slots
// (now local) in rank order.  The reference runs the combine
// (csrc/exl3/moe.cu:268 combine_routes) and the all-reduce
// (vllm_sm80/models/deepseek_v41/sm80_moe.py:464 moe_all_reduce) as two
// steps.
//
// Buffer halves alternate with the block's epoch parity: a rank can be at
// most one call ahead of a peer still reading (its next call needs that
// peer's flag of the current call), so a half is never overwritten while
// read.  Waits are bounded by %globaltimer and report kErrPeerTimeout.
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace fused {

constexpr int kThreads = 256;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__global__ void __launch_bounds__(kThreads) combine_allreduce_kernel(CombineArArgs p) {
  pdl_prologue();
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    s_epoch = p.epochs[b] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int hv = p.H / 8;
  const int64_t nv = (int64_t)p.T * hv;
  const int64_t per = (nv + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = b * per, v1 = min(nv, v0 + per);
  const int64_t half_off = p.data_off + (int64_t)(e & 1) * p.world * p.slot_bytes;
  // 1. this rank's partial output, pushed to every rank's slot `rank`
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const int t = (int)(v / hv);
    const int c = (int)(v % hv) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < p.k; j0 += 4) {  // fixed slot order; the slot, weight and row loads of 4 at once
      int s[4];
      float w[4];
      float4 a[4], bb[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) s[jj] = j0 + jj < p.k ? p.slot_of[(int64_t)t * p.k + j0 + jj] : -1;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        w[jj] = s[jj] >= 0 ? p.sorted_weight[s[jj]] : 0.f;
        if (s[jj] >= 0) {
          const float4* row = reinterpret_cast<const float4*>(p.y + (int64_t)s[jj] * p.ld_y + c);
          a[jj] = row[0];
          bb[jj] = row[1];
        } else {
          a[jj] = bb[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        acc[0] += w[jj] * a[jj].x;
        acc[1] += w[jj] * a[jj].y;
        acc[2] += w[jj] * a[jj].z;
        acc[3] += w[jj] * a[jj].w;
        acc[4] += w[jj] * bb[jj].x;
        acc[5] += w[jj] * bb[jj].y;
        acc[6] += w[jj] * bb[jj].z;
        acc[7] += w[jj] * bb[jj].w;
      }
    }
    if (p.add) {
      const uint4 a = *reinterpret_cast<const uint4*>(p.add + (int64_t)t * p.H + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&a);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(h[i]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    const int64_t off = half_off + (int64_t)p.rank * p.slot_bytes + v * 16;
    for (int dst = 0; dst < p.world; ++dst) *reinterpret_cast<uint4*>(p.peers[dst] + off) = o;
  }
  __threadfence_system();
  __syncthreads();
  // 2. publish, then wait for every rank's block b
  if (threadIdx.x < p.world) {
    st_release_sys(reinterpret_cast<uint32_t*>(p.peers[threadIdx.x] + p.flag_off) + b * p.world + p.rank, e);
    const uint32_t* f = reinterpret_cast<const uint32_t*>(p.peers[p.rank] + p.flag_off) + b * p.world + threadIdx.x;
    const uint64_t t0 = globaltimer();
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (globaltimer() - t0 > p.timeout_ns) {
        record_error(p.status, kErrPeerTimeout);
        s_fail = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (!s_fail) {
    // 3. sum the ranks' slots (pushed here) in rank order
    const uint8_t* mine = reinterpret_cast<const uint8_t*>(p.peers[p.rank]) + half_off;
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < p.world; ++r) {
        const uint4 x = ld_cg_v4(mine + (int64_t)r * p.slot_bytes + v * 16);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&x);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(h[i]);
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(p.out)[v] = o;
    }
  }
  if (threadIdx.x == 0) p.epochs[b] = e;
}

}  // namespace fused

cudaError_t combine_allreduce(const CombineArArgs& a, int blocks, cudaStream_t stream) {
  if (a.H % 8 || a.world < 1 || a.world > 32 || blocks < 1 || (a.ld_y % 4)) return cudaErrorInvalidValue;
  if ((int64_t)a.T * a.H * 2 > a.slot_bytes) return cudaErrorInvalidValue;
  if (a.T == 0) return cudaSuccess;
  launch_pdl(fused::combine_allreduce_kernel, dim3(blocks), dim3(fused::kThreads), 0, stream, a);
  return cudaGetLastError();
}

}  // namespace b200

// Collectives over NVLink peer memory (symmetric buffers mapped into every
// rank of the tensor-parallel group).
//
// one-shot all-reduce (decode-sized messages; the reference's flags-in-data
// P2P two-shot / one-shot kernels, vllm_sm80/distributed/
// custom_all_reduce_flags.py:376,688, play this role on PCIe):
//   * block b of every rank owns the same slice of the message;
//   * it copies its slice of the input into this rank's symmetric buffer
//     (double-buffered by call parity), then publishes a per-block epoch flag
//     into every peer's flag area (release, system scope) and waits until every
//     peer's flag for that block reached the same epoch (acquire);
//   * it then sums the slice over all ranks (peer loads, fp32, rank order, so
//     every rank gets the bitwise-same result) and writes the output.
// Epochs are per block and monotonic (a flag is never reset), so a fast peer
// that already entered the next call cannot be mistaken for this one, and the
// kernel is CUDA-graph capturable (no host-side state per call).  Every wait
// is bounded by %globaltimer; a rank that never arrives makes the kernel set
// kErrPeerTimeout in the status word and return (the host raises).
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace comm {

constexpr int kThreads = 512;

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
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

struct ArParams {
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  int64_t n;                // elements (multiple of 8)
  const uint64_t* peers;    // [world] base address of each rank's symmetric buffer
  int rank, world;
  int64_t data_off;         // bytes from a buffer's base to its data area
  int64_t half_bytes;       // bytes of one data half (double buffering)
  uint32_t* epochs;         // [gridDim.x] this rank's per-block call counters (local memory)
  uint32_t* status;
  uint64_t timeout_ns;
};

// Flag area at the start of each symmetric buffer: flags[block][src_rank].
__device__ __forceinline__ uint32_t* flag_ptr(uint64_t base, int block, int src, int world) {
  return reinterpret_cast<uint32_t*>(base) + block * world + src;
}

__global__ void __launch_bounds__(kThreads) oneshot_all_reduce_kernel(ArParams p) {
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
  const int64_t half = (e & 1) * p.half_bytes;
  const int64_t nv = p.n / 8;  // 16-byte vectors
  const int64_t per = (nv + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = b * per, v1 = min(nv, v0 + per);
  uint8_t* mine = reinterpret_cast<uint8_t*>(p.peers[p.rank]) + p.data_off + half;
  // 1. stage this block's slice of the input in my symmetric buffer
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x)
    reinterpret_cast<uint4*>(mine)[v] = reinterpret_cast<const uint4*>(p.in)[v];
  __syncthreads();
  // 2. publish, then wait for every peer's block b
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world) {
    st_release_sys(flag_ptr(p.peers[threadIdx.x], b, p.rank, p.world), e);
    const uint32_t* f = flag_ptr(p.peers[p.rank], b, threadIdx.x, p.world);
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
  if (s_fail) {
    if (threadIdx.x == 0) p.epochs[b] = e;
    return;
  }
  // 3. sum over ranks in rank order (fp32), write the output
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < p.world; ++r) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.peers[r]) + p.data_off + half;
      const uint4 x = ld_cg_v4(reinterpret_cast<const uint4*>(src) + v);
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
  if (threadIdx.x == 0) p.epochs[b] = e;
}

}  // namespace comm

cudaError_t symm_all_reduce(const void* in, void* out, int64_t n, const uint64_t* peers, int rank, int world,
                            int64_t data_off, int64_t half_bytes, uint32_t* epochs, int blocks, uint32_t* status,
                            uint64_t timeout_ns, cudaStream_t stream) {
  if (n % 8 || n * 2 > half_bytes || world > 32 || blocks < 1) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  comm::ArParams p{reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<__nv_bfloat16*>(out), n, peers, rank,
                   world, data_off, half_bytes, epochs, status, timeout_ns};
  launch_pdl(comm::oneshot_all_reduce_kernel, dim3(blocks), dim3(comm::kThreads), 0, stream, p);
  return cudaGetLastError();
}

}  // namespace b200

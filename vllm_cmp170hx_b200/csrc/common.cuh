// Shared device helpers for the sm_100a kernels of this package.
//
// Everything GEMM-shaped here runs on the 5th-generation tensor cores:
// operands are staged in shared memory (by TMA or by producer warps that
// decode quantised weights), one elected thread issues `tcgen05.mma`, the
// fp32 accumulator lives in tensor memory (TMEM) and the epilogue reads it
// back with `tcgen05.ld`.  Every spin-wait in this file is bounded: a wait
// that runs out records an error code in a device word the host reads, and
// the caller unwinds (it never traps).
#pragma once
#include <cstdlib>
#include <utility>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define B200_DEVICE __device__ __forceinline__

namespace b200 {

// ---------------------------------------------------------------------------
// Error words.  A kernel that gives up on a wait ORs one of these codes into
// the status word it was given (or the global fallback word) and returns.
// ---------------------------------------------------------------------------
enum ErrorCode : uint32_t {
  kErrNone = 0,
  kErrMbarTimeout = 1u << 0,   // an mbarrier phase never completed
  kErrPeerTimeout = 1u << 1,   // a peer rank's flag never arrived
  kErrBadIndex = 1u << 2,      // an index was out of range (access skipped)
  kErrTmemAlloc = 1u << 3,     // TMEM allocation did not return
};

// Upper bound on polls of one wait.  try_wait itself suspends for a
// hardware-chosen interval, so this is seconds of wall time, far longer than
// any legitimate wait in these kernels and short enough to unwind a broken
// pipeline before the host's own watchdog.
constexpr uint32_t kMaxPolls = 1u << 26;

B200_DEVICE void record_error(uint32_t* status, uint32_t code) {
  if (status != nullptr) atomicOr(status, code);
}

B200_DEVICE uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

B200_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

B200_DEVICE uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

B200_DEVICE bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
B200_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

B200_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

B200_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

B200_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel of this package is launched with
// programmatic stream serialisation (`launch_pdl`) and starts with `pdl_prologue()`:
// it waits for the previous kernel in the stream to complete (and its memory to
// be visible) before touching anything, then lets the next kernel launch.  So a
// kernel's CTAs are scheduled, and reach that wait, while its predecessor
// drains, instead of after it (the per-launch gap of CUDA-graph decode steps).
// ---------------------------------------------------------------------------
B200_DEVICE void pdl_prologue() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether launches may overlap their predecessor (programmatic dependent launch).  VLLM_B200_NO_PDL=1
// turns it off for diagnosis: a profiler then charges each kernel its own time only, not the time it
// spent launched early and waiting for its predecessor.  griddepcontrol.wait returns at once then.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VLLM_B200_NO_PDL");
    return !(v != nullptr && v[0] == '1');
  }();
  return on;
}

template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Thread-block clusters: rank, distributed shared memory, cluster-scope barriers
// ---------------------------------------------------------------------------
B200_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The address of `local` (a shared-memory address of this CTA) in CTA `cta` of the cluster.
B200_DEVICE uint32_t cluster_map(uint32_t local, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(cta));
  return r;
}

// All threads of every CTA of the cluster (aligned: every thread of each warp executes it).  Used
// once, right after the mbarrier initialisation, when every CTA reaches it unconditionally.
B200_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive (release, cluster scope) on the mbarrier at the same offset as `bar` in CTA `cta`.
B200_DEVICE void mbar_arrive_remote(uint64_t* bar, uint32_t cta) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_map(smem_u32(bar), cta))
               : "memory");
}

// Bulk copy of `bytes` (16-B multiple, both ends 16-B aligned) from this CTA's shared memory to the
// same-offset-independent address `dst_local` in CTA `cta` of the cluster; completion is signalled on
// that CTA's mbarrier `bar_local` (its offset), as transaction bytes.  Not a multicast: one
// destination, inside this GPU.
B200_DEVICE void bulk_copy_to_cta(uint32_t dst_local, const void* src, uint32_t bytes, uint64_t* bar_local, uint32_t cta) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          cluster_map(dst_local, cta)),
      "r"(smem_u32(src)), "r"(bytes), "r"(cluster_map(smem_u32(bar_local), cta))
      : "memory");
}

B200_DEVICE void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the source side of every committed bulk copy has been read (its shared memory may be reused)
B200_DEVICE void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

B200_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

B200_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

B200_DEVICE bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for a phase completed by arrivals of other CTAs of the cluster (acquire at cluster
// scope, so their writes before the arrive are visible).
B200_DEVICE bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t* status) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
  }
  record_error(status, kErrMbarTimeout);
  return false;
}

// Bounded wait for the phase with the given parity.  Returns false (and
// records kErrMbarTimeout) when the phase did not complete in kMaxPolls polls.
B200_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  record_error(status, kErrMbarTimeout);
  return false;
}

// Bounded wait that also gives up as soon as another role of the CTA raised
// the shared abort flag (checked every 256 polls).
B200_DEVICE bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && abort_flag != nullptr && *abort_flag) return false;
  }
  record_error(status, kErrMbarTimeout);
  if (abort_flag != nullptr) *abort_flag = 1;
  return false;
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor copies, no multicast anywhere in this package)
// ---------------------------------------------------------------------------
B200_DEVICE void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

B200_DEVICE void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

B200_DEVICE void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                             int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Untiled bulk copy global -> shared (both 16-B aligned, size multiple of 16).
B200_DEVICE void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA issue, commit, loads
// ---------------------------------------------------------------------------
// Allocates `ncols` TMEM columns (power of two, >= 32) for the whole warp;
// the base address is written to *dst_smem.  Must be called by one full warp.
B200_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

B200_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

B200_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

B200_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
B200_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T ; kind::f16 covers bf16 and fp16
// operands (A and B must have the same type), fp32 accumulate.
B200_DEVICE void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A is read from tensor
// memory, row m in lane m, K-major with two 16-bit elements per 32-bit column
// (a K = 16 step spans 8 columns).
B200_DEVICE void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// kind::f8f6f4 (e4m3 / e5m2 operands, fp32 accumulate), K = 32 per instruction.
B200_DEVICE void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (frees the operand stage / publishes the accumulator).
B200_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

B200_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
B200_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 16 consecutive columns: thread t of the warp gets
// columns [col, col+16) of TMEM lane (warp_quarter*32 + t).
B200_DEVICE void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}

B200_DEVICE void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr));
}

B200_DEVICE void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
      "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------
// Layout-type field (bits 61..63) of the sm_100 shared-memory descriptor.
enum SmemLayout : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

// Shared-memory matrix descriptor: start address, leading/stride byte
// offsets (all in 16-byte units), fixed version bits 46..47 = 1, layout type.
B200_DEVICE uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, SmemLayout layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 0x7) << 61;
  return d;
}

// K-major operand in 128-byte-swizzled rows (what TMA SWIZZLE_128B writes):
// 8-row atoms of 1024 bytes, consecutive atoms 1024 bytes apart.
B200_DEVICE uint64_t desc_kmajor_sw128(const void* tile) {
  return make_smem_desc(smem_u32(tile), 16, 1024, kSwizzle128B);
}

// K-major operand, no swizzle: 8x16-byte core matrices; `lbo` = bytes between
// core matrices adjacent in K, `sbo` = bytes between core matrices adjacent in M/N.
B200_DEVICE uint64_t desc_kmajor_plain(const void* tile, uint32_t lbo, uint32_t sbo) {
  return make_smem_desc(smem_u32(tile), lbo, sbo, kSwizzleNone);
}

// Instruction descriptor for kind::f16: fp32 accumulator, both operands
// K-major unless the *_mn flags say otherwise.  ab_format: 0 = f16, 1 = bf16.
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t m, uint32_t n, uint32_t ab_format,
                                                      bool a_mn = false, bool b_mn = false) {
  return (1u << 4)                      // D format f32
         | (ab_format << 7)             // A format
         | (ab_format << 10)            // B format
         | ((a_mn ? 1u : 0u) << 15)     // A major
         | ((b_mn ? 1u : 0u) << 16)     // B major
         | ((n >> 3) << 17)             // N / 8
         | ((m >> 4) << 24);            // M / 16
}

// Instruction descriptor for kind::f8f6f4 with e4m3 operands, fp32 accumulate.
__host__ __device__ constexpr uint32_t make_idesc_e4m3(uint32_t m, uint32_t n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
B200_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

B200_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

B200_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

B200_DEVICE uint32_t pack_half2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
B200_DEVICE float to_float(T v);
template <>
B200_DEVICE float to_float<float>(float v) { return v; }
template <>
B200_DEVICE float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
B200_DEVICE float to_float<__half>(__half v) { return __half2float(v); }

template <typename T>
B200_DEVICE T from_float(float v);
template <>
B200_DEVICE float from_float<float>(float v) { return v; }
template <>
B200_DEVICE __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16(v); }
template <>
B200_DEVICE __half from_float<__half>(float v) { return __float2half(v); }

B200_DEVICE float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
// softplus with torch's default threshold (x above 20 returns x)
B200_DEVICE float softplusf_(float x) { return x > 20.f ? x : log1pf(__expf(x)); }
B200_DEVICE float siluf_(float x) { return x / (1.0f + __expf(-x)); }

}  // namespace b200

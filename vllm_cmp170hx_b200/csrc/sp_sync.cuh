// Flag protocol of the sequence-parallel collectives (sp_comm.cu, and the GEMM / assignment kernels
// that push into or wait on them).
//
// Every rank owns one symmetric buffer (mapped into every peer over NVLink).  Its first bytes are the
// flag words flags[channel][src] (uint32): rank `src` stores the call number of its latest push on
// `channel` into the flag of every destination, with release semantics at system scope, after all of
// that call's data stores.  Data moves by plain peer stores into the destination's receive area of the
// channel; the receiver waits (acquire, bounded by %globaltimer) until every source's flag reached its
// own call number, then reads the area with L1-bypassing loads.
//
// Call numbers are kept per rank and channel in local device memory (`SpSync::state`, four uint32 per
// channel: pushes done, push arrivals, receives done, receive arrivals).  Every block of a launch reads
// the count at its start; the last block to arrive at the end (arrival counter) publishes the flags
// (push side) and stores the new count, and resets the arrival counter.  No block of a launch can read
// the count after the last block updated it (all blocks arrived before), and launches of one channel on
// one rank are ordered by the stream, so the counts need no host state and CUDA-graph replays advance
// them.  The grid size may differ from call to call.
//
// Receive areas are single-buffered.  A channel's next push to a peer always comes after this rank
// waited on a later push of that peer, which that peer issues after it finished reading the area (the
// layer's collectives alternate AG -> RS -> DISPATCH -> COMBINE), so a push never overwrites data still
// being read.
#pragma once
#include "common.cuh"
#include "launch.h"

namespace b200 {

// SpSync, the channels and the flag area size are declared in launch.h (shared with the host glue).

B200_DEVICE void sp_st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_DEVICE uint32_t sp_ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
B200_DEVICE uint4 sp_ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
B200_DEVICE uint32_t sp_ld_cg_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
B200_DEVICE uint32_t sp_ld_volatile(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }

B200_DEVICE uint32_t* sp_flag(uint64_t base, int ch, int src) {
  return reinterpret_cast<uint32_t*>(base) + ch * kSpMaxRanks + src;
}

// Receive side, at block start (thread 0): this call's number on `ch`.
B200_DEVICE uint32_t sp_recv_epoch(const SpSync& s, int ch) { return sp_ld_volatile(&s.state[ch * 4 + 2]) + 1; }

// Receive side: threads [0, world) of the calling group wait until every source's flag of `ch` reached
// `e`.  Returns false (and records kErrPeerTimeout) for a thread whose source never arrived; the caller
// combines the results over the group.
B200_DEVICE bool sp_wait_flag(const SpSync& s, int ch, uint32_t e, int src) {
  const uint32_t* f = sp_flag(s.peers[s.rank], ch, src);
  const uint64_t t0 = globaltimer();
  while ((int32_t)(sp_ld_acquire_sys(f) - e) < 0) {
    if (globaltimer() - t0 > s.timeout_ns) {
      record_error(s.status, kErrPeerTimeout);
      return false;
    }
  }
  return true;
}

// Block end (thread 0, after every thread of the block fenced its pushes and the block synchronised):
// count this block in; the last block of the launch publishes `ch` to every rank (push side) and
// stores the call count.
B200_DEVICE void sp_push_arrive(const SpSync& s, int ch, int nblocks) {
  const uint32_t old = atomicAdd(&s.state[ch * 4 + 1], 1u);
  if (old + 1 != (uint32_t)nblocks) return;
  __threadfence_system();
  const uint32_t e = sp_ld_volatile(&s.state[ch * 4 + 0]) + 1;
  for (int d = 0; d < s.world; ++d) sp_st_release_sys(sp_flag(s.peers[d], ch, s.rank), e);
  s.state[ch * 4 + 1] = 0;
  s.state[ch * 4 + 0] = e;
  __threadfence();
}

B200_DEVICE void sp_recv_arrive(const SpSync& s, int ch, int nblocks, uint32_t e) {
  const uint32_t old = atomicAdd(&s.state[ch * 4 + 3], 1u);
  if (old + 1 != (uint32_t)nblocks) return;
  s.state[ch * 4 + 3] = 0;
  s.state[ch * 4 + 2] = e;
  __threadfence();
}

}  // namespace b200

// Device side of the flag barrier between the GPUs of one node (one process per GPU).  Flag words live in memory every rank has mapped (mlb_ipc_alloc / mlb_ipc_open):
// flags[r][p] is written by rank p and read by rank r.
#pragma once

#include "common.cuh"

namespace mlb {

constexpr int64_t kPeerDefaultTimeoutNs = 2000000000LL;  // 2 s

// One rank's view of the barrier: every rank's flag array (flags[r] has `world` words, word p written by
// rank p), this rank's epoch counter (device memory, advanced by each barrier) and the wait limit.
struct PeerSync {
  uint32_t* flags[MLB_MAX_OUT_DESTS];
  uint32_t* epoch;
  int rank, world;
  int64_t timeout_ns;
};
constexpr uint32_t kPeerMaxSpins = 1u << 26;             // backstop on each wait besides the clock

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called by one whole warp after every write this rank owes its peers is ordered before it: advance the
// epoch, raise this rank's word in every peer's flag array to it (lane p talks to rank p),
// and wait until every peer has raised its word here.  Each wait gives up after timeout_ns or
// kPeerMaxSpins polls; returns true (on lane 0) if any wait gave up.
__device__ __forceinline__ bool peer_signal_and_wait(const PeerSync ps, int lane) {
  uint32_t e = 0;
  if (lane == 0) e = *ps.epoch + 1;
  e = __shfl_sync(0xffffffffu, e, 0);
  uint32_t* peer = nullptr;
  const uint32_t* mine = nullptr;
#pragma unroll
  for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i) {  // select without dynamic indexing of the parameter array
    if (i == lane) peer = ps.flags[i];
    if (i == ps.rank) mine = ps.flags[i];
  }
  const uint64_t limit = static_cast<uint64_t>(ps.timeout_ns > 0 ? ps.timeout_ns : kPeerDefaultTimeoutNs);
  bool timed_out = false;
  if (lane < ps.world) {
    __threadfence_system();
    st_release_sys(peer + ps.rank, e);
    const uint32_t* word = mine + lane;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if (static_cast<int32_t>(ld_acquire_sys(word) - e) >= 0) break;
      if (it >= kPeerMaxSpins || globaltimer_ns() - t0 > limit) {
        timed_out = true;
        break;
      }
      __nanosleep(64);
    }
  }
  const bool any = __any_sync(0xffffffffu, timed_out);
  if (lane == 0) *ps.epoch = e;
  return any;
}

}  // namespace mlb

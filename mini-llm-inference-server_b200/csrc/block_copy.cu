// K3 — block copy for prefix-cache copy-on-write and pool compaction.
//
// pool[dst[i]] = pool[src[i]] for every pool (every layer's K and V) in one launch.  The reference has
// no block COW or compaction; its only compaction by copy is SlotKVCache.move
// (src/minillm/cache/slot.py:41-46), a per-layer slice assignment.  One CTA copies one block of one
// pool per iteration: 256 threads move 16-byte vectors, eight loads in flight per thread before the
// stores, so a 32 KB block (16 tokens x 8 heads x 128 dims x bf16) is one pass.
#include "common.cuh"

namespace mlb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;

__global__ void __launch_bounds__(kThreads) block_copy_kernel(void* const* pools, int num_pools,
                                                              int64_t num_blocks, int64_t block_bytes,
                                                              const int32_t* src, const int32_t* dst,
                                                              int64_t num_pairs, int32_t* err) {
  griddep_begin();
  const int64_t items = num_pairs * num_pools;
  const int64_t nvec = block_bytes / 16;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t pair = it / num_pools;
    const int pool = static_cast<int>(it % num_pools);
    const int64_t s = __ldg(src + pair), d = __ldg(dst + pair);
    if (s < 0 || s >= num_blocks || d < 0 || d >= num_blocks) {
      if (threadIdx.x == 0 && pool == 0) flag_error(err, MLB_DEV_COPY_RANGE);
      continue;
    }
    char* base = static_cast<char*>(pools[pool]);
    const uint4* sp = reinterpret_cast<const uint4*>(base + s * block_bytes);
    uint4* dp = reinterpret_cast<uint4*>(base + d * block_bytes);
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += kThreads * kUnroll) {
      uint4 r[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t v = v0 + u * kThreads;
        if (v < nvec) r[u] = __ldcs(sp + v);  // streamed once: do not keep in L2 at the expense of others
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t v = v0 + u * kThreads;
        if (v < nvec) dp[v] = r[u];
      }
    }
  }
}

}  // namespace

cudaError_t launch_block_copy(void* const* pools, int num_pools, int64_t num_blocks, int64_t block_bytes,
                              const int32_t* src, const int32_t* dst, int64_t num_pairs, int32_t* err,
                              int num_sms, cudaStream_t s) {
  const int64_t items = num_pairs * num_pools;
  int64_t grid = items < static_cast<int64_t>(num_sms) * 8 ? items : static_cast<int64_t>(num_sms) * 8;
  if (grid < 1) return cudaSuccess;
  return launch_k(block_copy_kernel, dim3(static_cast<unsigned>(grid)), dim3(kThreads), 0, s, pools, num_pools,
                  num_blocks, block_bytes, src, dst, num_pairs, err);
}

}  // namespace mlb

// K3 — block copy for prefix-cache copy-on-write and pool compaction.
//
// pool[dst[i]] = pool[src[i]] for every pool (every layer's K and V) in one launch.  The reference has
// no block COW or compaction; its only compaction by copy is SlotKVCache.move
// (src/minillm/cache/slot.py:41-46), a per-layer slice assignment.
//
// Each thread keeps kInFlight 16-byte loads in flight before its stores, whatever the block size: a CTA
// item is PPC consecutive pairs of one pool (items spread over the grid) and each thread takes VU vectors
// of each pair's block, with PPC x VU = kInFlight.  A 32 KB block (16 tokens x 8 heads x 128 dims x bf16)
// is one pair per item; the 4 KB blocks of one KV head per GPU (KV-head sharding over 8 GPUs) are 8 pairs
// per item, where one pair per item left a single load in flight per thread (3.45 TB/s read + write
// measured, against 5.7 at 32 KB).
#include "common.cuh"

namespace mlb {
namespace {

constexpr int kThreads = 256;
constexpr int kInFlight = 8;

template <int PPC, int VU>
__global__ void __launch_bounds__(kThreads) block_copy_kernel(void* const* pools, int num_pools,
                                                              int64_t num_blocks, int64_t block_bytes,
                                                              const int32_t* src, const int32_t* dst,
                                                              int64_t num_pairs, int32_t* err) {
  static_assert(PPC * VU == kInFlight, "loads in flight per thread");
  griddep_begin();
  const int64_t nvec = block_bytes / 16;
  const int64_t groups = (num_pairs + PPC - 1) / PPC;
  // one item = PPC consecutive pairs of one pool; items spread over the grid
  for (int64_t it = blockIdx.x; it < groups * num_pools; it += gridDim.x) {
    const int64_t p0 = (it / num_pools) * PPC;
    const int pool = static_cast<int>(it % num_pools);
    int64_t s[PPC], d[PPC];
#pragma unroll
    for (int q = 0; q < PPC; ++q) {
      s[q] = d[q] = -1;
      if (p0 + q < num_pairs) {
        s[q] = __ldg(src + p0 + q);
        d[q] = __ldg(dst + p0 + q);
        if (s[q] < 0 || s[q] >= num_blocks || d[q] < 0 || d[q] >= num_blocks) {
          if (threadIdx.x == 0 && pool == 0) flag_error(err, MLB_DEV_COPY_RANGE);
          s[q] = -1;  // skipped
        }
      }
    }
    char* base = static_cast<char*>(pools[pool]);
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += static_cast<int64_t>(kThreads) * VU) {
      uint4 r[PPC][VU];
#pragma unroll
      for (int q = 0; q < PPC; ++q)
#pragma unroll
        for (int u = 0; u < VU; ++u) {
          const int64_t v = v0 + u * kThreads;
          if (s[q] >= 0 && v < nvec)  // streamed once: do not keep in L2 at the expense of others
            r[q][u] = __ldcs(reinterpret_cast<const uint4*>(base + s[q] * block_bytes) + v);
        }
#pragma unroll
      for (int q = 0; q < PPC; ++q)
#pragma unroll
        for (int u = 0; u < VU; ++u) {
          const int64_t v = v0 + u * kThreads;
          if (s[q] >= 0 && v < nvec) reinterpret_cast<uint4*>(base + d[q] * block_bytes)[v] = r[q][u];
        }
    }
  }
}

template <int PPC, int VU>
cudaError_t launch_copy(void* const* pools, int num_pools, int64_t num_blocks, int64_t block_bytes,
                        const int32_t* src, const int32_t* dst, int64_t num_pairs, int32_t* err, int num_sms,
                        cudaStream_t s) {
  const int64_t items = (num_pairs + PPC - 1) / PPC * num_pools;
  const int64_t grid = items < static_cast<int64_t>(num_sms) * 8 ? items : static_cast<int64_t>(num_sms) * 8;
  if (grid < 1) return cudaSuccess;
  return launch_k(block_copy_kernel<PPC, VU>, dim3(static_cast<unsigned>(grid)), dim3(kThreads), 0, s, pools,
                  num_pools, num_blocks, block_bytes, src, dst, num_pairs, err);
}

}  // namespace

cudaError_t launch_block_copy(void* const* pools, int num_pools, int64_t num_blocks, int64_t block_bytes,
                              const int32_t* src, const int32_t* dst, int64_t num_pairs, int32_t* err,
                              int num_sms, cudaStream_t s) {
  const int64_t vectors_per_thread = (block_bytes / 16 + kThreads - 1) / kThreads;
  if (vectors_per_thread >= 8)
    return launch_copy<1, 8>(pools, num_pools, num_blocks, block_bytes, src, dst, num_pairs, err, num_sms, s);
  if (vectors_per_thread >= 4)
    return launch_copy<2, 4>(pools, num_pools, num_blocks, block_bytes, src, dst, num_pairs, err, num_sms, s);
  if (vectors_per_thread >= 2)
    return launch_copy<4, 2>(pools, num_pools, num_blocks, block_bytes, src, dst, num_pairs, err, num_sms, s);
  return launch_copy<8, 1>(pools, num_pools, num_blocks, block_bytes, src, dst, num_pairs, err, num_sms, s);
}

}  // namespace mlb

// Device-side expansion of a step's attention metadata (the bulk of AttentionMetadata.build,
// src/minillm/attention/metadata.py:71-103, which walks every new token in Python and builds eleven host
// tensors).  The host sends one compact int64 upload (every sequence's block ids back to back plus O(S)
// prefix arrays) and this kernel writes the per-token and per-page arrays and the two padded block tables
// straight into the buffers the metadata tensors view.  At config 3 sizes (256 rows, tables 1314 wide)
// the padded tables alone are 4 MB of int64 + 2 MB of int32 that no longer cross PCIe or pass through
// numpy.
//
// One launch, four grid-stride loops (tokens, table cells, context pages, per-sequence values); each
// thread's loads are a binary search over a prefix array of S + 1 entries and one or two id loads.
#include "common.cuh"

namespace mlb {
namespace {

struct MetaArgs {
  const int64_t* ids;         // [num_ids]
  const int64_t* ids_indptr;  // [S + 1]
  const int64_t* qo;          // [S + 1]
  const int64_t* seq_lens;    // [S]
  const int64_t* kv_indptr;   // [S + 1]
  const int64_t* last_len;    // [S]
  int64_t num_tokens, num_pages;
  int num_seqs, width, block_size;
  int64_t* out64;  // positions [N] | slot_mapping [N] | block_tables [S, W] | logits_index [S]
  int32_t* out32;  // qo [S + 1] | seq_lens [S] | block_tables [S, W] | kv_indptr [S + 1] | kv_indices [P] | last [S]
};

// The sequence s with indptr[s] <= x < indptr[s + 1] (indptr non-decreasing, indptr[0] <= x < indptr[S]).
__device__ __forceinline__ int owner_of(const int64_t* indptr, int num_seqs, int64_t x) {
  int lo = 0, hi = num_seqs;  // invariant: indptr[lo] <= x < indptr[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(indptr + mid) <= x)
      lo = mid;
    else
      hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(256) build_metadata_kernel(MetaArgs a) {
  griddep_begin();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int S = a.num_seqs, W = a.width;
  const int64_t N = a.num_tokens, cells = static_cast<int64_t>(S) * W;
  int64_t* positions = a.out64;
  int64_t* slots = a.out64 + N;
  int64_t* table64 = a.out64 + 2 * N;
  int64_t* logits = table64 + cells;
  int32_t* qo32 = a.out32;
  int32_t* lens32 = qo32 + S + 1;
  int32_t* table32 = lens32 + S;
  int32_t* kv_indptr32 = table32 + cells;
  int32_t* kv_indices = kv_indptr32 + S + 1;
  int32_t* last32 = kv_indices + a.num_pages;
  // new tokens: position in the sequence (cached tokens first) and the pool slot it is written to
  for (int64_t t = tid; t < N; t += stride) {
    const int s = owner_of(a.qo, S, t);
    const int64_t q0 = __ldg(a.qo + s), n_new = __ldg(a.qo + s + 1) - q0;
    const int64_t pos = t - q0 + (__ldg(a.seq_lens + s) - n_new);
    const int64_t id = __ldg(a.ids + __ldg(a.ids_indptr + s) + pos / a.block_size);
    positions[t] = pos;
    slots[t] = id * a.block_size + pos % a.block_size;
  }
  // padded block tables, int64 and int32 (padding: block 0)
  for (int64_t i = tid; i < cells; i += stride) {
    const int s = static_cast<int>(i / W), c = static_cast<int>(i % W);
    const int64_t b0 = __ldg(a.ids_indptr + s), nblk = __ldg(a.ids_indptr + s + 1) - b0;
    const int64_t id = c < nblk ? __ldg(a.ids + b0 + c) : 0;
    table64[i] = id;
    table32[i] = static_cast<int32_t>(id);
  }
  // every sequence's context pages, concatenated
  for (int64_t p = tid; p < a.num_pages; p += stride) {
    const int s = owner_of(a.kv_indptr, S, p);
    kv_indices[p] = static_cast<int32_t>(__ldg(a.ids + __ldg(a.ids_indptr + s) + (p - __ldg(a.kv_indptr + s))));
  }
  // per-sequence values
  for (int64_t s = tid; s <= S; s += stride) {
    qo32[s] = static_cast<int32_t>(__ldg(a.qo + s));
    kv_indptr32[s] = static_cast<int32_t>(__ldg(a.kv_indptr + s));
    if (s < S) {
      lens32[s] = static_cast<int32_t>(__ldg(a.seq_lens + s));
      last32[s] = static_cast<int32_t>(__ldg(a.last_len + s));
      logits[s] = __ldg(a.qo + s + 1) - 1;
    }
  }
}

}  // namespace

cudaError_t launch_build_metadata(const int64_t* in, int64_t num_ids, int num_seqs, int64_t num_tokens,
                                  int64_t num_pages, int width, int block_size, int64_t* out64, int32_t* out32,
                                  cudaStream_t s) {
  MetaArgs a{};
  a.ids = in;
  a.ids_indptr = in + num_ids;
  a.qo = a.ids_indptr + num_seqs + 1;
  a.seq_lens = a.qo + num_seqs + 1;
  a.kv_indptr = a.seq_lens + num_seqs;
  a.last_len = a.kv_indptr + num_seqs + 1;
  a.num_tokens = num_tokens;
  a.num_pages = num_pages;
  a.num_seqs = num_seqs;
  a.width = width;
  a.block_size = block_size;
  a.out64 = out64;
  a.out32 = out32;
  int64_t work = num_tokens;
  work = work > static_cast<int64_t>(num_seqs) * width ? work : static_cast<int64_t>(num_seqs) * width;
  work = work > num_pages ? work : num_pages;
  work = work > num_seqs + 1 ? work : num_seqs + 1;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_k(build_metadata_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, a);
}

}  // namespace mlb

// Paged attention with split-K scratch in a library-owned static device array: an entry point that
// allocates nothing.
//
// Who needs it: some callers cannot allocate device memory at the time they attend.  An engine that, like
// the reference's (engine/process.py:91-115), hands nearly all free device memory to the KV pool at start-up
// has nothing left for a workspace later, and a caller outside PyTorch (a C or Go serving loop, an embedded
// runtime) may have no device allocator to draw one from and cannot afford cudaMalloc's implicit device
// synchronisation inside a decode step.  For them, mlb_paged_attention_noalloc runs the same attention and
// split-K reduction kernels as mlb_paged_attention + mlb_splitk_reduce, with the fp32 partial rows kept in
// `g_splitk_scratch` below instead of caller-provided buffers.
//
// Limits and sharing:
// - the array is MLB_NOALLOC_SCRATCH_BYTES (8 MiB) and every GPU that loads this library holds it until
//   the process exits; a plan whose partial rows need more (rows x heads x (head_dim + 1) x 4 bytes) is
//   rejected with MLB_ENOSPACE before anything is launched;
// - every call on a device shares the one array and it keeps the last call's contents.  Each partial row a
//   plan uses is written before it is read, so nothing needs clearing, but calls that overlap on the GPU
//   (concurrent streams) race on the array: serialise them;
// - the device address of the array is looked up once per device, on the first call with that device
//   current (cudaGetSymbolAddress); make that first call before any stream capture.
#include <mutex>
#include <string>

#include "attn_args.cuh"

namespace mlb {
int set_last_error(int code, const char* msg);  // the mlb_last_error() channel (capi.cu)
}  // namespace mlb

namespace {

constexpr size_t kNoallocScratchBytes = MLB_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// File-scope device scratch.  In host code this name is only a host-side stand-in: its device address must
// be fetched with cudaGetSymbolAddress on each device before a kernel can be given it.
static __device__ __align__(256) unsigned char g_splitk_scratch[kNoallocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_splitk_scratch on the current device (looked up once per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_splitk_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

int noalloc_fail(int code, const std::string& msg) { return mlb::set_last_error(code, msg.c_str()); }

}  // namespace

extern "C" {

int mlb_paged_attention_noalloc(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* k_cache,
                                const void* v_cache, int dtype, int64_t num_blocks, int block_size, int num_heads,
                                int num_kv_heads, int head_dim, float scale, const int32_t* block_tables,
                                int64_t bt_stride, const int32_t* seq_lens, const int32_t* qo_indptr, int num_seqs,
                                const mlb_work_unit* units, int64_t num_units, const mlb_shared_unit* shared_units,
                                int64_t num_shared_units, const mlb_share_member* members, int64_t num_partial_rows,
                                const int32_t* reduce_rows, const int32_t* reduce_chunks, int64_t num_tokens,
                                void* out, int64_t out_stride_tok, int64_t out_stride_head, int32_t* err_word,
                                void* stream) {
  if (num_partial_rows < 0 || num_heads <= 0 || head_dim <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads)
    return noalloc_fail(MLB_EINVAL, "paged_attention_noalloc: bad sizes");
  // Bound the row count before multiplying, so a huge caller-supplied count cannot wrap the byte total
  // below the array size: one row takes num_heads x (head_dim + 1) floats.
  const size_t row_bytes = static_cast<size_t>(num_heads) * (static_cast<size_t>(head_dim) + 1) * sizeof(float);
  if (static_cast<uint64_t>(num_partial_rows) > kNoallocScratchBytes / row_bytes)
    return noalloc_fail(MLB_ENOSPACE, "paged_attention_noalloc: the plan's " + std::to_string(num_partial_rows) +
                                          " split-K rows do not fit the " + std::to_string(kNoallocScratchBytes) +
                                          "-byte static array; use mlb_paged_attention with a workspace or a "
                                          "larger pages_per_unit");
  const size_t o_bytes = static_cast<size_t>(num_partial_rows) * num_heads * head_dim * sizeof(float);
  const size_t lse_bytes = static_cast<size_t>(num_partial_rows) * num_heads * sizeof(float);
  const size_t lse_off = (o_bytes + 255) & ~size_t(255);
  if (lse_off + lse_bytes > kNoallocScratchBytes)
    return noalloc_fail(MLB_ENOSPACE, "paged_attention_noalloc: the plan's " + std::to_string(num_partial_rows) +
                                          " split-K rows need " + std::to_string(lse_off + lse_bytes) +
                                          " bytes of scratch, more than the " +
                                          std::to_string(kNoallocScratchBytes) +
                                          "-byte static array; use mlb_paged_attention with a workspace or a "
                                          "larger pages_per_unit");
  if (num_partial_rows > 0 && (!reduce_rows || !reduce_chunks))
    return noalloc_fail(MLB_EINVAL, "paged_attention_noalloc: the plan splits sequences but reduce rows are null");
  void* scratch = nullptr;
  if (num_partial_rows > 0) {
    cudaError_t e = scratch_address(&scratch);
    if (e != cudaSuccess)
      return noalloc_fail(MLB_ECUDA, std::string("paged_attention_noalloc: cudaGetSymbolAddress: ") +
                                         cudaGetErrorString(e));
  }
  float* po = static_cast<float*>(scratch);
  float* plse = scratch ? reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + lse_off) : nullptr;
  const int rc = mlb_paged_attention(q, q_stride_tok, q_stride_head, k_cache, v_cache, dtype, num_blocks, block_size,
                                     num_heads, num_kv_heads, head_dim, scale, block_tables, bt_stride, seq_lens,
                                     qo_indptr, num_seqs, units, num_units, shared_units, num_shared_units, members,
                                     po, plse, num_partial_rows, out, out_stride_tok, out_stride_head, nullptr,
                                     err_word, stream);
  if (rc != MLB_OK || num_partial_rows == 0 || num_tokens == 0) return rc;  // mlb_last_error() says why
  return mlb_splitk_reduce(po, plse, num_partial_rows, reduce_rows, reduce_chunks,
                           mlb::tokens_per_tile(num_heads, num_kv_heads), num_tokens, num_heads,
                           head_dim, out, out_stride_tok, out_stride_head, dtype, nullptr, stream);
}

}  // extern "C"

/*
 * mlb_paged_kv.h — C ABI of the B200 (sm_100a) paged KV-cache hot path.
 *
 * Drop-in boundary for the paged path of prakhar-iit/mini-llm-inference-server.  Every entry point
 * below replaces one piece of the reference's Python/torch hot path (cited as file:line inside that
 * project).  Conventions shared by all of them:
 *   - pointers are raw device pointers (or host pointers where stated), sizes are element counts and
 *     strides are in ELEMENTS of the tensor they describe; the innermost (head_dim) stride is 1;
 *   - `stream` is a cudaStream_t passed as void* (0 = the legacy default stream);
 *   - the return value is MLB_OK (0) or an MLB_E* code; mlb_last_error() describes the last failure of
 *     the calling thread.  No C++ exception crosses this boundary;
 *   - the library allocates no device memory: pools, metadata, outputs and split-K workspace all
 *     belong to the caller (torch in the Python package);
 *   - `err_word` (optional, may be NULL) is a device int32 into which kernels OR an MLB_DEV_* bit when
 *     they meet an out-of-range slot / block id or a wait that never completes; the offending access
 *     is skipped instead of faulting.
 */
#ifndef MLB_PAGED_KV_H
#define MLB_PAGED_KV_H

#include <stdint.h>

#if defined(__GNUC__)
#define MLB_API __attribute__((visibility("default")))
#else
#define MLB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types of rows and pools */
enum { MLB_F32 = 0, MLB_F16 = 1, MLB_BF16 = 2 };

/* status codes */
enum { MLB_OK = 0, MLB_EINVAL = 1, MLB_EUNSUPPORTED = 2, MLB_ECUDA = 3, MLB_ENOSPACE = 4 };

/* bits a kernel ORs into *err_word */
enum {
  MLB_DEV_SLOT_RANGE = 1,   /* slot_mapping entry outside [0, num_blocks * block_size): row not written */
  MLB_DEV_BLOCK_RANGE = 2,  /* block_tables entry outside [0, num_blocks): page treated as empty        */
  MLB_DEV_WAIT_TIMEOUT = 4, /* a bounded wait on a page copy gave up: output of that unit is invalid    */
  MLB_DEV_COPY_RANGE = 8    /* block-copy pair outside [0, num_blocks): pair skipped                    */
};

/* Description of the last failing call on this thread ("" if none). */
MLB_API const char* mlb_last_error(void);

/* ABI version (bumped on any signature change). */
MLB_API int mlb_abi_version(void);  /* 10 */

/*
 * Programmatic dependent launch (process-wide, default on): every kernel is launched with programmatic
 * stream serialisation, so it becomes resident while its predecessor on the stream finishes and waits
 * on the device (griddepcontrol.wait) before reading anything; launch latency hides behind the previous
 * kernel's tail.  Results are identical either way.  Returns the previous setting.
 */
MLB_API int mlb_set_programmatic_launch(int enable);

/*
 * Shared-prefix units on the 5th-generation tensor cores (process-wide, default on): tcgen05.mma tiles of
 * 128 query columns x 128 keys with TMEM accumulators, for 16-bit pools with head_dim 64 or 128 and q rows
 * 16-byte aligned; otherwise (or when disabled) the warp-level mma.sync kernel.  Same plan either way.
 * Returns the previous setting.
 */
MLB_API int mlb_set_tensor_core_prefix(int enable);

/*
 * Shared-prefix units beside the per-sequence units (process-wide, default on): when a plan has both, the
 * shared-prefix kernel runs on a library-owned side stream of the greatest priority (one per host thread
 * and device, created on the first such call: make it before any stream capture) while the per-sequence
 * kernel runs on the caller's stream, forked from and joined back into the caller's stream with events, so
 * work queued after the call waits for both.  Results are identical either way.  Returns the previous
 * setting.
 */
MLB_API int mlb_set_concurrent_prefix(int enable);

/*
 * KV append.  Replaces write_kv (src/minillm/attention/paged_torch_ref.py:23-28), shared by all three
 * reference backends (torch_ref.py:47, flashinfer_backend.py:43, flash_attn_backend.py:44):
 *     k_cache.view(-1, Hkv, Dh)[slot_mapping[i]] = k[i].to(k_cache.dtype)   (and the same for v)
 * k, v: [num_tokens, num_kv_heads, head_dim] of in_dtype with strides (tok, head) in elements;
 * pools: [num_blocks, block_size, num_kv_heads, head_dim] of cache_dtype, contiguous;
 * slot_mapping: device int64 [num_tokens] (metadata.py:94).  Casts round to nearest even; bf16 NaN is
 * stored as 0xFFFF and fp16 NaN as sign|0x7E00 (the reference's CPU cast).  Slots must be distinct.
 */
MLB_API int mlb_kv_append(void* k_cache, void* v_cache, int cache_dtype, int64_t num_blocks, int block_size,
                  const int64_t* slot_mapping, const void* k, int64_t k_stride_tok, int64_t k_stride_head,
                  const void* v, int64_t v_stride_tok, int64_t v_stride_head, int in_dtype,
                  int64_t num_tokens, int num_kv_heads, int head_dim, int32_t* err_word, void* stream);

/*
 * One unit of paged-attention work: query tile `q_tile` of sequence `seq` over the pages
 * [page_begin, page_end) of its block table, for every KV head (the kernel's grid is units x heads).
 * part_row < 0: the unit covers the whole context and writes `out` itself; otherwise it writes
 * normalised fp32 partial rows part_row + t (t = token within the tile) for the split-K reduction.
 * q0 / num_new / seq_len repeat the sequence's qo_indptr[seq], new-token count and context length so
 * a CTA starts from one 32-byte record.
 */
typedef struct {
  int32_t seq;
  int32_t q_tile;
  int32_t page_begin;
  int32_t page_end;
  int32_t part_row;
  int32_t q0;
  int32_t num_new;
  int32_t seq_len;
} mlb_work_unit;

/*
 * Units of query-tile work for the tensor-core kernel (up to 128 query columns = tokens x query heads of
 * one KV head each).  They come in PAIRS: units 2i and 2i + 1 cover the same pages of the same table row,
 * with the same kind and piece, and one tensor-core CTA per (pair, KV head) loads each K / V tile once for
 * both (member_count 0 marks an empty partner).  num_shared_units is even.  Two kinds (reserved[0] & 0xff):
 * kind 0, a shared prefix (a prefix-cache hit seen by many decode rows): pages [page_begin, page_end) are
 *   the same blocks in the tables of members [member_begin, member_begin + member_count) of the members
 *   array (member_count <= 128 / group), and the table row of sequence `table_seq` holds them.  Each page
 *   is loaded once and applied to every member's query heads; every key is visible.  Each member writes
 *   its partial row members[m].part_base + piece * tokens_per_tile.
 * kind 1, a query tile of a multi-token row (a prefill chunk on cache): tokens member_begin ..
 *   member_begin + member_count - 1 (global token indices, member_count <= 128 / group) of sequence
 *   table_seq against its pages [page_begin, page_end), causal (token i of the row sees keys up to its own
 *   position; a pair of neighbouring tiles covers the later tile's keys).  piece < 0: the unit covers every key its tokens see and writes the final rows; otherwise
 *   it is piece `piece` of (reserved[0] >> 8) and token m's partial row is
 *   reserved[1] + (m * pieces + piece) * tokens_per_tile.
 */
typedef struct {
  int32_t member_begin;
  int32_t member_count;
  int32_t page_begin;
  int32_t page_end;
  int32_t piece;
  int32_t table_seq;
  int32_t reserved[2];
} mlb_shared_unit;

typedef struct {
  int32_t seq;       /* the member sequence (a decode row: one new token)   */
  int32_t q0;        /* qo_indptr[seq]: its token                          */
  int32_t part_base; /* its first partial row                              */
  int32_t reserved;
} mlb_share_member;

/*
 * Host-side planner (host pointers).  Plays the role of FlashInfer's per-step plan() that the reference
 * runs once per AttentionMetadata and reuses across layers (flashinfer_backend.py:44-45, :48-64).
 * Inputs: qo_indptr [num_seqs + 1] and seq_lens [num_seqs] exactly as AttentionMetadata holds them
 * (metadata.py:39-40, :97-98); max_blocks_per_seq = block_tables width (validates seq_lens).
 * block_tables_host (optional, may be NULL): a host copy of the int32 block tables with row stride
 * bt_stride_host; pass it for 16-bit pools only.  When given, decode rows whose tables start with the same
 * run of block ids (shared prefix blocks) get shared-prefix units (a cascade split), and rows of >= 16 new
 * tokens get query-tile units (kind 1 above) instead of 8-column work units.  pages_per_unit = 0 picks a
 * split size from the total work and num_sms.
 * With units == NULL only the counts are returned (*num_units, *num_shared_units, *num_members,
 * *num_partial_rows); otherwise every output array must hold its count (MLB_ENOSPACE if not).
 * reduce_rows / reduce_chunks [num_tokens]: first partial row and number of pieces per token (pieces
 * <= 1: nothing to reduce).  Query tokens per tile = max(1, 8 / (num_heads / num_kv_heads)).
 */
MLB_API int mlb_plan_attention(const int32_t* qo_indptr, const int32_t* seq_lens, int num_seqs, int max_blocks_per_seq,
                       const int32_t* block_tables_host, int64_t bt_stride_host,
                       int num_heads, int num_kv_heads, int block_size, int num_sms, int pages_per_unit,
                       mlb_work_unit* units, int64_t units_capacity, int64_t* num_units,
                       mlb_shared_unit* shared_units, int64_t shared_capacity, int64_t* num_shared_units,
                       mlb_share_member* members, int64_t members_capacity, int64_t* num_members,
                       int32_t* reduce_rows, int32_t* reduce_chunks, int64_t num_tokens,
                       int64_t* num_partial_rows);

/*
 * Where the final attention rows go.  NULL in the calls below means the call's own `out` (strides in
 * elements).  Otherwise every final row is stored into each of num_dests (1..MLB_MAX_OUT_DESTS)
 * destination buffers: row (token t, head h of this call) lands at element offset
 * t * stride_tok + (head_offset + h) * stride_head of dests[i].  KV-head sharding uses it to do the
 * output all-gather with the kernels' own stores: dests are every rank's gathered [N, H_total, head_dim]
 * output (peers' buffers opened with mlb_ipc_open, reached over NVLink), head_offset the rank's first
 * query head; mlb_peer_barrier then tells the ranks that the rows have landed.  No reference
 * counterpart (the reference runs on one GPU); it replaces the NCCL all-gather of the output.
 */
#define MLB_MAX_OUT_DESTS 8
typedef struct {
  int32_t num_dests;
  int32_t head_offset;
  int64_t stride_tok;
  int64_t stride_head;
  void* dests[MLB_MAX_OUT_DESTS];
} mlb_out_targets;

/*
 * Paged attention over block tables (decode rows and multi-token rows with the causal mask aligned to
 * the end of each context).  Replaces paged_attention (src/minillm/attention/paged_torch_ref.py:40-74)
 * and the FlashInfer decode/prefill wrappers' run() (flashinfer_backend.py:46).
 * q: [N, num_heads, head_dim] (strides in elements); pools as above, dtype == q's; block_tables:
 * device int32 [num_seqs, bt_stride] (metadata.py:48); seq_lens: device int32 [num_seqs];
 * qo_indptr: device int32 [num_seqs + 1]; units / shared_units / members: device copies of the plan
 * (shared_units may be NULL when num_shared_units == 0).  Scale is usually 1/sqrt(head_dim).
 * partial_o [num_partial_rows, num_heads, head_dim] and partial_lse [num_partial_rows, num_heads] (fp32,
 * caller-owned) may be NULL when the plan has no partial rows; when it has some, mlb_splitk_reduce
 * completes `out`.  out: [N, num_heads, head_dim] of q's dtype, or out_targets (then `out` may be NULL).
 * Supported: head_dim 64/128/256,
 * block_size 16, num_heads / num_kv_heads <= 8; f16/bf16 pools use tensor-core tiles, f32 pools CUDA
 * cores (f32 plans carry no shared-prefix units).
 */
MLB_API int mlb_paged_attention(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                        const void* k_cache, const void* v_cache, int dtype, int64_t num_blocks, int block_size,
                        int num_heads, int num_kv_heads, int head_dim, float scale,
                        const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens,
                        const int32_t* qo_indptr, int num_seqs, const mlb_work_unit* units, int64_t num_units,
                        const mlb_shared_unit* shared_units, int64_t num_shared_units, const mlb_share_member* members,
                        float* partial_o, float* partial_lse, int64_t num_partial_rows,
                        void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        const mlb_out_targets* out_targets, int32_t* err_word, void* stream);

/*
 * The step's new K/V rows for mlb_paged_attention_append: k / v [num_tokens, num_kv_heads, head_dim] in
 * the pools' dtype (strides in elements; bases and both strides x element bytes 16-byte aligned), and
 * slot_mapping [num_tokens] (device int64), as mlb_kv_append takes them.
 */
typedef struct {
  const void* k;
  const void* v;
  int64_t k_stride_tok, k_stride_head;
  int64_t v_stride_tok, v_stride_head;
  const int64_t* slot_mapping;
  int64_t num_tokens;
} mlb_append_rows;

/*
 * mlb_kv_append followed by mlb_paged_attention, as ONE attention launch (the order of the reference's
 * forward: write, then attend, src/minillm/attention/torch_ref.py:46-48).  Every attention CTA that loads
 * a page holding new rows takes those rows from k / v (never from the pool, which may not have them yet),
 * and the units of each row's last query tile store them into the pools at slot_mapping (out-of-range
 * slots are skipped and flagged MLB_DEV_SLOT_RANGE, as in mlb_kv_append).  16-bit pools only.
 * The caller guarantees, for the launch to equal the two calls:
 *   - slot_mapping[t] is the slot the block tables give token t (block_tables[s][pos / 16] * 16 + pos % 16,
 *     as AttentionMetadata.build makes it, metadata.py:81);
 *   - every block that receives a row appears once in all sequences' context pages (no other sequence,
 *     and no other position of the same sequence, reads it), so no other CTA needs the written values;
 *   - the plan has no query-tile units (kind 1 shared units, rows of >= 16 new tokens).
 * Otherwise call mlb_kv_append and mlb_paged_attention.  Other arguments as mlb_paged_attention.
 */
MLB_API int mlb_paged_attention_append(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                        void* k_cache, void* v_cache, int dtype, int64_t num_blocks, int block_size,
                        int num_heads, int num_kv_heads, int head_dim, float scale,
                        const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens,
                        const int32_t* qo_indptr, int num_seqs, const mlb_work_unit* units, int64_t num_units,
                        const mlb_shared_unit* shared_units, int64_t num_shared_units, const mlb_share_member* members,
                        float* partial_o, float* partial_lse, int64_t num_partial_rows,
                        void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        const mlb_out_targets* out_targets, const mlb_append_rows* append, int32_t* err_word,
                        void* stream);

/*
 * Split-K reduction: for every token whose reduce_chunks > 1, combine its rows
 * reduce_rows[t] + c * tokens_per_tile (c < reduce_chunks[t]) by their log-sum-exp weights and write
 * out[t] (or every out_targets destination).  Completes mlb_paged_attention; no reference counterpart
 * (the reference never splits).  Under programmatic launch the kernel reads reduce_rows / reduce_chunks
 * before it waits for the kernel launched just before it on the stream (normally the attention launch):
 * upload them before that launch, as the plan's other arrays, never from that kernel.
 */
MLB_API int mlb_splitk_reduce(const float* partial_o, const float* partial_lse, int64_t num_partial_rows,
                      const int32_t* reduce_rows, const int32_t* reduce_chunks, int tokens_per_tile,
                      int64_t num_tokens, int num_heads, int head_dim,
                      void* out, int64_t out_stride_tok, int64_t out_stride_head, int out_dtype,
                      const mlb_out_targets* out_targets, void* stream);

/*
 * Device-side expansion of a step's attention metadata: the per-token, per-page and padded-table parts of
 * AttentionMetadata.build (src/minillm/attention/metadata.py:71-103) computed on the GPU from a compact
 * upload.  `in` (device int64) holds, back to back:
 *   ids [num_ids]           every sequence's block ids, concatenated
 *   ids_indptr [S + 1]      offsets of each sequence's ids in `ids`
 *   qo_indptr [S + 1]       token offsets (query_start_loc, metadata.py:84)
 *   seq_lens [S]            context lengths after this step
 *   kv_indptr [S + 1]       offsets of each sequence's context pages, ceil(seq_len / block_size) each
 *   kv_last_page_len [S]
 * (S = num_seqs; every sequence's ids must cover its seq_len).  The call fills
 *   out64: positions [N] | slot_mapping [N] | block_tables [S, width] | logits_index [S]
 *   out32: qo_indptr [S + 1] | seq_lens [S] | block_tables [S, width] | kv_indptr [S + 1] |
 *          kv_indices [num_pages] | kv_last_page_len [S]
 * with N = num_tokens = qo_indptr[S] and num_pages = kv_indptr[S]: the reference's fields (metadata.py:94-102),
 * tables padded with block 0 and int32 values the int64 ones truncated, as Tensor.to(torch.int32) does.
 */
MLB_API int mlb_build_metadata(const int64_t* in, int64_t num_ids, int num_seqs, int64_t num_tokens,
                               int64_t num_pages, int width, int block_size, int64_t* out64, int32_t* out32,
                               void* stream);

/*
 * Block copy for prefix-cache copy-on-write and compaction: pool[dst[i]] = pool[src[i]] for every pool
 * in `pools` (a DEVICE array of num_pools base pointers: every layer's K and V).  block_bytes = one
 * block of one pool (block_size * Hkv * Dh * elt).  The destination set must be disjoint from the
 * source set.  No reference counterpart: the reference has no COW or compaction; its compaction by
 * copy is SlotKVCache.move (src/minillm/cache/slot.py:41-46), which this generalises to blocks.
 */
MLB_API int mlb_block_copy(void* const* pools, int num_pools, int64_t num_blocks, int64_t block_bytes,
                   const int32_t* src, const int32_t* dst, int64_t num_pairs, int32_t* err_word, void* stream);

/*
 * Paged attention that allocates nothing.  No counterpart in the reference: it is this library's answer to
 * callers that cannot allocate device memory when they attend, e.g. an engine that gave nearly all free
 * device memory to the KV pool at start-up (as the reference sizes its pool, engine/process.py:91-115), or a
 * non-PyTorch serving loop with no device allocator and no room for cudaMalloc's implicit synchronisation.
 * Same arguments and results as mlb_paged_attention followed by mlb_splitk_reduce (out gets q's dtype),
 * with the split-K partial rows kept in a static device array of MLB_NOALLOC_SCRATCH_BYTES that every GPU
 * loading the library holds until exit.  Plans whose partial rows need more than that (rows x num_heads x
 * (head_dim + 1) x 4 bytes, each part 256-byte aligned) return MLB_ENOSPACE.  All calls share the array and
 * it keeps the last call's contents; calls that overlap on the GPU race.  The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) with that device current: make it before any stream
 * capture.  reduce_rows / reduce_chunks / num_tokens are the plan's (mlb_plan_attention).
 */
#define MLB_NOALLOC_SCRATCH_BYTES (8u << 20)
MLB_API int mlb_paged_attention_noalloc(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                        const void* k_cache, const void* v_cache, int dtype, int64_t num_blocks, int block_size,
                        int num_heads, int num_kv_heads, int head_dim, float scale,
                        const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens,
                        const int32_t* qo_indptr, int num_seqs, const mlb_work_unit* units, int64_t num_units,
                        const mlb_shared_unit* shared_units, int64_t num_shared_units, const mlb_share_member* members,
                        int64_t num_partial_rows, const int32_t* reduce_rows, const int32_t* reduce_chunks,
                        int64_t num_tokens, void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        int32_t* err_word, void* stream);

/*
 * Device memory shared between the processes of one node (one process per GPU), for the output
 * all-gather above.  No reference counterpart.  mlb_ipc_alloc: cudaMalloc `bytes` on the current device,
 * zero it, and export a handle of MLB_IPC_HANDLE_BYTES bytes that other processes pass to mlb_ipc_open
 * (which maps it, enabling peer access, and returns this process's address of it).  Close what you
 * opened before the owner frees it.
 */
#define MLB_IPC_HANDLE_BYTES 64
MLB_API int mlb_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle);
MLB_API int mlb_ipc_open(const void* handle, void** dev_ptr);
MLB_API int mlb_ipc_close(void* dev_ptr);
MLB_API int mlb_ipc_free(void* dev_ptr);

/*
 * Barrier of `world` ranks, one GPU each, over flag words in shared device memory: flags[r] is rank r's
 * array of `world` uint32 (flags[rank] local, the others peer addresses from mlb_ipc_open).  One launch
 * on `stream`: makes every write of the earlier work on the stream (the kernels' stores into peers'
 * buffers) visible to the node, raises this rank's word in every peer's array to the next epoch, then
 * waits until every peer has done the same here.  `epoch` is this rank's device counter (one uint32,
 * zero at the start, advanced by the kernel, so CUDA-graph replays stay in step).  The wait gives up after
 * timeout_ns (0: 2 s) and ORs MLB_DEV_WAIT_TIMEOUT into *err_word.  Every rank must make the same
 * sequence of calls.  No reference counterpart.
 */
MLB_API int mlb_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t* epoch, int64_t timeout_ns,
                     int32_t* err_word, void* stream);

/*
 * The output all-gather carried by the split-K reduction: one launch that finishes every row of a step
 * and puts it in every rank's gathered buffer.  Call it after mlb_paged_attention was given
 * out_targets = { 1 destination: out_targets->dests[self_dest], same head_offset and strides } (the rank's
 * own buffer).  Split tokens are reduced from their partial rows into every destination; unsplit tokens'
 * rows are copied from dests[self_dest] to the others (NVLink stores into peers' buffers).  Follow it
 * with mlb_peer_barrier on the same stream: the kernel boundary and the barrier's system-scope fence make
 * the rows visible before the flags.  reduce_rows / reduce_chunks / tokens_per_tile / num_partial_rows are
 * the plan's (num_partial_rows may be 0: nothing was split).  No reference counterpart (it replaces the
 * NCCL all-gather of KV-head sharding).
 */
MLB_API int mlb_splitk_reduce_gather(const float* partial_o, const float* partial_lse, int64_t num_partial_rows,
                      const int32_t* reduce_rows, const int32_t* reduce_chunks, int tokens_per_tile,
                      int64_t num_tokens, int num_heads, int head_dim, int out_dtype,
                      const mlb_out_targets* out_targets, int self_dest, void* stream);

/*
 * The same all-gather without the barrier: one launch that finishes this rank's rows, sends them to every
 * peer and waits for the peers' rows.  Each 32-bit word of a row goes to a peer as one 8-byte packet
 * {word, epoch} (single-copy-atomic store), so a row is complete when its packets carry the current
 * epoch: no system-scope fence and no flag round trip, at twice the NVLink bytes of
 * mlb_splitk_reduce_gather.  Call it after mlb_paged_attention left this rank's unsplit rows in `out`
 * (this rank's gathered [num_tokens, world * num_heads, head_dim] buffer, element strides, rows 4-byte
 * aligned), heads [rank * num_heads, (rank + 1) * num_heads).  packets: 2 x world addresses,
 * packets[a * world + p] = rank p's packet area a (this rank's own, the others from mlb_ipc_open), each
 * packet_capacity x world x num_heads x (head_dim x element bytes / 4) uint64, zero when allocated.  Calls
 * alternate between the two areas by the epoch's parity (a peer may still be reading the previous call's).
 * state: this rank's two uint32 device words {epoch, arrivals}, zero at the start and advanced by the
 * kernel (CUDA-graph replays stay in step).  Each wait gives up after timeout_ns (0: 2 s) and ORs MLB_DEV_WAIT_TIMEOUT into
 * *err_word.  Every rank must make the same sequence of calls.  No reference counterpart (it replaces the
 * NCCL all-gather of KV-head sharding).
 */
MLB_API int mlb_splitk_reduce_exchange(const float* partial_o, const float* partial_lse, int64_t num_partial_rows,
                      const int32_t* reduce_rows, const int32_t* reduce_chunks, int tokens_per_tile,
                      int64_t num_tokens, int num_heads, int head_dim, int out_dtype, void* out,
                      int64_t out_stride_tok, int64_t out_stride_head, void* const* packets,
                      int64_t packet_capacity, int rank, int world, uint32_t* state, int64_t timeout_ns,
                      int32_t* err_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLB_PAGED_KV_H */

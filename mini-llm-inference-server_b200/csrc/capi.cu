// The extern "C" boundary (include/mlb_paged_kv.h): argument validation, the host-side split planner,
// dispatch to the kernels, and error reporting by status code + mlb_last_error().  No exception and no
// device allocation crosses or happens behind this boundary.
#include <algorithm>
#include <array>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "attn_args.cuh"

namespace mlb {
cudaError_t launch_kv_append(void* k_cache, void* v_cache, int cache_dtype, int64_t num_slots, const int64_t* slots,
                             const void* k, int64_t k_st, int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                             int in_dtype, int64_t num_tokens, int hkv, int dh, bool vec, int32_t* err,
                             cudaStream_t s);
cudaError_t launch_paged_attention(const AttnArgs& a, int dtype, int dh, int64_t num_units, cudaStream_t s);
cudaError_t launch_shared_prefix_attention(const AttnArgs& a, int dtype, int dh, int64_t num_units, cudaStream_t s);
bool shared_prefix_tc_supported(const AttnArgs& a, int dtype, int dh);
cudaError_t launch_shared_prefix_tc(const AttnArgs& a, int dtype, int dh, int64_t num_units, cudaStream_t s);
bool tensor_core_prefix();
bool concurrent_prefix();  // mlb_set_concurrent_prefix
cudaError_t launch_splitk_reduce(const float* po, const float* plse, const int32_t* rrows, const int32_t* rchunks,
                                 int tpt, int64_t ntok, int h, int dh, const mlb_out_targets& out,
                                 int out_dtype, cudaStream_t s);
cudaError_t launch_splitk_reduce_gather(const float* po, const float* plse, const int32_t* rrows,
                                        const int32_t* rchunks, int tpt, int64_t ntok, int h, int dh,
                                        const mlb_out_targets& out, int self, int out_dtype, cudaStream_t s);
cudaError_t launch_splitk_reduce_exchange(const float* po, const float* plse, const int32_t* rrows,
                                          const int32_t* rchunks, int tpt, int64_t ntok, int h, int dh, int out_dtype,
                                          void* out, int64_t out_st, int64_t out_sh, void* const* packets, int rank,
                                          int world, uint32_t* state, int64_t timeout_ns, int32_t* err, int num_sms,
                                          cudaStream_t s);
cudaError_t launch_block_copy(void* const* pools, int num_pools, int64_t num_blocks, int64_t block_bytes,
                              const int32_t* src, const int32_t* dst, int64_t num_pairs, int32_t* err, int num_sms,
                              cudaStream_t s);
cudaError_t launch_build_metadata(const int64_t* in, int64_t num_ids, int num_seqs, int64_t num_tokens,
                                  int64_t num_pages, int width, int block_size, int64_t* out64, int32_t* out32,
                                  cudaStream_t s);
}  // namespace mlb

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MLB_OK;
  return fail(MLB_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int elt_bytes(int dtype) { return dtype == MLB_F32 ? 4 : (dtype == MLB_F16 || dtype == MLB_BF16) ? 2 : 0; }
bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr int kMinPagesPerUnit = 8;  // below this a unit's pipeline start-up dominates
constexpr int kCtasPerSm = 3;        // resident paged-attention CTAs per SM (shared memory bound)
constexpr int kWaveTenths = 13;      // the auto split aims for 1.3 waves of resident CTAs (measured best) ...
constexpr int kEqualWaveHundredths = 155;  // ... 1.55 waves when every row's pages are the same length ...
constexpr int kSmallWorkPages = 64;        // ... and 0.55 waves when the step has under 64 page-heads per
constexpr int kSmallWaveHundredths = 55;   //     CTA slot (per-CTA start and split-K rows then dominate)
constexpr int kSharedColumns = 128;  // query columns (member rows x group) per shared-prefix unit: MMA M
constexpr int kSharedCtasPerSm = 1;  // resident shared-prefix CTAs per SM (the tcgen05 kernel's smem/TMEM)
// SM time of one shared-prefix tile (128 query columns x 128 keys, a single-tile tensor-core CTA) in
// page-heads streamed by the per-sequence kernel (head_dim 128; measured on config 4: ~2 us per tile per SM
// against ~0.1 us per 8 KB page-head)
#ifndef MLB_TILE_PAGE_HEADS
#define MLB_TILE_PAGE_HEADS 19
#endif
constexpr int kTilePageHeads = MLB_TILE_PAGE_HEADS;
constexpr int kMinSharedSmPct = 25;  // the shared-prefix kernel gets at least this share of the SMs
constexpr int kMinShareSeqs = 4;     // a shared prefix is planned once only for this many decode rows ...
constexpr int kMinSharePages = 8;    // ... sharing at least this many full pages
constexpr int kPrefillMinTokens = 16;   // multi-token rows this long go to tensor-core query tiles ...
constexpr int kPrefillPiecePages = 128;  // ... split into pieces of at most this many pages (16 MMA tiles)

// The destinations of a call's final rows: its own `out`, or the caller's targets (checked).
int resolve_targets(const char* what, void* out, int64_t st, int64_t sh, const mlb_out_targets* t,
                    mlb_out_targets* r) {
  if (!t) {
    if (!out) return fail(MLB_EINVAL, "%s: null out", what);
    *r = mlb_out_targets{};
    r->num_dests = 1;
    r->stride_tok = st;
    r->stride_head = sh;
    r->dests[0] = out;
    return MLB_OK;
  }
  if (t->num_dests < 1 || t->num_dests > MLB_MAX_OUT_DESTS || t->head_offset < 0)
    return fail(MLB_EINVAL, "%s: out_targets has %d destinations (1..%d), head_offset %d", what, t->num_dests,
                MLB_MAX_OUT_DESTS, t->head_offset);
  for (int i = 0; i < t->num_dests; ++i)
    if (!t->dests[i]) return fail(MLB_EINVAL, "%s: out_targets destination %d is null", what, i);
  *r = *t;
  return MLB_OK;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// A side stream of the greatest priority and two events, per host thread and device, created on first use
// and kept for the thread's life: the shared-prefix kernel runs there beside the per-sequence kernel.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

cudaError_t side_stream(SideStream** out) {
  constexpr int kMaxDevices = 64;
  thread_local SideStream pool[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  SideStream& s = pool[dev];
  if (!s.join) {
    int least = 0, greatest = 0;
    if ((e = cudaDeviceGetStreamPriorityRange(&least, &greatest)) != cudaSuccess) return e;
    if (!s.stream && (e = cudaStreamCreateWithPriority(&s.stream, cudaStreamNonBlocking, greatest)) != cudaSuccess)
      return e;
    if (!s.fork && (e = cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming)) != cudaSuccess) return e;
    if ((e = cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming)) != cudaSuccess) return e;
  }
  *out = &s;
  return cudaSuccess;
}

struct Group {
  int seq, tile, pages;
  int start = 0;  // pages before this are planned as shared-prefix units (0: none)
  int shared_pieces = 0;
};

// Sets of decode rows whose block tables begin with the same run of block ids (shared prefix-cache blocks).
struct ShareSet {
  std::vector<int> seqs;
  int pages;  // shared pages: identical ids, full, and wholly before every member's new token
};

std::vector<ShareSet> find_shared_prefixes(const int32_t* qo, const int32_t* lens, int num_seqs, const int32_t* tables,
                                           int64_t stride, int bs) {
  // Candidates: decode rows with enough full pages before their new token.  Sorting their tables
  // lexicographically puts rows that share a long run of leading block ids next to each other; a set is a
  // maximal run whose neighbours share at least kMinSharePages pages, and it shares the run's minimum.
  std::vector<int> cand;
  std::vector<int> full(num_seqs, 0);
  for (int s = 0; s < num_seqs; ++s) {
    const int n = qo[s + 1] - qo[s];
    full[s] = (lens[s] - n) / bs;  // pages wholly before the row's new token
    if (n == 1 && full[s] >= kMinSharePages) cand.push_back(s);
  }
  auto row = [&](int s) { return tables + static_cast<int64_t>(s) * stride; };
  auto lcp = [&](int a, int b) {
    const int lim = std::min(full[a], full[b]);
    const int32_t *ra = row(a), *rb = row(b);
    int c = 0;
    while (c < lim && ra[c] == rb[c]) ++c;
    return c;
  };
  std::sort(cand.begin(), cand.end(), [&](int a, int b) {
    const int c = lcp(a, b);
    const int lim = std::min(full[a], full[b]);
    if (c < lim) return row(a)[c] < row(b)[c];
    return full[a] != full[b] ? full[a] < full[b] : a < b;
  });
  std::vector<ShareSet> sets;
  for (size_t i = 0; i < cand.size();) {
    size_t j = i + 1;
    int shared = full[cand[i]];
    while (j < cand.size()) {
      const int c = lcp(cand[j - 1], cand[j]);
      if (c < kMinSharePages) break;
      shared = std::min(shared, c);
      ++j;
    }
    if (j - i >= static_cast<size_t>(kMinShareSeqs)) {
      ShareSet set;
      set.pages = shared;
      set.seqs.assign(cand.begin() + i, cand.begin() + j);
      std::sort(set.seqs.begin(), set.seqs.end());
      sets.push_back(std::move(set));
    }
    i = j;
  }
  return sets;
}

// Enumerate (sequence, query tile) groups and the pages each must read; validates the step.
int plan_groups(const int32_t* qo, const int32_t* lens, int num_seqs, int max_blocks, int h, int hkv, int bs,
                std::vector<Group>& groups, int64_t* total_pages) {
  const int tpt = mlb::tokens_per_tile(h, hkv);
  *total_pages = 0;
  groups.clear();
  for (int s = 0; s < num_seqs; ++s) {
    const int n = qo[s + 1] - qo[s], L = lens[s];
    if (n < 0) return fail(MLB_EINVAL, "qo_indptr must be non-decreasing (sequence %d)", s);
    if (L < n) return fail(MLB_EINVAL, "sequence %d: seq_len %d < %d new tokens", s, L, n);
    if (max_blocks >= 0 && static_cast<int64_t>(L) > static_cast<int64_t>(max_blocks) * bs)
      return fail(MLB_EINVAL, "sequence %d: %d blocks can't hold %d tokens", s, max_blocks, L);
    if ((n + tpt - 1) / tpt > (1 << 20)) return fail(MLB_EINVAL, "sequence %d: %d new tokens is too many query tiles", s, n);
    for (int t = 0; t * tpt < n; ++t) {
      const int last = std::min((t + 1) * tpt, n) - 1;
      const int extent = L - n + last + 1;
      const int pages = (extent + bs - 1) / bs;
      groups.push_back({s, t, pages});
      *total_pages += pages;
    }
  }
  return MLB_OK;
}

}  // namespace

namespace mlb {
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

namespace {
std::atomic<int> g_programmatic_launch{1};
std::atomic<int> g_tensor_core_prefix{1};
std::atomic<int> g_concurrent_prefix{1};
}  // namespace
bool programmatic_launch() { return g_programmatic_launch.load(std::memory_order_relaxed) != 0; }
bool tensor_core_prefix() { return g_tensor_core_prefix.load(std::memory_order_relaxed) != 0; }
bool concurrent_prefix() { return g_concurrent_prefix.load(std::memory_order_relaxed) != 0; }
}  // namespace mlb

extern "C" {

const char* mlb_last_error(void) { return g_last_error.c_str(); }

int mlb_abi_version(void) { return 10; }

int mlb_set_programmatic_launch(int enable) {
  return mlb::g_programmatic_launch.exchange(enable ? 1 : 0, std::memory_order_relaxed);
}

int mlb_set_tensor_core_prefix(int enable) {
  return mlb::g_tensor_core_prefix.exchange(enable ? 1 : 0, std::memory_order_relaxed);
}

int mlb_set_concurrent_prefix(int enable) {
  return mlb::g_concurrent_prefix.exchange(enable ? 1 : 0, std::memory_order_relaxed);
}

int mlb_kv_append(void* k_cache, void* v_cache, int cache_dtype, int64_t num_blocks, int block_size,
                  const int64_t* slot_mapping, const void* k, int64_t k_stride_tok, int64_t k_stride_head,
                  const void* v, int64_t v_stride_tok, int64_t v_stride_head, int in_dtype, int64_t num_tokens,
                  int num_kv_heads, int head_dim, int32_t* err_word, void* stream) {
  const int ob = elt_bytes(cache_dtype), ib = elt_bytes(in_dtype);
  if (!ob || !ib) return fail(MLB_EINVAL, "kv_append: unknown dtype (cache %d, rows %d)", cache_dtype, in_dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_blocks <= 0 || block_size <= 0)
    return fail(MLB_EINVAL, "kv_append: bad sizes");
  if ((head_dim * ob) % 16 != 0)
    return fail(MLB_EUNSUPPORTED, "kv_append: head_dim * element size must be a multiple of 16 bytes");
  if (num_tokens == 0) return MLB_OK;
  if (!k_cache || !v_cache || !slot_mapping || !k || !v) return fail(MLB_EINVAL, "kv_append: null pointer");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(MLB_EINVAL, "kv_append: pools must be 16-byte aligned");
  // Wide loads need every vector of every input row aligned to the load width.
  const int in_vec = ob == ib ? 16 : 8;
  const int64_t per_vec_bytes = static_cast<int64_t>(16 / ob) * ib;
  const bool vec = aligned(k, in_vec) && aligned(v, in_vec) && per_vec_bytes % in_vec == 0 &&
                   (k_stride_tok * ib) % in_vec == 0 && (k_stride_head * ib) % in_vec == 0 &&
                   (v_stride_tok * ib) % in_vec == 0 && (v_stride_head * ib) % in_vec == 0;
  return cuda_status(mlb::launch_kv_append(k_cache, v_cache, cache_dtype, num_blocks * block_size, slot_mapping, k,
                                           k_stride_tok, k_stride_head, v, v_stride_tok, v_stride_head, in_dtype,
                                           num_tokens, num_kv_heads, head_dim, vec, err_word,
                                           static_cast<cudaStream_t>(stream)),
                     "kv_append launch");
}

int mlb_plan_attention(const int32_t* qo_indptr, const int32_t* seq_lens, int num_seqs, int max_blocks_per_seq,
                       const int32_t* block_tables_host, int64_t bt_stride_host, int num_heads, int num_kv_heads,
                       int block_size, int num_sms, int pages_per_unit, mlb_work_unit* units, int64_t units_capacity,
                       int64_t* num_units, mlb_shared_unit* shared_units, int64_t shared_capacity,
                       int64_t* num_shared_units, mlb_share_member* members, int64_t members_capacity,
                       int64_t* num_members, int32_t* reduce_rows, int32_t* reduce_chunks, int64_t num_tokens,
                       int64_t* num_partial_rows) {
  if (!qo_indptr || !seq_lens || !num_units || !num_shared_units || !num_members || !num_partial_rows ||
      num_seqs < 0)
    return fail(MLB_EINVAL, "plan: null pointer or negative sequence count");
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads)
    return fail(MLB_EINVAL, "plan: num_heads (%d) must be a positive multiple of num_kv_heads (%d)", num_heads,
                num_kv_heads);
  if (block_size <= 0 || num_sms <= 0) return fail(MLB_EINVAL, "plan: bad block_size or num_sms");
  if (num_seqs > 0 && qo_indptr[num_seqs] > num_tokens)
    return fail(MLB_EINVAL, "plan: qo_indptr ends at %d > num_tokens %lld", qo_indptr[num_seqs],
                static_cast<long long>(num_tokens));
  std::vector<Group> groups;
  int64_t total = 0;
  int rc = plan_groups(qo_indptr, seq_lens, num_seqs, max_blocks_per_seq, num_heads, num_kv_heads, block_size, groups,
                       &total);
  if (rc != MLB_OK) return rc;
  const int tpt = mlb::tokens_per_tile(num_heads, num_kv_heads);
  const int group_size = num_heads / num_kv_heads;

  // ---- multi-token rows (prefill chunks on cache) of >= kPrefillMinTokens tokens: with host tables
  // (16-bit pools) they are planned as query tiles of 128 columns below instead of 8-column groups
  std::vector<int> prefill_seqs;
  if (block_tables_host && bt_stride_host > 0) {
    std::vector<char> is_prefill(num_seqs, 0);
    for (int s = 0; s < num_seqs; ++s)
      if (qo_indptr[s + 1] - qo_indptr[s] >= kPrefillMinTokens) is_prefill[s] = 1, prefill_seqs.push_back(s);
    if (!prefill_seqs.empty())
      groups.erase(std::remove_if(groups.begin(), groups.end(), [&](const Group& g) { return is_prefill[g.seq]; }),
                   groups.end());
  }

  // ---- shared prefixes: planned once per block of member rows, cut into `pieces` page runs
  std::vector<ShareSet> sets;
  if (block_tables_host && bt_stride_host > 0)
    sets = find_shared_prefixes(qo_indptr, seq_lens, num_seqs, block_tables_host, bt_stride_host, block_size);
  std::vector<int> seq_group(num_seqs, -1);  // the (single) group of each decode row
  for (size_t g = 0; g < groups.size(); ++g)
    if (groups[g].tile == 0) seq_group[groups[g].seq] = static_cast<int>(g);
  const int per_cta = std::max(1, kSharedColumns / group_size);  // member rows per shared unit
  for (const ShareSet& set : sets)
    for (int s : set.seqs) groups[seq_group[s]].start = set.pages;  // members' own pages follow the prefix
  int64_t rest = 0;  // pages left to the per-sequence kernel
  for (const Group& g : groups) rest += g.pages - g.start;
  // The shared-prefix kernel runs beside the per-sequence kernel, one CTA per SM: it gets the share of the
  // SMs that balances the two kernels' estimated SM time (all of them when no per-sequence work is left)
  int64_t tc_work = 0;
  // a tensor-core CTA takes one member block of a shared prefix (its single-tile pipeline double-buffers S,
  // which measured faster there than two blocks per CTA)
  auto blocks_of = [&](const ShareSet& set) {
    return (static_cast<int64_t>(set.seqs.size()) + per_cta - 1) / per_cta;
  };
  for (const ShareSet& set : sets)
    tc_work += blocks_of(set) * num_kv_heads * ((set.pages + kMinPagesPerUnit - 1) / kMinPagesPerUnit) *
               kTilePageHeads;
  const int64_t priv_work = rest * num_kv_heads;
  const int64_t share_pct =
      tc_work > 0 ? std::max<int64_t>(kMinSharedSmPct, 100 * tc_work / (tc_work + priv_work)) : 100;
  struct SetPlan {
    int pieces, per;
  };
  std::vector<SetPlan> set_plans;
  for (const ShareSet& set : sets) {
    // as many pieces as keep every CTA in one wave of that share, each a whole number of 8-page (128-key)
    // tiles
    const int64_t target = std::max<int64_t>(1, static_cast<int64_t>(num_sms) * kSharedCtasPerSm * share_pct / 100);
    int64_t pieces = std::max<int64_t>(1, target / (blocks_of(set) * num_kv_heads));
    pieces = std::min<int64_t>(pieces, std::max(1, set.pages / kMinPagesPerUnit));
    int per = static_cast<int>((set.pages + pieces - 1) / pieces);
    per = (per + kMinPagesPerUnit - 1) / kMinPagesPerUnit * kMinPagesPerUnit;
    pieces = (set.pages + per - 1) / per;
    set_plans.push_back({static_cast<int>(pieces), per});
    for (int s : set.seqs) groups[seq_group[s]].shared_pieces = static_cast<int>(pieces);
  }

  // ---- regular units over each group's pages [start, pages)
  // Split size (pages per unit).  Measured on B200 with every layer's launch back to back, one rank of
  // KV-head sharding emulated on one GPU (1 / 2 / 4 / 8 KV heads):
  // - rows of varied length (config 2, 64 rows): 1.3 waves of resident CTAs is best while the work is large
  //   (8 heads: 101 us; 1.5 waves 105, 2.2 waves 108), but with under 64 page-heads per CTA slot fewer,
  //   longer units win (1 head: 0.5 waves 19.8 us against 24.3 at 1.3; 2 heads: 32.8 against 37.2);
  // - rows of one length (config 5, 29 x 8192 pages): a last wave under half full costs a whole unit time
  //   (4 heads: 1.31 waves 1358 us, 1.05 waves 1444, 1.57 waves 1190 = 1/2 of the 8-head time), so every row
  //   gets the same number of units and they fill ~1.55 waves.
  int64_t chunk = pages_per_unit;
  if (chunk <= 0) {
    const int64_t slots = static_cast<int64_t>(num_sms) * kCtasPerSm;
    const int64_t work = rest * num_kv_heads;  // page-heads left to the per-sequence kernel
    int64_t gmin = INT64_MAX, gmax = 0, ngroups = 0;
    for (const Group& g : groups) {
      const int64_t own = g.pages - g.start;
      if (own <= 0) continue;
      gmin = std::min(gmin, own);
      gmax = std::max(gmax, own);
      ++ngroups;
    }
    if (ngroups > 0 && gmax - gmin <= gmax / 64 && gmax >= 2 * kMinPagesPerUnit) {
      const int64_t want = (slots * kEqualWaveHundredths + 99) / 100;  // CTAs
      int64_t k = (want + ngroups * num_kv_heads - 1) / (ngroups * num_kv_heads);  // units per row
      k = std::max<int64_t>(1, std::min<int64_t>(k, gmax / kMinPagesPerUnit));
      chunk = (gmax + k - 1) / k;
    } else {
      const int64_t hundredths = work < slots * kSmallWorkPages ? kSmallWaveHundredths : kWaveTenths * 10;
      const int64_t target_ctas = std::max<int64_t>(1, slots * hundredths / 100);
      chunk = std::max<int64_t>(kMinPagesPerUnit, (work + target_ctas - 1) / target_ctas);
    }
  }
  std::vector<mlb_work_unit> out;
  out.reserve(groups.size());
  std::vector<int64_t> base(groups.size(), -1);
  if (reduce_rows && reduce_chunks)
    for (int64_t t = 0; t < num_tokens; ++t) reduce_rows[t] = -1, reduce_chunks[t] = 0;
  int64_t rows = 0;
  for (size_t gi = 0; gi < groups.size(); ++gi) {
    const Group& g = groups[gi];
    const int64_t own = g.pages - g.start;
    const int64_t nch = std::max<int64_t>(1, (own + chunk - 1) / chunk);
    const int64_t per = std::max<int64_t>(1, (own + nch - 1) / nch);
    const int64_t pieces = g.shared_pieces + nch;
    if (pieces > 1) base[gi] = rows, rows += pieces * tpt;
    for (int64_t c = 0; c < nch; ++c) {
      mlb_work_unit u{};
      u.seq = g.seq;
      u.q_tile = g.tile;
      u.page_begin = static_cast<int32_t>(g.start + c * per);
      u.page_end = static_cast<int32_t>(std::min<int64_t>(g.start + (c + 1) * per, g.pages));
      u.part_row = pieces > 1 ? static_cast<int32_t>(base[gi] + (g.shared_pieces + c) * tpt) : -1;
      u.q0 = qo_indptr[g.seq];
      u.num_new = qo_indptr[g.seq + 1] - qo_indptr[g.seq];
      u.seq_len = seq_lens[g.seq];
      if (u.page_end > u.page_begin) out.push_back(u);
    }
    if (reduce_rows && reduce_chunks) {
      const int n = qo_indptr[g.seq + 1] - qo_indptr[g.seq];
      for (int i = 0; i < tpt && g.tile * tpt + i < n; ++i) {
        const int64_t tok = qo_indptr[g.seq] + static_cast<int64_t>(g.tile) * tpt + i;
        reduce_rows[tok] = pieces > 1 ? static_cast<int32_t>(base[gi] + i) : -1;
        reduce_chunks[tok] = static_cast<int32_t>(pieces);
      }
    }
  }
  // ---- query tiles of the prefill rows (mlb_shared_unit of kind 1): 128 / group consecutive tokens of one
  // sequence over the keys its last token sees (causal), in pieces of <= kPrefillPiecePages pages whose
  // partial rows are token-major: row(token i, piece p) = part_base + (i * pieces + p) * tpt.  Neighbouring
  // tiles go in pairs over the later tile's keys (one tensor-core CTA takes both; the earlier tile's causal
  // limit masks the few keys it does not see); a row's last odd tile gets an empty partner.
  std::vector<std::array<mlb_shared_unit, 2>> tile_pairs;
  const int tile_tokens = std::max(1, kSharedColumns / group_size);
  for (int s : prefill_seqs) {
    const int n = qo_indptr[s + 1] - qo_indptr[s], L = seq_lens[s];
    for (int t0 = 0; t0 < n; t0 += 2 * tile_tokens) {
      const int ntok[2] = {std::min(tile_tokens, n - t0), std::max(0, std::min(tile_tokens, n - t0 - tile_tokens))};
      const int key_end = L - n + t0 + ntok[0] + ntok[1];  // keys 0 .. key_end - 1: the pair's last token
      const int pages = (key_end + block_size - 1) / block_size;
      int pieces = std::min(255, std::max(1, (pages + kPrefillPiecePages - 1) / kPrefillPiecePages));
      int per = (pages + pieces - 1) / pieces;
      per = (per + kMinPagesPerUnit - 1) / kMinPagesPerUnit * kMinPagesPerUnit;  // whole 8-page MMA tiles
      pieces = (pages + per - 1) / per;
      int64_t part_base[2] = {-1, -1};
      for (int h = 0; h < 2; ++h)
        if (pieces > 1 && ntok[h] > 0) part_base[h] = rows, rows += static_cast<int64_t>(ntok[h]) * pieces * tpt;
      for (int p = 0; p < pieces; ++p) {
        std::array<mlb_shared_unit, 2> pair{};
        for (int h = 0; h < 2; ++h) {
          mlb_shared_unit& u = pair[h];
          u.member_begin = qo_indptr[s] + t0 + h * tile_tokens;  // kind 1: the tile's first token
          u.member_count = ntok[h];
          u.page_begin = p * per;
          u.page_end = std::min(pages, (p + 1) * per);
          u.piece = pieces > 1 ? p : -1;
          u.table_seq = s;
          u.reserved[0] = 1 | (pieces << 8);
          u.reserved[1] = static_cast<int32_t>(part_base[h]);
        }
        tile_pairs.push_back(pair);
      }
      if (reduce_rows && reduce_chunks)
        for (int h = 0; h < 2; ++h)
          for (int i = 0; i < ntok[h]; ++i) {
            const int64_t tok = qo_indptr[s] + t0 + h * tile_tokens + i;
            reduce_rows[tok] =
                pieces > 1 ? static_cast<int32_t>(part_base[h] + static_cast<int64_t>(i) * pieces * tpt) : -1;
            reduce_chunks[tok] = pieces;
          }
    }
  }
  if (rows > INT32_MAX) return fail(MLB_EINVAL, "plan: too many partial rows");
  // Largest units first, so the short tail units fill in behind them.
  std::stable_sort(out.begin(), out.end(), [](const mlb_work_unit& x, const mlb_work_unit& y) {
    return (x.page_end - x.page_begin) > (y.page_end - y.page_begin);
  });

  // shared-prefix units: per piece, one member block per pair with an empty partner (a single-tile CTA);
  // every pair of units (2i, 2i + 1) covers the same pages of the same table row, and pairs are ordered
  // largest first as whole pairs
  std::vector<std::array<mlb_shared_unit, 2>> pairs;
  std::vector<mlb_share_member> mems;
  for (size_t k = 0; k < sets.size(); ++k) {
    const ShareSet& set = sets[k];
    const int first = static_cast<int>(mems.size());
    for (int s : set.seqs)
      mems.push_back({s, qo_indptr[s], static_cast<int32_t>(base[seq_group[s]]), 0});
    const int nm = static_cast<int>(set.seqs.size());
    for (int piece = 0; piece < set_plans[k].pieces; ++piece)
      for (int m = 0; m < nm; m += per_cta) {
        std::array<mlb_shared_unit, 2> pair{};
        for (int h = 0; h < 2; ++h) {
          mlb_shared_unit& u = pair[h];
          u.member_begin = first + m;
          u.member_count = h == 0 ? std::min(per_cta, nm - m) : 0;
          u.page_begin = piece * set_plans[k].per;
          u.page_end = std::min(set.pages, (piece + 1) * set_plans[k].per);
          u.piece = piece;
          u.table_seq = set.seqs[0];
        }
        pairs.push_back(pair);
      }
  }
  pairs.insert(pairs.end(), tile_pairs.begin(), tile_pairs.end());
  std::stable_sort(pairs.begin(), pairs.end(),
                   [](const std::array<mlb_shared_unit, 2>& x, const std::array<mlb_shared_unit, 2>& y) {
                     return (x[0].page_end - x[0].page_begin) > (y[0].page_end - y[0].page_begin);  // largest first
                   });
  std::vector<mlb_shared_unit> sunits;
  sunits.reserve(2 * pairs.size());
  for (const auto& pair : pairs) sunits.insert(sunits.end(), pair.begin(), pair.end());
  *num_units = static_cast<int64_t>(out.size());
  *num_shared_units = static_cast<int64_t>(sunits.size());
  *num_members = static_cast<int64_t>(mems.size());
  *num_partial_rows = rows;
  if (!units) return MLB_OK;  // count only
  if (static_cast<int64_t>(out.size()) > units_capacity || static_cast<int64_t>(sunits.size()) > shared_capacity ||
      static_cast<int64_t>(mems.size()) > members_capacity)
    return fail(MLB_ENOSPACE, "plan: output arrays too small (%zu units, %zu shared units, %zu members)", out.size(),
                sunits.size(), mems.size());
  if ((!sunits.empty() && !shared_units) || (!mems.empty() && !members))
    return fail(MLB_EINVAL, "plan: the plan has shared-prefix units but no arrays for them");
  std::copy(out.begin(), out.end(), units);
  std::copy(sunits.begin(), sunits.end(), shared_units);
  std::copy(mems.begin(), mems.end(), members);
  return MLB_OK;
}

}  // extern "C"

namespace {

// mlb_paged_attention and mlb_paged_attention_append: `app` (validated by the caller) or nullptr.
int attention_call(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* k_cache,
                   const void* v_cache, int dtype, int64_t num_blocks, int block_size, int num_heads,
                   int num_kv_heads, int head_dim, float scale, const int32_t* block_tables, int64_t bt_stride,
                   const int32_t* seq_lens, const int32_t* qo_indptr, int num_seqs, const mlb_work_unit* units,
                   int64_t num_units, const mlb_shared_unit* shared_units, int64_t num_shared_units,
                   const mlb_share_member* members, float* partial_o, float* partial_lse, int64_t num_partial_rows,
                   void* out, int64_t out_stride_tok, int64_t out_stride_head, const mlb_out_targets* out_targets,
                   const mlb_append_rows* app, int32_t* err_word, void* stream) {
  if (!elt_bytes(dtype)) return fail(MLB_EINVAL, "paged_attention: unknown dtype %d", dtype);
  if (block_size != mlb::kBlockSize)
    return fail(MLB_EUNSUPPORTED, "paged_attention: block_size %d (kernels are built for 16)", block_size);
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(MLB_EUNSUPPORTED, "paged_attention: head_dim %d (supported: 64, 128, 256)", head_dim);
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads)
    return fail(MLB_EINVAL, "paged_attention: num_heads %d not a multiple of num_kv_heads %d", num_heads,
                num_kv_heads);
  if (num_heads / num_kv_heads > 8)
    return fail(MLB_EUNSUPPORTED, "paged_attention: %d query heads per KV head (at most 8)",
                num_heads / num_kv_heads);
  if (num_units < 0 || num_shared_units < 0 || num_seqs < 0 || num_blocks <= 0)
    return fail(MLB_EINVAL, "paged_attention: bad sizes");
  if (num_units == 0 && num_shared_units == 0) return MLB_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !seq_lens || !qo_indptr || (num_units && !units))
    return fail(MLB_EINVAL, "paged_attention: null pointer");
  mlb_out_targets targets;
  if (int rc = resolve_targets("paged_attention", out, out_stride_tok, out_stride_head, out_targets, &targets))
    return rc;
  if (num_shared_units > 0 && (!shared_units || dtype == MLB_F32))  // members: only kind-0 units read them
    return fail(MLB_EINVAL, "paged_attention: query-tile units need their array and a 16-bit pool");
  if (num_shared_units % 2)
    return fail(MLB_EINVAL, "paged_attention: query-tile units come in pairs (%lld units)",
                static_cast<long long>(num_shared_units));
  if (num_partial_rows > 0 && (!partial_o || !partial_lse))
    return fail(MLB_EINVAL, "paged_attention: the plan has %lld partial rows but no workspace",
                static_cast<long long>(num_partial_rows));
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(MLB_EINVAL, "paged_attention: pools must be 16-byte aligned");
  if (num_units * num_kv_heads > INT32_MAX || num_shared_units * num_kv_heads > INT32_MAX)
    return fail(MLB_EINVAL, "paged_attention: grid too large");
  mlb::AttnArgs a{};
  a.q = static_cast<const char*>(q);
  a.q_st = q_stride_tok;
  a.q_sh = q_stride_head;
  a.k_cache = static_cast<const char*>(k_cache);
  a.v_cache = static_cast<const char*>(v_cache);
  a.num_blocks = num_blocks;
  a.h = num_heads;
  a.hkv = num_kv_heads;
  a.group = num_heads / num_kv_heads;
  a.tile_tokens = mlb::tokens_per_tile(num_heads, num_kv_heads);
  a.sl2 = scale * mlb::kLog2e;
  a.bt = block_tables;
  a.bt_stride = bt_stride;
  a.seq_lens = seq_lens;
  a.qo = qo_indptr;
  a.units = units;
  a.shared_units = shared_units;
  a.members = members;
  a.part_o = partial_o;
  a.part_lse = partial_lse;
  a.part_rows = num_partial_rows;
  a.out = targets;
  a.out_vec = mlb::out_vec_ok(targets, elt_bytes(dtype)) ? 1 : 0;
  a.err = err_word;
  if (app) {
    a.app_k = static_cast<const char*>(app->k);
    a.app_v = static_cast<const char*>(app->v);
    a.app_k_st = app->k_stride_tok;
    a.app_k_sh = app->k_stride_head;
    a.app_v_st = app->v_stride_tok;
    a.app_v_sh = app->v_stride_head;
    a.app_slots = app->slot_mapping;
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tc = num_shared_units > 0 && mlb::tensor_core_prefix() && mlb::shared_prefix_tc_supported(a, dtype, head_dim);
  auto launch_shared = [&](cudaStream_t s) {
    return tc ? mlb::launch_shared_prefix_tc(a, dtype, head_dim, num_shared_units, s)
              : mlb::launch_shared_prefix_attention(a, dtype, head_dim, num_shared_units, s);
  };
  if (num_shared_units > 0 && num_units > 0 && mlb::concurrent_prefix()) {
    // The two kernels write disjoint rows and neither reads what the other writes (a page written by the
    // fused append is private to its row, never part of a shared unit): fork the shared-prefix kernel onto
    // a high-priority side stream (its CTAs, one per SM, are placed first), run the per-sequence kernel
    // beside it on the caller's stream (it fills the free SMs and the shared kernel's tail), and join, so
    // whatever the caller queues next (the split-K reduction) waits for both.  Captures into CUDA graphs
    // as a fork and a join.
    SideStream* ss = nullptr;
    cudaError_t e = side_stream(&ss);
    if (e == cudaSuccess) e = cudaEventRecord(ss->fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ss->stream, ss->fork, 0);
    if (e != cudaSuccess) return cuda_status(e, "paged_attention: side stream fork");
    cudaError_t el = launch_shared(ss->stream);
    if (el == cudaSuccess) el = mlb::launch_paged_attention(a, dtype, head_dim, num_units, st);
    // joined whatever happened above, so a stream capture never ends with the side stream still forked
    cudaError_t ej = cudaEventRecord(ss->join, ss->stream);
    if (ej == cudaSuccess) ej = cudaStreamWaitEvent(st, ss->join, 0);
    return cuda_status(el != cudaSuccess ? el : ej, "paged_attention launch (shared-prefix kernel on a side stream)");
  }
  if (num_shared_units > 0) {
    const int rc = cuda_status(launch_shared(st), "shared-prefix attention launch");
    if (rc != MLB_OK) return rc;
  }
  if (num_units == 0) return MLB_OK;
  return cuda_status(mlb::launch_paged_attention(a, dtype, head_dim, num_units, st), "paged_attention launch");
}

}  // namespace

extern "C" {

int mlb_paged_attention(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const void* k_cache,
                        const void* v_cache, int dtype, int64_t num_blocks, int block_size, int num_heads,
                        int num_kv_heads, int head_dim, float scale, const int32_t* block_tables, int64_t bt_stride,
                        const int32_t* seq_lens, const int32_t* qo_indptr, int num_seqs, const mlb_work_unit* units,
                        int64_t num_units, const mlb_shared_unit* shared_units, int64_t num_shared_units,
                        const mlb_share_member* members, float* partial_o, float* partial_lse,
                        int64_t num_partial_rows, void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        const mlb_out_targets* out_targets, int32_t* err_word, void* stream) {
  return attention_call(q, q_stride_tok, q_stride_head, k_cache, v_cache, dtype, num_blocks, block_size, num_heads,
                        num_kv_heads, head_dim, scale, block_tables, bt_stride, seq_lens, qo_indptr, num_seqs, units,
                        num_units, shared_units, num_shared_units, members, partial_o, partial_lse, num_partial_rows,
                        out, out_stride_tok, out_stride_head, out_targets, nullptr, err_word, stream);
}

int mlb_paged_attention_append(const void* q, int64_t q_stride_tok, int64_t q_stride_head, void* k_cache,
                               void* v_cache, int dtype, int64_t num_blocks, int block_size, int num_heads,
                               int num_kv_heads, int head_dim, float scale, const int32_t* block_tables,
                               int64_t bt_stride, const int32_t* seq_lens, const int32_t* qo_indptr, int num_seqs,
                               const mlb_work_unit* units, int64_t num_units, const mlb_shared_unit* shared_units,
                               int64_t num_shared_units, const mlb_share_member* members, float* partial_o,
                               float* partial_lse, int64_t num_partial_rows, void* out, int64_t out_stride_tok,
                               int64_t out_stride_head, const mlb_out_targets* out_targets,
                               const mlb_append_rows* append, int32_t* err_word, void* stream) {
  if (!append || !append->k || !append->v || !append->slot_mapping)
    return fail(MLB_EINVAL, "paged_attention_append: null append rows");
  if (append->num_tokens < 0) return fail(MLB_EINVAL, "paged_attention_append: bad num_tokens");
  if (dtype != MLB_F16 && dtype != MLB_BF16)
    return fail(MLB_EUNSUPPORTED, "paged_attention_append: 16-bit pools only (dtype %d)", dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(MLB_EUNSUPPORTED, "paged_attention_append: head_dim %d (supported: 64, 128)", head_dim);
  if (!aligned(append->k, 16) || !aligned(append->v, 16) || (append->k_stride_tok * 2) % 16 ||
      (append->k_stride_head * 2) % 16 || (append->v_stride_tok * 2) % 16 || (append->v_stride_head * 2) % 16)
    return fail(MLB_EINVAL, "paged_attention_append: k / v rows must be 16-byte aligned");
  if (append->num_tokens == 0) append = nullptr;  // nothing new: plain attention
  return attention_call(q, q_stride_tok, q_stride_head, k_cache, v_cache, dtype, num_blocks, block_size, num_heads,
                        num_kv_heads, head_dim, scale, block_tables, bt_stride, seq_lens, qo_indptr, num_seqs, units,
                        num_units, shared_units, num_shared_units, members, partial_o, partial_lse, num_partial_rows,
                        out, out_stride_tok, out_stride_head, out_targets, append, err_word, stream);
}

int mlb_splitk_reduce(const float* partial_o, const float* partial_lse, int64_t num_partial_rows,
                      const int32_t* reduce_rows, const int32_t* reduce_chunks, int tokens_per_tile_,
                      int64_t num_tokens, int num_heads, int head_dim, void* out, int64_t out_stride_tok,
                      int64_t out_stride_head, int out_dtype, const mlb_out_targets* out_targets, void* stream) {
  if (!elt_bytes(out_dtype)) return fail(MLB_EINVAL, "splitk_reduce: unknown dtype %d", out_dtype);
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(MLB_EUNSUPPORTED, "splitk_reduce: head_dim %d", head_dim);
  if (num_tokens < 0 || num_heads <= 0 || tokens_per_tile_ <= 0) return fail(MLB_EINVAL, "splitk_reduce: bad sizes");
  if (num_tokens == 0 || num_partial_rows == 0) return MLB_OK;
  if (!partial_o || !partial_lse || !reduce_rows || !reduce_chunks)
    return fail(MLB_EINVAL, "splitk_reduce: null pointer");
  mlb_out_targets targets;
  if (int rc = resolve_targets("splitk_reduce", out, out_stride_tok, out_stride_head, out_targets, &targets))
    return rc;
  return cuda_status(mlb::launch_splitk_reduce(partial_o, partial_lse, reduce_rows, reduce_chunks, tokens_per_tile_,
                                               num_tokens, num_heads, head_dim, targets, out_dtype,
                                               static_cast<cudaStream_t>(stream)),
                     "splitk_reduce launch");
}

int mlb_splitk_reduce_gather(const float* partial_o, const float* partial_lse, int64_t num_partial_rows,
                             const int32_t* reduce_rows, const int32_t* reduce_chunks, int tokens_per_tile_,
                             int64_t num_tokens, int num_heads, int head_dim, int out_dtype,
                             const mlb_out_targets* out_targets, int self_dest, void* stream) {
  if (!elt_bytes(out_dtype)) return fail(MLB_EINVAL, "splitk_reduce_gather: unknown dtype %d", out_dtype);
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(MLB_EUNSUPPORTED, "splitk_reduce_gather: head_dim %d", head_dim);
  if (num_tokens < 0 || num_heads <= 0 || tokens_per_tile_ <= 0 || num_partial_rows < 0)
    return fail(MLB_EINVAL, "splitk_reduce_gather: bad sizes");
  if (!out_targets) return fail(MLB_EINVAL, "splitk_reduce_gather: null out_targets");
  mlb_out_targets targets;
  if (int rc = resolve_targets("splitk_reduce_gather", nullptr, 0, 0, out_targets, &targets)) return rc;
  if (self_dest < 0 || self_dest >= targets.num_dests)
    return fail(MLB_EINVAL, "splitk_reduce_gather: self_dest %d outside the %d destinations", self_dest,
                targets.num_dests);
  if (num_tokens == 0) return MLB_OK;
  if (num_partial_rows > 0 && (!partial_o || !partial_lse || !reduce_rows || !reduce_chunks))
    return fail(MLB_EINVAL, "splitk_reduce_gather: null pointer");
  return cuda_status(mlb::launch_splitk_reduce_gather(partial_o, partial_lse, reduce_rows,
                                                      num_partial_rows > 0 ? reduce_chunks : nullptr,
                                                      tokens_per_tile_, num_tokens, num_heads, head_dim, targets,
                                                      self_dest, out_dtype, static_cast<cudaStream_t>(stream)),
                     "splitk_reduce_gather launch");
}

int mlb_splitk_reduce_exchange(const float* partial_o, const float* partial_lse, int64_t num_partial_rows,
                               const int32_t* reduce_rows, const int32_t* reduce_chunks, int tokens_per_tile_,
                               int64_t num_tokens, int num_heads, int head_dim, int out_dtype, void* out,
                               int64_t out_stride_tok, int64_t out_stride_head, void* const* packets,
                               int64_t packet_capacity, int rank, int world, uint32_t* state, int64_t timeout_ns,
                               int32_t* err_word, void* stream) {
  const int eb = elt_bytes(out_dtype);
  if (!eb) return fail(MLB_EINVAL, "splitk_reduce_exchange: unknown dtype %d", out_dtype);
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(MLB_EUNSUPPORTED, "splitk_reduce_exchange: head_dim %d", head_dim);
  if (world < 1 || world > MLB_MAX_OUT_DESTS || rank < 0 || rank >= world)
    return fail(MLB_EINVAL, "splitk_reduce_exchange: rank %d of %d (1..%d ranks)", rank, world, MLB_MAX_OUT_DESTS);
  if (num_tokens < 0 || num_heads <= 0 || tokens_per_tile_ <= 0 || num_partial_rows < 0 || timeout_ns < 0)
    return fail(MLB_EINVAL, "splitk_reduce_exchange: bad sizes");
  if (num_tokens > packet_capacity)
    return fail(MLB_EINVAL, "splitk_reduce_exchange: %lld tokens > packet capacity %lld",
                static_cast<long long>(num_tokens), static_cast<long long>(packet_capacity));
  if (!out || !packets || !state) return fail(MLB_EINVAL, "splitk_reduce_exchange: null pointer");
  for (int p = 0; p < 2 * world; ++p)
    if (!packets[p]) return fail(MLB_EINVAL, "splitk_reduce_exchange: packet area %d of rank %d is null", p / world,
                                 p % world);
  // every lane moves head_dim / 32 elements as whole 32-bit words: rows 4-byte aligned
  if ((reinterpret_cast<uintptr_t>(out) | static_cast<uintptr_t>(out_stride_tok * eb) |
       static_cast<uintptr_t>(out_stride_head * eb)) & 3)
    return fail(MLB_EUNSUPPORTED, "splitk_reduce_exchange: out rows must be 4-byte aligned");
  if (num_tokens == 0) return MLB_OK;
  if (num_partial_rows > 0 && (!partial_o || !partial_lse || !reduce_rows || !reduce_chunks))
    return fail(MLB_EINVAL, "splitk_reduce_exchange: null pointer");
  return cuda_status(mlb::launch_splitk_reduce_exchange(
                         partial_o, partial_lse, reduce_rows, num_partial_rows > 0 ? reduce_chunks : nullptr,
                         tokens_per_tile_, num_tokens, num_heads, head_dim, out_dtype, out, out_stride_tok,
                         out_stride_head, packets, rank, world, state, timeout_ns > 0 ? timeout_ns : 2000000000LL,
                         err_word, sm_count(), static_cast<cudaStream_t>(stream)),
                     "splitk_reduce_exchange launch");
}

int mlb_block_copy(void* const* pools, int num_pools, int64_t num_blocks, int64_t block_bytes, const int32_t* src,
                   const int32_t* dst, int64_t num_pairs, int32_t* err_word, void* stream) {
  if (num_pools < 0 || num_pairs < 0 || num_blocks <= 0 || block_bytes <= 0)
    return fail(MLB_EINVAL, "block_copy: bad sizes");
  if (block_bytes % 16) return fail(MLB_EUNSUPPORTED, "block_copy: block_bytes must be a multiple of 16");
  if (num_pools == 0 || num_pairs == 0) return MLB_OK;
  if (!pools || !src || !dst) return fail(MLB_EINVAL, "block_copy: null pointer");
  return cuda_status(mlb::launch_block_copy(pools, num_pools, num_blocks, block_bytes, src, dst, num_pairs, err_word,
                                            sm_count(), static_cast<cudaStream_t>(stream)),
                     "block_copy launch");
}

int mlb_build_metadata(const int64_t* in, int64_t num_ids, int num_seqs, int64_t num_tokens, int64_t num_pages,
                       int width, int block_size, int64_t* out64, int32_t* out32, void* stream) {
  if (num_ids < 0 || num_seqs < 0 || num_tokens < 0 || num_pages < 0 || width < 0 || block_size <= 0)
    return fail(MLB_EINVAL, "build_metadata: bad sizes");
  if (num_tokens > INT32_MAX || num_pages > INT32_MAX)
    return fail(MLB_EINVAL, "build_metadata: more than 2^31 tokens or pages (int32 offsets)");
  if (num_seqs == 0) return MLB_OK;
  if (!in || !out64 || !out32) return fail(MLB_EINVAL, "build_metadata: null pointer");
  return cuda_status(mlb::launch_build_metadata(in, num_ids, num_seqs, num_tokens, num_pages, width, block_size, out64,
                                                out32, static_cast<cudaStream_t>(stream)),
                     "build_metadata launch");
}

}  // extern "C"

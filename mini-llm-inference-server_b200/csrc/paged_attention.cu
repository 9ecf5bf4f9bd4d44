// K2a — paged attention over block tables, split-K partials; K2b — the split-K reduction.
//
// Replaces paged_attention (src/minillm/attention/paged_torch_ref.py:40-74), which gathers every
// sequence's context into a contiguous copy and runs SDPA, and the FlashInfer decode wrapper the
// reference's CUDA backend calls (attention/flashinfer_backend.py:46).  Here the pages are read in place.
//
// Work decomposition (one CTA = one work unit x one KV head):
//   unit = (sequence, query tile, page range).  A query tile is up to 8 "columns" = (query token,
//   query head) pairs that share this KV head; a decode row of GQA group 4 is 4 columns.
//   The CTA's warps take the unit's pages round robin.  Each warp streams its pages through a private
//   ring of shared-memory slots filled with 16-byte cp.async (a page of one head = 16 K rows + 16 V rows);
//   rows are padded by 16 bytes so ldmatrix reads are free of bank conflicts.  (On B200 this load path
//   measured 6.75-6.86 TB/s for these 256-byte rows, equal to tensor-map TMA with 2 KB boxes and above
//   1-D bulk copies of single rows.)
//   Per page and warp: S^T[16 tok x 8 col] = K[16 x Dh] . Q^T (m16n8k16 MMAs, fp32 accumulate),
//   online softmax per column (exp2 domain), P^T goes back to a B fragment with movmatrix.trans, and
//   O^T[Dh x 8] += V^T . P^T.  The warps' (m, l, O) are merged through shared memory at the end.
//   A sequence split over several units writes normalised fp32 partial rows that K2b merges.
// Shared prefixes (K2s): pages that many decode rows' tables share (prefix-cache hits) are attended once per
//   block of up to 16 rows: one CTA loads each shared page into shared memory once and its 8 warps apply it
//   to 2 rows x 4 query heads each, writing partial rows that K2b merges with the rows' private pages.
// f32 pools take a CUDA-core path with the same decomposition (fp32 accuracy, 1e-5).
#include <algorithm>
#include <climits>

#include "attn_args.cuh"

namespace mlb {

// Ring shape of the 16-bit kernel (head_dim 64 / 128): warps per CTA and slots per warp.  Two slots of
// 8.5 KB per warp keep 3 CTAs resident per SM; these are the values measured best on B200.
#ifndef MLB_ATTN_STAGES
#define MLB_ATTN_STAGES 2
#endif
#ifndef MLB_ATTN_WARPS
#define MLB_ATTN_WARPS 4
#endif

namespace {

constexpr int kWarps = 4;  // warps per CTA of the f32 kernel
constexpr float kNegInf = -__builtin_huge_valf();

struct UnitInfo {
  int seq, q0, n_new, L, t0, ncols, pb, pe, part_row;
};

__device__ __forceinline__ UnitInfo unit_info(const AttnArgs& a, int unit_idx) {
  const int4* rec = reinterpret_cast<const int4*>(a.units + unit_idx);  // one 32-byte record, two loads
  const int4 x = __ldg(rec), y = __ldg(rec + 1);
  UnitInfo r;
  r.seq = x.x;
  r.t0 = x.y * a.tile_tokens;
  r.pb = x.z;
  r.pe = x.w;
  r.part_row = y.x;
  r.q0 = y.y;
  r.n_new = y.z;
  r.L = y.w;
  r.ncols = min(a.tile_tokens, r.n_new - r.t0) * a.group;
  return r;
}

// Exclusive key limit of column j: its query token sits at position L - n_new + qi and sees keys up to
// and including itself (causal, aligned to the end of the context; a decode row sees all L keys).
__device__ __forceinline__ int column_limit(const AttnArgs& a, const UnitInfo& ui, int j) {
  if (j >= ui.ncols) return 0;
  return ui.L - ui.n_new + ui.t0 + j / a.group + 1;
}

// Merge the warps' (m, l, O[col][dim]) states and write the unit's result: the final row when the unit
// covers the whole context, else a normalised fp32 partial row plus its log2-sum-exp.
template <int DH, int OUT_DT, int NW>
__device__ __forceinline__ void merge_and_store(const AttnArgs& a, const UnitInfo& ui, int kvh,
                                                const float* const* so, const float* const* sm,
                                                const float* const* sl) {
  constexpr int V = 4, DV = DH / V;  // each thread takes 4 consecutive dims of one column (16-byte reads)
  for (int idx = threadIdx.x; idx < ui.ncols * DV; idx += blockDim.x) {
    const int j = idx / DV, d = (idx % DV) * V;
    float M = kNegInf;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm[w][j]);
    float lsum = 0.f, acc[V] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = sm[w][j];
      const float e = mw == kNegInf ? 0.f : fast_exp2(mw - M);
      lsum += e * sl[w][j];
      const float4 x = *reinterpret_cast<const float4*>(so[w] + j * DH + d);
      acc[0] += e * x.x;
      acc[1] += e * x.y;
      acc[2] += e * x.z;
      acc[3] += e * x.w;
    }
    float val[V];
#pragma unroll
    for (int k = 0; k < V; ++k) val[k] = lsum > 0.f ? acc[k] / lsum : 0.f;
    const int qi = ui.t0 + j / a.group;
    const int head = kvh * a.group + j % a.group;
    if (ui.part_row < 0) {
      store_out_n<OUT_DT, V>(a.out, a.out_vec, ui.q0 + qi, head, d, val);
    } else {
      const int64_t row = ui.part_row + j / a.group;
      *reinterpret_cast<float4*>(a.part_o + (row * a.h + head) * DH + d) = make_float4(val[0], val[1], val[2], val[3]);
      if (d == 0) a.part_lse[row * a.h + head] = lsum > 0.f ? M + log2f(lsum) : kNegInf;
    }
  }
}

// One page of one KV head against up to 8 query columns (one warp): S^T = K . Q^T on m16n8k16 tensor-core
// tiles, the online-softmax update of the columns' running max m / sum l / output O^T, and O^T += V^T . P^T.
// kaddr / vaddr: this lane's ldmatrix addresses in the page's K and V tiles; tk0: token index of this lane's
// first S^T row (the second is tk0 + 8); lim0 / lim1: exclusive key limits of the lane's two columns.
template <int DT, int DH>
__device__ __forceinline__ void attend_page(uint32_t kaddr, uint32_t vaddr, const uint32_t (&qb)[DH / 16][2], int tk0,
                                            int lim0, int lim1, float sl2, float (&o)[DH / 16][4], float& m0,
                                            float& m1, float& l0, float& l1) {
  constexpr int KSTEPS = DH / 16;
  // S^T = K . Q^T, two accumulators to halve the dependent-MMA chain
  float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    uint32_t x0, x1, x2, x3;
    ldsm_x4(kaddr + ks * 32, x0, x1, x2, x3);
    mma16816<DT>((ks & 1) ? sb : sa, x0, x1, x2, x3, qb[ks][0], qb[ks][1]);
  }
  const int tk1 = tk0 + 8;
  const float x0 = tk0 < lim0 ? (sa[0] + sb[0]) * sl2 : kNegInf;
  const float x1 = tk0 < lim1 ? (sa[1] + sb[1]) * sl2 : kNegInf;
  const float x2 = tk1 < lim0 ? (sa[2] + sb[2]) * sl2 : kNegInf;
  const float x3 = tk1 < lim1 ? (sa[3] + sb[3]) * sl2 : kNegInf;
  // online softmax per column; columns j0, j1 are shared by the 8 lanes with equal lane % 4
  float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
  const float b0 = mn0 == kNegInf ? 0.f : mn0, b1 = mn1 == kNegInf ? 0.f : mn1;
  const float al0 = fast_exp2(m0 - b0), al1 = fast_exp2(m1 - b1);
  const float p0 = fast_exp2(x0 - b0), p2 = fast_exp2(x2 - b0);
  const float p1 = fast_exp2(x1 - b1), p3 = fast_exp2(x3 - b1);
  l0 = l0 * al0 + p0 + p2;
  l1 = l1 * al1 + p1 + p3;
  m0 = mn0;
  m1 = mn1;
#pragma unroll
  for (int mt = 0; mt < DH / 16; ++mt) {
    o[mt][0] *= al0;
    o[mt][1] *= al1;
    o[mt][2] *= al0;
    o[mt][3] *= al1;
  }
  // P (C layout: token rows, column pairs) -> P^T as the B operand (token = k, column = n)
  const uint32_t pb0 = movm_t(pack2<DT>(p0, p1));
  const uint32_t pb1 = movm_t(pack2<DT>(p2, p3));
#pragma unroll
  for (int mt = 0; mt < DH / 16; ++mt) {
    uint32_t y0, y1, y2, y3;
    ldsm_x4_t(vaddr + mt * 32, y0, y1, y2, y3);
    mma16816<DT>(o[mt], y0, y1, y2, y3, pb0, pb1);
  }
}

// Fused append (mlb_paged_attention_append): rows of this page that are new this step (positions
// [L - n_new, L)) are taken from the call's k / v rows, not from the pool, which need not hold them yet (the
// page's copy may have read the old slot contents).  The units of the row's last query tile also store them
// into the pools at slot_mapping; that tile's units split its pages between them, so each new (token, KV
// head) row is stored once.  Lanes take 16-byte chunks of the rows, K then V.  tok_base: key position of
// the page's first slot; slot: the page's K tile in the warp's ring (the V tile follows at TILE).
template <int DH, int ROWB, int TILE>
__device__ __forceinline__ void take_new_rows(const AttnArgs& a, const UnitInfo& ui, int kvh, uint8_t* slot,
                                              int tok_base, int lane) {
  constexpr int CH_ROW = DH * 2 / 16;
  const int new0 = ui.L - ui.n_new;
  const int r_lo = max(new0 - tok_base, 0), r_hi = min(ui.L - tok_base, kBlockSize);
  if (r_lo >= r_hi) return;  // warp-uniform
  const bool writer = ui.t0 + a.tile_tokens >= ui.n_new;
  const int64_t slot_end = a.num_blocks * kBlockSize;
  for (int e = lane; e < (r_hi - r_lo) * 2 * CH_ROW; e += 32) {
    const int r = r_lo + e / (2 * CH_ROW), kv = (e / CH_ROW) & 1, c = e % CH_ROW;
    const int64_t t = ui.q0 + (tok_base + r - new0);
    const char* src = kv ? a.app_v + (t * a.app_v_st + kvh * a.app_v_sh) * 2
                         : a.app_k + (t * a.app_k_st + kvh * a.app_k_sh) * 2;
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(src) + c);
    *reinterpret_cast<uint4*>(slot + kv * TILE + r * ROWB + c * 16) = x;
    if (writer) {
      const int64_t sl = __ldg(a.app_slots + t);
      if (sl >= 0 && sl < slot_end) {
        char* dst = const_cast<char*>(kv ? a.v_cache : a.k_cache) + (sl * a.hkv + kvh) * (DH * 2);
        reinterpret_cast<uint4*>(dst)[c] = x;
      } else if (kv == 0 && c == 0) {
        flag_error(a.err, MLB_DEV_SLOT_RANGE);
      }
    }
  }
  __syncwarp();
}

// ------------------------------------------------------------------ 16-bit pools: tensor-core tiles

// NW warps per CTA, each streaming its pages through a private ring of STAGES shared-memory slots.
template <int DT, int DH, int STAGES, int NW>
__global__ void __launch_bounds__(NW * 32) paged_attn_mma_kernel(AttnArgs a) {
  constexpr int ROWB = DH * 2 + 16;  // padded shared row: 8 consecutive rows hit 8 distinct 16B bank groups
  constexpr int TILE = 16 * ROWB;    // one page of one head, K or V
  constexpr int STAGE = 2 * TILE;
  constexpr int KSTEPS = DH / 16;
  constexpr int CH_ROW = DH * 2 / 16;         // 16-byte chunks per row
  constexpr int CH_LANE = 2 * 16 * CH_ROW / 32;  // chunks each lane copies per page (K and V)
  static_assert(8 * DH * 4 + 64 <= STAGES * STAGE, "merge state must fit in a warp's ring");
  static_assert(32 % CH_ROW == 0 || CH_ROW % 32 == 0, "row chunks must tile a warp");

  extern __shared__ __align__(128) uint8_t smem[];
  griddep_begin();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x % a.hkv;
  const UnitInfo ui = unit_info(a, blockIdx.x / a.hkv);
  uint8_t* ring = smem + warp * STAGES * STAGE;

  const int pb = ui.pb + warp;
  const int npages = pb < ui.pe ? (ui.pe - pb + NW - 1) / NW : 0;
  const int32_t* table = a.bt + static_cast<int64_t>(ui.seq) * a.bt_stride;

  // Block ids of this warp's pages, 32 at a time (lane i holds page i of the window); the next window
  // is loaded one window ahead so its latency hides behind the current one.
  auto load_window = [&](int w) -> int {
    const int i = w * 32 + lane;
    return i < npages ? __ldg(table + pb + i * NW) : 0;
  };
  int ids_cur = load_window(0), ids_nxt = load_window(1), win = 0;
  uint32_t bad_mask = 0;  // bit s: the page in slot s had a block id outside the pool

  // Copy page j (this warp's j-th) into slot j % STAGES with 16-byte cp.async: chunk e = c * 32 + lane of
  // the page's 2 x 16 rows, consecutive lanes on consecutive chunks of a row (coalesced).  Every call
  // commits one group (possibly empty) so the group count stays in step with the page count.
  const int64_t row_stride = static_cast<int64_t>(a.hkv) * DH * 2;  // bytes between tokens of one head
  auto issue = [&](int j) {
    if (j < npages) {
      if ((j >> 5) != win) {
        ++win;
        ids_cur = ids_nxt;
        ids_nxt = load_window(win + 1);
      }
      const int bid = __shfl_sync(0xffffffffu, ids_cur, j & 31);
      const int s = j % STAGES;
      const bool ok = bid >= 0 && bid < a.num_blocks;
      bad_mask = ok ? (bad_mask & ~(1u << s)) : (bad_mask | (1u << s));
      if (!ok) {
        if (lane == 0) flag_error(a.err, MLB_DEV_BLOCK_RANGE);
      } else {
        const int64_t page_off = (static_cast<int64_t>(bid) * kBlockSize * a.hkv + kvh) * (DH * 2);
        uint8_t* slot = ring + s * STAGE;
#pragma unroll
        for (int c = 0; c < CH_LANE; ++c) {
          const int e = c * 32 + lane;
          const int kv = e / (16 * CH_ROW), row = (e / CH_ROW) % 16, ch = e % CH_ROW;
          const char* src = (kv ? a.v_cache : a.k_cache) + page_off + row * row_stride + ch * 16;
          cp_async16(slot + kv * TILE + row * ROWB + ch * 16, src);
        }
      }
    }
    cp_async_commit();
  };

#pragma unroll
  for (int j = 0; j < STAGES - 1; ++j) issue(j);

  // Q^T as B fragments (column n = lane / 4, dims 2 * (lane % 4) + {0, 1} (+8)), loaded once.
  uint32_t qb[KSTEPS][2];
  {
    const int n = lane >> 2, c2 = (lane & 3) * 2;
    const bool live = n < ui.ncols;
    const int tok = ui.q0 + ui.t0 + (live ? n / a.group : 0);
    const int head = kvh * a.group + (live ? n % a.group : 0);
    const uint16_t* qrow = reinterpret_cast<const uint16_t*>(a.q) + static_cast<int64_t>(tok) * a.q_st +
                           static_cast<int64_t>(head) * a.q_sh;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      if (live) {
        const int d = ks * 16 + c2;
        qb[ks][0] = static_cast<uint32_t>(__ldg(qrow + d)) | (static_cast<uint32_t>(__ldg(qrow + d + 1)) << 16);
        qb[ks][1] = static_cast<uint32_t>(__ldg(qrow + d + 8)) | (static_cast<uint32_t>(__ldg(qrow + d + 9)) << 16);
      } else {
        qb[ks][0] = qb[ks][1] = 0u;
      }
    }
  }

  const int r0 = lane >> 2;
  const int j0 = (lane & 3) * 2, j1 = j0 + 1;
  const int lim0 = column_limit(a, ui, j0), lim1 = column_limit(a, ui, j1);
  float o[DH / 16][4];
#pragma unroll
  for (int mt = 0; mt < DH / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;

  // lane-constant parts of the ldmatrix addresses
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t k_off = ((lane & 7) + 8 * ((lane >> 3) & 1)) * ROWB + (lane >> 4) * 16;
  const uint32_t v_off = ((lane & 7) + 8 * (lane >> 4)) * ROWB + ((lane >> 3) & 1) * 16;

  for (int i = 0; i < npages; ++i) {
    issue(i + STAGES - 1);           // refill the slot page i - 1 used
    cp_async_wait<STAGES - 1>();     // this lane's copies of page i have landed
    __syncwarp();                    // ... and every other lane's
    const int s = i % STAGES;
    if (a.app_k) take_new_rows<DH, ROWB, TILE>(a, ui, kvh, ring + s * STAGE, (pb + i * NW) * kBlockSize, lane);
    if (!((bad_mask >> s) & 1u)) {
      const int tok_base = (pb + i * NW) * kBlockSize;
      uint8_t* vt = ring + s * STAGE + TILE;
      const int live_rows = ui.L - tok_base;
      if (live_rows < 16) {
        // Rows past the context end hold another request's data or junk; P is 0 there, but 0 * NaN
        // would still poison O, so clear those V rows.
        const int r_begin = live_rows < 0 ? 0 : live_rows;
        for (int e = lane; e < (16 - r_begin) * CH_ROW; e += 32) {
          const int r = r_begin + e / CH_ROW, c = e % CH_ROW;
          *reinterpret_cast<uint4*>(vt + r * ROWB + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }

      attend_page<DT, DH>(ring_u32 + s * STAGE + k_off, ring_u32 + s * STAGE + TILE + v_off, qb, tok_base + r0,
                          lim0, lim1, a.sl2, o, m0, m1, l0, l1);
    }
    __syncwarp();  // every lane is done with slot s before the next iteration refills it
  }
  cp_async_wait<0>();

#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  // Stash this warp's state in its own ring: every copy into it has landed and been consumed.
  __syncwarp();
  float* so = reinterpret_cast<float*>(ring);
  float* sm = so + 8 * DH;
  float* sl = sm + 8;
#pragma unroll
  for (int mt = 0; mt < DH / 16; ++mt) {
    const int d = mt * 16 + r0;
    so[j0 * DH + d] = o[mt][0];
    so[j1 * DH + d] = o[mt][1];
    so[j0 * DH + d + 8] = o[mt][2];
    so[j1 * DH + d + 8] = o[mt][3];
  }
  if (lane < 4) {
    sm[j0] = m0;
    sm[j1] = m1;
    sl[j0] = l0;
    sl[j1] = l1;
  }
  __syncthreads();
  const float* so_w[NW];
  const float* sm_w[NW];
  const float* sl_w[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    so_w[w] = reinterpret_cast<const float*>(smem + w * STAGES * STAGE);
    sm_w[w] = so_w[w] + 8 * DH;
    sl_w[w] = sm_w[w] + 8;
  }
  merge_and_store<DH, DT, NW>(a, ui, kvh, so_w, sm_w, sl_w);
}

// ------------------------------------------------------------------ shared prefixes (K2s)

constexpr int kSharedWarps = 8;   // warps per shared-prefix CTA (the planner sizes member blocks with it)
constexpr int kSharedStages = 4;  // CTA-wide ring slots: 3 pages in flight while one is read

// One CTA = (shared unit, KV head).  Every page of the unit's range is loaded once into a CTA-wide ring and
// read by all warps; warp w owns member rows [w * mpw, (w + 1) * mpw) of the unit (mpw = 8 / group), i.e.
// up to 8 (row, query head) columns.  Shared pages hold only tokens every member sees (no mask).  Each warp
// ends with normalised partial rows of its members for the split-K reduction.
template <int DT, int DH>
__global__ void __launch_bounds__(kSharedWarps * 32) shared_prefix_kernel(AttnArgs a) {
  constexpr int NW = kSharedWarps, S = kSharedStages;
  constexpr int ROWB = DH * 2 + 16;
  constexpr int TILE = 16 * ROWB;
  constexpr int STAGE = 2 * TILE;
  constexpr int KSTEPS = DH / 16;
  constexpr int CH_ROW = DH * 2 / 16;
  constexpr int CHUNKS = 2 * 16 * CH_ROW;  // 16-byte chunks of one page (K and V rows of one head)
  extern __shared__ __align__(128) uint8_t smem[];
  griddep_begin();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x % a.hkv;
  const int4* rec = reinterpret_cast<const int4*>(a.shared_units + blockIdx.x / a.hkv);
  const int4 x = __ldg(rec), y = __ldg(rec + 1);
  const int mb = x.x, mc = x.y, pb = x.z, pe = x.w, piece = y.x, tseq = y.y;
  // kind 0: shared prefix (members mb.., all keys visible); kind 1: query tile of sequence tseq (tokens
  // mb .. mb + mc - 1, causal keys)
  const bool tile_unit = (y.z & 0xff) == 1;
  const int tile_pieces = y.z >> 8, tile_part_base = y.w;
  const int seq_len = tile_unit ? __ldg(a.seq_lens + tseq) : INT_MAX;
  const int first_pos = tile_unit ? seq_len - (__ldg(a.qo + tseq + 1) - __ldg(a.qo + tseq)) + (mb - __ldg(a.qo + tseq))
                                  : 0;
  const bool final_rows = tile_unit && piece < 0;
  const int npages = pe - pb;
  const int32_t* table = a.bt + static_cast<int64_t>(tseq) * a.bt_stride;
  const int64_t row_stride = static_cast<int64_t>(a.hkv) * DH * 2;
  const int mpw = a.group >= 8 ? 1 : 8 / a.group;  // member rows per warp
  // A unit may hold more members than one pass covers (NW * mpw rows): the pages are walked once per
  // block of NW * mpw member rows.
  for (int sub = 0; sub * NW * mpw < mc; ++sub) {
    const int wm = sub * NW * mpw + warp * mpw;
    const int ncols = max(0, min(mpw, mc - wm)) * a.group;

    uint32_t bad_mask = 0;
    auto issue = [&](int j) {
      if (j < npages) {
        const int bid = __ldg(table + pb + j);
        const int s = j % S;
        const bool ok = bid >= 0 && bid < a.num_blocks;
        bad_mask = ok ? (bad_mask & ~(1u << s)) : (bad_mask | (1u << s));
        if (!ok) {
          if (threadIdx.x == 0) flag_error(a.err, MLB_DEV_BLOCK_RANGE);
        } else {
          const int64_t page_off = (static_cast<int64_t>(bid) * kBlockSize * a.hkv + kvh) * (DH * 2);
          uint8_t* slot = smem + s * STAGE;
          for (int e = threadIdx.x; e < CHUNKS; e += NW * 32) {
            const int kv = e / (16 * CH_ROW), row = (e / CH_ROW) % 16, ch = e % CH_ROW;
            cp_async16(slot + kv * TILE + row * ROWB + ch * 16,
                       (kv ? a.v_cache : a.k_cache) + page_off + row * row_stride + ch * 16);
          }
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < S - 1; ++j) issue(j);

    // Q^T fragments: column n = lane / 4 is member wm + n / group (its one new token), head kvh * group + n % group
    uint32_t qb[KSTEPS][2];
    {
      const int n = lane >> 2, c2 = (lane & 3) * 2;
      const bool live = n < ncols;
      const int tok = !live ? 0 : tile_unit ? mb + wm + n / a.group : __ldg(&a.members[mb + wm + n / a.group].q0);
      const int head = kvh * a.group + (live ? n % a.group : 0);
      const uint16_t* qrow = reinterpret_cast<const uint16_t*>(a.q) + static_cast<int64_t>(tok) * a.q_st +
                             static_cast<int64_t>(head) * a.q_sh;
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int d = ks * 16 + c2;
        qb[ks][0] =
            live ? static_cast<uint32_t>(__ldg(qrow + d)) | (static_cast<uint32_t>(__ldg(qrow + d + 1)) << 16) : 0u;
        qb[ks][1] =
            live ? static_cast<uint32_t>(__ldg(qrow + d + 8)) | (static_cast<uint32_t>(__ldg(qrow + d + 9)) << 16) : 0u;
      }
    }
    const int r0 = lane >> 2, j0 = (lane & 3) * 2, j1 = j0 + 1;
    const bool live0 = j0 < ncols, live1 = j1 < ncols;
    // exclusive key limits: a shared prefix is visible whole; a query tile's token sees keys up to itself
    const int lim0 = !live0 ? 0 : tile_unit ? first_pos + wm + j0 / a.group + 1 : INT_MAX;
    const int lim1 = !live1 ? 0 : tile_unit ? first_pos + wm + j1 / a.group + 1 : INT_MAX;
    float o[DH / 16][4];
#pragma unroll
    for (int mt = 0; mt < DH / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
    const uint32_t base_u32 = smem_u32(smem);
    const uint32_t k_off = ((lane & 7) + 8 * ((lane >> 3) & 1)) * ROWB + (lane >> 4) * 16;
    const uint32_t v_off = ((lane & 7) + 8 * (lane >> 4)) * ROWB + ((lane >> 3) & 1) * 16;

    for (int i = 0; i < npages; ++i) {
      issue(i + S - 1);            // refill the slot page i - 1 used (every warp left it at the last barrier)
      cp_async_wait<S - 1>();      // this thread's copies of page i have landed
      __syncthreads();             // ... and every other thread's
      const int s = i % S;
      const int key0 = (pb + i) * kBlockSize;  // key position of the page's first slot
      if (key0 + kBlockSize > seq_len) {       // the sequence's last page: zero V rows past its end (0 x NaN)
        uint8_t* vt = smem + s * STAGE + TILE;
        for (int e = threadIdx.x; e < kBlockSize * CH_ROW; e += NW * 32) {
          const int row = e / CH_ROW, ch = e % CH_ROW;
          if (key0 + row >= seq_len) *reinterpret_cast<uint4*>(vt + row * ROWB + ch * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncthreads();
      }
      if (ncols > 0 && !((bad_mask >> s) & 1u))
        attend_page<DT, DH>(base_u32 + s * STAGE + k_off, base_u32 + s * STAGE + TILE + v_off, qb,
                            tile_unit ? key0 + r0 : 0, lim0, lim1, a.sl2, o, m0, m1, l0, l1);
      __syncthreads();  // every warp is done with slot s before it is refilled
    }
    cp_async_wait<0>();

#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    // partial row of member m: members[m].part_base + piece * tokens_per_tile (its one token); of token m of
    // a split query tile: part_base + (m * pieces + piece) * tokens_per_tile
    auto part_row = [&](int m) -> int64_t {
      return tile_unit ? tile_part_base + (static_cast<int64_t>(m) * tile_pieces + piece) * a.tile_tokens
                       : __ldg(&a.members[mb + m].part_base) + static_cast<int64_t>(piece) * a.tile_tokens;
    };
    const int h0 = kvh * a.group + j0 % a.group, h1 = kvh * a.group + j1 % a.group;
    const int m0i = wm + j0 / a.group, m1i = wm + j1 / a.group;
    if (final_rows) {  // an unsplit query tile: its rows are final
#pragma unroll
      for (int mt = 0; mt < DH / 16; ++mt) {
        const int d = mt * 16 + r0;
        if (live0) {
          store_out1<DT>(a.out, mb + m0i, h0, d, o[mt][0] * inv0);
          store_out1<DT>(a.out, mb + m0i, h0, d + 8, o[mt][2] * inv0);
        }
        if (live1) {
          store_out1<DT>(a.out, mb + m1i, h1, d, o[mt][1] * inv1);
          store_out1<DT>(a.out, mb + m1i, h1, d + 8, o[mt][3] * inv1);
        }
      }
    } else {
      const int64_t slot0 = live0 ? part_row(m0i) * a.h + h0 : 0;
      const int64_t slot1 = live1 ? part_row(m1i) * a.h + h1 : 0;
#pragma unroll
      for (int mt = 0; mt < DH / 16; ++mt) {
        const int d = mt * 16 + r0;
        if (live0) {
          a.part_o[slot0 * DH + d] = o[mt][0] * inv0;
          a.part_o[slot0 * DH + d + 8] = o[mt][2] * inv0;
        }
        if (live1) {
          a.part_o[slot1 * DH + d] = o[mt][1] * inv1;
          a.part_o[slot1 * DH + d + 8] = o[mt][3] * inv1;
        }
      }
      if (r0 == 0) {
        if (live0) a.part_lse[slot0] = l0 > 0.f ? m0 + log2f(l0) : kNegInf;
        if (live1) a.part_lse[slot1] = l1 > 0.f ? m1 + log2f(l1) : kNegInf;
      }
    }
    __syncthreads();  // the ring is reused by the next block of members
  }
}

// ------------------------------------------------------------------ f32 pools: CUDA cores

template <int DH>
__global__ void __launch_bounds__(kWarps * 32) paged_attn_f32_kernel(AttnArgs a) {
  constexpr int HALF = DH / 2;
  constexpr int DPL = DH / 32;  // dims per lane in the P.V product
  constexpr int MSTRIDE = 8 * DH + 16;
  extern __shared__ __align__(128) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem);  // [8][DH]
  float* ms = qs + 8 * DH;                     // [warps][8 * DH + 16]
  griddep_begin();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x % a.hkv;
  const UnitInfo ui = unit_info(a, blockIdx.x / a.hkv);
  const float* q = reinterpret_cast<const float*>(a.q);
  for (int idx = threadIdx.x; idx < 8 * DH; idx += blockDim.x) {
    const int j = idx / DH, d = idx % DH;
    float x = 0.f;
    if (j < ui.ncols) {
      const int tok = ui.q0 + ui.t0 + j / a.group, head = kvh * a.group + j % a.group;
      x = q[static_cast<int64_t>(tok) * a.q_st + static_cast<int64_t>(head) * a.q_sh + d];
    }
    qs[idx] = x;
  }
  __syncthreads();

  int lim[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) lim[j] = column_limit(a, ui, j);
  float o[8][DPL], m[8], l[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    m[j] = kNegInf;
    l[j] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[j][i] = 0.f;
  }
  const int t = lane & 15, half = lane >> 4;
  const int32_t* table = a.bt + static_cast<int64_t>(ui.seq) * a.bt_stride;
  const float* kc = reinterpret_cast<const float*>(a.k_cache);
  const float* vc = reinterpret_cast<const float*>(a.v_cache);

  for (int page = ui.pb + warp; page < ui.pe; page += kWarps) {
    const int bid = __ldg(table + page);
    if (bid < 0 || bid >= a.num_blocks) {
      if (lane == 0) flag_error(a.err, MLB_DEV_BLOCK_RANGE);
      continue;
    }
    const int tok = page * kBlockSize + t;
    const float* krow = kc + ((static_cast<int64_t>(bid) * kBlockSize + t) * a.hkv + kvh) * DH + half * HALF;
    float sc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j] = 0.f;
#pragma unroll 4
    for (int c = 0; c < HALF; c += 4) {
      const float4 kv = __ldg(reinterpret_cast<const float4*>(krow + c));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < ui.ncols) {
          const float4 qv = *reinterpret_cast<const float4*>(qs + j * DH + half * HALF + c);
          sc[j] = fmaf(kv.x, qv.x, fmaf(kv.y, qv.y, fmaf(kv.z, qv.z, fmaf(kv.w, qv.w, sc[j]))));
        }
      }
    }
    float p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= ui.ncols) {
        p[j] = 0.f;
        continue;
      }
      const float s = sc[j] + __shfl_xor_sync(0xffffffffu, sc[j], 16);
      const float x = tok < lim[j] ? s * a.sl2 : kNegInf;
      float mx = x;
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[j], mx);
      const float b = mn == kNegInf ? 0.f : mn;
      const float al = fast_exp2(m[j] - b);
      p[j] = fast_exp2(x - b);
      float ps = p[j];
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[j] = l[j] * al + ps;
      m[j] = mn;
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[j][i] *= al;
    }
    const int live = min(kBlockSize, ui.L - page * kBlockSize);  // rows past the context end are skipped
    for (int r = 0; r < live; ++r) {
      const float* vrow = vc + ((static_cast<int64_t>(bid) * kBlockSize + r) * a.hkv + kvh) * DH;
      float vv[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) vv[i] = __ldg(vrow + lane + 32 * i);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < ui.ncols) {
          const float pj = __shfl_sync(0xffffffffu, p[j], r);
#pragma unroll
          for (int i = 0; i < DPL; ++i) o[j][i] = fmaf(pj, vv[i], o[j][i]);
        }
      }
    }
  }

  float* so = ms + warp * MSTRIDE;
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < DPL; ++i) so[j * DH + lane + 32 * i] = o[j][i];
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      so[8 * DH + j] = m[j];
      so[8 * DH + 8 + j] = l[j];
    }
  }
  __syncthreads();
  const float* so_w[kWarps];
  const float* sm_w[kWarps];
  const float* sl_w[kWarps];
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    so_w[w] = ms + w * MSTRIDE;
    sm_w[w] = so_w[w] + 8 * DH;
    sl_w[w] = sm_w[w] + 8;
  }
  merge_and_store<DH, MLB_F32, kWarps>(a, ui, kvh, so_w, sm_w, sl_w);
}

// ------------------------------------------------------------------ split-K reduction

template <int N>
__device__ __forceinline__ void load_f32(const float* p, float (&x)[N]) {
  if constexpr (N == 2) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    x[0] = v.x;
    x[1] = v.y;
  } else {
#pragma unroll
    for (int k = 0; k < N / 4; ++k) {
      const float4 v = reinterpret_cast<const float4*>(p)[k];
      x[4 * k] = v.x;
      x[4 * k + 1] = v.y;
      x[4 * k + 2] = v.z;
      x[4 * k + 3] = v.w;
    }
  }
}

// Combine the `nc` partial rows of one (token, head): lane l ends with dims [l * DPL, (l + 1) * DPL) of the
// normalised result (8- or 16-byte loads of the rows; weights 2^(lse_c - max)).
template <int DH>
__device__ __forceinline__ void reduce_token_head(const float* po, const float* plse, int64_t r0, int nc, int tpt,
                                                  int h, int head, int lane, float (&acc)[DH / 32]) {
  constexpr int DPL = DH / 32, BATCH = 4;
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  float lw = 0.f;
  if (nc <= 32) {
    // the first BATCH pieces' rows and lane c's log2-sum-exp of piece c load together (one round trip for
    // most tokens); max, weights and their sum by shuffles; further pieces then load BATCH at a time
    float x0[BATCH][DPL];
#pragma unroll
    for (int j = 0; j < BATCH; ++j)
      if (j < nc) load_f32<DPL>(po + ((r0 + static_cast<int64_t>(j) * tpt) * h + head) * DH + lane * DPL, x0[j]);
    const float lse = lane < nc ? plse[(r0 + static_cast<int64_t>(lane) * tpt) * h + head] : kNegInf;
    float M = lse;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float w_lane = (lse == kNegInf || M == kNegInf) ? 0.f : fast_exp2(lse - M);
    lw = w_lane;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const float w = __shfl_sync(0xffffffffu, w_lane, j);
      if (j < nc) {
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] = fmaf(w, x0[j][i], acc[i]);
      }
    }
    for (int c0 = BATCH; c0 < nc; c0 += BATCH) {
      float x[BATCH][DPL];
#pragma unroll
      for (int j = 0; j < BATCH; ++j)
        if (c0 + j < nc)
          load_f32<DPL>(po + ((r0 + static_cast<int64_t>(c0 + j) * tpt) * h + head) * DH + lane * DPL, x[j]);
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const float w = __shfl_sync(0xffffffffu, w_lane, (c0 + j) & 31);
        if (c0 + j < nc) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[i] = fmaf(w, x[j][i], acc[i]);
        }
      }
    }
  } else {
    float M = kNegInf;
    for (int c = lane; c < nc; c += 32) M = fmaxf(M, plse[(r0 + static_cast<int64_t>(c) * tpt) * h + head]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    for (int c = 0; c < nc; ++c) {
      const int64_t row = r0 + static_cast<int64_t>(c) * tpt;
      const float lse = plse[row * h + head];
      const float w = (lse == kNegInf || M == kNegInf) ? 0.f : fast_exp2(lse - M);
      lw += w;
      float x[DPL];
      load_f32<DPL>(po + (row * h + head) * DH + lane * DPL, x);
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = fmaf(w, x[i], acc[i]);
    }
  }
  const float inv = lw > 0.f ? 1.f / lw : 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] *= inv;
}

// One warp per (token, query head) whose sequence was split.
template <int DH, int OUT_DT>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* po, const float* plse,
                                                            const int32_t* rrows, const int32_t* rchunks, int tpt,
                                                            int64_t ntok, int h, const mlb_out_targets out,
                                                            int out_vec) {
  constexpr int DPL = DH / 32;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const bool live = wid < ntok * h;
  const int64_t tok = live ? wid / h : 0;
  const int head = static_cast<int>(wid % h);
  // The plan's reduce arrays are uploaded before the attention launch and not written by it: read them
  // before the wait, while the attention grid drains (one round trip fewer after it)
  const int nc = live ? rchunks[tok] : 0;
  const int r0 = live ? rrows[tok] : 0;
  griddep_begin();
  if (nc <= 1) return;
  float acc[DPL];
  reduce_token_head<DH>(po, plse, r0, nc, tpt, h, head, lane, acc);
  store_out_n<OUT_DT, DPL>(out, out_vec != 0, tok, head, lane * DPL, acc);
}

// The split-K reduction carrying the output all-gather: one warp per (token, query head) of this rank.
// Split tokens are reduced into every destination; unsplit tokens' rows (written by the attention kernel
// into destination `self` only) are copied from there to the others.  No fence here: the barrier kernel
// that follows on the stream orders these stores before its flags (a per-CTA system-scope fence measured
// ~12 us slower per launch than the kernel boundary).
template <int DH, int OUT_DT>
__global__ void __launch_bounds__(256) splitk_reduce_gather_kernel(const float* po, const float* plse,
                                                                   const int32_t* rrows, const int32_t* rchunks,
                                                                   int tpt, int64_t ntok, int h,
                                                                   const mlb_out_targets out, int out_vec,
                                                                   int self) {
  constexpr int DPL = DH / 32;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const bool live = wid < ntok * h;
  const int64_t tok = live ? wid / h : 0;
  const int head = static_cast<int>(wid % h);
  const int nc = live && rchunks ? rchunks[tok] : 1;  // plan arrays: read before the wait, as above
  const int r0 = live && rchunks ? rrows[tok] : 0;
  griddep_begin();
  if (!live) return;
  if (nc > 1) {
    float acc[DPL];
    reduce_token_head<DH>(po, plse, r0, nc, tpt, h, head, lane, acc);
    store_out_n<OUT_DT, DPL>(out, out_vec != 0, tok, head, lane * DPL, acc);
  } else {
    copy_out_n<OUT_DT, DPL>(out, out_vec != 0, self, tok, head, lane * DPL);
  }
}

// The split-K reduction carrying the output all-gather as flagged packets, with no barrier kernel after
// it.  Every 32-bit word of a row travels to each peer as one 64-bit packet {word, epoch}, stored with
// one single-copy-atomic 8-byte store, so a receiver that reads the packet with the current epoch holds
// that word: no fence, no flag round trip.  Phase 1 (send): one warp per (token, head of this rank),
// grid-stride: finish the row (reduce a split token, or read the unsplit row the attention kernel left
// in this rank's own buffer) and store its packets into every peer's packet area.  Phase 2 (receive): the
// same warp waits (bounded) for the packets of the same (token, head index) from every peer in this
// rank's area and writes those rows into its own buffer.  The grid is at most one CTA per SM, so every
// CTA is resident and all ranks' warps make progress.  The epoch (state[0]) is read by every CTA first
// and advanced by the last CTA to finish (state[1] counts arrivals).  Calls alternate between two packet
// areas by the epoch's parity: a peer may still be reading the area of the call before (a rank finishes a
// call once it holds every peer's rows, not once every peer holds its), never the one of two calls back.
struct ExchangeArgs {
  const float* po;
  const float* plse;
  const int32_t* rrows;
  const int32_t* rchunks;
  int tpt, h, rank, world;
  int64_t ntok;
  char* out;  // this rank's gathered rows [ntok, world * h, DH] (element strides below)
  int64_t out_st, out_sh;
  uint64_t* packets[2][MLB_MAX_OUT_DESTS];  // area a of rank p: [ntok][world][h][row words]
  uint32_t* state;                       // this rank's {epoch, arrivals}
  int64_t timeout_ns;
  int32_t* err;
};

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <int DH, int OUT_DT>
__global__ void __launch_bounds__(256) splitk_reduce_exchange_kernel(const ExchangeArgs x) {
  constexpr int EB = Elt<OUT_DT>::bytes;
  constexpr int DPL = DH / 32;       // output elements per lane
  constexpr int WPL = DPL * EB / 4;  // 32-bit words per lane
  constexpr int WPR = 32 * WPL;      // words per row
  griddep_begin();
  const uint32_t e = *reinterpret_cast<volatile const uint32_t*>(x.state) + 1u;
  const int area = static_cast<int>(e & 1u);
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t items = x.ntok * x.h;
  auto row_at = [&](int64_t tok, int head) {
    return x.out + (tok * x.out_st + static_cast<int64_t>(head) * x.out_sh + lane * DPL) * EB;
  };
  for (int64_t it = warp0; it < items; it += nwarps) {
    const int64_t tok = it / x.h;
    const int hl = static_cast<int>(it % x.h);
    char* row = row_at(tok, x.rank * x.h + hl);
    uint32_t w[WPL];
    const int nc = x.rchunks ? x.rchunks[tok] : 1;
    if (nc > 1) {
      float acc[DPL];
      reduce_token_head<DH>(x.po, x.plse, x.rrows[tok], nc, x.tpt, x.h, hl, lane, acc);
      if constexpr (OUT_DT == MLB_F32) {
#pragma unroll
        for (int k = 0; k < DPL; ++k) w[k] = __float_as_uint(acc[k]);
      } else {
#pragma unroll
        for (int k = 0; k < DPL / 2; ++k) {
          const uint32_t lo = OUT_DT == MLB_BF16 ? f32_to_bf16_bits(acc[2 * k]) : f32_to_f16_bits(acc[2 * k]);
          const uint32_t hi = OUT_DT == MLB_BF16 ? f32_to_bf16_bits(acc[2 * k + 1]) : f32_to_f16_bits(acc[2 * k + 1]);
          w[k] = lo | (hi << 16);
        }
      }
      store_bytes<DPL * EB>(row, w);
    } else {
      load_bytes<DPL * EB>(row, w);
    }
    const int64_t at = ((tok * x.world + x.rank) * x.h + hl) * WPR + lane * WPL;
#pragma unroll
    for (int p = 0; p < MLB_MAX_OUT_DESTS; ++p) {
      if (p >= x.world || p == x.rank) continue;
#pragma unroll
      for (int i = 0; i < WPL; ++i)
        st_relaxed_sys_u64(x.packets[area][p] + at + i, (static_cast<uint64_t>(e) << 32) | w[i]);
    }
  }
  // receive: one deadline for the whole phase, so a missing peer costs one timeout, not one per row
  const uint64_t* mine = nullptr;
#pragma unroll
  for (int p = 0; p < MLB_MAX_OUT_DESTS; ++p)
    if (p == x.rank) mine = x.packets[area][p];
  const uint64_t deadline = globaltimer_ns() + static_cast<uint64_t>(x.timeout_ns);
  bool late = false;
  for (int64_t it = warp0; it < items && !late; it += nwarps) {
    const int64_t tok = it / x.h;
    const int hl = static_cast<int>(it % x.h);
    for (int p = 0; p < x.world && !late; ++p) {
      if (p == x.rank) continue;
      const uint64_t* src = mine + ((tok * x.world + p) * x.h + hl) * WPR + lane * WPL;
      uint32_t w[WPL];
#pragma unroll
      for (int i = 0; i < WPL; ++i) {
        uint64_t v = ld_relaxed_sys_u64(src + i);
        for (uint32_t polls = 1; static_cast<uint32_t>(v >> 32) != e; ++polls) {
          if ((polls & 63) == 0 && (globaltimer_ns() > deadline || polls >= (1u << 26))) {
            late = true;
            break;
          }
          v = ld_relaxed_sys_u64(src + i);
        }
        w[i] = static_cast<uint32_t>(v);
      }
      if (!late) store_bytes<DPL * EB>(row_at(tok, p * x.h + hl), w);
    }
  }
  if (late) flag_error(x.err, MLB_DEV_WAIT_TIMEOUT);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(x.state + 1, 1u) == gridDim.x - 1) {  // every CTA has read the epoch
      x.state[1] = 0u;
      x.state[0] = e;
      __threadfence();
    }
  }
}

// Opt in to > 48 KB of dynamic shared memory once per kernel instance and device (`done` is the
// caller's per-instance bit set of device ordinals < 64).
template <typename K>
cudaError_t set_smem(K kernel, int bytes, unsigned long long& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && (done >> dev) & 1ull) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev < 64) __atomic_fetch_or(&done, 1ull << dev, __ATOMIC_RELAXED);
  return e;
}

template <int DT, int DH, int STAGES, int NW>
cudaError_t launch_mma(const AttnArgs& a, int64_t ctas, cudaStream_t s) {
  constexpr int bytes = NW * STAGES * 2 * 16 * (DH * 2 + 16);
  static unsigned long long done = 0;
  auto k = paged_attn_mma_kernel<DT, DH, STAGES, NW>;
  cudaError_t e = set_smem(k, bytes, done);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(static_cast<unsigned>(ctas)), dim3(NW * 32), bytes, s, a);
}

template <int DH>
cudaError_t launch_f32(const AttnArgs& a, int64_t ctas, cudaStream_t s) {
  constexpr int bytes = (8 * DH + kWarps * (8 * DH + 16)) * 4;
  static unsigned long long done = 0;
  auto k = paged_attn_f32_kernel<DH>;
  cudaError_t e = set_smem(k, bytes, done);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(static_cast<unsigned>(ctas)), dim3(kWarps * 32), bytes, s, a);
}

template <int DT, int DH>
cudaError_t launch_shared(const AttnArgs& a, int64_t units, cudaStream_t s) {
  constexpr int bytes = kSharedStages * 2 * 16 * (DH * 2 + 16);
  static unsigned long long done = 0;
  auto k = shared_prefix_kernel<DT, DH>;
  cudaError_t e = set_smem(k, bytes, done);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(static_cast<unsigned>(units * a.hkv)), dim3(kSharedWarps * 32), bytes, s, a);
}

}  // namespace

cudaError_t launch_shared_prefix_attention(const AttnArgs& a, int dtype, int dh, int64_t num_units, cudaStream_t s) {
  if (dtype == MLB_BF16) {
    if (dh == 64) return launch_shared<MLB_BF16, 64>(a, num_units, s);
    if (dh == 128) return launch_shared<MLB_BF16, 128>(a, num_units, s);
    if (dh == 256) return launch_shared<MLB_BF16, 256>(a, num_units, s);
  } else if (dtype == MLB_F16) {
    if (dh == 64) return launch_shared<MLB_F16, 64>(a, num_units, s);
    if (dh == 128) return launch_shared<MLB_F16, 128>(a, num_units, s);
    if (dh == 256) return launch_shared<MLB_F16, 256>(a, num_units, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_paged_attention(const AttnArgs& a, int dtype, int dh, int64_t num_units, cudaStream_t s) {
  const int64_t ctas = num_units * a.hkv;
  if (dtype == MLB_BF16) {
    if (dh == 64) return launch_mma<MLB_BF16, 64, MLB_ATTN_STAGES, MLB_ATTN_WARPS>(a, ctas, s);
    if (dh == 128) return launch_mma<MLB_BF16, 128, MLB_ATTN_STAGES, MLB_ATTN_WARPS>(a, ctas, s);
    if (dh == 256) return launch_mma<MLB_BF16, 256, 2, 4>(a, ctas, s);
  } else if (dtype == MLB_F16) {
    if (dh == 64) return launch_mma<MLB_F16, 64, MLB_ATTN_STAGES, MLB_ATTN_WARPS>(a, ctas, s);
    if (dh == 128) return launch_mma<MLB_F16, 128, MLB_ATTN_STAGES, MLB_ATTN_WARPS>(a, ctas, s);
    if (dh == 256) return launch_mma<MLB_F16, 256, 2, 4>(a, ctas, s);
  } else if (dtype == MLB_F32) {
    if (dh == 64) return launch_f32<64>(a, ctas, s);
    if (dh == 128) return launch_f32<128>(a, ctas, s);
    if (dh == 256) return launch_f32<256>(a, ctas, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_splitk_reduce(const float* po, const float* plse, const int32_t* rrows, const int32_t* rchunks,
                                 int tpt, int64_t ntok, int h, int dh, const mlb_out_targets& out,
                                 int out_dtype, cudaStream_t s) {
  const int64_t warps = ntok * h;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  const int vec = out_vec_ok(out, out_dtype == MLB_F32 ? 4 : 2) ? 1 : 0;
#define MLB_RED(D, O)                                                                                    \
  if (dh == D && out_dtype == O) {                                                                       \
    return launch_k(splitk_reduce_kernel<D, O>, dim3(blocks), dim3(256), 0, s, po, plse, rrows, rchunks, tpt, \
                    ntok, h, out, vec);                                                                  \
  }
  MLB_RED(64, MLB_F32) MLB_RED(64, MLB_F16) MLB_RED(64, MLB_BF16)
  MLB_RED(128, MLB_F32) MLB_RED(128, MLB_F16) MLB_RED(128, MLB_BF16)
  MLB_RED(256, MLB_F32) MLB_RED(256, MLB_F16) MLB_RED(256, MLB_BF16)
#undef MLB_RED
  return cudaErrorInvalidValue;
}

cudaError_t launch_splitk_reduce_gather(const float* po, const float* plse, const int32_t* rrows,
                                        const int32_t* rchunks, int tpt, int64_t ntok, int h, int dh,
                                        const mlb_out_targets& out, int self, int out_dtype, cudaStream_t s) {
  const int64_t warps = ntok * h;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  const int vec = out_vec_ok(out, out_dtype == MLB_F32 ? 4 : 2) ? 1 : 0;
#define MLB_REDG(D, O)                                                                                          \
  if (dh == D && out_dtype == O)                                                                                \
    return launch_k(splitk_reduce_gather_kernel<D, O>, dim3(blocks), dim3(256), 0, s, po, plse, rrows, rchunks, \
                    tpt, ntok, h, out, vec, self);
  MLB_REDG(64, MLB_F32) MLB_REDG(64, MLB_F16) MLB_REDG(64, MLB_BF16)
  MLB_REDG(128, MLB_F32) MLB_REDG(128, MLB_F16) MLB_REDG(128, MLB_BF16)
  MLB_REDG(256, MLB_F32) MLB_REDG(256, MLB_F16) MLB_REDG(256, MLB_BF16)
#undef MLB_REDG
  return cudaErrorInvalidValue;
}

cudaError_t launch_splitk_reduce_exchange(const float* po, const float* plse, const int32_t* rrows,
                                          const int32_t* rchunks, int tpt, int64_t ntok, int h, int dh, int out_dtype,
                                          void* out, int64_t out_st, int64_t out_sh, void* const* packets, int rank,
                                          int world, uint32_t* state, int64_t timeout_ns, int32_t* err, int num_sms,
                                          cudaStream_t s) {
  ExchangeArgs x{};
  x.po = po;
  x.plse = plse;
  x.rrows = rrows;
  x.rchunks = rchunks;
  x.tpt = tpt;
  x.h = h;
  x.rank = rank;
  x.world = world;
  x.ntok = ntok;
  x.out = static_cast<char*>(out);
  x.out_st = out_st;
  x.out_sh = out_sh;
  for (int a = 0; a < 2; ++a)
    for (int p = 0; p < world; ++p) x.packets[a][p] = static_cast<uint64_t*>(packets[a * world + p]);
  x.state = state;
  x.timeout_ns = timeout_ns;
  x.err = err;
  // one warp per (token, head) up to one CTA per SM: every CTA resident at once
  const int64_t ctas = (ntok * h + 7) / 8;
  const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ctas, num_sms)));
#define MLB_EXCH(D, O) \
  if (dh == D && out_dtype == O) return launch_k(splitk_reduce_exchange_kernel<D, O>, dim3(blocks), dim3(256), 0, s, x);
  MLB_EXCH(64, MLB_F32) MLB_EXCH(64, MLB_F16) MLB_EXCH(64, MLB_BF16)
  MLB_EXCH(128, MLB_F32) MLB_EXCH(128, MLB_F16) MLB_EXCH(128, MLB_BF16)
  MLB_EXCH(256, MLB_F32) MLB_EXCH(256, MLB_F16) MLB_EXCH(256, MLB_BF16)
#undef MLB_EXCH
  return cudaErrorInvalidValue;
}

}  // namespace mlb

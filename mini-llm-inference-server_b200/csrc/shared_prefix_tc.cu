// K2s on the 5th-generation tensor cores: shared-prefix (cascade) attention and prefill query tiles with
// tcgen05.mma, TMEM accumulators and an mbarrier pipeline.
//
// A unit is up to 128 query columns of one KV head over a run of pages: a shared prefix that every member
// row's block table holds (kind 0, 128 / group member rows, every key visible), or consecutive tokens of one
// multi-token row (kind 1, causal keys).  That is a small FlashAttention forward: S = Q . K^T over the pages,
// online softmax, O = P . V, with M = 128 query columns (the TMEM lanes) and 128 keys (8 pages) per tile.
//
// A CTA takes a PAIR of units over the same pages (the planner makes them: two neighbouring query tiles of
// one row over the later tile's keys), so every K / V tile is loaded once for 256 query columns and two
// softmax warpgroups work side by side, or a SINGLE unit (a shared prefix's member block), whose scores are
// triple-buffered in TMEM so the tensor core computes the next two tiles' scores while the softmax works.
//
// Roles in one CTA of 384 threads (1 CTA per SM: two Q tiles + 3 K and 2 V stages (Dh 128) or 4 + 4 (Dh 64)
// of shared memory, all 512 TMEM columns):
// - warp 0 fills the K ring and warp 2 the V ring (one lane per page; warp 3 idles).  Each page of a tile is
//   Dh/64 TMA boxes (tensor maps over the K and V pools: {64 dims, 1 KV head, 16 slots}, 128-byte swizzle),
//   landing in the K-major layout the MMA reads ([Dh/64][128 rows][64]); the stage's "full" barrier counts
//   the bytes (expect_tx).  With a warp per ring a K tile never waits behind a V slot.  A block id out of
//   range gets a slot coordinate past the pool's end: TMA fills zeros there and the softmax masks the page.
//   No multicast.
// - warp 1, one thread: the MMA issuer.  Paired, per tile j and query tile x (A, then B): O_x += P_x(j) . V_j
//   with P read from TMEM (A operand) and V as an MN-major B operand (one k-step of 16 keys per loaded page,
//   so pages past the unit's end are never read), then S_x(j+1) = Q_x . K_{j+1}^T, committed to s_full[x].
//   Single: S(0), S(1), then per tile j: O += P(j) . V_j and S(j+2) into the buffer P(j-1) held.
// - warps 4-7 (tile A) and 8-11 (tile B), one thread = one query column = one TMEM lane: the whole S row
//   comes out of TMEM in one go (4 loads, one wait) for the masked max (exp2 domain), and P = 2^(s - m),
//   packed to 16 bits, goes back over the first 64 columns of the same S buffer; row sums in fp32.  The 128
//   scores per thread need more than the 168 registers 384 threads get at launch: warps 0-3 give theirs up
//   (setmaxnreg.dec to 56) and the softmax warps take them (setmaxnreg.inc to 224).  O is rescaled (TMEM load /
//   scale / store) only when a row's max grows by more than 8 (a factor 256 of headroom keeps P and the
//   sums finite), which after the first tiles is rare; the rescale first waits for the P . V products
//   before it.  At the end (the "final" barrier, committed behind the last MMA) every column's normalised O
//   row and log2-sum-exp go to its split-K partial row, merged by the reduction (an unsplit query tile
//   stores its final rows).
// TMEM columns, paired: S_A [0,128), S_B [128,256), O_A [256, 256 + Dh), O_B [256 + Dh, 256 + 2 Dh);
// single: S buffers [0,128), [128,256), [256,384), O [384, 384 + Dh).
//
// Every wait is bounded (time and polls); on expiry the CTA raises MLB_DEV_WAIT_TIMEOUT, drains its own
// copies and MMAs, frees TMEM and returns.
#include <cuda.h>

#include <climits>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>

#include "attn_args.cuh"

namespace mlb {

namespace {

constexpr int kTcThreads = 384;     // 12 warps: 3 producers, the MMA issuer, two softmax warpgroups
constexpr int kTcRows = 128;        // query columns per tile = MMA M = TMEM lanes
constexpr int kTcTileTokens = 128;  // keys per tile = N of S = Q . K^T
constexpr int kTcTilePages = kTcTileTokens / kBlockSize;
constexpr uint32_t kTmemCols = 512;
// registers per thread: at launch (384 threads on one SM), after the split for warps 0-3 and for the softmax
constexpr int kRegsLaunch = 168, kRegsLow = 56, kRegsHigh = 224;
static_assert(128 * (kRegsLaunch - kRegsLow) == 256 * (kRegsHigh - kRegsLaunch), "the split must balance");
static_assert(kRegsLaunch * kTcThreads <= 65536, "one CTA per SM");
// TMEM columns: S_A [0,128), S_B [128,256), O_A [256, 256 + Dh), O_B after it; P_x (16-bit pairs) over the
// first 64 columns of S_x
__device__ __forceinline__ uint32_t col_s(int x) { return x ? 128u : 0u; }
// a single-tile CTA: S buffers b = 0, 1, 2 at [128 b, 128 b + 128), O at [384, 384 + Dh)
constexpr uint32_t kSingleO = 384;
template <int DH>
__device__ __forceinline__ uint32_t col_o(int x) {
  return 256u + (x ? static_cast<uint32_t>(DH) : 0u);
}
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

template <int DH>
struct TcLayout {
  // K and V tiles in separate rings beside the two Q tiles: a K tile is free once both S products of its
  // key tile are done, well before the V tile (both P . V products), so K runs further ahead
  static constexpr int kKStages = DH == 128 ? 3 : 4;
  static constexpr int kVStages = DH == 128 ? 2 : 4;
  static constexpr int kTileBytes = kTcTileTokens * DH * 2;  // one K or V tile, [DH/64][128][64] swizzled
  static constexpr int kQBytes = kTcRows * DH * 2;           // one query tile
  static constexpr int kKOffset = 2 * kQBytes;
  static constexpr int kVOffset = kKOffset + kKStages * kTileBytes;
  static constexpr int kBarOffset = kVOffset + kVStages * kTileBytes;
  // barriers: kfull[KS], kempty[KS], vfull[VS], vempty[VS], s_full[3], p_full[3], final, q_ready, o_done;
  // then the TMEM base and the abort flag
  static constexpr int kNumBars = 2 * kKStages + 2 * kVStages + 9;
  static constexpr int kBytes = kBarOffset + 8 * kNumBars + 16;
  static constexpr int kLaunchBytes = kBytes + 1024;  // slack to align the base to 1024 (swizzle atoms)
};

// ---------------------------------------------------------------- tcgen05 / proxy wrappers

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// One tiled TMA box (this GPU's memory, no multicast) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm100 version 1.  Addresses and
// offsets in bytes (multiples of 16).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator, A and B of one 16-bit type (fmt 0 = f16,
// 1 = bf16), A K-major, B K-major or MN-major, shape M x N.
__host__ __device__ constexpr uint32_t f16_idesc(uint32_t fmt, bool b_mn_major, int m, int n) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns (this warp's lane quarter)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%"
      "18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The compiler takes a tcgen05.ld's destination registers as written by the ld itself, so arithmetic on them
// may be scheduled above tcgen05.wait::ld (the wait's memory clobber orders memory, not registers).  This
// empty asm "rewrites" the 32 registers after the wait (volatile asms keep their order), which pins every use.
__device__ __forceinline__ void tmem_pin32(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded wait on an mbarrier phase; gives up (and tells the CTA to stop) when another role aborted or
// after kWaitLimitNs.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  *abort_flag = 1;
  flag_error(err, MLB_DEV_WAIT_TIMEOUT);
  return false;
}

// Bounded wait that ignores the abort flag (draining this CTA's own MMAs before TMEM is freed).
__device__ __forceinline__ bool tc_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  return false;
}

// Byte offset of 16-byte chunk c (of a DH x 2-byte row) of row r in a [DH/64][128][64] swizzled tile.
__device__ __forceinline__ uint32_t sw_chunk(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * (kTcRows * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int DT, int DH>
__global__ void __launch_bounds__(kTcThreads, 1) shared_prefix_tc_kernel(AttnArgs a, const __grid_constant__ CUtensorMap tk,
                                                                          const __grid_constant__ CUtensorMap tv) {
  using L = TcLayout<DH>;
  constexpr int NK = L::kKStages, NV = L::kVStages;
  constexpr int CH = DH * 2 / 16;  // 16-byte chunks per row
  constexpr uint32_t kFmt = DT == MLB_BF16 ? 1u : 0u;
  constexpr uint32_t kIdescS = f16_idesc(kFmt, false, kTcRows, kTcTileTokens);
  constexpr uint32_t kIdescO = f16_idesc(kFmt, true, kTcRows, DH);
  constexpr float kNegInfF = -__builtin_huge_valf();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* kfull = bars;                   // [NK] a K stage has landed
  uint64_t* kempty = bars + NK;             // [NK] both S products reading the K stage have completed
  uint64_t* vfull = bars + 2 * NK;          // [NV] a V stage has landed
  uint64_t* vempty = bars + 2 * NK + NV;    // [NV] both P . V products reading the V stage have completed
  uint64_t* s_full = bars + 2 * (NK + NV);  // [3] an S buffer holds its tile's scores (paired: S_x, x < 2)
  uint64_t* p_full = s_full + 3;            // [3] P written over that buffer (128 softmax threads)
  uint64_t* final_bar = s_full + 6;         // every MMA of the CTA has completed
  uint64_t* q_ready = s_full + 7;           // both Q tiles are in shared memory (256 softmax threads)
  uint64_t* o_done = s_full + 8;            // single-tile CTA: the P . V products of a tile have completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + L::kNumBars) + 1;
  const uint32_t q_smem = smem_u32(smem);  // Q_A, then Q_B
  const uint32_t k_smem = q_smem + L::kKOffset, v_smem = q_smem + L::kVOffset;

  griddep_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x % a.hkv;
  // the CTA's pair of units: 2 * pair (tile A) and 2 * pair + 1 (tile B) share the page range, the table row
  // and the kind; a B without members leaves the CTA one tile
  const int4* rec = reinterpret_cast<const int4*>(a.shared_units + 2 * (blockIdx.x / a.hkv));
  const int4 xa = __ldg(rec), ya = __ldg(rec + 1), xb = __ldg(rec + 2), yb = __ldg(rec + 3);
  const int pb = xa.z, pe = xa.w, tseq = ya.y;
  // kind 0: a shared prefix, members mb .. mb + mc - 1 (one decode token each), every key visible.
  // kind 1: a query tile of sequence tseq: mc consecutive tokens from token mb, causal keys.
  const bool tile_unit = (ya.z & 0xff) == 1;
  bool two = xb.y > 0;
  if (two && (xb.z != pb || xb.w != pe || yb.y != tseq || (yb.z & 0xff) != (ya.z & 0xff) || yb.x != ya.x)) {
    two = false;  // a pair the planner would not make: tile B is left out and the plan flagged
    if (threadIdx.x == 0) flag_error(a.err, MLB_DEV_BLOCK_RANGE);
  }
  const int npages = pe - pb;
  const int ntiles = (npages + kTcTilePages - 1) / kTcTilePages;
  const int32_t* table = a.bt + static_cast<int64_t>(tseq) * a.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NK; ++s) {
      mbar_init(kfull + s, 1);
      mbar_init(kempty + s, 1);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(vfull + s, 1);
      mbar_init(vempty + s, 1);
    }
    for (int b = 0; b < 3; ++b) {
      mbar_init(s_full + b, 1);
      mbar_init(p_full + b, 128);
    }
    mbar_init(final_bar, 1);
    mbar_init(q_ready, 256);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the whole warp allocates TMEM; the address lands in shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Register split: the producer / MMA warpgroup (warps 0-3) drops to kRegsLow, the two softmax warpgroups
  // take what it frees (kRegsHigh each).  The launch gives every thread kRegsLaunch (checked on the host
  // against the compiled kernel before any launch), so 128 x (launch - low) = 256 x (high - launch) exactly.
  if (warp < 4) {
    // warpgroup 0 gives up registers, all four warps at the same instruction
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (warp != 1) {
      // ------------------------------------------------------------ producers: warp 0 fills the K ring,
      // warp 2 the V ring (warp 3 has no role), so a K tile never queues behind a V slot: the K ring runs up
      // to kKStages tiles ahead of the scores while V stages wait for their P . V products.  Lane p loads
      // page p's block id one tile ahead (the table round trip overlaps the previous tile) and issues the
      // page's Dh/64 boxes; lane 0 declares the tile's bytes on the stage barrier (one arrival per phase).
      if (warp != 3) {
        constexpr uint32_t kBoxBytes = 64 * 2 * kBlockSize;  // {64 dims, 1 head, 16 slots}
        constexpr int kHalves = DH / 64;
        const bool is_v = warp == 2;
        const int stages = is_v ? NV : NK;
        uint64_t* full = is_v ? vfull : kfull;
        uint64_t* empty = is_v ? vempty : kempty;
        const uint32_t ring = is_v ? v_smem : k_smem;
        const CUtensorMap* map = is_v ? &tv : &tk;
        const int oob_slot = static_cast<int>(a.num_blocks * kBlockSize);  // past the end: zero fill
        auto load_bid = [&](int j) {
          const int page = j * kTcTilePages + lane;
          return lane < kTcTilePages && page < npages ? __ldg(table + pb + page) : 0;
        };
        int bid = load_bid(0);
        for (int j = 0; j < ntiles; ++j) {
          const int st = j % stages;
          const int live_pages = min(kTcTilePages, npages - j * kTcTilePages);
          const uint32_t bytes = static_cast<uint32_t>(live_pages) * kHalves * kBoxBytes;
          const int next = load_bid(j + 1);
          int slot = oob_slot;
          if (lane < live_pages) {
            if (bid >= 0 && bid < a.num_blocks)
              slot = bid * kBlockSize;
            else
              flag_error(a.err, MLB_DEV_BLOCK_RANGE);
          }
          if (j >= stages) {  // the warp waits for the ring slot on lane 0 and follows it (uniform exit)
            int ok = 1;
            if (lane == 0) ok = tc_wait(empty + st, ((j / stages) + 1) & 1, abort_flag, a.err) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok, 0) == 0) break;
          }
          if (lane == 0) mbar_arrive_expect_tx(full + st, bytes);
          __syncwarp();
          if (lane < live_pages) {
#pragma unroll
            for (int h = 0; h < kHalves; ++h)
              tma_load_3d(ring + st * L::kTileBytes + h * (kTcTileTokens * 128) + lane * (kBlockSize * 128), map,
                          h * 64, kvh, slot, full + st);
          }
          bid = next;
        }
      }
    } else {
      // ------------------------------------------------------------ MMA issuer (one thread)
      // Paired CTA, per tile j: O_A += P_A(j) . V_j, S_A(j+1) = Q_A . K_{j+1}^T, commit s_full[A]; then the
      // same for B; a K stage is released once both S products of its tile are issued, a V stage once both
      // P . V products are.  While softmax A works on its scores the tensor core runs B's products, and the
      // other way round.  Issued MMAs execute in order, so S_x(j+1) overwrites the TMEM columns holding
      // P_x(j) only after P_x(j) . V_j has read them.
      // Single-tile CTA: S is triple-buffered in TMEM (tile j in buffer j % 3), so two tiles of scores are
      // issued ahead of the softmax and P(j) . V_j -> S(j+2) runs while it works on tile j+1 (with two
      // buffers, S(j+1) queued behind P(j-1) . V and the softmax waited for it about a quarter of every
      // tile); o_done tells the softmax when the P . V products before its tile have completed.
      if (lane == 0) {
        auto issue_s = [&](uint32_t s_col, int x, int j) {  // S = Q_x . K_j^T (K = Dh in steps of 16)
          const uint32_t kb = k_smem + (j % NK) * L::kTileBytes, qx = q_smem + x * L::kQBytes;
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) {
            const uint32_t off = (ks >> 2) * (kTcRows * 128) + (ks & 3) * 32;
            umma_ss(tmem + s_col, sw128_desc(qx + off, 16, 1024), sw128_desc(kb + off, 16, 1024), kIdescS,
                    ks > 0 ? 1u : 0u);
          }
        };
        auto issue_pv = [&](uint32_t o_col, uint32_t p_col, int j) {  // O += P . V_j, one k-step per loaded page
          const uint32_t vb = v_smem + (j % NV) * L::kTileBytes;
          const int live_pages = min(kTcTilePages, npages - j * kTcTilePages);
          for (int ks = 0; ks < live_pages; ++ks)
            umma_ts(tmem + o_col, tmem + p_col + ks * 8, sw128_desc(vb + ks * 16 * 128, kTcRows * 128, 1024),
                    kIdescO, (j > 0 || ks > 0) ? 1u : 0u);
        };
        auto wait_k = [&](int j) {
          if (!tc_wait(kfull + j % NK, (j / NK) & 1, abort_flag, a.err)) return false;
          fence_proxy_async_smem();
          tc_fence_after();
          return true;
        };
        auto wait_v = [&](int j) {
          if (!tc_wait(vfull + j % NV, (j / NV) & 1, abort_flag, a.err)) return false;
          fence_proxy_async_smem();
          tc_fence_after();
          return true;
        };
        bool ok = ntiles > 0 && tc_wait(q_ready, 0, abort_flag, a.err);
        if (two) {
          if (ok && wait_k(0)) {
            issue_s(col_s(0), 0, 0);
            umma_commit(s_full);
            issue_s(col_s(1), 1, 0);
            umma_commit(s_full + 1);
            umma_commit(kempty);  // K tile 0 is free once both its S products are done
          } else {
            ok = false;
          }
          for (int j = 0; ok && j < ntiles && !*abort_flag; ++j) {
            const bool more = j + 1 < ntiles;
            if (!tc_wait(p_full, j & 1, abort_flag, a.err) || !wait_v(j)) break;
            issue_pv(col_o<DH>(0), col_s(0), j);
            if (more) {
              if (!wait_k(j + 1)) break;
              issue_s(col_s(0), 0, j + 1);
            }
            umma_commit(s_full);
            if (!tc_wait(p_full + 1, j & 1, abort_flag, a.err)) break;
            tc_fence_after();
            issue_pv(col_o<DH>(1), col_s(1), j);
            umma_commit(vempty + j % NV);
            if (more) {
              issue_s(col_s(1), 1, j + 1);
              umma_commit(kempty + (j + 1) % NK);
            }
            umma_commit(s_full + 1);
          }
        } else {
          // single tile, S triple-buffered (buffer j % 3 at column 128 (j % 3), O after them): S(0) and S(1)
          // first, then per tile j: O += P(j) . V_j once P(j) is in, and S(j + 2) into the buffer P(j - 1)
          // held (its P . V was issued before it: in order).  The scores of the next two tiles are computed
          // while the softmax works, so P(j) . V -> S(j + 2) is off the softmax's path.
          for (int j = 0; ok && j < ntiles && j < 2; ++j) {
            if (!wait_k(j)) {
              ok = false;
              break;
            }
            issue_s(kTcRows * j, 0, j);
            umma_commit(s_full + j);
            umma_commit(kempty + j % NK);
          }
          for (int j = 0; ok && j < ntiles && !*abort_flag; ++j) {
            const int b = j % 3;
            if (!tc_wait(p_full + b, (j / 3) & 1, abort_flag, a.err) || !wait_v(j)) break;
            issue_pv(kSingleO, kTcRows * b, j);
            umma_commit(vempty + j % NV);
            umma_commit(o_done);
            if (j + 2 < ntiles) {
              if (!wait_k(j + 2)) break;
              issue_s(kTcRows * ((j + 2) % 3), 0, j + 2);
              umma_commit(s_full + (j + 2) % 3);
              umma_commit(kempty + (j + 2) % NK);
            }
          }
        }
        umma_commit(final_bar);  // every MMA issued above has completed when this arrives
        if (!tc_drain(final_bar, 0)) flag_error(a.err, MLB_DEV_WAIT_TIMEOUT);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax warpgroups: warps 4-7 take tile A,
    // warps 8-11 tile B; one thread = one query column = one TMEM lane
    const int x = warp >= 8 ? 1 : 0;
    const int row = threadIdx.x - 128 * (1 + x);
    const int mb = x ? xb.x : xa.x, mc = x ? xb.y : xa.y, piece = x ? yb.x : ya.x;
    const int tile_pieces = (x ? yb.z : ya.z) >> 8, tile_part_base = x ? yb.w : ya.w;
    // the Q rows first, straight into the swizzled K-major A tile (zero for absent columns); the producers
    // are already fetching the first K/V tiles, and only the MMA issuer waits for q_ready
    {
      const int m = row / a.group;
      const bool live = m < mc && (x == 0 || two);
      const uint4* src = nullptr;
      if (live) {
        const int tok = tile_unit ? mb + m : __ldg(&a.members[mb + m].q0);
        const int head = kvh * a.group + row % a.group;
        src = reinterpret_cast<const uint4*>(
            a.q + (static_cast<int64_t>(tok) * a.q_st + static_cast<int64_t>(head) * a.q_sh) * 2);
      }
      uint8_t* qx = smem + x * L::kQBytes;
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) {
        const uint4 v = live ? __ldg(src + ch) : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(qx + sw_chunk(row, ch)) = v;
      }
      fence_proxy_async_smem();  // generic-proxy stores, read by the tensor core (async proxy)
    }
    mbar_arrive(q_ready);
    const bool active = x == 0 || two;
    // this column's destination: an unsplit query tile writes its final row, everything else a split-K
    // partial row (its index read now, off the epilogue's path)
    const int out_m = row / a.group, out_head = kvh * a.group + row % a.group;
    const bool final_rows = tile_unit && piece < 0;
    bool out_live = active && out_m < mc;
    int64_t out_slot = 0;
    if (out_live && !final_rows) {
      const int64_t prow = tile_unit ? tile_part_base + (static_cast<int64_t>(out_m) * tile_pieces + piece) * a.tile_tokens
                                     : __ldg(&a.members[mb + out_m].part_base) + static_cast<int64_t>(piece) * a.tile_tokens;
      out_slot = prow * a.h + out_head;
      if (out_slot < 0 || out_slot >= a.part_rows * a.h) {  // a plan inconsistent with the workspace
        flag_error(a.err, MLB_DEV_BLOCK_RANGE);
        out_live = false;
      }
    }
    const uint32_t lanes = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t o_cols = tmem + lanes + (two ? col_o<DH>(x) : kSingleO);
    // kind 1: key position of the tile's first token, and this column's exclusive causal key limit
    const int first_pos = tile_unit ? __ldg(a.seq_lens + tseq) - (__ldg(a.qo + tseq + 1) - __ldg(a.qo + tseq)) +
                                          (mb - __ldg(a.qo + tseq))
                                    : 0;
    const int key_lim = first_pos + row / a.group + 1;
    const int seq_len = tile_unit ? __ldg(a.seq_lens + tseq) : INT_MAX;
    float m_used = kNegInfF, l = 0.f;
    bool ok = true;
    // a wait before warp-collective TMEM loads / stores: every lane gets the same answer, so a timeout seen
    // by some lanes never splits the warp at a tcgen05 .sync.aligned instruction
    auto wait_warp = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc_wait(bar, parity, abort_flag, a.err) ? 1 : 0) != 0;
    };
    for (int j = 0; active && j < ntiles; ++j) {
      // keys of this tile: full pages up to the unit's end, minus pages with an out-of-range block id
      // (lane p checks page p; loaded before the wait so the round trip overlaps it), minus (kind 1) keys
      // past the column's causal limit: key k of the tile is live iff k < valid_end and its page is good
      const int live_pages = min(kTcTilePages, npages - j * kTcTilePages);
      int my_bid = 0;
      if (lane < live_pages) my_bid = __ldg(table + pb + j * kTcTilePages + lane);
      // S buffer of this tile: the tile's own (paired) or tile j's of the three (single)
      const int buf = two ? x : j % 3;
      const uint32_t s_cols = tmem + lanes + kTcRows * buf;  // col_s(x) = 128 x when paired
      if (!wait_warp(s_full + buf, two ? (j & 1) : ((j / 3) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t bad = __ballot_sync(0xffffffffu, lane < live_pages && (my_bid < 0 || my_bid >= a.num_blocks));
      const int tile_key0 = (pb + j * kTcTilePages) * kBlockSize;  // key position of element 0
      const int valid_end = tile_unit ? min(live_pages * kBlockSize, key_lim - tile_key0) : live_pages * kBlockSize;
      const bool masked = valid_end < kTcTileTokens || bad != 0u;
      // the whole S row: 4 TMEM loads in flight, one wait (the softmax warps hold 224 registers)
      uint32_t sr[kTcTileTokens];
#pragma unroll
      for (int c = 0; c < kTcTileTokens / 32; ++c) tmem_ld32(s_cols + 32 * c, sr + 32 * c);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < kTcTileTokens / 32; ++c) tmem_pin32(sr + 32 * c);
      if (masked) {  // only a tile with a partial page range, a bad page or a causal edge
#pragma unroll
        for (int k = 0; k < kTcTileTokens; ++k)
          if (k >= valid_end || ((bad >> (k / kBlockSize)) & 1u)) sr[k] = __float_as_uint(kNegInfF);
      }
      // 8 independent max chains (one serial chain of 128 dependent FMNMX would be the critical path)
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = __uint_as_float(sr[i]);
#pragma unroll
      for (int k = 8; k < kTcTileTokens; ++k) mx8[k % 8] = fmaxf(mx8[k % 8], __uint_as_float(sr[k]));
      const float mraw = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      if (tile_unit && x == 0) {
        // V rows of slots past the sequence's end (its last page) are junk: 0 x NaN would poison P . V, so
        // they are zeroed in shared memory before the tile goes to the tensor core (tile A's threads do it
        // before they release P_A; the MMA issues P_B . V after P_A . V)
        const int r0 = max(0, seq_len - tile_key0), r1 = live_pages * kBlockSize;
        if (r0 < r1) {
          // the V tile has its own barrier: its rows must have landed before they are cleared
          if (!wait_warp(vfull + j % NV, (j / NV) & 1)) {
            ok = false;
            break;
          }
          const uint32_t vb = v_smem + (j % NV) * L::kTileBytes;
          constexpr int kRowItems = (DH / 64) * 8;  // 16-byte chunks of one row, both halves
          for (int e = row; e < (r1 - r0) * kRowItems; e += 128) {
            const int r = r0 + e / kRowItems, h = (e % kRowItems) / 8, c = e % 8;
            st_shared_zero16(vb + h * (kTcRows * 128) + r * 128 + c * 16);
          }
          fence_proxy_async_smem();
        }
      }
      const float mx = mraw * a.sl2;  // the scale is positive: max commutes with it
      const bool need = mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? fmaxf(m_used, mx) : m_used;
        if (j > 0) {  // paired: P_x(j-1) . V has completed (s_full[x] of this tile was committed after it)
          if (!two && !wait_warp(o_done, (j - 1) & 1)) {  // single: wait for it
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = m_new == m_used ? 1.f : fast_exp2(m_used - m_new);
#pragma unroll
          for (int i = 0; i < DH / 32; ++i) {
            uint32_t orow[32];
            tmem_ld32(o_cols + 32 * i, orow);
            tmem_wait_ld();
            tmem_pin32(orow);
#pragma unroll
            for (int k = 0; k < 32; ++k) orow[k] = __float_as_uint(__uint_as_float(orow[k]) * alpha);
            tmem_st32(o_cols + 32 * i, orow);
          }
          tmem_wait_st();
          l *= alpha;
        }
        m_used = m_new;
      }
      // p = 2^(s * scale * log2 e - m) packed to 16 bits over the first 64 columns of S_x (the row is in
      // registers already), in two halves of 32 packed columns.  The scale-and-subtract and the row sums run
      // on packed pairs of fp32 (fma.rn.f32x2 / add.f32x2, each lane rounded as fmaf / fadd); the
      // exponentials stay on the special-function unit.  4 pair sums = 8 independent sum chains.
      const float nbase = m_used == kNegInfF ? 0.f : -m_used;
      uint64_t sl2v, nbv, s4[4];
      asm("mov.b64 %0, {%1, %1};" : "=l"(sl2v) : "f"(a.sl2));
      asm("mov.b64 %0, {%1, %1};" : "=l"(nbv) : "f"(nbase));
#pragma unroll
      for (int i = 0; i < 4; ++i) s4[i] = 0ull;  // +0.0f in both halves
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int k = 0; k < 64; k += 2) {
          uint64_t sv, xv, pv;
          asm("mov.b64 %0, {%1, %2};" : "=l"(sv) : "r"(sr[64 * h + k]), "r"(sr[64 * h + k + 1]));
          asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(xv) : "l"(sv), "l"(sl2v), "l"(nbv));
          float x0, x1;
          asm("mov.b64 {%0, %1}, %2;" : "=f"(x0), "=f"(x1) : "l"(xv));
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          asm("mov.b64 %0, {%1, %2};" : "=l"(pv) : "f"(p0), "f"(p1));
          asm("add.f32x2 %0, %0, %1;" : "+l"(s4[(k / 2) % 4]) : "l"(pv));
          pk[k / 2] = pack2<DT>(p0, p1);
        }
        tmem_st32(s_cols + 32 * h, pk);
      }
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float lo, hi;
        asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(s4[i]));
        sum += lo + hi;
      }
      l += sum;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full + buf);
    }
    // O is complete when final_bar (committed once, after every MMA) arrives; the whole O row comes out of
    // TMEM in one go (Dh / 32 loads, one wait), and the row's destination was worked out before the tiles
    if (active && ok && ntiles > 0 && wait_warp(final_bar, 0) && !*abort_flag) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint32_t orow[DH];
#pragma unroll
      for (int i = 0; i < DH / 32; ++i) tmem_ld32(o_cols + 32 * i, orow + 32 * i);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < DH / 32; ++i) tmem_pin32(orow + 32 * i);
      if (out_live && final_rows) {
#pragma unroll
        for (int k = 0; k < DH / 8; ++k) {
          float v8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v8[e] = __uint_as_float(orow[8 * k + e]) * inv;
          store_out_n<DT, 8>(a.out, a.out_vec != 0, mb + out_m, out_head, 8 * k, v8);
        }
      } else if (out_live) {
        float4* dst = reinterpret_cast<float4*>(a.part_o + out_slot * DH);
#pragma unroll
        for (int k = 0; k < DH / 4; ++k)
          dst[k] = make_float4(__uint_as_float(orow[4 * k]) * inv, __uint_as_float(orow[4 * k + 1]) * inv,
                               __uint_as_float(orow[4 * k + 2]) * inv, __uint_as_float(orow[4 * k + 3]) * inv);
        a.part_lse[out_slot] = l > 0.f ? m_used + log2f(l) : kNegInfF;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tensor map of one pool for the K/V boxes: dims {Dh, Hkv, num_blocks * 16}, box {64, 1, 16}, 128-byte
// swizzle, zero fill out of bounds.  Encoded maps are cached per (address, shape, dtype): a serving loop
// reuses the same pools every step.
cudaError_t pool_tensor_map(CUtensorMap* out, const void* pool, int dtype, int64_t num_blocks, int hkv, int dh) {
  static std::mutex mu;
  static EncodeTiledFn encode = nullptr;
  static std::unordered_map<std::string, CUtensorMap> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  char key[96];
  snprintf(key, sizeof key, "%p/%d/%lld/%d/%d", pool, dtype, static_cast<long long>(num_blocks), hkv, dh);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(dh), static_cast<cuuint64_t>(hkv),
                              static_cast<cuuint64_t>(num_blocks) * kBlockSize};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(dh) * 2, static_cast<cuuint64_t>(hkv) * dh * 2};
  const cuuint32_t box[3] = {64, 1, kBlockSize};
  const cuuint32_t elem[3] = {1, 1, 1};
  const CUresult r = encode(out, dtype == MLB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            3, const_cast<void*>(pool), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (cache.size() >= 1024) cache.clear();  // bounded: pools are few, a churn of new ones restarts it
  cache.emplace(key, *out);
  return cudaSuccess;
}

template <int DT, int DH>
cudaError_t launch_tc(const AttnArgs& a, int64_t units, cudaStream_t s) {
  constexpr int bytes = TcLayout<DH>::kLaunchBytes;
  static_assert(bytes <= 232448, "shared memory budget of one sm_100 CTA");
  static unsigned long long done = 0;
  auto k = shared_prefix_tc_kernel<DT, DH>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!(dev < 64 && (done >> dev) & 1ull)) {
    // the register split inside the kernel (setmaxnreg) balances only if every thread starts with exactly
    // kRegsLaunch registers; a build that compiled to another count is refused instead of launched
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kRegsLaunch) return cudaErrorInvalidKernelImage;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    if (dev < 64) __atomic_fetch_or(&done, 1ull << dev, __ATOMIC_RELAXED);
  }
  CUtensorMap tk, tv;
  e = pool_tensor_map(&tk, a.k_cache, DT, a.num_blocks, a.hkv, DH);
  if (e == cudaSuccess) e = pool_tensor_map(&tv, a.v_cache, DT, a.num_blocks, a.hkv, DH);
  if (e != cudaSuccess) return e;
  // one CTA per pair of units (2i, 2i + 1) and KV head
  return launch_k(k, dim3(static_cast<unsigned>(units / 2 * a.hkv)), dim3(kTcThreads), bytes, s, a, tk, tv);
}

}  // namespace

// True when the tcgen05 kernel takes this launch: 16-bit pools, head_dim 64 or 128, q rows 16-byte aligned,
// pool slots addressable by the tensor maps' 32-bit coordinates.
bool shared_prefix_tc_supported(const AttnArgs& a, int dtype, int dh) {
  if ((dtype != MLB_BF16 && dtype != MLB_F16) || (dh != 64 && dh != 128)) return false;
  if (a.num_blocks * kBlockSize >= INT32_MAX) return false;
  return reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && a.q_st % 8 == 0 && a.q_sh % 8 == 0;
}

cudaError_t launch_shared_prefix_tc(const AttnArgs& a, int dtype, int dh, int64_t num_units, cudaStream_t s) {
  if (dtype == MLB_BF16) {
    if (dh == 64) return launch_tc<MLB_BF16, 64>(a, num_units, s);
    if (dh == 128) return launch_tc<MLB_BF16, 128>(a, num_units, s);
  } else if (dtype == MLB_F16) {
    if (dh == 64) return launch_tc<MLB_F16, 64>(a, num_units, s);
    if (dh == 128) return launch_tc<MLB_F16, 128>(a, num_units, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mlb

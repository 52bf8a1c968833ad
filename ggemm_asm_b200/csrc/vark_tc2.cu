// vark_tc2.cu - persistent sm_100a tcgen05 kernel for the variable-K grouped FP8 wgrad on CTA
// pairs (cta_group::2). This is the default tensor-core path.
//
// Computes, for every group g, C[g] = sL*sR * LHS[off_g:off_{g+1}]^T . RHS[off_g:off_{g+1}]
// (ggemm-asm README.md:5,45-48; bench.py:182-193 "dW = lhs^T @ rhs" per expert).
//
// Tile and operands. One work item is (group g, up to 256 rows of C, up to 256 columns of C) and
// is computed by a cluster of two CTAs with tcgen05.mma.cta_group::2 (M=256, N<=256, K=32), in
// one of two orientations:
//   * C rows on TMEM lanes, for every item of a full 256-row tile. MMA-M runs along OUT_M:
//     operand A = LHS (e4m3), CTA r of the pair holds C rows [m0 + 128r, m0 + 128r + 128), one
//     per TMEM lane. MMA-N runs along OUT_N: operand B = RHS (e5m2), N/2 columns per CTA, the
//     MMA reading both halves across the pair. N is 256 except in the last column tile, where it
//     is the remaining columns rounded up to 32 (128 at OUT_N = 5760 = 22 x 256 + 128, 64 at
//     2880). An epilogue lane holds 32 consecutive columns of one C row: one 64-byte row of the
//     stored box.
//   * C columns on TMEM lanes, for the last row tile when OUT_M is not a multiple of 256 (64 rows
//     at 2880 = 11 x 256 + 64), where most of a 256-row MMA-M would be padding. MMA-M runs along
//     OUT_N (A = RHS, 128 C columns per CTA) and MMA-N along the tile's rows rounded up to 32
//     (B = LHS, half per CTA), so ragged OUT_M costs no tensor work. An epilogue lane holds 32
//     rows of one C column, so the epilogue transposes through shared memory (lane pairs exchange
//     values so that each lane writes 4-byte words).
// Either orientation moves the same bytes (2 x 128 x TK per CTA and TK tokens for 128 x 256 x TK
// MACs); the first takes the cheaper epilogue. Measured against C columns on the lanes for every
// item (one process, 9 interleaved rounds, bit-identical outputs): gate_up +1.4%, down +1.1%,
// skewed routing +1.3%, the reference's exponential routing +2.4%.
// Both operands stay in their token-major layout, which for the MMA is MN-major: a TMA box of
// 128 contiguous features x TK tokens lands with the 128-byte swizzle of the canonical MN-major
// layout. Per CTA and TK tokens that is 2 x 128 x TK bytes for 128 x 256 x TK MACs. Boxes that
// run past a tensor edge are zero-filled by TMA without memory traffic; the epilogue's TMA
// stores clip them.
//
// Warp roles (64 + 32 x EPI_WARPS threads per CTA, one CTA per SM, 74 pairs on 148 SMs,
// persistent over a static round-robin schedule of work items by cluster):
//   warp 0      TMA producer (both CTAs): ring of ST stages {A 128 x TK, B N/2 x TK},
//               completion counted on the pair leader's full barrier
//   warp 1      TMEM owner (both CTAs, cta_group::2 allocation of all 512 columns = two
//               128-lane x 256-column fp32 accumulators); in the leader also the MMA issuer
//   warps 2..   epilogue (both CTAs): tcgen05.ld 32 TMEM columns -> * (sL*sR) -> bf16 (RNE)
//               -> a 64B-swizzled 32x32 smem box -> TMA store; warp w owns TMEM lanes
//               32*(w%4)..+31 = 32 C rows (or, C columns on the lanes, 32 C columns) of this
//               CTA's half
// The leader's commits arrive on both CTAs' barriers (tcgen05.commit multicast); the epilogue
// warps of both CTAs release an accumulator on the leader's barrier.
//
// Variable K. Loads go through the launch's own tensor maps over all M_total tokens (no map is
// built on the device). A group's tokens [off_g, off_{g+1}) are walked in blocks of TK aligned
// to the group's START. The main ring carries only whole K steps (32 tokens): the last block
// issues only the steps it holds, and its rows past them are loaded but never multiplied. A
// group that ends inside a step has a tail of 1..31 tokens. It is loaded at the item's start,
// one 32-token chunk (second maps with 32-row boxes), into one of two tail buffers per CTA, on
// the CTA's own barrier. At its next stop the producer zeroes the chunk's rows past the group
// in both boxes (both, so that an Inf or NaN in a neighbour's token can never meet a zero and
// enter the sum as NaN), makes the writes visible to the tensor core (proxy fence) and releases
// the tail to the leader at cluster scope. The MMA warp takes it after the item's whole steps,
// with a cluster-scope acquire, so the zeroing is off the MMA's critical path. Empty groups
// skip the pipeline and the epilogue stores zeros.
//
// Unknown M_total (the 14-argument drop-in). The maps then end at the int32 coordinate limit, so
// TMA would not clip anything; instead every role reads group_offs[G] once and no load touches a
// token row at or past it: a group's last block whose box would cross it is loaded shifted back
// by whole K steps, so that it ends with the block's last whole step (the MMA warp starts that
// many steps into the stage), and a tail chunk that would cross it is loaded as the 32 tokens
// that end with the group, its first 32 - ragged rows (the group's earlier tokens, already
// multiplied) being the ones the producer zeroes. Offsets past group_offs[G] are invalid. With
// M_total known the maps end there and TMA clips boxes without reading memory, so nothing moves.
// The producer records, per operand, the end of the highest token row any of its loads can read
// (status words 4 = LHS, 5 = RHS).
//
// Every mbarrier wait is bounded (TcParams::timeout_ns). On expiry the CTA flags
// GGEMM_VARK_DEV_TIMEOUT, sets the abort flag of both CTAs of the pair, every role leaves its
// loop, in-flight loads and MMAs are drained with bounded waits, and the pair meets at a
// cluster barrier before TMEM is freed.
#include <cuda_bf16.h>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"
#include "vark_ptx.cuh"

namespace vark {
namespace {

#ifndef VARK_PAIR_EPI_WARPS
#define VARK_PAIR_EPI_WARPS 4
#endif
constexpr int EPI_WARP0 = 2;
constexpr int EPI_WARPS = VARK_PAIR_EPI_WARPS;  // 4 or 8: one or two warps per TMEM lane quarter
constexpr int EPI_SPLIT = EPI_WARPS / 4;        // warps sharing one lane quarter's columns
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
constexpr int ITEM_COLS = 2 * PAIR_HALF;   // C columns per work item (MMA M)
constexpr int ITEM_ROWS = PAIR_ROWS_MAX;   // C rows per work item at most (MMA N)
constexpr int TK = PAIR_TOKENS;            // tokens per stage (TK/32 MMAs)
constexpr int ST = PAIR_STAGES;

constexpr uint32_t BOX_BYTES = 128 * TK;                 // one operand box per CTA
constexpr int SPB = TK / 32;                             // K steps (MMAs) per full stage
constexpr uint32_t TAIL_BYTES = 128 * 32;                // one operand's 32-token tail chunk
// Narrow B: an item whose B half (MMA N / 2) fits in 32 or 64 bytes - the last column tile
// (B = RHS) or the last row tile (B = LHS) - loads B in boxes that wide, with the matching
// swizzle, instead of 128 wide: the 128-wide boxes were mostly past the operand's edge (zero
// fill) yet took the same TMA time per K step. B's token rows are then bw bytes apart.
constexpr uint32_t ACC_COLS = 256;                       // TMEM columns per accumulator
constexpr uint32_t TMEM_COLS = 512;
constexpr int NACC = 2;
constexpr int EPI_COLS = 32;                             // C columns per epilogue box (one warp)
constexpr int EPI_ROWS = 32;                             // C rows per epilogue box
constexpr uint32_t EPI_BUF_BYTES = EPI_COLS * EPI_ROWS * 2;  // 2 KiB

static_assert(PAIR_HALF == 128 && ITEM_ROWS == 256, "pair tile is 256 x 256");
static_assert(TK % 32 == 0 && TK >= 64 && TK <= 256, "token block: a multiple of the MMA K (32), TMA box rows <= 256");

// Shared-memory map (offsets from a 1024-byte aligned base; identical in both CTAs).
constexpr uint32_t OFF_A = 0;                            // operand A stages
constexpr uint32_t OFF_B = OFF_A + ST * BOX_BYTES;       // operand B stages
constexpr uint32_t OFF_EPI = OFF_B + ST * BOX_BYTES;
constexpr uint32_t OFF_TAIL = OFF_EPI + EPI_WARPS * 2 * EPI_BUF_BYTES;  // 2 x {A, B} tails
constexpr uint32_t OFF_BARS = OFF_TAIL + 2 * 2 * TAIL_BYTES;
constexpr uint32_t NUM_BARS = 2 * ST + 2 + 2 + 1 + 1 + 2 + 2;
constexpr uint32_t OFF_MISC = OFF_BARS + NUM_BARS * 8;
constexpr uint32_t SMEM_USED = OFF_MISC + 16;
constexpr uint32_t SMEM_ALLOC = SMEM_USED + 1024;
static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
static_assert(OFF_EPI % 1024 == 0 && OFF_TAIL % 1024 == 0, "alignment");

// Instruction descriptors without N (or-ed in per item): C rows on the TMEM lanes (A = LHS) and
// C columns on the lanes (A = RHS).
constexpr uint32_t IDESC_ROWS_NO_N = idesc_f8f6f4(/*A=LHS e4m3*/ 0, /*B=RHS e5m2*/ 1,
                                                  /*A MN-major*/ 1, /*B MN-major*/ 1, 256, 0);
constexpr uint32_t IDESC_COLS_NO_N = idesc_f8f6f4(/*A=RHS e5m2*/ 1, /*B=LHS e4m3*/ 0,
                                                  /*A MN-major*/ 1, /*B MN-major*/ 1, 256, 0);

struct Ctl {
  volatile int* abort;
  uint32_t peer_abort;  // shared::cluster address of the peer CTA's abort flag
  uint32_t* status;
  uint64_t timeout_ns;
};

__device__ __noinline__ void report_timeout(const Ctl& ctl, uint32_t where) {
  *ctl.abort = 1;
  st_shared_cluster_u32(ctl.peer_abort, 1u);
  if (ctl.status != nullptr) {
    atomicOr(ctl.status, GGEMM_VARK_DEV_TIMEOUT);
    atomicExch(ctl.status + 1, where);
  }
}

// Bounded wait by every lane of a warp; warp-uniform verdict (see vark_tc.cu). CLUSTER: acquire
// at cluster scope (a stage the peer CTA wrote with generic stores).
template <bool CLUSTER = false>
__device__ __forceinline__ bool warp_wait(const Ctl& ctl, uint32_t bar, uint32_t parity,
                                          uint32_t where) {
  auto try_wait = [&] {
    return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
  bool ok = try_wait();
  if (!ok) {
    const uint64_t t0 = globaltimer_ns();
    while (!(ok = try_wait())) {
      if (*ctl.abort) break;
      if (globaltimer_ns() - t0 > ctl.timeout_ns) {
        report_timeout(ctl, where);
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

struct Item {
  int g, r;        // group, and the item's index within it
  int m0, n0;      // first C row and first C column of the pair tile (set by place_item)
  int nrows;       // C rows of the item rounded up to 32 (<= 256): MMA N with C columns on lanes
  int tokens;      // K_g (0 for empty or invalid groups)
  int64_t end;     // off_{g+1}
  bool rows_lanes; // C rows on the TMEM lanes (every full row tile; see the file comment)
  int ecols;       // C columns of the item rounded up to 32 (<= 256): MMA N with C rows on lanes
  uint32_t bw;     // B bytes per token row in shared memory: 128, or 64 / 32 (narrow maps)
};

// Token rows [0, lim) hold valid offsets and, with offs_bound, bound every load.
__device__ __forceinline__ int64_t token_rows_limit(const TcParams& p) {
  if (!p.offs_bound) return p.token_limit;
  const int64_t e = __ldg(p.group_offs + p.G);
  return e < 0 ? 0 : (e < p.token_limit ? e : p.token_limit);
}

// The lookahead half of an item: its group and token count (loads of group_offs, issued one
// item ahead so that their latency is hidden). place_item finishes the item once it is current:
// nothing in the tile's placement waits for the loads.
__device__ __forceinline__ Item decode_item(const TcParams& p, int64_t lim, int item,
                                            bool report) {
  const int per_group = p.row_tiles * p.col_tiles;
  Item t;
  t.g = item / per_group;
  t.r = item - t.g * per_group;
  const int64_t lo = __ldg(p.group_offs + t.g);
  const int64_t hi = __ldg(p.group_offs + t.g + 1);
  if (lo < 0 || hi < lo || hi > lim) {
    if (report && p.status != nullptr) atomicOr(p.status, GGEMM_VARK_DEV_BAD_OFFS);
    t.tokens = 0;
    t.end = 0;
  } else {
    t.tokens = static_cast<int>(hi - lo);
    t.end = hi;
  }
  return t;
}

// The tile of a decoded item. A group's items are walked column-major (row tile fastest): the
// 74 items in flight at once then span all row tiles and ~6 column tiles instead of all column
// tiles and ~3 row tiles, so for an expert whose slice exceeds L2 a wave streams 4.5 instead of
// 6.6 KB per token from DRAM at 2880 x 5760. Measured against the row-major walk (one process,
// 9 interleaved rounds, bit-identical outputs): skewed routing +5.5%, the reference's
// exponential routing +3.6%, one 43229-token expert among 31 small ones +2.1%, gate_up and
// down -0.4% and -0.3% (within run-to-run noise). Walking only the groups larger than half of
// L2 column-major gained less on the skewed workloads (+4.1%, +2.4%).
__device__ __forceinline__ Item place_item(const TcParams& p, Item t) {
  t.m0 = (t.r % p.row_tiles) * ITEM_ROWS;
  t.n0 = (t.r / p.row_tiles) * ITEM_COLS;
  t.nrows = min(ITEM_ROWS, (p.OUT_M - t.m0 + 31) & ~31);
  t.rows_lanes = t.m0 + ITEM_ROWS <= p.OUT_M;
  t.ecols = min(ITEM_COLS, (p.OUT_N - t.n0 + 31) & ~31);
  const int b_half = (t.rows_lanes ? t.ecols : t.nrows) >> 1;
  const int nw = t.rows_lanes ? p.bw_rhs : p.bw_lhs;
  t.bw = (nw > 0 && b_half <= nw) ? static_cast<uint32_t>(nw) : 128u;
  return t;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    vark_tc2_kernel(const __grid_constant__ CUtensorMap map_lhs,
                    const __grid_constant__ CUtensorMap map_rhs,
                    const __grid_constant__ CUtensorMap map_lhs32,
                    const __grid_constant__ CUtensorMap map_rhs32,
                    const __grid_constant__ CUtensorMap map_lhs_n,
                    const __grid_constant__ CUtensorMap map_lhs32_n,
                    const __grid_constant__ CUtensorMap map_rhs_n,
                    const __grid_constant__ CUtensorMap map_rhs32_n,
                    const __grid_constant__ CUtensorMap map_c, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  const uint32_t bar_full = base + OFF_BARS;         // [ST]  used in the leader only
  const uint32_t bar_empty = bar_full + 8 * ST;      // [ST]  both CTAs
  const uint32_t bar_tfull = bar_empty + 8 * ST;     // [2]   both CTAs
  const uint32_t bar_tempty = bar_tfull + 16;        // [2]   used in the leader only
  const uint32_t bar_drain = bar_tempty + 16;        // [1]   leader
  const uint32_t bar_zfill = bar_drain + 8;          // [1]   both CTAs: a tail's own loads
  const uint32_t bar_tail_full = bar_zfill + 8;      // [2]   leader: both tails zeroed
  const uint32_t bar_tail_empty = bar_tail_full + 16;  // [2] both CTAs: the leader's commit
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(sbase + OFF_MISC);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(sbase + OFF_MISC + 4);

  // ---- set-up -------------------------------------------------------------------------------
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < ST; ++s) {
      mbar_init(bar_full + 8 * s, 2);   // one expect-tx arrival from each CTA's producer
      mbar_init(bar_empty + 8 * s, 1);  // the leader's commit
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);                // the leader's commit
      mbar_init(bar_tempty + 8 * a, 2 * EPI_WARPS);   // every epilogue warp of the pair
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_zfill, 1);  // this CTA's producer
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_tail_full + 8 * i, 2);   // each CTA's producer, after zeroing
      mbar_init(bar_tail_empty + 8 * i, 1);  // the leader's commit
    }
    fence_mbar_init();
    tma_prefetch_desc(&map_lhs);
    tma_prefetch_desc(&map_rhs);
    tma_prefetch_desc(&map_lhs32);
    tma_prefetch_desc(&map_rhs32);
    tma_prefetch_desc(&map_lhs_n);
    tma_prefetch_desc(&map_lhs32_n);
    tma_prefetch_desc(&map_rhs_n);
    tma_prefetch_desc(&map_rhs32_n);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive/commit
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const Ctl ctl{abort_flag, mapa_shared(smem_u32(const_cast<int*>(abort_flag)), rank ^ 1u),
                p.status, p.timeout_ns};
  const int num_items = p.G * p.row_tiles * p.col_tiles;
  const int64_t lim = token_rows_limit(p);
  const bool bounded = p.offs_bound != 0;
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(num_clusters_x());

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) =======================================
    const uint64_t policy = l2_policy_evict_last();
    // Failure-detection test hook (GGEMM_VARK_TEST_STALL_MAGIC): withhold the first stage.
    bool withhold =
        p.status != nullptr && *reinterpret_cast<volatile uint32_t*>(p.status + 3) ==
                                   GGEMM_VARK_TEST_STALL_MAGIC;
    uint32_t stage = 0, phase = 0, zphase = 0, ntail = 0;
    bool ok = true;
    // A tail whose rows past the group still have to be zeroed (-1: none). The zeroing is
    // finished at the producer's next stop, when the tail has usually landed; the MMA warp only
    // needs the tail after the item's whole K steps.
    int ztail = -1;
    // Byte ranges of the pending tail to zero: A rows are 128 B, B rows 128, 64 or 32 B.
    uint32_t za0 = 0, za1 = 0, zb0 = 0, zb1 = 0;
    // End of the highest token row a load of each operand can read (TMA clips at token_limit).
    int64_t rows_lhs = 0, rows_rhs = 0;
    auto note_rows = [&](bool a_is_lhs, int64_t end_a, int64_t end_b) {
      const int64_t ea = end_a < p.token_limit ? end_a : p.token_limit;
      const int64_t eb = end_b < p.token_limit ? end_b : p.token_limit;
      if (a_is_lhs) {
        rows_lhs = ea > rows_lhs ? ea : rows_lhs;
        rows_rhs = eb > rows_rhs ? eb : rows_rhs;
      } else {
        rows_rhs = ea > rows_rhs ? ea : rows_rhs;
        rows_lhs = eb > rows_lhs ? eb : rows_lhs;
      }
    };
    auto finish_zfill = [&]() -> bool {
      if (ztail < 0) return true;
      if (!warp_wait(ctl, bar_zfill, zphase, 0x600u)) return false;
      zphase ^= 1u;
      const uint32_t ta = base + OFF_TAIL + static_cast<uint32_t>(ztail) * 2u * TAIL_BYTES;
      smem_zero_warp(ta + za0, za1 - za0, lane);
      smem_zero_warp(ta + TAIL_BYTES + zb0, zb1 - zb0, lane);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive_release_cluster(mapa_shared(bar_tail_full + 8 * ztail, 0));
      ztail = -1;
      return true;
    };
    Item nxt = decode_item(p, lim, cluster, false);
    for (int item = cluster; item < num_items && ok; item += nclusters) {
      const Item t = place_item(p, nxt);  // decoded one item ahead: the offsets' latency is hidden
      if (item + nclusters < num_items) nxt = decode_item(p, lim, item + nclusters, false);
      if (t.tokens == 0) continue;
      const int steps = t.tokens >> 5;                 // whole 32-token K steps
      const int ragged = t.tokens & 31;                // tokens of the tail step
      const int nkb = (steps + SPB - 1) / SPB;         // main-ring blocks
      // First token of the group as a TMA row coordinate (token_limit <= INT32_MAX).
      const int32_t lo = static_cast<int32_t>(t.end - t.tokens);
      // C rows on the lanes: A = this CTA's 128 C rows (LHS), B = this CTA's half of the item's
      // columns (RHS). C columns on the lanes: A = 128 C columns (RHS), B = half of the rows
      // (LHS). Every N/2 is a multiple of 16, so the TMA x coordinates stay 16-byte aligned.
      const int32_t r = static_cast<int32_t>(rank);
      const int32_t xa = t.rows_lanes ? t.m0 + PAIR_HALF * r : t.n0 + PAIR_HALF * r;
      const int32_t xb = t.rows_lanes ? t.n0 + (t.ecols >> 1) * r : t.m0 + (t.nrows >> 1) * r;
      if (ragged != 0) {
        // The tail: one 32-token chunk from the group's last whole step on, into a tail buffer
        // (two, used in turn), loaded first so that its zeroing is long done when the MMA warp
        // reaches it. Rows [ragged, 32) of it are not the group's (another group's tokens, or
        // TMA zero fill past M_total); in a chunk moved back, rows [0, 32 - ragged) are not.
        const uint32_t tb = ntail & 1u;
        const uint32_t tpar = ((ntail >> 1) & 1u) ^ 1u;
        if (!finish_zfill() || !warp_wait(ctl, bar_tail_empty + 8 * tb, tpar, 0x700u | tb)) {
          ok = false;
          break;
        }
        ++ntail;
        const uint32_t ta = base + OFF_TAIL + tb * 2u * TAIL_BYTES;
        const int32_t y0 = lo + 32 * steps;
        // Unknown M_total and a chunk that would cross group_offs[G]: the 32 tokens ending with
        // the group instead, whose first 32 - ragged rows are zeroed (see the file comment).
        const bool back = bounded && static_cast<int64_t>(y0) + 32 > lim;
        const int32_t y = back ? y0 + ragged - 32 : y0;
        const bool nb = t.bw != 128u;
        const uint32_t tail_b = t.bw * 32u;
        if (lane == 0) {
          mbar_arrive_expect_tx(bar_zfill, TAIL_BYTES + tail_b);
          tma_load_2d_hint(ta, t.rows_lanes ? &map_lhs32 : &map_rhs32, bar_zfill, xa, y, policy);
          tma_load_2d_hint(ta + TAIL_BYTES,
                           t.rows_lanes ? (nb ? &map_rhs32_n : &map_rhs32)
                                  : (nb ? &map_lhs32_n : &map_lhs32),
                           bar_zfill, xb, y, policy);
          note_rows(t.rows_lanes, static_cast<int64_t>(y) + 32, static_cast<int64_t>(y) + 32);
        }
        ztail = static_cast<int>(tb);
        const uint32_t keep = static_cast<uint32_t>(back ? 32 - ragged : ragged);
        za0 = back ? 0u : keep * 128u;
        za1 = back ? keep * 128u : TAIL_BYTES;
        zb0 = back ? 0u : keep * t.bw;
        zb1 = back ? keep * t.bw : tail_b;
      }
      const CUtensorMap* const map_a = t.rows_lanes ? &map_lhs : &map_rhs;
      const bool nb = t.bw != 128u;
      const CUtensorMap* const map_b =
          t.rows_lanes ? (nb ? &map_rhs_n : &map_rhs) : (nb ? &map_lhs_n : &map_lhs);
      const uint32_t stage_bytes = BOX_BYTES + t.bw * TK;
      for (int kb = 0; kb < nkb; ++kb) {
        // Neither wait depends on the pending tail: the MMA warp takes it after the item's
        // whole steps, and this stage's previous fill is older than all of them.
        if (!warp_wait(ctl, bar_empty + 8 * stage, phase ^ 1u, 0x100u | stage) ||
            !finish_zfill()) {
          ok = false;
          break;
        }
        if (lane == 0 && !withhold) {
          // The last block's rows past the whole steps are loaded but never multiplied. With
          // M_total unknown, a last block whose box would cross group_offs[G] is moved back by
          // whole steps so that it ends with its last whole step.
          const uint32_t fb = mapa_shared(bar_full + 8 * stage, 0);  // leader's barrier
          int32_t y = lo + TK * kb;
          if (bounded && static_cast<int64_t>(y) + TK > lim) y += 32 * (steps - SPB * kb) - TK;
          mbar_arrive_expect_tx_cluster(fb, stage_bytes);
          tma_load_2d_pair(base + OFF_A + stage * BOX_BYTES, map_a, fb, xa, y, policy);
          tma_load_2d_pair(base + OFF_B + stage * BOX_BYTES, map_b, fb, xb, y, policy);
          note_rows(t.rows_lanes, static_cast<int64_t>(y) + TK, static_cast<int64_t>(y) + TK);
        }
        __syncwarp();
        withhold = false;
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (ok && !finish_zfill()) ok = false;
    if (lane == 0 && p.status != nullptr) {
      atomicMax(p.status + 4, static_cast<uint32_t>(rows_lhs));
      atomicMax(p.status + 5, static_cast<uint32_t>(rows_rhs));
    }
    // Loads still in flight are drained through the empty barriers: every stage and tail this
    // producer filled is released by the leader's commit once its MMAs (which waited for the
    // data) finish; a tail still pending after an abort is drained on its own barrier. After an
    // abort the waits are bounded.
    if (lane == 0) {
      for (int s = 0; s < ST; ++s) {
        const uint64_t t0 = globaltimer_ns();
        // A stage filled k times has had k commits when drained: its parity equals the fill
        // parity. Waiting for "phase ^ 1" of the CURRENT position covers the stages ahead.
        const uint32_t par = (static_cast<uint32_t>(s) < stage) ? phase : (phase ^ 1u);
        while (!mbar_try_wait(bar_empty + 8 * s, par)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
      for (uint32_t tb = 0; tb < 2; ++tb) {
        const uint32_t uses = (ntail + 1u - tb) >> 1;  // tail buffer tb holds uses 0, 2, 4 ... or 1, 3 ...
        if (uses == 0) continue;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_tail_empty + 8 * tb, (uses - 1u) & 1u)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
      if (ztail >= 0) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_zfill, zphase)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ======================= MMA issuer (pair leader only) ==================================
    if (leader) {
      uint32_t stage = 0, phase = 0, ntail = 0;
      uint32_t acc = 0, acc_phase = 0;
      bool ok = true;
      Item nxt = decode_item(p, lim, cluster, false);
      for (int item = cluster; item < num_items && ok; item += nclusters) {
        const Item t = place_item(p, nxt);
        if (item + nclusters < num_items) nxt = decode_item(p, lim, item + nclusters, false);
        if (t.tokens == 0) continue;
        const int steps = t.tokens >> 5;
        const int ragged = t.tokens & 31;
        const int nkb = (steps + SPB - 1) / SPB;
        if (!warp_wait(ctl, bar_tempty + 8 * acc, acc_phase ^ 1u, 0x200u | acc)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        const uint32_t idesc =
            t.rows_lanes ? IDESC_ROWS_NO_N | (static_cast<uint32_t>(t.ecols >> 3) << 17)
                         : IDESC_COLS_NO_N | (static_cast<uint32_t>(t.nrows >> 3) << 17);
        // Descriptors without their start address, built once per item. A: 32 token rows of 128
        // bytes per K step. B: 32 token rows of bw bytes with the bw-byte swizzle, 8-row K groups
        // 8 * bw bytes apart. A K step adds its byte offset / 16 to the address field (the
        // stage addresses stay far below the field's 2^18-byte range).
        const uint32_t bw = t.bw;
        const uint64_t b_layout = bw == 128u ? kSmemSw128 : (bw == 64u ? kSmemSw64 : kSmemSw32);
        const uint64_t a_fixed = smem_desc_sw128(0u, BOX_BYTES, 1024u);
        const uint64_t b_fixed = smem_desc(0u, BOX_BYTES, 8u * bw, b_layout);
        const uint32_t b_step = 2u * bw;  // (32 rows * bw bytes) / 16
        for (int kb = 0; kb < nkb; ++kb) {
          if (!warp_wait(ctl, bar_full + 8 * stage, phase, 0x300u | stage)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_stage = base + OFF_A + stage * BOX_BYTES;
          const uint32_t b_stage = base + OFF_B + stage * BOX_BYTES;
          if (lane == 0) {
            const int ks_n = kb < nkb - 1 ? SPB : steps - SPB * (nkb - 1);
            const uint64_t a0 = a_fixed | (a_stage >> 4);
            const uint64_t b0 = b_fixed | (b_stage >> 4);
            if (ks_n == SPB) {
#pragma unroll
              for (int ks = 0; ks < SPB; ++ks)
                mma_f8f6f4_pair(d_tmem, a0 + ks * 256u, b0 + ks * b_step, idesc,
                                (kb > 0 || ks > 0) ? 1u : 0u);
            } else {  // the last block: only its whole steps
              // A block the producer moved back (M_total unknown) holds them at its end.
              const int64_t y = t.end - t.tokens + static_cast<int64_t>(TK) * kb;
              const int ks0 = (bounded && y + TK > lim) ? SPB - ks_n : 0;
              for (int ks = ks0; ks < ks0 + ks_n; ++ks)
                mma_f8f6f4_pair(d_tmem, a0 + ks * 256u, b0 + ks * b_step, idesc,
                                (kb > 0 || ks > ks0) ? 1u : 0u);
            }
            mma_commit_pair(bar_empty + 8 * stage, 0x3);  // frees the stage in both CTAs
          }
          __syncwarp();
          if (++stage == ST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (ragged != 0) {
          // The tail step: its rows past the group were zeroed by both producers (generic
          // stores released at cluster scope).
          const uint32_t tb = ntail & 1u;
          const uint32_t tpar = (ntail >> 1) & 1u;
          ++ntail;
          if (!warp_wait<true>(ctl, bar_tail_full + 8 * tb, tpar, 0x800u | tb)) break;
          tc_fence_after_sync();
          if (lane == 0) {
            const uint32_t ta = base + OFF_TAIL + tb * 2u * TAIL_BYTES;
            const uint64_t tb_desc = b_fixed | ((ta + TAIL_BYTES) >> 4);
            mma_f8f6f4_pair(d_tmem, a_fixed | (ta >> 4), tb_desc, idesc,
                            steps > 0 ? 1u : 0u);
            mma_commit_pair(bar_tail_empty + 8 * tb, 0x3);  // frees the tail in both CTAs
          }
          __syncwarp();
        }
        if (lane == 0) mma_commit_pair(bar_tfull + 8 * acc, 0x3);  // accumulator ready
        __syncwarp();
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (lane == 0) {
        mma_commit_pair(bar_drain, 0x1);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_drain, 0)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
      __syncwarp();
    }
  } else {
    // ======================= epilogue (EPI_WARPS warps, both CTAs) ===========================
    const int ew = warp - EPI_WARP0;
    const int quarter = warp & 3;        // TMEM lanes this warp may access
    const int half = ew >> 2;            // which of the quarter's warps (0 when EPI_SPLIT == 1)
    const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t epi_sh = base + OFF_EPI + ew * 2 * EPI_BUF_BYTES;
    const uint32_t leader_tempty = mapa_shared(bar_tempty, 0);
    uint32_t acc = 0, acc_phase = 0;
    uint32_t nstore = 0;
    // Next free staging buffer: wait until the TMA store that last read it has finished.
    auto next_buf = [&]() -> uint32_t {
      const uint32_t buf = epi_sh + (nstore & 1u) * EPI_BUF_BYTES;
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
      return buf;
    };
    const bool reporter = leader && ew == 0 && lane == 0;
    Item nxt = decode_item(p, lim, cluster, reporter);
    for (int item = cluster; item < num_items; item += nclusters) {
      const Item t = place_item(p, nxt);
      if (item + nclusters < num_items) nxt = decode_item(p, lim, item + nclusters, reporter);
      // This warp's 32 TMEM lanes are 32 C rows starting at row0 (C rows on the lanes) or 32 C
      // columns starting at xcol; TMEM column chunk c is 32 C columns or 32 C rows of those.
      const int xcol = t.n0 + PAIR_HALF * static_cast<int>(rank) + quarter * 32;
      const int row0 = t.m0 + PAIR_HALF * static_cast<int>(rank) + quarter * 32;
      const bool live = t.rows_lanes ? row0 < p.OUT_M : xcol < p.OUT_N;
      const int span = t.rows_lanes ? min(t.ecols, p.OUT_N - t.n0) : min(t.nrows, p.OUT_M - t.m0);
      const int nchunks = (span + 31) / 32;
      if (t.tokens == 0) {
        if (live) {
          const uint32_t buf = next_buf();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(
                             buf + static_cast<uint32_t>(lane) * 64u + k * 16u),
                         "r"(0u)
                         : "memory");
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int c = half; c < nchunks; c += EPI_SPLIT) {
              if (t.rows_lanes)
                tma_store_3d(&map_c, buf, t.n0 + c * EPI_COLS, row0, t.g);
              else
                tma_store_3d(&map_c, buf, xcol, t.m0 + c * EPI_ROWS, t.g);
            }
            bulk_commit_group();
          }
          ++nstore;
        }
        continue;
      }
      const float scale = __ldg(p.lhs_scale + static_cast<int64_t>(t.g) * p.scale_stride) *
                          __ldg(p.rhs_scale + static_cast<int64_t>(t.g) * p.scale_stride);
      if (!warp_wait(ctl, bar_tfull + 8 * acc, acc_phase, 0x400u | acc)) break;
      tc_fence_after_sync();
      if (live) {
        const uint32_t t_acc = tmem_base + lane_field + acc * ACC_COLS;
        // The 32x32 box is stored row-major (64-byte rows) with the 64-byte swizzle the C tensor
        // map expects (16-byte chunk ^= (row >> 1) & 3). With C columns on the lanes, this lane
        // holds C column xcol + lane for the 32 C rows of TMEM columns [32c, 32c+32); lanes 2i
        // and 2i+1 (columns 2i, 2i+1)
        // swap one value per row pair so that each writes a 4-byte word of one row: the even
        // lane row j, the odd lane row j+1 - 32 lanes cover two 64-byte rows, no bank conflict.
        const uint32_t pr = static_cast<uint32_t>(lane) >> 1;  // column pair index i
        const uint32_t odd = static_cast<uint32_t>(lane) & 1u;
        auto emit = [&](uint32_t (&r)[32], int c) {
          const uint32_t buf = next_buf();
          if (t.rows_lanes) {
            // C rows on the lanes: this lane holds 32 consecutive C columns of C row row0 + lane:
            // one 64-byte row of the box, four 16-byte pieces at the 64-byte swizzle's positions.
            const uint32_t row = static_cast<uint32_t>(lane);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint32_t v[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 b2 =
                    __floats2bfloat162_rn(__uint_as_float(r[8 * q4 + 2 * e]) * scale,
                                          __uint_as_float(r[8 * q4 + 2 * e + 1]) * scale);
                v[e] = *reinterpret_cast<const uint32_t*>(&b2);
              }
              const uint32_t addr =
                  buf + row * 64u + ((static_cast<uint32_t>(q4) ^ ((row >> 1) & 3u)) << 4);
              asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]),
                           "r"(v[1]), "r"(v[2]), "r"(v[3])
                           : "memory");
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&map_c, buf, t.n0 + c * EPI_COLS, row0, t.g);
              bulk_commit_group();
            }
            ++nstore;
            return;
          }
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float v0 = __uint_as_float(r[j]) * scale;
            const float v1 = __uint_as_float(r[j + 1]) * scale;
            const float other = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
            const __nv_bfloat162 w =
                odd ? __floats2bfloat162_rn(other, v1) : __floats2bfloat162_rn(v0, other);
            const uint32_t row = static_cast<uint32_t>(j) + odd;
            const uint32_t addr = buf + row * 64u + ((((pr >> 2) ^ (row >> 1)) & 3u) << 4) +
                                  (pr & 3u) * 4u;
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr),
                         "r"(*reinterpret_cast<const uint32_t*>(&w))
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&map_c, buf, xcol, t.m0 + c * EPI_ROWS, t.g);
            bulk_commit_group();
          }
          ++nstore;
        };
        // Two register sets: the load of the next chunk overlaps the conversion of this one.
        uint32_t ra[32], rb[32];
        int c = half;
        if (c < nchunks) tmem_ld_32x32b_x32(t_acc + c * EPI_ROWS, ra);
        tmem_ld_wait();
        tmem_regs_fence(ra);
        while (c < nchunks) {
          int cn = c + EPI_SPLIT;
          if (cn < nchunks) tmem_ld_32x32b_x32(t_acc + cn * EPI_ROWS, rb);
          emit(ra, c);
          tmem_ld_wait();
          tmem_regs_fence(rb);
          c = cn;
          if (c >= nchunks) break;
          cn = c + EPI_SPLIT;
          if (cn < nchunks) tmem_ld_32x32b_x32(t_acc + cn * EPI_ROWS, ra);
          emit(rb, c);
          tmem_ld_wait();
          tmem_regs_fence(ra);
          c = cn;
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty + 8 * acc);
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  // ---- teardown -----------------------------------------------------------------------------
  tc_fence_before_sync();
  cluster_sync_all();  // the leader's MMAs into the peer's TMEM/smem are done
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace

size_t tc2_smem_bytes() { return SMEM_ALLOC; }

cudaError_t tc2_launch(const PairMaps& m, const TcParams& p, int grid, cudaStream_t stream) {
  vark_tc2_kernel<<<grid, NUM_THREADS, SMEM_ALLOC, stream>>>(
      m.lhs, m.rhs, m.lhs32, m.rhs32, m.lhs_n, m.lhs32_n, m.rhs_n, m.rhs32_n, m.c, p);
  return cudaGetLastError();
}

cudaError_t tc2_set_attributes() {
  return cudaFuncSetAttribute(vark_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(SMEM_ALLOC));
}

}  // namespace vark

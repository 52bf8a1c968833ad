// vark_fwd.cu - persistent sm_100a tcgen05 kernel for the fixed-K grouped FP8 GEMM of the MoE
// forward and data-gradient sites, on CTA pairs (cta_group::2).
//
// Computes, for every token t of expert g (off_g <= t < off_{g+1}),
//     C[t, n] = sA * sB_g * sum_k A[t, k] * B[g, n, k]                 (fp32 accumulate -> bf16)
// with A [M_total, K] (e4m3 for the forward sites, e5m2 for the data gradient) and B e4m3,
// stored [G, N, K] ("trans_b", K contiguous: the harness's layout) or [G, K, N] (N contiguous).
// These are the four "persistent" call
// sites of the ggemm-asm harness (bench.py:154-181: gate_up_fwd, down_fwd, down_dgrad,
// gate_up_dgrad) with the argument layout of bench.py:312-338 (A, B, C, A_scale, B_scale,
// group_offs, G, N, K, stride_am, stride_bg, stride_bn, stride_cm, stride_cn).
//
// Tile and operands. A work item is (expert g, 256 tokens of g, up to 256 columns of N) and is
// computed by a cluster of two CTAs with tcgen05.mma.cta_group::2 (M=256, N<=256, K=32):
//   * MMA-M runs along tokens: operand A. CTA r holds tokens [m0 + 128r, +128) of the expert,
//     one per TMEM lane.
//   * MMA-N runs along N: operand B = B[g]. The item's N columns are split N/2 per CTA. N is 256
//     except on the last column tile, where it is the remaining columns rounded up to 16 (128 at
//     N = 5760, 64 at N = 2880), so ragged N costs no tensor work.
//   * A is K-major (K contiguous in memory): TMA boxes of 128 K-bytes x 128 rows land in the
//     canonical 128-byte-swizzled K-major layout; a stage is TK = 256 K values (two boxes), i.e.
//     8 MMAs per stage, the K advance inside a box being +32 bytes on the descriptor's start
//     address. B is the same when stored [G, N, K]; stored [G, K, N] it is MN-major for the MMA:
//     one box of 128 N-bytes x 256 K rows in the canonical 128-byte-swizzled MN-major layout,
//     the K advance being 32 rows (4096 bytes). Then the item's N is a multiple of 32 so that
//     each CTA's half starts on a 16-byte boundary (the TMA inner-coordinate rule). The last
//     stage of a K that is not a multiple of TK issues only ceil(K_rest / 32) MMAs (TMA
//     zero-fills the part of a box beyond K).
//   * Rows past the expert: A and C go through the launch's own tensor maps over all M_total
//     rows (no map is built on the device). The A rows of a partial last token tile are the
//     next expert's tokens (or zero fill past M_total); their accumulator rows are computed and
//     never stored. C is stored 32 rows at a time: a warp whose 32 rows all belong to the
//     expert stores them with TMA; the warp holding the expert's ragged last rows writes only
//     those rows with plain stores, clipped to N, so no expert's output touches another's rows.
//     A TMA store writes a row up to the next 16-byte boundary, so when N is not a multiple of
//     8 the 32-column chunk that crosses N is written with plain stores as well: nothing past
//     column N - 1 is touched.
//   * Unknown M_total (offs_bound, the 14-argument entry point): the A map then ends at the int32
//     coordinate limit, so every role reads group_offs[G] and no A load touches a row at or past
//     it. A CTA whose 128-row box would cross it loads the 128 rows that end there instead; its
//     TMEM lane i then holds token row (group_offs[G] - 128 + i), and the epilogue stores only
//     the lanes whose rows are this CTA's rows of the expert. Offsets past group_offs[G] are
//     invalid. The producer records the end of the highest A row any of its loads can read
//     (status word 4).
//
// Warp roles (6 warps, one CTA per SM, 74 pairs on 148 SMs, persistent over a static round-robin
// of work items by cluster; items ordered expert, token tile, column tile):
//   warp 0      TMA producer (both CTAs): ring of ST stages {A 128 x 256, B N/2 x 256},
//               completion counted on the pair leader's barrier
//   warp 1      TMEM owner (both CTAs; all 512 columns = two 128-lane x 256-column fp32
//               accumulators); in the leader also the MMA issuer
//   warps 2..5  epilogue (both CTAs): tcgen05.ld 32 TMEM columns of this warp's 32 rows ->
//               * (sA * sB_g) -> bf16 (RNE) -> one 64-byte row per lane of a 64B-swizzled
//               32 x 32 smem box -> TMA store (or, for the expert's ragged last rows, plain
//               16-byte stores straight from the registers)
//
// Every mbarrier wait is bounded (FwdParams::timeout_ns). On expiry the CTA flags
// GGEMM_VARK_DEV_TIMEOUT, sets the abort flag of both CTAs, every role leaves its loop,
// in-flight loads and MMAs are drained with bounded waits, and the pair meets at a cluster
// barrier before TMEM is freed.
#include <cuda_bf16.h>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"
#include "vark_ptx.cuh"

namespace vark {
namespace {

constexpr int EPI_WARP0 = 2;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr int TILE_M = 256;                  // tokens per item (MMA M)
constexpr int TILE_N = 256;                  // columns per item at most (MMA N)
constexpr int TK = 256;                      // K per stage (two 128-byte boxes per operand)
constexpr int KBOX = 128;                    // K bytes per TMA box (one swizzle atom row)
constexpr int ST = 3;                        // stages
constexpr uint32_t BOX_BYTES = 128 * KBOX;   // 128 rows x 128 K-bytes
constexpr uint32_t OP_STAGE = 2 * BOX_BYTES; // per operand per stage (TK = 2 boxes)
constexpr uint32_t STAGE_BYTES = 2 * OP_STAGE;
constexpr uint32_t ACC_COLS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr int NACC = 2;
constexpr int EPI_COLS = 32, EPI_ROWS = 32;
constexpr uint32_t EPI_BUF_BYTES = EPI_COLS * EPI_ROWS * 2;

constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_B = OFF_A + ST * OP_STAGE;
constexpr uint32_t OFF_EPI = OFF_B + ST * OP_STAGE;
constexpr uint32_t OFF_BARS = OFF_EPI + EPI_WARPS * 2 * EPI_BUF_BYTES;
constexpr uint32_t NUM_BARS = 2 * ST + 2 + 2 + 1;
constexpr uint32_t OFF_MISC = OFF_BARS + NUM_BARS * 8;
constexpr uint32_t SMEM_USED = OFF_MISC + 16;
constexpr uint32_t SMEM_ALLOC = SMEM_USED + 1024;
static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
static_assert(OFF_EPI % 1024 == 0 && OP_STAGE % 1024 == 0, "alignment");

struct Ctl {
  volatile int* abort;
  uint32_t peer_abort;
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

// Bounded wait by every lane of a warp; warp-uniform verdict.
__device__ __forceinline__ bool warp_wait(const Ctl& ctl, uint32_t bar, uint32_t parity,
                                          uint32_t where) {
  bool ok = mbar_try_wait(bar, parity);
  if (!ok) {
    const uint64_t t0 = globaltimer_ns();
    while (!(ok = mbar_try_wait(bar, parity))) {
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
  int g;          // expert
  int m0;         // first token of the tile, relative to off_g
  int rows;       // tokens of the expert in this tile (<= 256)
  int n0;         // first column
  int ncols;      // MMA N: columns of the item, a multiple of 16 (<= 256)
  int64_t lo;     // off_g
  int tokens;     // M_g
};

// Walks the item sequence expert by expert. Items of an expert: ceil(M_g / 256) token tiles x
// n_tiles column tiles, column tile fastest. Invalid offsets make an expert empty (reported by
// the walker created with report = true).
struct Walker {
  const FwdParams* p;
  int64_t lim;  // offsets above this are invalid
  bool report;
  int g = -1;
  int64_t base = 0;   // items before expert g
  int64_t count = 0;  // items of expert g
  int64_t lo = 0;
  int tokens = 0;
  __device__ __forceinline__ void next_expert() {
    base += count;
    ++g;
    count = 0;
    if (g >= p->G) return;
    const int64_t a = __ldg(p->group_offs + g), b = __ldg(p->group_offs + g + 1);
    if (a < 0 || b < a || b > lim || b - a > INT32_MAX) {
      if (report && p->status != nullptr) atomicOr(p->status, GGEMM_VARK_DEV_BAD_OFFS);
      tokens = 0;
      return;
    }
    lo = a;
    tokens = static_cast<int>(b - a);
    count = static_cast<int64_t>((tokens + TILE_M - 1) / TILE_M) * p->n_tiles;
  }
  // Item `i` (i never decreases between calls). False past the last item.
  __device__ __forceinline__ bool seek(int64_t i, Item* t) {
    if (g < 0) next_expert();
    while (g < p->G && i >= base + count) next_expert();
    if (g >= p->G) return false;
    const int64_t r = i - base;
    const int mt = static_cast<int>(r / p->n_tiles);
    const int nt = static_cast<int>(r - static_cast<int64_t>(mt) * p->n_tiles);
    t->g = g;
    t->lo = lo;
    t->tokens = tokens;
    t->m0 = mt * TILE_M;
    t->rows = min(TILE_M, tokens - t->m0);
    const int rem = p->N - (p->n_tiles - 1) * TILE_N;  // columns of the last tile
    if (rem > 0 && rem <= 64 && p->n_tiles > 1) {
      // A last tile of at most 64 columns (N = 2880 = 11 x 256 + 64) costs nearly a whole item
      // for a quarter of its work. The columns are spread evenly over the same number of tiles
      // in 32-column chunks instead (2880 = 6 x 256 + 6 x 224; each half stays 16-byte aligned
      // in either B layout). One-process A/B, bit-identical output: N x K = 2880 x 5760 +2.0 to
      // +4.7% over three runs, 2880 x 2880 -1.4 to +2.4% (noise). A larger remainder keeps
      // whole tiles: at 5760 = 22 x 256 + 128 the spread measured -1.7%.
      const int chunks = (p->N + 31) >> 5;
      const int cb = chunks / p->n_tiles;
      const int crem = chunks - cb * p->n_tiles;
      t->n0 = 32 * (nt * cb + min(nt, crem));
      t->ncols = 32 * (cb + (nt < crem ? 1 : 0));
    } else {
      t->n0 = nt * TILE_N;
      const int align = p->b_mn_major ? 32 : 16;  // MN-major B: each half 16-byte aligned
      t->ncols = min(TILE_N, (p->N - t->n0 + align - 1) & ~(align - 1));
    }
    return true;
  }
};

// Token rows [0, lim) hold valid offsets and, with offs_bound, bound every A load.
__device__ __forceinline__ int64_t token_rows_limit(const FwdParams& p) {
  if (!p.offs_bound) return p.token_limit;
  const int64_t e = __ldg(p.group_offs + p.G);
  return e < 0 ? 0 : (e < p.token_limit ? e : p.token_limit);
}

// First A row of CTA `rank`'s box for item t: its own rows (off_g + m0 + 128 rank), or, with
// M_total unknown and a box that would cross lim, the 128 rows that end at lim.
__device__ __forceinline__ int64_t a_box_row(const FwdParams& p, int64_t lim, const Item& t,
                                             uint32_t rank) {
  const int64_t ya = t.lo + t.m0 + 128 * static_cast<int64_t>(rank);
  return (p.offs_bound && ya + 128 > lim) ? lim - 128 : ya;
}

// Shared-memory descriptor offsets of MMA ks (K step of 32) inside a stage, in descriptor units
// (16 bytes): A and K-major B advance 32 bytes inside a 128-byte box and then jump to the next
// box; MN-major B advances 32 rows of 128 bytes.
__device__ __forceinline__ uint64_t kmajor_step(int ks) {
  return static_cast<uint64_t>(((ks >> 2) * BOX_BYTES + (ks & 3) * 32u) >> 4);
}
__device__ __forceinline__ uint64_t mnmajor_step(int ks) {
  return static_cast<uint64_t>((ks * 4096u) >> 4);
}

template <bool BMN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    vark_fwd2_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  const uint32_t bar_full = base + OFF_BARS;         // [ST]  leader
  const uint32_t bar_empty = bar_full + 8 * ST;      // [ST]  both CTAs
  const uint32_t bar_tfull = bar_empty + 8 * ST;     // [2]   both CTAs
  const uint32_t bar_tempty = bar_tfull + 16;        // [2]   leader
  const uint32_t bar_drain = bar_tempty + 16;        // [1]   leader
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(sbase + OFF_MISC);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(sbase + OFF_MISC + 4);

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < ST; ++s) {
      mbar_init(bar_full + 8 * s, 2);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, 2 * EPI_WARPS);
    }
    mbar_init(bar_drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const Ctl ctl{abort_flag, mapa_shared(smem_u32(const_cast<int*>(abort_flag)), rank ^ 1u),
                p.status, p.timeout_ns};
  const int64_t cluster = cluster_id_x();
  const int64_t nclusters = num_clusters_x();
  const int64_t lim = token_rows_limit(p);

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) =======================================
    const uint64_t policy = l2_policy_evict_last();
    bool withhold =
        p.status != nullptr && *reinterpret_cast<volatile uint32_t*>(p.status + 3) ==
                                   GGEMM_VARK_TEST_STALL_MAGIC;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    int64_t rows_end = 0;  // end of the highest A row a load can read (TMA clips at token_limit)
    Walker w{&p, lim, false};
    Item t;
    const int nkb = (p.K + TK - 1) / TK;
    for (int64_t item = cluster; ok && w.seek(item, &t); item += nclusters) {
      // Token rows of this CTA's half of the tile, as rows of the whole A (off_g + m0 + 128r,
      // or moved back to end at group_offs[G]; below the token coordinate limit, so it fits the
      // TMA's int32 coordinate).
      const int32_t ya = static_cast<int32_t>(a_box_row(p, lim, t, rank));
      if (lane == 0) {
        const int64_t e = static_cast<int64_t>(ya) + 128;
        rows_end = e > rows_end ? (e < p.token_limit ? e : p.token_limit) : rows_end;
      }
      const int32_t yb = t.n0 + (t.ncols >> 1) * static_cast<int32_t>(rank);
      for (int kb = 0; kb < nkb; ++kb) {
        if (!warp_wait(ctl, bar_empty + 8 * stage, phase ^ 1u, 0x100u | stage)) {
          ok = false;
          break;
        }
        if (lane == 0 && !withhold) {
          const uint32_t fb = mapa_shared(bar_full + 8 * stage, 0);
          mbar_arrive_expect_tx_cluster(fb, STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int32_t x = kb * TK + h * KBOX;
            tma_load_2d_pair(base + OFF_A + stage * OP_STAGE + h * BOX_BYTES, &map_a, fb, x, ya,
                             policy);
            if (!BMN)
              tma_load_3d_pair(base + OFF_B + stage * OP_STAGE + h * BOX_BYTES, &map_b, fb, x, yb,
                               t.g, policy);
          }
          if (BMN)  // one box: this CTA's N/2 columns x the stage's 256 K rows
            tma_load_3d_pair(base + OFF_B + stage * OP_STAGE, &map_b, fb, yb, kb * TK, t.g,
                             policy);
        }
        __syncwarp();
        withhold = false;
        if (++stage == ST) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (lane == 0 && p.status != nullptr) atomicMax(p.status + 4, static_cast<uint32_t>(rows_end));
    if (lane == 0) {
      for (int s = 0; s < ST; ++s) {
        const uint64_t t0 = globaltimer_ns();
        const uint32_t par = (static_cast<uint32_t>(s) < stage) ? phase : (phase ^ 1u);
        while (!mbar_try_wait(bar_empty + 8 * s, par)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ======================= MMA issuer (pair leader only) ==================================
    if (leader) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t idesc0 = idesc_f8f6f4(static_cast<uint32_t>(p.a_fmt), /*B e4m3*/ 0,
                                           /*A K-major*/ 0, BMN ? 1u : 0u, TILE_M, 0);
      const int nkb = (p.K + TK - 1) / TK;
      Walker w{&p, lim, false};
      Item t;
      for (int64_t item = cluster; ok && w.seek(item, &t); item += nclusters) {
        if (!warp_wait(ctl, bar_tempty + 8 * acc, acc_phase ^ 1u, 0x200u | acc)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        const uint32_t idesc = idesc0 | (static_cast<uint32_t>(t.ncols >> 3) << 17);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!warp_wait(ctl, bar_full + 8 * stage, phase, 0x300u | stage)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const int kmma = min(TK / 32, (p.K - kb * TK + 31) / 32);
          if (lane == 0) {
            // Stage descriptors; each MMA adds a constant offset. MN-major B: the box holds one
            // MN atom (the N/2 <= 128 columns of this CTA), LBO = box bytes.
            const uint64_t a0 = smem_desc_sw128(base + OFF_A + stage * OP_STAGE, 16u, 1024u);
            const uint64_t b0 = BMN ? smem_desc_sw128(base + OFF_B + stage * OP_STAGE, OP_STAGE,
                                                      1024u)
                                    : smem_desc_sw128(base + OFF_B + stage * OP_STAGE, 16u, 1024u);
            if (kmma == TK / 32) {
#pragma unroll
              for (int ks = 0; ks < TK / 32; ++ks)
                mma_f8f6f4_pair(d_tmem, a0 + kmajor_step(ks),
                                b0 + (BMN ? mnmajor_step(ks) : kmajor_step(ks)), idesc,
                                (kb > 0 || ks > 0) ? 1u : 0u);
            } else {  // the K tail
              for (int ks = 0; ks < kmma; ++ks)
                mma_f8f6f4_pair(d_tmem, a0 + kmajor_step(ks),
                                b0 + (BMN ? mnmajor_step(ks) : kmajor_step(ks)), idesc,
                                (kb > 0 || ks > 0) ? 1u : 0u);
            }
            mma_commit_pair(bar_empty + 8 * stage, 0x3);
          }
          __syncwarp();
          if (++stage == ST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) mma_commit_pair(bar_tfull + 8 * acc, 0x3);
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
    // ======================= epilogue (4 warps, both CTAs) ===================================
    const int quarter = warp & 3;  // TMEM lanes 32*quarter.. = tokens m0 + 128*rank + 32*quarter..
    const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t epi_sh = base + OFF_EPI + (warp - EPI_WARP0) * 2 * EPI_BUF_BYTES;
    const uint32_t leader_tempty = mapa_shared(bar_tempty, 0);
    uint32_t acc = 0, acc_phase = 0, nstore = 0;
    Walker w{&p, lim, leader && warp == EPI_WARP0 && lane == 0};
    Item t;
    for (int64_t item = cluster; w.seek(item, &t); item += nclusters) {
      const float scale = __ldg(p.a_scale + static_cast<int64_t>(t.g) * p.scale_stride) *
                          __ldg(p.b_scale + static_cast<int64_t>(t.g) * p.scale_stride);
      if (!warp_wait(ctl, bar_tfull + 8 * acc, acc_phase, 0x400u | acc)) break;
      tc_fence_after_sync();
      // Expert row of this warp's lane 0: TMEM lane i holds A row (box row + i). This CTA's
      // own rows of the expert start at m0 + 128 rank; a box moved back (M_total unknown) starts
      // `shift` rows before them, and its lanes below the CTA's rows are not stored.
      const int own0 = t.m0 + 128 * static_cast<int>(rank);
      const int shift = static_cast<int>(t.lo + own0 - a_box_row(p, lim, t, rank));
      const int row0 = own0 - shift + 32 * quarter;
      const int lane_lo = max(0, own0 - row0);
      const int lane_hi = min(EPI_ROWS, t.tokens - row0);
      if (lane_lo < lane_hi) {
        const uint32_t t_acc = tmem_base + lane_field + acc * ACC_COLS;
        // 32-column chunks up to the last real column (the store clips columns >= N).
        const int nchunks = (min(t.ncols, p.N - t.n0) + EPI_COLS - 1) / EPI_COLS;
        // This warp's rows of the expert: all 32, or a ragged range of lanes.
        const bool whole = lane_lo == 0 && lane_hi == EPI_ROWS;
        const int32_t crow0 = static_cast<int32_t>(t.lo + row0);  // lane 0 as a row of C
        // Lane = token row; a chunk is 32 consecutive columns. Eight of them -> four bf16 pairs.
        auto pack = [&](const uint32_t (&r)[32], int q, uint32_t (&v)[4]) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 b2 =
                __floats2bfloat162_rn(__uint_as_float(r[8 * q + 2 * e]) * scale,
                                      __uint_as_float(r[8 * q + 2 * e + 1]) * scale);
            v[e] = *reinterpret_cast<const uint32_t*>(&b2);
          }
        };
        auto emit = [&](uint32_t (&r)[32], int c) {
          const int col0 = t.n0 + c * EPI_COLS;
          // A TMA store writes each row up to the next 16-byte boundary, so the chunk that
          // crosses an N that is not a multiple of 8 goes the plain way too.
          if (!whole || ((p.N & 7) != 0 && col0 + EPI_COLS > p.N)) {
            // The expert's last rows, the live lanes of a box moved back, or the last chunk of
            // a ragged N: each live lane writes its row's 32 columns (clipped to N) as 16-byte
            // pieces; C rows are 16-byte aligned (the row pitch is a multiple of 8 elements) and
            // col0 is a multiple of 32.
            if (lane >= lane_lo && lane < lane_hi) {
              const int ncv = min(EPI_COLS, p.N - col0);
              uint16_t* const dst = p.c + static_cast<int64_t>(crow0 + lane) * p.stride_cm + col0;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t v[4];
                pack(r, q, v);
                if (8 * q + 8 <= ncv) {
                  *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(v[0], v[1], v[2], v[3]);
                } else {
#pragma unroll
                  for (int e = 0; e < 8; ++e)
                    if (8 * q + e < ncv)
                      dst[8 * q + e] = static_cast<uint16_t>(v[e >> 1] >> (16 * (e & 1)));
                }
              }
            }
            return;
          }
          // Full 32 rows: one 64-byte row per lane of a 64B-swizzled box, written as four
          // 16-byte pieces at the swizzle's positions (piece ^ (row>>1)&3), then one TMA store.
          const uint32_t buf = epi_sh + (nstore & 1u) * EPI_BUF_BYTES;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          const uint32_t row = static_cast<uint32_t>(lane);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t v[4];
            pack(r, q, v);
            const uint32_t addr = buf + row * 64u + ((static_cast<uint32_t>(q) ^ ((row >> 1) & 3u)) << 4);
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]),
                         "r"(v[1]), "r"(v[2]), "r"(v[3])
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_c, buf, col0, crow0);
            bulk_commit_group();
          }
          ++nstore;
        };
        uint32_t ra[32], rb[32];
        int c = 0;
        if (c < nchunks) tmem_ld_32x32b_x32(t_acc + c * EPI_COLS, ra);
        tmem_ld_wait();
        tmem_regs_fence(ra);
        while (c < nchunks) {
          int cn = c + 1;
          if (cn < nchunks) tmem_ld_32x32b_x32(t_acc + cn * EPI_COLS, rb);
          emit(ra, c);
          tmem_ld_wait();
          tmem_regs_fence(rb);
          c = cn;
          if (c >= nchunks) break;
          cn = c + 1;
          if (cn < nchunks) tmem_ld_32x32b_x32(t_acc + cn * EPI_COLS, ra);
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

  tc_fence_before_sync();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace

size_t fwd2_smem_bytes() { return SMEM_ALLOC; }

cudaError_t fwd2_launch(const CUtensorMap& map_a, const CUtensorMap& map_b,
                        const CUtensorMap& map_c, const FwdParams& p, int grid,
                        cudaStream_t stream) {
  if (p.b_mn_major)
    vark_fwd2_kernel<true><<<grid, NUM_THREADS, SMEM_ALLOC, stream>>>(map_a, map_b, map_c, p);
  else
    vark_fwd2_kernel<false><<<grid, NUM_THREADS, SMEM_ALLOC, stream>>>(map_a, map_b, map_c, p);
  return cudaGetLastError();
}

cudaError_t fwd2_set_attributes() {
  cudaError_t e = cudaFuncSetAttribute(vark_fwd2_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(SMEM_ALLOC));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(vark_fwd2_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(SMEM_ALLOC));
}

}  // namespace vark

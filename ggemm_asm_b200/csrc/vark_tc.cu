// vark_tc.cu - persistent sm_100a tcgen05 kernel for the variable-K grouped FP8 wgrad.
//
// Computes, for every group g, C[g] = sL*sR * LHS[off_g:off_{g+1}]^T . RHS[off_g:off_{g+1}]
// (ggemm-asm README.md:5,45-48; bench.py:182-193 "dW = lhs^T @ rhs" per expert).
//
// Formulation on the tensor core. One work item ("tile") is (group g, row tile, column tile)
// of C. The MMA computes the TRANSPOSED tile  D[n][m] = sum_t RHS[t][n] * LHS[t][m], so that
//   * MMA-M (128 TMEM lanes) runs along OUT_N (C columns): operand A = RHS (e5m2),
//   * MMA-N (240 TMEM columns) runs along OUT_M (C rows):  operand B = LHS (e4m3),
// and both operands are consumed in their natural token-major layout, which for the MMA is
// "MN-major" (the M/N index is contiguous). A TMA box of 128 contiguous features x 128 tokens
// lands in shared memory with the 128-byte swizzle that the MN-major canonical layout expects.
// 5760 = 45 x 128 and 2880 = 12 x 240, so the GPT-OSS shapes have no ragged tiles.
//
// Warp roles (192 threads, one CTA per SM, persistent over a static round-robin schedule):
//   warp 0      TMA producer: 4-stage ring of {RHS 128x128, LHS 2 x 128x128} token blocks
//   warp 1      TMEM owner + MMA issuer: tcgen05.mma.kind::f8f6f4 into one of two fp32
//               accumulators (TMEM columns [0,240) and [256,496))
//   warps 2..5  epilogue: tcgen05.ld -> * (sL*sR) -> bf16 (RNE) -> smem -> TMA store;
//               warp w owns TMEM lanes 32*(w%4)..+31, i.e. 32 C columns of the tile
// The epilogue of one tile overlaps the MMAs of the next through the two accumulators.
//
// Variable K. A group's tokens [off_g, off_{g+1}) are walked in blocks of 128 that are aligned
// to the START of the group, through the launch's own tensor maps over all M_total tokens (no
// map is built on the device). Only the last block can hold rows that are not the group's
// (another group's tokens, or TMA zero fill past M_total); the MMA warp issues only its K steps
// (32 tokens) that hold group tokens. When the group ends inside a step, that block completes on
// a second barrier; the producer zeroes the step's rows past the group in every box of the stage
// (all operands, so that a neighbour's Inf or NaN never meets a zero and enters the sum as NaN),
// makes the writes visible to the tensor core (proxy fence) and then releases the stage to the
// MMA warp. Empty groups skip the pipeline: the epilogue TMA-stores zeros for them.
//
// Unknown M_total (offs_bound): every role reads group_offs[G] and no load touches a token row at
// or past it. A group's last block whose box would cross it is loaded as the 128 tokens that end
// with the group; its tokens then occupy the last ceil(rem / 32) K steps of the stage, the first
// of them starting with (32 - rem % 32) % 32 earlier tokens, which the producer zeroes. Offsets
// past group_offs[G] are invalid. The producer records the end of the highest token row any of
// its loads can read (status words 4 = LHS, 5 = RHS).
//
// Every mbarrier wait is bounded (TcParams::timeout_ns). On expiry the CTA sets the abort
// flag and GGEMM_VARK_DEV_TIMEOUT in the status block, every role leaves its loop, in-flight
// TMA loads and MMAs are drained with bounded waits, TMEM is freed and the CTA returns.
#include <cuda_bf16.h>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"
#include "vark_ptx.cuh"

namespace vark {
namespace {

constexpr int NUM_THREADS = 192;
constexpr int EPI_WARP0 = 2;
constexpr int EPI_WARPS = 4;

constexpr uint32_t RHS_STAGE_BYTES = TILE_COLS * TILE_TOKENS;      // 16 KiB at 128 tokens
constexpr uint32_t LHS_BOX_BYTES = 128 * TILE_TOKENS;              // 16 KiB at 128 tokens
constexpr uint32_t LHS_STAGE_BYTES = LHS_BOXES * LHS_BOX_BYTES;    // 32 KiB at 128 tokens
constexpr uint32_t STAGE_TX_BYTES = RHS_STAGE_BYTES + LHS_STAGE_BYTES;
constexpr uint32_t ACC_STRIDE_COLS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t EPI_BUF_BYTES = EPI_BOX_COLS * EPI_BOX_ROWS * 2;  // 1 KiB

static_assert(TILE_COLS == 128, "MMA M is 128 (one CTA, TMEM lane == tile column)");
static_assert(TILE_ROWS % 16 == 0 && TILE_ROWS <= 256, "MMA N must be a multiple of 16, <= 256");
static_assert(TILE_TOKENS == 64 || TILE_TOKENS == 128, "a token block is 2 or 4 MMAs of K=32");
static_assert(TILE_ROWS <= ACC_STRIDE_COLS, "accumulators must not overlap");
static_assert(EPI_BOX_COLS == 32, "one epilogue warp covers 32 TMEM lanes");

// Shared-memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t OFF_RHS = 0;
constexpr uint32_t OFF_LHS = OFF_RHS + STAGES * RHS_STAGE_BYTES;
constexpr uint32_t OFF_EPI = OFF_LHS + STAGES * LHS_STAGE_BYTES;
constexpr uint32_t OFF_ZERO = OFF_EPI + EPI_WARPS * 2 * EPI_BUF_BYTES;
constexpr uint32_t OFF_BARS = OFF_ZERO + EPI_BUF_BYTES;
constexpr uint32_t NUM_BARS = 2 * STAGES + 2 + 2 + 1 + 1;
constexpr uint32_t OFF_MISC = OFF_BARS + NUM_BARS * 8;
constexpr uint32_t SMEM_USED = OFF_MISC + 16;
constexpr uint32_t SMEM_ALLOC = SMEM_USED + 1024;  // alignment slack
static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
static_assert(OFF_BARS % 8 == 0, "mbarriers are 8-byte aligned");

constexpr uint32_t IDESC = idesc_f8f6f4(/*A=RHS e5m2*/ 1, /*B=LHS e4m3*/ 0,
                                        /*A MN-major*/ 1, /*B MN-major*/ 1, 128, TILE_ROWS);

struct Ctl {
  volatile int* abort;
  uint32_t* status;
  uint64_t timeout_ns;
};

// Record a wait that exceeded its limit: stop every role of this CTA and flag the host.
__device__ __noinline__ void report_timeout(const Ctl& ctl, uint32_t where) {
  *ctl.abort = 1;
  if (ctl.status != nullptr) {
    atomicOr(ctl.status, GGEMM_VARK_DEV_TIMEOUT);
    atomicExch(ctl.status + 1, where);
  }
}

// Bounded wait on an mbarrier phase, executed by every lane of a warp (inline: the waits sit on
// the critical path between the TMA, MMA and epilogue warps). Returns a warp-uniform verdict:
// false if the limit expired in any lane or another role already aborted.
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

struct TileInfo {
  int g, row0, col0;
  int tokens;      // K_g (0 for empty or invalid groups)
  int64_t end;     // off_{g+1}
};

// Token rows [0, lim) hold valid offsets and, with offs_bound, bound every load.
__device__ __forceinline__ int64_t token_rows_limit(const TcParams& p) {
  if (!p.offs_bound) return p.token_limit;
  const int64_t e = __ldg(p.group_offs + p.G);
  return e < 0 ? 0 : (e < p.token_limit ? e : p.token_limit);
}

// First K step of a group's last block that holds its tokens: nonzero when the block was moved
// back to end with the group (M_total unknown and the box would cross group_offs[G]).
__device__ __forceinline__ int last_block_slot0(bool bounded, int64_t y, int rem, int64_t lim) {
  return (bounded && y + TILE_TOKENS > lim) ? (TILE_TOKENS - rem) >> 5 : 0;
}

__device__ __forceinline__ TileInfo decode_tile(const TcParams& p, int64_t lim, int tile,
                                                bool report) {
  const int per_group = p.row_tiles * p.col_tiles;
  TileInfo t;
  t.g = tile / per_group;
  const int r = tile - t.g * per_group;
  t.row0 = (r % p.row_tiles) * TILE_ROWS;
  t.col0 = (r / p.row_tiles) * TILE_COLS;
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

__global__ void __launch_bounds__(NUM_THREADS, 1)
    vark_tc_kernel(const __grid_constant__ CUtensorMap map_rhs,
                   const __grid_constant__ CUtensorMap map_lhs,
                   const __grid_constant__ CUtensorMap map_c, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const uint32_t bar_full = base + OFF_BARS;                 // [STAGES]
  const uint32_t bar_empty = bar_full + 8 * STAGES;          // [STAGES]
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;         // [2]
  const uint32_t bar_tempty = bar_tfull + 16;                // [2]
  const uint32_t bar_drain = bar_tempty + 16;                // [1]
  const uint32_t bar_zfill = bar_drain + 8;                  // [1] a group's last block
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(sbase + OFF_MISC);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(sbase + OFF_MISC + 4);

  // ---- set-up -------------------------------------------------------------------------------
  {
    uint32_t* z = reinterpret_cast<uint32_t*>(sbase + OFF_ZERO);
    for (int i = threadIdx.x; i < static_cast<int>(EPI_BUF_BYTES / 4); i += NUM_THREADS) z[i] = 0u;
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, EPI_WARPS);
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_zfill, 1);
    fence_mbar_init();
    tma_prefetch_desc(&map_rhs);
    tma_prefetch_desc(&map_lhs);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const Ctl ctl{abort_flag, p.status, p.timeout_ns};
  const int num_tiles = p.G * p.row_tiles * p.col_tiles;
  const int64_t lim = token_rows_limit(p);
  const bool bounded = p.offs_bound != 0;

  if (warp == 0) {
    // ======================= TMA producer (lane 0 issues; the warp stays converged) ==========
    const uint64_t policy = l2_policy_evict_last();
    // Failure-detection test hook (GGEMM_VARK_TEST_STALL_MAGIC): withhold the first stage.
    bool withhold =
        p.status != nullptr && *reinterpret_cast<volatile uint32_t*>(p.status + 3) ==
                                   GGEMM_VARK_TEST_STALL_MAGIC;
    uint32_t stage = 0, phase = 0, zphase = 0;
    uint32_t used_mask = 0, parity_mask = 0;  // per stage: issued at least once / last parity
    bool ok = true, zpending = false;
    int64_t rows_end = 0;  // end of the highest token row a load can read (TMA clips at token_limit)
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const TileInfo t = decode_tile(p, lim, tile, false);
      if (t.tokens == 0) continue;
      const int nkb = (t.tokens + TILE_TOKENS - 1) / TILE_TOKENS;
      const int rem = t.tokens - TILE_TOKENS * (nkb - 1);  // the group's tokens in its last block
      // First token of the group as a TMA row coordinate (token_limit <= INT32_MAX).
      const int32_t lo = static_cast<int32_t>(t.end - t.tokens);
      for (int kb = 0; kb < nkb; ++kb) {
        if (!warp_wait(ctl, bar_empty + 8 * stage, phase ^ 1u, 0x100u | stage)) {
          ok = false;
          break;
        }
        const uint32_t fb = bar_full + 8 * stage;
        const uint32_t rhs_dst = base + OFF_RHS + stage * RHS_STAGE_BYTES;
        const uint32_t lhs_dst = base + OFF_LHS + stage * LHS_STAGE_BYTES;
        const int64_t y_block = static_cast<int64_t>(lo) + TILE_TOKENS * kb;
        // M_total unknown and the last block's box would cross group_offs[G]: the block is
        // moved back so that it ends with the group's rem tokens.
        const bool back = kb == nkb - 1 && bounded && y_block + TILE_TOKENS > lim;
        const int32_t y = static_cast<int32_t>(back ? y_block + rem - TILE_TOKENS : y_block);
        // A group's last block that ends inside a K step (32 tokens): the MMA warp multiplies
        // that step, so its rows [rem, ceil32(rem)) must be zero. The block lands on bar_zfill
        // instead and those rows are zeroed before the stage is released to the MMA warp. (The
        // MMA warp issues only the steps that hold group tokens, so a block ending on a step
        // boundary needs nothing.)
        const bool last_partial = kb == nkb - 1 && (rem & 31) != 0;
        if (!withhold) {
          const uint32_t lb = last_partial ? bar_zfill : fb;
          if (lane == 0) {
            mbar_arrive_expect_tx(lb, STAGE_TX_BYTES);
            const int64_t e = static_cast<int64_t>(y) + TILE_TOKENS;
            rows_end = e > rows_end ? (e < p.token_limit ? e : p.token_limit) : rows_end;
            tma_load_2d_hint(rhs_dst, &map_rhs, lb, t.col0, y, policy);
#pragma unroll
            for (int b = 0; b < LHS_BOXES; ++b)
              tma_load_2d_hint(lhs_dst + b * LHS_BOX_BYTES, &map_lhs, lb, t.row0 + 128 * b, y,
                               policy);
          }
          if (last_partial) {
            zpending = true;
            if (!warp_wait(ctl, bar_zfill, zphase, 0x600u)) {
              ok = false;
              break;
            }
            zpending = false;
            zphase ^= 1u;
            // Whole 128-byte token rows, so the 128-byte swizzle does not matter. A block moved
            // back zeroes the earlier tokens in front of its first step instead.
            const uint32_t z0 = back ? static_cast<uint32_t>((TILE_TOKENS - rem) & ~31) * 128u
                                     : static_cast<uint32_t>(rem) * 128u;
            const uint32_t zbytes = back ? static_cast<uint32_t>(TILE_TOKENS - rem) * 128u - z0
                                         : static_cast<uint32_t>((rem + 31) & ~31) * 128u - z0;
            smem_zero_warp(rhs_dst + z0, zbytes, lane);
#pragma unroll
            for (int b = 0; b < LHS_BOXES; ++b)
              smem_zero_warp(lhs_dst + b * LHS_BOX_BYTES + z0, zbytes, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(fb);
          }
        }
        __syncwarp();
        withhold = false;
        used_mask |= 1u << stage;
        parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (lane == 0 && p.status != nullptr) {
      atomicMax(p.status + 4, static_cast<uint32_t>(rows_end));  // LHS and RHS boxes alike
      atomicMax(p.status + 5, static_cast<uint32_t>(rows_end));
    }
    // Drain: every issued load must have landed before the CTA may exit. On the normal path
    // they all have (the MMA warp consumed them); after an abort the wait is bounded.
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) {
        if ((used_mask & (1u << s)) == 0) continue;
        const uint32_t par = (parity_mask >> s) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_full + 8 * s, par)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
      if (zpending) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_zfill, zphase)) {
          if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ======================= MMA issuer =====================================================
    uint32_t stage = 0, phase = 0;
    uint32_t acc = 0, acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const TileInfo t = decode_tile(p, lim, tile, false);
      if (t.tokens == 0) continue;
      const int nkb = (t.tokens + TILE_TOKENS - 1) / TILE_TOKENS;
      const int rem = t.tokens - TILE_TOKENS * (nkb - 1);
      const int last_steps = (rem + 31) >> 5;  // of the last block
      const int64_t lo = t.end - t.tokens;
      if (!warp_wait(ctl, bar_tempty + 8 * acc, acc_phase ^ 1u, 0x200u | acc)) break;
      tc_fence_after_sync();
      const uint32_t d_tmem = tmem_base + acc * ACC_STRIDE_COLS;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!warp_wait(ctl, bar_full + 8 * stage, phase, 0x300u | stage)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t a_stage = base + OFF_RHS + stage * RHS_STAGE_BYTES;
        const uint32_t b_stage = base + OFF_LHS + stage * LHS_STAGE_BYTES;
        if (lane == 0) {
          if (kb < nkb - 1 || last_steps == TILE_TOKENS / 32) {
#pragma unroll
            for (int ks = 0; ks < TILE_TOKENS / 32; ++ks) {
              const uint64_t adesc = smem_desc_sw128(a_stage + ks * 4096u, RHS_STAGE_BYTES, 1024u);
              const uint64_t bdesc = smem_desc_sw128(b_stage + ks * 4096u, LHS_BOX_BYTES, 1024u);
              mma_f8f6f4(d_tmem, adesc, bdesc, IDESC, (kb > 0 || ks > 0) ? 1u : 0u);
            }
          } else {  // the group's last block: only the K steps that hold its tokens
            const int ks0 = last_block_slot0(bounded, lo + TILE_TOKENS * kb, rem, lim);
            for (int ks = ks0; ks < ks0 + last_steps; ++ks) {
              const uint64_t adesc = smem_desc_sw128(a_stage + ks * 4096u, RHS_STAGE_BYTES, 1024u);
              const uint64_t bdesc = smem_desc_sw128(b_stage + ks * 4096u, LHS_BOX_BYTES, 1024u);
              mma_f8f6f4(d_tmem, adesc, bdesc, IDESC, (kb > 0 || ks > ks0) ? 1u : 0u);
            }
          }
          mma_commit(bar_empty + 8 * stage);  // frees the stage once these MMAs finish
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) mma_commit(bar_tfull + 8 * acc);  // accumulator ready for the epilogue
      __syncwarp();
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    // Drain outstanding MMAs before TMEM can be released.
    if (lane == 0) {
      mma_commit(bar_drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar_drain, 0)) {
        if (globaltimer_ns() - t0 > ctl.timeout_ns) break;
      }
    }
    __syncwarp();
  } else {
    // ======================= epilogue (warps 2..5) ==========================================
    const int ew = warp - EPI_WARP0;
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t zero_buf = base + OFF_ZERO;
    __nv_bfloat16* const epi_gen =
        reinterpret_cast<__nv_bfloat16*>(sbase + OFF_EPI + ew * 2 * EPI_BUF_BYTES);
    const uint32_t epi_sh = base + OFF_EPI + ew * 2 * EPI_BUF_BYTES;
    uint32_t acc = 0, acc_phase = 0;
    uint32_t nstore = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const TileInfo t = decode_tile(p, lim, tile, quarter == 0 && lane == 0);
      const int xcol = t.col0 + quarter * 32;
      const bool col_live = xcol < p.OUT_N;
      const int rows_here = min(TILE_ROWS, p.OUT_M - t.row0);
      const int nchunks = (rows_here + EPI_BOX_ROWS - 1) / EPI_BOX_ROWS;
      if (t.tokens == 0) {
        if (col_live && lane == 0) {
          for (int c = 0; c < nchunks; ++c)
            tma_store_3d(&map_c, zero_buf, xcol, t.row0 + c * EPI_BOX_ROWS, t.g);
          bulk_commit_group();
        }
        __syncwarp();
        continue;
      }
      const float scale = __ldg(p.lhs_scale + static_cast<int64_t>(t.g) * p.scale_stride) *
                          __ldg(p.rhs_scale + static_cast<int64_t>(t.g) * p.scale_stride);
      if (!warp_wait(ctl, bar_tfull + 8 * acc, acc_phase, 0x400u | acc)) break;
      tc_fence_after_sync();
      if (col_live) {
        const uint32_t t_acc = tmem_base + lane_field + acc * ACC_STRIDE_COLS;
        for (int c = 0; c < nchunks; ++c) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_acc + c * EPI_BOX_ROWS, r);
          tmem_ld_wait();
          tmem_regs_fence(r);
          const uint32_t buf = nstore & 1u;
          if (lane == 0) bulk_wait_group_read<1>();  // the store that used `buf` has read it
          __syncwarp();
          __nv_bfloat16* dst = epi_gen + buf * (EPI_BUF_BYTES / 2);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            dst[j * EPI_BOX_COLS + lane] = __float2bfloat16_rn(__uint_as_float(r[j]) * scale);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&map_c, epi_sh + buf * EPI_BUF_BYTES, xcol, t.row0 + c * EPI_BOX_ROWS,
                         t.g);
            bulk_commit_group();
          }
          ++nstore;
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  // ---- teardown -----------------------------------------------------------------------------
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace

size_t tc_smem_bytes() { return SMEM_ALLOC; }

cudaError_t tc_launch(const CUtensorMap& map_rhs, const CUtensorMap& map_lhs,
                      const CUtensorMap& map_c, const TcParams& p, int grid,
                      cudaStream_t stream) {
  vark_tc_kernel<<<grid, NUM_THREADS, SMEM_ALLOC, stream>>>(map_rhs, map_lhs, map_c, p);
  return cudaGetLastError();
}

cudaError_t tc_set_attributes() {
  return cudaFuncSetAttribute(vark_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(SMEM_ALLOC));
}

}  // namespace vark

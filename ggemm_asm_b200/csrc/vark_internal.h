// vark_internal.h - host-side interface between the C ABI (vark_capi.cu) and the kernels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace vark {

// Tile geometry of the tcgen05 path. One output tile is TILE_COLS columns of C (along OUT_N;
// the MMA M dimension) by TILE_ROWS rows of C (along OUT_M; the MMA N dimension); the token
// (reduction) dimension is consumed TILE_TOKENS rows per pipeline stage.
#ifndef VARK_TILE_TOKENS
#define VARK_TILE_TOKENS 128
#endif
#ifndef VARK_STAGES
#define VARK_STAGES 4
#endif
constexpr int TILE_COLS = 128;
constexpr int TILE_ROWS = 240;
constexpr int TILE_TOKENS = VARK_TILE_TOKENS;  // 64 or 128 (a multiple of the MMA K of 32)
constexpr int STAGES = VARK_STAGES;
constexpr int LHS_BOXES = (TILE_ROWS + 127) / 128;  // 128-wide TMA boxes per LHS stage

// Geometry of the CTA-pair (cta_group::2) kernel: a work item is 256 C columns (128 per CTA,
// the MMA M) by up to 256 C rows (the MMA N); PAIR_TOKENS tokens per pipeline stage.
// Stage shape: 192 tokens (6 MMAs per commit) x 4 stages measured best on B200 (81-84% of the
// tensor peak in cycles at the gate_up shape vs 76% for 128 x 6 and 79% for 256 x 3): fewer
// commit/wait hand-offs per MMA against enough stages to cover TMA latency.
#ifndef VARK_PAIR_TK
#define VARK_PAIR_TK 192
#endif
#ifndef VARK_PAIR_STAGES
#define VARK_PAIR_STAGES 4
#endif
constexpr int PAIR_HALF = 128;              // C columns per CTA of a pair
constexpr int PAIR_COLS = 2 * PAIR_HALF;    // C columns per work item
constexpr int PAIR_ROWS_MAX = 256;          // C rows per work item (the last one may be fewer)
constexpr int PAIR_STAGES = VARK_PAIR_STAGES;
constexpr int PAIR_TOKENS = VARK_PAIR_TK;   // tokens per pipeline stage of the pair kernel

// Per-warp C staging box of the epilogue (columns x rows), written with one TMA store.
constexpr int EPI_BOX_COLS = 32;
constexpr int EPI_BOX_ROWS = 16;

struct TcParams {
  const int64_t* group_offs;
  const float* lhs_scale;
  const float* rhs_scale;
  int32_t scale_stride;  // 0: one scale per tensor, 1: one per group
  int32_t G;
  int32_t OUT_M;
  int32_t OUT_N;
  int32_t row_tiles;     // number of row (OUT_M) tiles of the launched kernel's geometry
  int32_t col_tiles;     // number of column (OUT_N) tiles
  int64_t token_limit;   // group offsets above this are invalid
  uint32_t* status;      // device status block (bit flags in word 0)
  uint64_t timeout_ns;   // limit on one pipeline wait
  uint16_t* c;           // C (bf16 bits) and its element strides, for direct stores
  int64_t stride_cg;
  int64_t stride_cm;
  int32_t bw_lhs;        // pair kernel: width in bytes (32 or 64) of the narrow LHS maps, 0: none
  int32_t bw_rhs;        // pair kernel: the same for the narrow RHS maps
  // 1 when the caller did not state m_total (the 14-argument drop-in): the kernel reads
  // group_offs[G] and no load touches a token row at or past it (boxes that would cross it are
  // moved to end there), and offsets past it are invalid. 0: the maps end at token_limit and TMA
  // clips boxes there.
  int32_t offs_bound;
};

// Dynamic shared memory the tcgen05 kernel needs (bytes, including alignment slack).
size_t tc_smem_bytes();

// Launch the persistent tcgen05 kernel. Tensor maps are encoded by the caller.
cudaError_t tc_launch(const CUtensorMap& map_rhs, const CUtensorMap& map_lhs,
                      const CUtensorMap& map_c, const TcParams& p, int grid,
                      cudaStream_t stream);

struct SimtParams {
  const uint8_t* lhs;
  const uint8_t* rhs;
  uint16_t* c;  // bf16 bits
  const float* lhs_scale;
  const float* rhs_scale;
  int32_t scale_stride;
  const int64_t* group_offs;
  int32_t G, OUT_M, OUT_N;
  int64_t stride_lhs_m, stride_rhs_m, stride_cg, stride_cm, stride_cn;
  int64_t token_limit;
  uint32_t* status;
  int32_t offs_bound;  // as TcParams::offs_bound: offsets past group_offs[G] are invalid
};

cudaError_t simt_launch(const SimtParams& p, cudaStream_t stream);

// Raise the tcgen05 kernel's dynamic shared-memory limit (once per device).
cudaError_t tc_set_attributes();

// CTA-pair kernel (vark_tc2.cu): same parameters; row_tiles = ceil(OUT_M / PAIR_ROWS_MAX),
// col_tiles = ceil(OUT_N / PAIR_COLS), and `grid` must be even (one cluster of two CTAs per pair
// of SMs).
size_t tc2_smem_bytes();
// map_lhs / map_rhs: 2-D u8 {features, tokens}, box {128, PAIR_TOKENS}, 128-byte swizzle.
// map_lhs32 / map_rhs32: the same operands with 32-token boxes (a group's ragged last K step).
// map_lhs_n / map_lhs32_n and map_rhs_n / map_rhs32_n: boxes {w, PAIR_TOKENS} and {w, 32} with
// the w-byte swizzle, w = p.bw_lhs / p.bw_rhs (32 or 64; any valid map when 0). An item whose
// B half (MMA N / 2) fits in w bytes loads B through them: the last row tile (B = LHS, C columns
// on the TMEM lanes) and the last column tile (B = RHS, C rows on the lanes).
// Narrow width for a last tile of MMA N = n: 32 or 64 bytes when N / 2 fits, else 0.
inline int32_t pair_narrow_width(int32_t n) { return n <= 64 ? 32 : (n <= 128 ? 64 : 0); }
struct PairMaps {
  CUtensorMap lhs, rhs, lhs32, rhs32, lhs_n, lhs32_n, rhs_n, rhs32_n;
  CUtensorMap c;     // C as {OUT_N, OUT_M, G} bf16, box {32, 32, 1}, 64-byte swizzle
  int32_t bw_lhs;    // narrow width of lhs_n / lhs32_n (TcParams::bw_lhs)
  int32_t bw_rhs;    // the same for rhs_n / rhs32_n
};
cudaError_t tc2_launch(const PairMaps& maps, const TcParams& p, int grid, cudaStream_t stream);

// The driver's cuTensorMapEncodeTiled, resolved once per process (vark_capi.cu); nullptr if the
// driver lacks it. Resolving it touches no device memory.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Every map of one pair-kernel launch (vark_capi.cu), shared by all entry points that launch it:
// operands with `token_dim` rows (row pitches slm / srm bytes), C with element strides scg / scm.
// A NULL operand (a call without tokens) is mapped onto c, which is then never loaded through.
// False if the driver rejects a map.
bool encode_pair_maps(PairMaps* m, const void* lhs, const void* rhs, void* c, int32_t G,
                      int32_t OUT_M, int32_t OUT_N, int32_t slm, int32_t srm, int32_t scg,
                      int32_t scm, uint64_t token_dim);
cudaError_t tc2_set_attributes();

// Fixed-K grouped GEMM (vark_fwd.cu): C[t, :] = sA * sB_g * A[t, :] . B[g]^T for the tokens t of
// expert g; A [tokens, K] is K-major fp8, B [G, N, K] (K-major) or [G, K, N] (N-major) e4m3, C
// bf16. Tensor maps (encoded by the caller): A 2D u8 {K, rows} box {128, 128}; B 3D u8 {K, N, G}
// box {128, 128, 1} or {N, K, G} box {128, 256, 1}; C 2D bf16 {N, rows} box {32, 32} with the
// 64-byte swizzle. The kernel rebuilds the A and C maps per expert.
struct FwdParams {
  const int64_t* group_offs;
  const float* a_scale;   // one value, or G values when scale_stride == 1
  const float* b_scale;   // likewise
  int32_t scale_stride;
  int32_t b_mn_major;     // 0: B [G, N, K] (K contiguous); 1: B [G, K, N] (N contiguous)
  int32_t G, N, K;
  int32_t n_tiles;        // ceil(N / 256)
  int32_t a_fmt;          // 0: e4m3, 1: e5m2 (B is e4m3)
  int64_t token_limit;    // group offsets above this are invalid
  uint32_t* status;
  uint64_t timeout_ns;
  uint16_t* c;            // C base (bf16 bits); row pitch in elements (a multiple of 8)
  int64_t stride_cm;
  int32_t offs_bound;     // as TcParams::offs_bound, for the rows of A
};
size_t fwd2_smem_bytes();
cudaError_t fwd2_launch(const CUtensorMap& map_a, const CUtensorMap& map_b,
                        const CUtensorMap& map_c, const FwdParams& p, int grid,
                        cudaStream_t stream);
cudaError_t fwd2_set_attributes();

// Library-wide helpers (vark_capi.cu): the current device's status block and SM count (set up
// on first use; returns a GGEMM_VARK_E* code), and recording of a failed CUDA call for
// ggemm_vark_last_cuda_error (returns GGEMM_VARK_ECUDA).
int device_status_block(uint32_t** status, int* sm_count);
int record_cuda_error(cudaError_t e);

// Workspace bytes of the quantisation kernel (vark_quant.cu) for `units` scaling units.
size_t quant_workspace_bytes(int32_t units);

}  // namespace vark

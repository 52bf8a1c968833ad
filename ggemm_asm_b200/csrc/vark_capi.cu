// vark_capi.cu - the C ABI (include/ggemm_vark.h): argument checks, path choice, TMA tensor
// maps, per-device state, launch.
//
// Replaces the reference's launch boundary: prepare_variable_k_args / launch_variable_k_kernel
// (ggemm-asm bench.py:364-413) and the KernelArgs packing + hipModuleLaunchKernel of
// launcher.cpp:16-33,123-168. The reference launches a fixed grid (#CUs x 512 threads, 64 KiB
// LDS); here the grid is one persistent CTA per SM and the geometry is internal.
#include <cudaTypedefs.h>

#include <climits>
#include <cstring>
#include <mutex>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"

namespace vark {
cudaError_t tc_set_attributes();
}

namespace {

constexpr int kMaxDevices = 64;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s per pipeline wait
constexpr int64_t kTokenCoordLimit = INT32_MAX;        // TMA coordinates are int32
constexpr size_t kStatusBytes = 4096;  // status words

thread_local int t_last_cuda_error = 0;

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  uint32_t* status = nullptr;    // status block owned by the library
};

std::mutex g_mutex;
DeviceState g_dev[kMaxDevices];

int fail_cuda(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return GGEMM_VARK_ECUDA;
}

// Resolve per-device state once (SM count, compute capability, status block, kernel
// attributes). Returns a GGEMM_VARK_E* code.
int get_device(DeviceState** out, int* dev_out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return GGEMM_VARK_ENO_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return GGEMM_VARK_ENO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& s = g_dev[dev];
  if (!s.ready) {
    if ((e = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return fail_cuda(e);
    if ((e = cudaDeviceGetAttribute(&s.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return fail_cuda(e);
    if ((e = cudaDeviceGetAttribute(&s.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return fail_cuda(e);
    if (s.cc_major != 10 || s.cc_minor != 0) return GGEMM_VARK_ENO_DEVICE;  // sm_100 only
    if ((e = vark::tc_set_attributes()) != cudaSuccess) return fail_cuda(e);
    if ((e = vark::tc2_set_attributes()) != cudaSuccess) return fail_cuda(e);
    if ((e = vark::fwd2_set_attributes()) != cudaSuccess) return fail_cuda(e);
    // One allocation per device, kept until exit: the status block.
    void* blk = nullptr;
    const size_t bytes = kStatusBytes;
    if ((e = cudaMalloc(&blk, bytes)) != cudaSuccess) return fail_cuda(e);
    if ((e = cudaMemset(blk, 0, bytes)) != cudaSuccess) {
      cudaFree(blk);
      return fail_cuda(e);
    }
    s.status = static_cast<uint32_t*>(blk);
    if (vark::tensor_map_encoder() == nullptr) return fail_cuda(cudaErrorSymbolNotFound);
    s.ready = true;
  }
  *out = &s;
  if (dev_out) *dev_out = dev;
  return GGEMM_VARK_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool tc_layout_ok(const void* lhs, const void* rhs, void* c, int32_t OUT_M, int32_t OUT_N,
                  int32_t slm, int32_t srm, int32_t scg, int32_t scm, int32_t scn) {
  (void)OUT_M;
  if (!aligned16(lhs) || !aligned16(rhs) || !aligned16(c)) return false;
  if (slm % 16 != 0 || srm % 16 != 0) return false;              // fp8 row pitch, bytes
  if (scn != 1) return false;                                     // C rows contiguous
  if ((2ll * scm) % 16 != 0 || (2ll * scg) % 16 != 0) return false;  // bf16 pitches
  // A TMA store writes a C row up to the next 16-byte boundary: with OUT_N % 8 != 0 it would
  // overwrite up to 7 of the caller's columns past OUT_N.
  if (OUT_N % 8 != 0) return false;
  return true;
}

// lhs/rhs may be NULL only when the caller states that there are no tokens (m_total == 0):
// every group is then empty and the operands are never read.
int check_args(const void* lhs, const void* rhs, void* c, const float* ls, const float* rs,
               const int64_t* offs, int32_t G, int32_t OUT_M, int32_t OUT_N, int32_t slm,
               int32_t srm, int32_t scg, int32_t scm, int32_t scn, int64_t m_total) {
  if (m_total != 0 && (lhs == nullptr || rhs == nullptr)) return GGEMM_VARK_EINVAL_PTR;
  if (c == nullptr || ls == nullptr || rs == nullptr || offs == nullptr)
    return GGEMM_VARK_EINVAL_PTR;
  if (G < 0 || OUT_M <= 0 || OUT_N <= 0) return GGEMM_VARK_EINVAL_SHAPE;
  if (slm < OUT_M || srm < OUT_N) return GGEMM_VARK_EINVAL_STRIDE;
  if (scn <= 0 || scm <= 0 || scg <= 0) return GGEMM_VARK_EINVAL_STRIDE;
  return GGEMM_VARK_OK;
}

CUresult encode_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_pitch, uint32_t box_tokens, uint32_t box_inner = 128,
                      CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_pitch};
  const cuuint32_t box[2] = {box_inner, box_tokens};
  const cuuint32_t estr[2] = {1, 1};
  const auto enc = vark::tensor_map_encoder();
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Narrow-box maps of an operand (boxes {w, box_tokens} and {w, 32}, w-byte swizzle); w = 0 (no
// narrow items) still encodes valid 32-byte maps, which the kernel never loads through.
CUresult encode_narrow(CUtensorMap* map, CUtensorMap* map32, const void* base, int32_t features,
                       uint64_t tokens, int32_t pitch, uint32_t box_tokens, int32_t w) {
  const uint32_t bw = w == 64 ? 64u : 32u;
  const CUtensorMapSwizzle sw = w == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUresult r = encode_2d_u8(map, base, static_cast<uint64_t>(features), tokens,
                                  static_cast<uint64_t>(pitch), box_tokens, bw, sw);
  if (r != CUDA_SUCCESS) return r;
  return encode_2d_u8(map32, base, static_cast<uint64_t>(features), tokens,
                      static_cast<uint64_t>(pitch), 32, bw, sw);
}

// C as a 3-D bf16 tensor {OUT_N, OUT_M, G}; the box and swizzle follow the kernel's epilogue.
CUresult encode_c(CUtensorMap* map, void* c, int32_t G, int32_t OUT_M, int32_t OUT_N,
                  int32_t scg, int32_t scm, uint32_t box_cols, uint32_t box_rows,
                  CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(OUT_N), static_cast<cuuint64_t>(OUT_M),
                              static_cast<cuuint64_t>(G)};
  const cuuint64_t strides[2] = {2ull * static_cast<cuuint64_t>(scm),
                                 2ull * static_cast<cuuint64_t>(scg)};
  const cuuint32_t box[3] = {box_cols, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const auto enc = vark::tensor_map_encoder();
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, c, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int run(const void* lhs, const void* rhs, void* c, const float* ls, const float* rs,
        const int64_t* offs, int32_t G, int32_t OUT_M, int32_t OUT_N, int32_t slm, int32_t srm,
        int32_t scg, int32_t scm, int32_t scn, int64_t m_total, int32_t scale_stride,
        int32_t path, void* status, uint64_t timeout_ns, void* stream) {
  int rc = check_args(lhs, rhs, c, ls, rs, offs, G, OUT_M, OUT_N, slm, srm, scg, scm, scn,
                      m_total);
  if (rc != GGEMM_VARK_OK) return rc;
  if (scale_stride != 0 && scale_stride != 1) return GGEMM_VARK_EINVAL_ARG;
  if (path < GGEMM_VARK_PATH_AUTO || path > GGEMM_VARK_PATH_TCGEN05_1SM)
    return GGEMM_VARK_EINVAL_ARG;
  if (m_total < -1) return GGEMM_VARK_EINVAL_ARG;
  if (status != nullptr && !aligned16(status)) return GGEMM_VARK_EINVAL_ARG;
  if (G == 0) return GGEMM_VARK_OK;

  DeviceState* dev = nullptr;
  rc = get_device(&dev, nullptr);
  if (rc != GGEMM_VARK_OK) return rc;

  const int64_t token_limit =
      m_total >= 0 ? (m_total < kTokenCoordLimit ? m_total : kTokenCoordLimit) : kTokenCoordLimit;
  uint32_t* st = status != nullptr ? static_cast<uint32_t*>(status) : dev->status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const bool tc_ok = tc_layout_ok(lhs, rhs, c, OUT_M, OUT_N, slm, srm, scg, scm, scn);
  bool use_tc = tc_ok;
  if ((path == GGEMM_VARK_PATH_TCGEN05 || path == GGEMM_VARK_PATH_TCGEN05_1SM) && !tc_ok)
    return GGEMM_VARK_ELAYOUT;
  if (path == GGEMM_VARK_PATH_SIMT) use_tc = false;

  if (!use_tc) {
    vark::SimtParams sp;
    sp.lhs = static_cast<const uint8_t*>(lhs);
    sp.rhs = static_cast<const uint8_t*>(rhs);
    sp.c = static_cast<uint16_t*>(c);
    sp.lhs_scale = ls;
    sp.rhs_scale = rs;
    sp.scale_stride = scale_stride;
    sp.group_offs = offs;
    sp.G = G;
    sp.OUT_M = OUT_M;
    sp.OUT_N = OUT_N;
    sp.stride_lhs_m = slm;
    sp.stride_rhs_m = srm;
    sp.stride_cg = scg;
    sp.stride_cm = scm;
    sp.stride_cn = scn;
    sp.token_limit = token_limit;
    sp.status = st;
    sp.offs_bound = m_total < 0 ? 1 : 0;
    if (G > 65535) return GGEMM_VARK_ETOO_LARGE;
    cudaError_t e = vark::simt_launch(sp, s);
    return e == cudaSuccess ? GGEMM_VARK_OK : fail_cuda(e);
  }

  // Tensor-core paths.
  const bool pair = path != GGEMM_VARK_PATH_TCGEN05_1SM && dev->sm_count >= 2;
  const int32_t rt = pair ? vark::PAIR_ROWS_MAX : vark::TILE_ROWS;
  const int32_t ct = pair ? vark::PAIR_COLS : vark::TILE_COLS;
  const int32_t row_tiles = (OUT_M + rt - 1) / rt;
  const int32_t col_tiles = (OUT_N + ct - 1) / ct;
  const int64_t tiles = static_cast<int64_t>(G) * row_tiles * col_tiles;
  if (tiles > INT32_MAX) return GGEMM_VARK_ETOO_LARGE;

  // With no tokens the operand maps are never used for a load; they only need to be valid
  // descriptors, so they point at C.
  const uint64_t token_dim = token_limit > 0 ? static_cast<uint64_t>(token_limit) : 1u;
  vark::PairMaps pm;
  CUtensorMap map_rhs, map_lhs, map_c;  // the single-CTA kernel's maps
  if (pair) {
    // The pair kernel loads a group's ragged last K step as one 32-token chunk, and the B of
    // its last row tile (LHS) and last column tile (RHS) through narrow boxes when their B
    // halves fit in 32 or 64 bytes.
    if (!vark::encode_pair_maps(&pm, lhs, rhs, c, G, OUT_M, OUT_N, slm, srm, scg, scm,
                                token_dim))
      return GGEMM_VARK_ELAYOUT;
  } else if (encode_2d_u8(&map_rhs, rhs != nullptr ? rhs : c, static_cast<uint64_t>(OUT_N),
                          token_dim, static_cast<uint64_t>(srm), vark::TILE_TOKENS) !=
                 CUDA_SUCCESS ||
             encode_2d_u8(&map_lhs, lhs != nullptr ? lhs : c, static_cast<uint64_t>(OUT_M),
                          token_dim, static_cast<uint64_t>(slm), vark::TILE_TOKENS) !=
                 CUDA_SUCCESS ||
             encode_c(&map_c, c, G, OUT_M, OUT_N, scg, scm, vark::EPI_BOX_COLS,
                      vark::EPI_BOX_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS) {
    return GGEMM_VARK_ELAYOUT;
  }

  vark::TcParams tp;
  tp.group_offs = offs;
  tp.lhs_scale = ls;
  tp.rhs_scale = rs;
  tp.scale_stride = scale_stride;
  tp.G = G;
  tp.OUT_M = OUT_M;
  tp.OUT_N = OUT_N;
  tp.row_tiles = row_tiles;
  tp.col_tiles = col_tiles;
  tp.token_limit = token_limit;
  tp.status = st;
  tp.timeout_ns = timeout_ns != 0 ? timeout_ns : kDefaultTimeoutNs;
  tp.c = static_cast<uint16_t*>(c);
  tp.stride_cg = scg;
  tp.stride_cm = scm;
  tp.bw_lhs = pair ? pm.bw_lhs : 0;
  tp.bw_rhs = pair ? pm.bw_rhs : 0;
  tp.offs_bound = m_total < 0 ? 1 : 0;
  cudaError_t e;
  if (pair) {
    const int64_t clusters = tiles < dev->sm_count / 2 ? tiles : dev->sm_count / 2;
    e = vark::tc2_launch(pm, tp, static_cast<int>(2 * clusters), s);
  } else {
    const int grid = static_cast<int>(tiles < dev->sm_count ? tiles : dev->sm_count);
    e = vark::tc_launch(map_rhs, map_lhs, map_c, tp, grid, s);
  }
  return e == cudaSuccess ? GGEMM_VARK_OK : fail_cuda(e);
}

// The fixed-K grouped GEMM (forward / data-gradient sites): argument checks, tensor maps, launch.
int run_fwd(const void* a, const void* b, void* c, const float* a_scale, const float* b_scale,
            const int64_t* offs, int32_t G, int32_t N, int32_t K, int32_t sam, int32_t sbg,
            int32_t sbn, int32_t scm, int32_t scn, int64_t m_total, int32_t a_fmt,
            int32_t scale_stride, int32_t b_layout, void* status, uint64_t timeout_ns,
            void* stream) {
  if (a_scale == nullptr || b_scale == nullptr || offs == nullptr) return GGEMM_VARK_EINVAL_PTR;
  if (m_total != 0 && (a == nullptr || b == nullptr || c == nullptr)) return GGEMM_VARK_EINVAL_PTR;
  if (G < 0 || N <= 0 || K <= 0) return GGEMM_VARK_EINVAL_SHAPE;
  if (b_layout != 0 && b_layout != 1) return GGEMM_VARK_EINVAL_ARG;
  // B rows: N rows of K (layout 0) or K rows of N (layout 1), stride_bn apart.
  const int32_t b_rows = b_layout == 0 ? N : K, b_row = b_layout == 0 ? K : N;
  if (sam < K || sbn < b_row || scn <= 0 || scm < N ||
      static_cast<int64_t>(sbg) < static_cast<int64_t>(b_rows - 1) * sbn + b_row)
    return GGEMM_VARK_EINVAL_STRIDE;
  if ((a_fmt != 0 && a_fmt != 1) || (scale_stride != 0 && scale_stride != 1) || m_total < -1)
    return GGEMM_VARK_EINVAL_ARG;
  if (status != nullptr && !aligned16(status)) return GGEMM_VARK_EINVAL_ARG;
  if (a != nullptr && (!aligned16(a) || !aligned16(b) || !aligned16(c) || sam % 16 != 0 ||
                       sbn % 16 != 0 || sbg % 16 != 0 || scn != 1 || (2ll * scm) % 16 != 0))
    return GGEMM_VARK_ELAYOUT;
  if (G == 0 || m_total == 0) return GGEMM_VARK_OK;

  DeviceState* dev = nullptr;
  int rc = get_device(&dev, nullptr);
  if (rc != GGEMM_VARK_OK) return rc;
  if (dev->sm_count < 2) return GGEMM_VARK_ENO_DEVICE;
  const int64_t token_limit =
      m_total >= 0 ? (m_total < kTokenCoordLimit ? m_total : kTokenCoordLimit) : kTokenCoordLimit;

  // A [rows, K] u8 and C [rows, N] bf16 over all M_total rows: the kernel addresses an expert's
  // rows by coordinate (off_g + row) and writes each expert's ragged last rows without TMA.
  CUtensorMap map_a, map_b, map_c;
  const auto enc = vark::tensor_map_encoder();
  const uint64_t rows = token_limit > 0 ? static_cast<uint64_t>(token_limit) : 1u;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(sam)};
    const cuuint32_t box[2] = {128, 128};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GGEMM_VARK_ELAYOUT;
  }
  {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(b_row), static_cast<cuuint64_t>(b_rows),
                                static_cast<cuuint64_t>(G)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(sbn), static_cast<cuuint64_t>(sbg)};
    const cuuint32_t box[3] = {128, b_layout == 0 ? 128u : 256u, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(b), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GGEMM_VARK_ELAYOUT;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), rows};
    const cuuint64_t strides[1] = {2ull * static_cast<cuuint64_t>(scm)};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GGEMM_VARK_ELAYOUT;
  }
  vark::FwdParams fp;
  fp.group_offs = offs;
  fp.a_scale = a_scale;
  fp.b_scale = b_scale;
  fp.scale_stride = scale_stride;
  fp.b_mn_major = b_layout;
  fp.G = G;
  fp.N = N;
  fp.K = K;
  fp.n_tiles = (N + 255) / 256;
  fp.a_fmt = a_fmt;
  fp.token_limit = token_limit;
  fp.status = status != nullptr ? static_cast<uint32_t*>(status) : dev->status;
  fp.timeout_ns = timeout_ns != 0 ? timeout_ns : kDefaultTimeoutNs;
  fp.c = static_cast<uint16_t*>(c);
  fp.stride_cm = scm;
  fp.offs_bound = m_total < 0 ? 1 : 0;
  // The item count depends on the group sizes, which stay on the device: one cluster per pair
  // of SMs, each walking the items round-robin (clusters without items exit at once).
  const cudaError_t e = vark::fwd2_launch(map_a, map_b, map_c, fp, 2 * (dev->sm_count / 2),
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GGEMM_VARK_OK : fail_cuda(e);
}

}  // namespace

namespace vark {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess && p != nullptr)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

bool encode_pair_maps(PairMaps* m, const void* lhs, const void* rhs, void* c, int32_t G,
                      int32_t OUT_M, int32_t OUT_N, int32_t slm, int32_t srm, int32_t scg,
                      int32_t scm, uint64_t token_dim) {
  if (tensor_map_encoder() == nullptr) return false;
  const void* lb = lhs != nullptr ? lhs : c;
  const void* rb = rhs != nullptr ? rhs : c;
  const int32_t row_tiles = (OUT_M + PAIR_ROWS_MAX - 1) / PAIR_ROWS_MAX;
  const int32_t col_tiles = (OUT_N + PAIR_COLS - 1) / PAIR_COLS;
  const int32_t last_rows = OUT_M - PAIR_ROWS_MAX * (row_tiles - 1);
  const int32_t last_cols = OUT_N - PAIR_COLS * (col_tiles - 1);
  m->bw_lhs = pair_narrow_width((last_rows + 31) & ~31);
  m->bw_rhs = last_cols < PAIR_COLS ? pair_narrow_width((last_cols + 31) & ~31) : 0;
  const uint64_t fm = static_cast<uint64_t>(OUT_M), fn = static_cast<uint64_t>(OUT_N);
  return encode_2d_u8(&m->rhs, rb, fn, token_dim, static_cast<uint64_t>(srm), PAIR_TOKENS) ==
             CUDA_SUCCESS &&
         encode_2d_u8(&m->lhs, lb, fm, token_dim, static_cast<uint64_t>(slm), PAIR_TOKENS) ==
             CUDA_SUCCESS &&
         encode_2d_u8(&m->rhs32, rb, fn, token_dim, static_cast<uint64_t>(srm), 32) ==
             CUDA_SUCCESS &&
         encode_2d_u8(&m->lhs32, lb, fm, token_dim, static_cast<uint64_t>(slm), 32) ==
             CUDA_SUCCESS &&
         encode_narrow(&m->lhs_n, &m->lhs32_n, lb, OUT_M, token_dim, slm, PAIR_TOKENS,
                       m->bw_lhs) == CUDA_SUCCESS &&
         encode_narrow(&m->rhs_n, &m->rhs32_n, rb, OUT_N, token_dim, srm, PAIR_TOKENS,
                       m->bw_rhs) == CUDA_SUCCESS &&
         encode_c(&m->c, c, G, OUT_M, OUT_N, scg, scm, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) ==
             CUDA_SUCCESS;
}

// Shared with the other entry points of the library (vark_quant.cu): the current device's status
// block and SM count, set up on first use.
int device_status_block(uint32_t** status, int* sm_count) {
  DeviceState* dev = nullptr;
  const int rc = get_device(&dev, nullptr);
  if (rc != GGEMM_VARK_OK) return rc;
  *status = dev->status;
  *sm_count = dev->sm_count;
  return GGEMM_VARK_OK;
}

int record_cuda_error(cudaError_t e) {
  cudaGetLastError();
  return fail_cuda(e);
}

}  // namespace vark

extern "C" {

int ggemm_vark_fp8_wgrad(const void* lhs, const void* rhs, void* c, const float* lhs_scale,
                         const float* rhs_scale, const int64_t* group_offs, int32_t G,
                         int32_t OUT_M, int32_t OUT_N, int32_t stride_lhs_m,
                         int32_t stride_rhs_m, int32_t stride_cg, int32_t stride_cm,
                         int32_t stride_cn, void* stream) {
  return run(lhs, rhs, c, lhs_scale, rhs_scale, group_offs, G, OUT_M, OUT_N, stride_lhs_m,
             stride_rhs_m, stride_cg, stride_cm, stride_cn, /*m_total=*/-1, /*scale_stride=*/0,
             GGEMM_VARK_PATH_AUTO, /*status=*/nullptr, /*timeout_ns=*/0, stream);
}

int ggemm_vark_fp8_wgrad_ex(const void* lhs, const void* rhs, void* c, const float* lhs_scale,
                            const float* rhs_scale, const int64_t* group_offs, int32_t G,
                            int32_t OUT_M, int32_t OUT_N, int32_t stride_lhs_m,
                            int32_t stride_rhs_m, int32_t stride_cg, int32_t stride_cm,
                            int32_t stride_cn, int64_t m_total, int32_t scale_stride,
                            int32_t path, void* status, uint64_t timeout_ns, void* stream) {
  return run(lhs, rhs, c, lhs_scale, rhs_scale, group_offs, G, OUT_M, OUT_N, stride_lhs_m,
             stride_rhs_m, stride_cg, stride_cm, stride_cn, m_total, scale_stride, path, status,
             timeout_ns, stream);
}

int ggemm_vark_grouped_fp8_fwd(const void* a, const void* b, void* c, const float* a_scale,
                               const float* b_scale, const int64_t* group_offs, int32_t G,
                               int32_t N, int32_t K, int32_t stride_am, int32_t stride_bg,
                               int32_t stride_bn, int32_t stride_cm, int32_t stride_cn,
                               void* stream) {
  return run_fwd(a, b, c, a_scale, b_scale, group_offs, G, N, K, stride_am, stride_bg, stride_bn,
                 stride_cm, stride_cn, /*m_total=*/-1, /*a_fmt=*/0, /*scale_stride=*/0,
                 /*b_layout=*/0, /*status=*/nullptr, /*timeout_ns=*/0, stream);
}

int ggemm_vark_grouped_fp8_fwd_ex(const void* a, const void* b, void* c, const float* a_scale,
                                  const float* b_scale, const int64_t* group_offs, int32_t G,
                                  int32_t N, int32_t K, int32_t stride_am, int32_t stride_bg,
                                  int32_t stride_bn, int32_t stride_cm, int32_t stride_cn,
                                  int64_t m_total, int32_t a_fmt, int32_t scale_stride,
                                  int32_t b_layout, void* status, uint64_t timeout_ns,
                                  void* stream) {
  return run_fwd(a, b, c, a_scale, b_scale, group_offs, G, N, K, stride_am, stride_bg, stride_bn,
                 stride_cm, stride_cn, m_total, a_fmt, scale_stride, b_layout, status,
                 timeout_ns, stream);
}

int ggemm_vark_read_status(void* status, int clear, uint32_t* bits_out) {
  if (bits_out == nullptr) return GGEMM_VARK_EINVAL_PTR;
  uint32_t* blk = static_cast<uint32_t*>(status);
  if (blk == nullptr) {
    DeviceState* dev = nullptr;
    const int rc = get_device(&dev, nullptr);
    if (rc != GGEMM_VARK_OK) return rc;
    blk = dev->status;
  }
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail_cuda(e);
  uint32_t words[2] = {0, 0};
  if ((e = cudaMemcpy(words, blk, sizeof(words), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return fail_cuda(e);
  *bits_out = words[0];
  if (clear && (e = cudaMemset(blk, 0, 256)) != cudaSuccess) return fail_cuda(e);
  if (clear && (e = cudaDeviceSynchronize()) != cudaSuccess) return fail_cuda(e);
  return GGEMM_VARK_OK;
}

int ggemm_vark_read_status_stream(void* status, int clear, uint32_t* words_out, int32_t nwords,
                                  void* stream) {
  if (words_out == nullptr) return GGEMM_VARK_EINVAL_PTR;
  if (nwords < 1 || nwords > 8) return GGEMM_VARK_EINVAL_ARG;
  if (status != nullptr && !aligned16(status)) return GGEMM_VARK_EINVAL_ARG;
  uint32_t* blk = static_cast<uint32_t*>(status);
  if (blk == nullptr) {
    DeviceState* dev = nullptr;
    const int rc = get_device(&dev, nullptr);
    if (rc != GGEMM_VARK_OK) return rc;
    blk = dev->status;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t words[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(words, blk, sizeof(uint32_t) * nwords, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail_cuda(e);
  for (int i = 0; i < nwords; ++i) words_out[i] = words[i];
  // Clear only the words this library writes (0, 1, 4, 5): word 3 holds the test hook.
  if (clear) {
    if ((e = cudaMemsetAsync(blk, 0, 2 * sizeof(uint32_t), s)) != cudaSuccess) return fail_cuda(e);
    if ((e = cudaMemsetAsync(blk + 4, 0, 2 * sizeof(uint32_t), s)) != cudaSuccess)
      return fail_cuda(e);
  }
  return GGEMM_VARK_OK;
}

int ggemm_vark_device_bytes(int32_t device, uint64_t* bytes_out) {
  if (bytes_out == nullptr) return GGEMM_VARK_EINVAL_PTR;
  if (device < 0 || device >= kMaxDevices) return GGEMM_VARK_EINVAL_ARG;
  std::lock_guard<std::mutex> lock(g_mutex);
  *bytes_out = g_dev[device].status != nullptr ? kStatusBytes : 0;
  return GGEMM_VARK_OK;
}

int ggemm_vark_tc_supported(const void* lhs, const void* rhs, void* c, int32_t OUT_M,
                            int32_t OUT_N, int32_t stride_lhs_m, int32_t stride_rhs_m,
                            int32_t stride_cg, int32_t stride_cm, int32_t stride_cn) {
  return tc_layout_ok(lhs, rhs, c, OUT_M, OUT_N, stride_lhs_m, stride_rhs_m, stride_cg,
                      stride_cm, stride_cn)
             ? 1
             : 0;
}

const char* ggemm_vark_strerror(int code) {
  switch (code) {
    case GGEMM_VARK_OK: return "success";
    case GGEMM_VARK_EINVAL_PTR: return "a required pointer is NULL";
    case GGEMM_VARK_EINVAL_SHAPE: return "G < 0, OUT_M <= 0 or OUT_N <= 0";
    case GGEMM_VARK_EINVAL_STRIDE: return "a stride is not positive or is smaller than its row";
    case GGEMM_VARK_EINVAL_ARG: return "an argument is outside its documented range";
    case GGEMM_VARK_ENO_DEVICE: return "no CUDA device, or the current device is not sm_100";
    case GGEMM_VARK_ECUDA: return "a CUDA runtime or driver call failed";
    case GGEMM_VARK_ELAYOUT: return "layout cannot be expressed for the tensor-core path";
    case GGEMM_VARK_ETOO_LARGE: return "a size exceeds the documented maximum";
    default: return "unknown error code";
  }
}

int ggemm_vark_last_cuda_error(void) { return t_last_cuda_error; }

int ggemm_vark_version(void) { return 0x000100; }

}  // extern "C"

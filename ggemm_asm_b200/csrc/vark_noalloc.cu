// vark_noalloc.cu - ggemm_vark_fp8_wgrad_noalloc: the grouped wgrad without any allocation.
//
// Who needs this. Some callers cannot let a library call cudaMalloc: code that runs inside a
// memory pool or arena owned by a framework (every byte must come from the arena), allocators
// with strict accounting, processes that fixed their device footprint up front, and paths that
// must not hit the device-wide synchronisation cudaMalloc/cudaFree can imply. The regular entry
// points make one cudaMalloc per device on first use (the status words). This entry point runs
// the same CTA-pair tensor-core kernel with that scratch taken from a fixed, file-scope device
// array instead, so it never allocates.
//
// What it costs. The array below (NOALLOC_SCRATCH_BYTES = 4 KiB) exists on every GPU that
// loads this library, for the life of the process, whether or not this entry point is called.
// All calls on a device share it and it keeps the last call's contents; the status words are
// cleared (cudaMemsetAsync on the caller's stream) at the start of every call. Calls that
// overlap on the GPU (different streams, no ordering between them) race on the status words.
#include <cudaTypedefs.h>

#include <climits>
#include <mutex>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"

namespace {

constexpr size_t kScratchBytes = 4096;  // status words
static_assert(kScratchBytes == GGEMM_VARK_NOALLOC_SCRATCH_BYTES, "header and file disagree");

// The scratch. In host code this name is only a stand-in for the device object: the device
// address comes from cudaGetSymbolAddress below and is what the kernel receives.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
constexpr int64_t kTokenCoordLimit = INT32_MAX;
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct Device {
  bool ready = false;
  int sm_count = 0;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
};

std::mutex g_mu;
Device g_devs[kMaxDevices];

// Once per device, with that device current: resolve the scratch array's device address and
// the kernel attributes. Nothing here allocates.
int setup(Device** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return GGEMM_VARK_ENO_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  Device& d = g_devs[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      cudaGetLastError();
      return GGEMM_VARK_ECUDA;
    }
    if (major != 10 || minor != 0) return GGEMM_VARK_ENO_DEVICE;
    if (d.sm_count < 2) return GGEMM_VARK_ENO_DEVICE;  // the kernel runs on CTA pairs
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return GGEMM_VARK_ECUDA;
    }
    if (vark::tc2_set_attributes() != cudaSuccess) {
      cudaGetLastError();
      return GGEMM_VARK_ECUDA;
    }
    // The same encoder and map layout as the regular entry points (vark_capi.cu).
    if (vark::tensor_map_encoder() == nullptr) return GGEMM_VARK_ECUDA;
    d.scratch = static_cast<uint8_t*>(ptr);
    d.ready = true;
  }
  *out = &d;
  return GGEMM_VARK_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int ggemm_vark_fp8_wgrad_noalloc(const void* lhs, const void* rhs, void* c,
                                            const float* lhs_scale, const float* rhs_scale,
                                            const int64_t* group_offs, int32_t G, int32_t OUT_M,
                                            int32_t OUT_N, int32_t stride_lhs_m,
                                            int32_t stride_rhs_m, int32_t stride_cg,
                                            int32_t stride_cm, int32_t stride_cn,
                                            int64_t m_total, int32_t scale_stride,
                                            void* status, void* stream) {
  // Same argument rules as ggemm_vark_fp8_wgrad_ex (lhs and rhs may be NULL only with
  // m_total == 0), restricted to layouts the tensor-core kernel takes (this entry point has no
  // CUDA-core fallback).
  if (c == nullptr || lhs_scale == nullptr || rhs_scale == nullptr || group_offs == nullptr)
    return GGEMM_VARK_EINVAL_PTR;
  if (m_total != 0 && (lhs == nullptr || rhs == nullptr)) return GGEMM_VARK_EINVAL_PTR;
  if (G < 0 || OUT_M <= 0 || OUT_N <= 0) return GGEMM_VARK_EINVAL_SHAPE;
  if (stride_lhs_m < OUT_M || stride_rhs_m < OUT_N || stride_cn <= 0 || stride_cm <= 0 ||
      stride_cg <= 0)
    return GGEMM_VARK_EINVAL_STRIDE;
  if ((scale_stride != 0 && scale_stride != 1) || m_total < -1) return GGEMM_VARK_EINVAL_ARG;
  if (status != nullptr && !aligned16(status)) return GGEMM_VARK_EINVAL_ARG;
  if (!aligned16(lhs) || !aligned16(rhs) || !aligned16(c) || stride_lhs_m % 16 != 0 ||
      stride_rhs_m % 16 != 0 || stride_cn != 1 || (2ll * stride_cm) % 16 != 0 ||
      (2ll * stride_cg) % 16 != 0 || OUT_N % 8 != 0)  // TMA stores write 16-byte row pieces
    return GGEMM_VARK_ELAYOUT;
  if (G == 0) return GGEMM_VARK_OK;

  Device* d = nullptr;
  int rc = setup(&d);
  if (rc != GGEMM_VARK_OK) return rc;

  const int32_t row_tiles = (OUT_M + vark::PAIR_ROWS_MAX - 1) / vark::PAIR_ROWS_MAX;
  const int32_t col_tiles = (OUT_N + vark::PAIR_COLS - 1) / vark::PAIR_COLS;
  const int64_t items = static_cast<int64_t>(G) * row_tiles * col_tiles;
  if (items > INT32_MAX) return GGEMM_VARK_ETOO_LARGE;

  const int64_t token_limit =
      m_total >= 0 ? (m_total < kTokenCoordLimit ? m_total : kTokenCoordLimit) : kTokenCoordLimit;
  const uint64_t token_dim = token_limit > 0 ? static_cast<uint64_t>(token_limit) : 1u;
  vark::PairMaps maps;
  if (!vark::encode_pair_maps(&maps, lhs, rhs, c, G, OUT_M, OUT_N, stride_lhs_m, stride_rhs_m,
                              stride_cg, stride_cm, token_dim))
    return GGEMM_VARK_ELAYOUT;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* st = status != nullptr ? static_cast<uint32_t*>(status)
                                   : reinterpret_cast<uint32_t*>(d->scratch);
  if (status == nullptr && cudaMemsetAsync(d->scratch, 0, 32, s) != cudaSuccess) {
    cudaGetLastError();
    return GGEMM_VARK_ECUDA;
  }

  vark::TcParams tp;
  tp.group_offs = group_offs;
  tp.lhs_scale = lhs_scale;
  tp.rhs_scale = rhs_scale;
  tp.scale_stride = scale_stride;
  tp.G = G;
  tp.OUT_M = OUT_M;
  tp.OUT_N = OUT_N;
  tp.row_tiles = row_tiles;
  tp.col_tiles = col_tiles;
  tp.token_limit = token_limit;
  tp.status = st;
  tp.timeout_ns = kTimeoutNs;
  tp.c = static_cast<uint16_t*>(c);
  tp.stride_cg = stride_cg;
  tp.stride_cm = stride_cm;
  tp.bw_lhs = maps.bw_lhs;
  tp.bw_rhs = maps.bw_rhs;
  tp.offs_bound = m_total < 0 ? 1 : 0;
  const int64_t clusters = items < d->sm_count / 2 ? items : d->sm_count / 2;
  const cudaError_t e = vark::tc2_launch(maps, tp, static_cast<int>(2 * clusters), s);
  if (e != cudaSuccess) return GGEMM_VARK_ECUDA;
  return GGEMM_VARK_OK;
}

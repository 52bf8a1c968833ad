// vark_simt.cu - CUDA-core variable-K grouped FP8 wgrad for arbitrary strides.
//
// Same contract as the tcgen05 kernel (C[g] = sL*sR * LHS_g^T . RHS_g, bf16 out, empty group
// -> zeros), used when the layout cannot be described to TMA (unaligned base or strides,
// stride_cn != 1). Each CTA computes a 64x64 block of one C[g]; tokens are staged 32 at a
// time in shared memory as fp32 and accumulated in fp32 in token order.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"

namespace vark {
namespace {

constexpr int BM = 64, BN = 64, BT = 32;

__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw(v, __NV_E4M3)));
}
__device__ __forceinline__ float e5m2_to_f32(uint8_t v) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw(v, __NV_E5M2)));
}

__global__ void __launch_bounds__(256) vark_simt_kernel(const SimtParams p) {
  __shared__ float sl[BT][BM];
  __shared__ float sr[BT][BN];
  const int g = blockIdx.z;
  const int m0 = blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;
  const int tx = threadIdx.x & 15;  // n direction
  const int ty = threadIdx.x >> 4;  // m direction

  int64_t lo = p.group_offs[g];
  int64_t hi = p.group_offs[g + 1];
  // Without m_total, group_offs[G] is the token count (rows are read only inside groups).
  const int64_t lim = p.offs_bound ? min(p.group_offs[p.G], p.token_limit) : p.token_limit;
  if (lo < 0 || hi < lo || hi > lim) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && p.status != nullptr)
      atomicOr(p.status, GGEMM_VARK_DEV_BAD_OFFS);
    lo = hi = 0;
  }

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int64_t t0 = lo; t0 < hi; t0 += BT) {
    for (int i = threadIdx.x; i < BT * BM; i += 256) {
      const int tt = i / BM, mm = i - tt * BM;
      const int64_t t = t0 + tt;
      const int m = m0 + mm;
      sl[tt][mm] = (t < hi && m < p.OUT_M) ? e4m3_to_f32(p.lhs[t * p.stride_lhs_m + m]) : 0.f;
    }
    for (int i = threadIdx.x; i < BT * BN; i += 256) {
      const int tt = i / BN, nn = i - tt * BN;
      const int64_t t = t0 + tt;
      const int n = n0 + nn;
      sr[tt][nn] = (t < hi && n < p.OUT_N) ? e5m2_to_f32(p.rhs[t * p.stride_rhs_m + n]) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int tt = 0; tt < BT; ++tt) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sl[tt][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sr[tt][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

  const float scale = p.lhs_scale[static_cast<int64_t>(g) * p.scale_stride] *
                      p.rhs_scale[static_cast<int64_t>(g) * p.scale_stride];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= p.OUT_M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= p.OUT_N) continue;
      const __nv_bfloat16 v = __float2bfloat16_rn(acc[i][j] * scale);
      p.c[g * p.stride_cg + m * p.stride_cm + n * p.stride_cn] =
          *reinterpret_cast<const uint16_t*>(&v);
    }
  }
}

}  // namespace

cudaError_t simt_launch(const SimtParams& p, cudaStream_t stream) {
  dim3 grid((p.OUT_N + BN - 1) / BN, (p.OUT_M + BM - 1) / BM, p.G);
  if (grid.y > 65535u || grid.z > 65535u) return cudaErrorInvalidConfiguration;
  vark_simt_kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace vark

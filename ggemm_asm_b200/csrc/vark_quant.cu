// vark_quant.cu - per-expert FP8 quantisation of a token-major bf16 operand: the producer step
// that feeds the grouped wgrad (x -> e4m3 LHS, dy -> e5m2 RHS), and its C-ABI entry point.
//
//   unit u      expert g's rows [off_g, off_{g+1}) (per_group = 1), or all rows (per_group = 0)
//   amax_u      max |x| over the unit's rows (a NaN anywhere in the unit makes it NaN)
//   s_u         amax_u / FMAX in fp32 (IEEE division); 1.0 when the unit is empty or amax_u == 0
//   q[t][f]     fp8( x[t][f] / s_u ), IEEE division, round to nearest even, saturated to +-FMAX
//   FMAX        448 (e4m3fn) or 57344 (e5m2)
//
// The reference harness makes its fp8 operands on the host (ggemm-asm bench.py:221-223: a direct
// bf16 -> fp8 cast, scales fixed at 0.1 by bench.py:266-267); the amax-scaled form above is the one
// the wgrad's test configurations use and the one an FP8 training step applies to x and dy.
//
// Design (HBM bound; 2 bytes read + 1 byte written per element):
//  - One co-resident grid (cooperative launch: SMs x CTAs per SM). Every unit is split into equal
//    contiguous slices of 16-byte vectors, slice c to CTA c.
//  - A CTA reduces the amax of its slice of unit u, publishes it (one atomicMax on the unit's
//    word, then an arrival count), waits until every CTA has published, and quantises the same
//    slice. All CTAs hold equal shares of a unit, so the wait is short.
//  - The second read of a row mostly comes from L2: at most about two units (up to ~94 MB at
//    4096 x 5760 bf16) lie between the two reads, and B200's L2 is 126 MB.
//  - Contiguous rows (the usual layout): the consumer warps work in two roles at once, 4 warps
//    reducing the amax of unit u from one ring of shared-memory chunks while 12 warps quantise
//    unit u-1 from a second ring; a producer warp per ring streams the CTA's slices into it with
//    1-D bulk copies (cp.async.bulk), and chunks are released through mbarriers. Other layouts
//    (padded rows, unaligned bases, F % 8 != 0) take a register-load kernel with the one-role
//    schedule and the same results.
//  - The quotient x / s is exact without a division per element (Markstein's correction below).
//  - Every wait is bounded (globaltimer): on expiry the CTA records GGEMM_VARK_DEV_TIMEOUT, raises
//    an abort word in the workspace that the other CTAs' waits watch, and returns.
#include <cuda_fp8.h>

#include <climits>

#include "../../include/ggemm_vark.h"
#include "vark_internal.h"
#include "vark_ptx.cuh"

namespace vark {
namespace {

constexpr int kThreads = 512;  // threads doing the arithmetic (register-load kernel: all of them)
constexpr int kUnroll = 4;
constexpr int kWarps = kThreads / 32;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;
// Bulk-copy kernel (contiguous rows), one CTA per SM: 16 consumer warps in two roles plus one
// producer warp per role. WS_AMAX_WARPS warps reduce the amax of unit s from the "amax ring"
// (WS_A_STAGES chunks of up to WS_A_CAP bytes: the first, DRAM read of every chunk) while the
// other warps quantise unit s-1 from the "quantise ring" (WS_Q_STAGES chunks of up to WS_Q_CAP
// bytes: the re-read, mostly from L2). Shapes measured in one process at the gate_up shapes
// (x [131072, 2880], dy [131072, 5760], and dy under skewed routing; ms; bit-identical output):
//   all 16 warps on each chunk in turn, one ring of 64 KB x 3 (96 KB x 2 for x)
//                                                            0.291 / 0.501 / 0.613
//   4 amax warps, amax ring 40 KB x 2, quantise ring 64 KB x 2 (kept)   0.226 / 0.446 / 0.567
//   4 amax warps, 48 KB x 2 each                                        0.231 / 0.487 / 0.577
//   4 amax warps, 32 KB x 2 and 64 KB x 2                               0.242 / 0.443 / 0.573
//   3 amax warps, 40 KB x 2 and 56 KB x 2                               0.233 / 0.455 / 0.578
//   2 amax warps, 48 KB x 2 each                                        0.248 / 0.460 / 0.581
//   quantise chunks of 24 or 32 KB (amax 48 KB x 3 or 32 KB x 4)       0.244-0.291 / 0.56-0.63
// With one set of warps on every chunk, the amax reads (DRAM latency, little arithmetic) and
// the quantisation (L2 reads, most of the arithmetic) took turns on the SM instead of
// overlapping; the quantise ring wants the larger chunks.
constexpr int kQtThreads = 512;                   // consumer threads (both roles)
constexpr int kQtWarps = kQtThreads / 32;
constexpr int WS_AMAX_WARPS = 4;
constexpr int WS_QUANT_WARPS = kQtWarps - WS_AMAX_WARPS;
constexpr int WS_AMAX_THREADS = 32 * WS_AMAX_WARPS;
constexpr int WS_QUANT_THREADS = 32 * WS_QUANT_WARPS;
constexpr int WS_THREADS = kQtThreads + 64;       // + one producer warp per ring
constexpr int WS_A_STAGES = 2, WS_Q_STAGES = 2;
constexpr uint32_t WS_A_CAP = 40u * 1024u, WS_Q_CAP = 64u * 1024u;
// The amax warps take unit s once the quantise warps have finished unit s - WS_LEAD: about two
// units lie between the two reads of a unit, and every wait points at a lower unit index. A lead
// of 3 measured dy -2 to -10% (more second reads missing L2), skewed dy +3 to +4%.
constexpr int WS_LEAD = 2;
constexpr size_t WS_SMEM = static_cast<size_t>(WS_A_STAGES) * WS_A_CAP +
                           static_cast<size_t>(WS_Q_STAGES) * WS_Q_CAP +
                           16 * (WS_A_STAGES + WS_Q_STAGES) + 128;
static_assert(WS_A_CAP % 16 == 0 && WS_Q_CAP % 16 == 0, "chunks: whole 16-byte vectors");
static_assert(WS_QUANT_WARPS > 0 && WS_SMEM <= 220 * 1024, "one CTA per SM, both rings");

struct QuantParams {
  const uint8_t* x;          // bf16 rows
  uint8_t* q;                // fp8 rows
  float* scales;             // [units]
  const int64_t* group_offs; // [G + 1]
  int32_t G;
  int32_t units;             // G (per group) or 1 (per tensor)
  int32_t per_group;
  int32_t F;                 // features per row
  int64_t stride_x;          // bytes
  int64_t stride_q;          // bytes
  int64_t token_limit;       // offsets above this are invalid
  float fmax;
  uint32_t* ws;              // [0]: abort word; [4, 4 + units): amax bits; then arrival counts
  uint32_t* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// First read of a row vector: normal L1 bypass, kept in L2 for the second read.
__device__ __forceinline__ uint4 ld_keep(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

// ---------------------------------------------------------------------------------------------
// Exact quotient without a division per element: Markstein's correction step (P. Markstein,
// IBM J. Res. Dev. 34(1), 1990), with y = RN(1/s) computed once per unit:
//     q = RN(x*y),  r = RN(s*(-q) + x) (exact, one fma),  q' = RN(r*y + q) (one fma)
// q' equals the IEEE quotient RN(x/s) for every bf16 significand x and every fp32 s in [1, 2)
// - all 2^30 pairs, checked exhaustively against IEEE division by the test suite - and every
// step scales exactly by powers of two while operands and results stay normal, so it holds for
// all normal x and s. The rest of the domain:
//  - x = +-0: q = +-0 is kept (the correction would lose the sign of zero).
//  - s within [2^-80, 2^100]: any x whose quotient can reach a nonzero fp8 code (|x/s| >= 2^-18)
//    has |x| >= 2^-98, so q, r and q' are normal. Smaller quotients round to +-0 on every route
//    (q' keeps the sign of x). Bf16 subnormal x gives |x/s| < 2^-46: +-0.
//  - s = NaN (the unit holds a NaN - the only way an input NaN can occur): every code is NaN,
//    as x/NaN is. s = +Inf (the unit holds an Inf - the only way an input Inf can occur):
//    q = +-0 for finite x, NaN for x = +-Inf, as x/Inf is.
// Units with a finite s outside [2^-80, 2^100] divide each element instead.
// ---------------------------------------------------------------------------------------------
template <bool E5M2>
__device__ __forceinline__ uint32_t cvt_pair(float a, float b) {
  return __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, E5M2 ? __NV_E5M2 : __NV_E4M3);
}

__device__ __forceinline__ bool fast_route_ok(float s) {
  return isnan(s) || isinf(s) || (s >= 0x1p-80f && s <= 0x1p100f);
}

__device__ __forceinline__ float quotient(float x, float s, float y) {
  const float q = __fmul_rn(x, y);
  const float r = __fmaf_rn(-s, q, x);
  const float q2 = __fmaf_rn(r, y, q);
  return q == 0.0f ? q : q2;
}

// Two bf16 in one 32-bit word -> two fp8 codes (low element in the low byte). FAST selects the
// division-free quotient (the caller checked fast_route_ok) or IEEE division.
template <bool E5M2, bool FAST>
__device__ __forceinline__ uint32_t quant_word(uint32_t w, float s, float y) {
  const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
  if constexpr (FAST) return cvt_pair<E5M2>(quotient(lo, s, y), quotient(hi, s, y)) & 0xffffu;
  return cvt_pair<E5M2>(__fdiv_rn(lo, s), __fdiv_rn(hi, s)) & 0xffffu;
}

// Eight bf16 (one 16-byte vector) -> eight fp8 codes.
template <bool E5M2, bool FAST>
__device__ __forceinline__ uint2 quant_vec(uint4 v, float s, float y) {
  const uint32_t c0 = quant_word<E5M2, FAST>(v.x, s, y), c1 = quant_word<E5M2, FAST>(v.y, s, y);
  const uint32_t c2 = quant_word<E5M2, FAST>(v.z, s, y), c3 = quant_word<E5M2, FAST>(v.w, s, y);
  return make_uint2(c0 | (c1 << 16), c2 | (c3 << 16));
}

// Scale of a unit from its amax bit pattern (|bf16| bits).
__device__ __forceinline__ float unit_scale(uint32_t amax_bits, float fmax) {
  const float a = __uint_as_float(amax_bits << 16);
  return (a == 0.0f) ? 1.0f : __fdiv_rn(a, fmax);
}

// Unit u's rows and whether its offsets are valid.
__device__ __forceinline__ bool unit_rows(const QuantParams& p, int u, int64_t* lo, int64_t* hi) {
  if (p.per_group) {
    *lo = __ldg(p.group_offs + u);
    *hi = __ldg(p.group_offs + u + 1);
  } else {
    *lo = __ldg(p.group_offs);
    *hi = __ldg(p.group_offs + p.G);
  }
  return *lo >= 0 && *hi >= *lo && *hi <= p.token_limit;
}

// This CTA's slice [v0, v1) of a unit with `total` vectors.
__device__ __forceinline__ void slice_of(int64_t total, int64_t* v0, int64_t* v1) {
  const int64_t n = gridDim.x, c = blockIdx.x;
  const int64_t base = total / n, rem = total % n;
  *v0 = base * c + (c < rem ? c : rem);
  *v1 = *v0 + base + (c < rem ? 1 : 0);
}

// Publish this CTA's amax of unit u: one atomicMax, then the arrival count (thread 0).
__device__ __forceinline__ void publish(const QuantParams& p, int u, uint32_t mm, bool withhold) {
  if (withhold) return;
  if (mm != 0) atomicMax(p.ws + 4 + u, mm);
  __threadfence();
  atomicAdd(p.ws + 4 + p.units + u, 1u);
}

__device__ __forceinline__ void report_timeout(const QuantParams& p, uint32_t where) {
  if (p.status != nullptr) {
    atomicOr(p.status, GGEMM_VARK_DEV_TIMEOUT);
    atomicExch(p.status + 1, where);
  }
  atomicExch(p.ws, 1u);
}

// Thread 0: wait until every CTA has published unit u's amax. False on expiry or abort.
__device__ bool wait_unit(const QuantParams& p, int u) {
  const uint32_t* arrived = p.ws + 4 + p.units + u;
  const uint32_t need = gridDim.x;
  if (ld_acquire_u32(arrived) >= need) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t ns = 32;
  while (true) {
    if (ld_acquire_u32(arrived) >= need) return true;
    if (ld_relaxed_u32(p.ws) != 0) return false;  // another CTA gave up
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      report_timeout(p, 0x51000000u | static_cast<uint32_t>(u & 0xffffff));
      return false;
    }
    __nanosleep(ns);
    if (ns < 128) ns *= 2;
  }
}

__device__ __forceinline__ bool test_withhold(const QuantParams& p) {
  return blockIdx.x == 0 && p.status != nullptr &&
         *reinterpret_cast<volatile const uint32_t*>(p.status + 3) == GGEMM_VARK_TEST_STALL_MAGIC;
}

// ---------------------------------------------------------------------------------------------
// Register-load kernel (any layout): threads stride over the slice in 16-byte vectors (VEC) or
// single elements.
// ---------------------------------------------------------------------------------------------

// Walks a thread's strided vector indices as (row, column-vector) pairs without a division per
// step: the stride kThreads is split once into whole rows and a column remainder.
struct RowWalk {
  int64_t row;
  int32_t col;
  int32_t vpr, drow, dcol;
  __device__ __forceinline__ void init(int64_t index, int32_t vectors_per_row) {
    vpr = vectors_per_row;
    row = index / vpr;
    col = static_cast<int32_t>(index - row * vpr);
    drow = kThreads / vpr;
    dcol = kThreads - drow * vpr;
  }
  __device__ __forceinline__ void step() {
    row += drow;
    col += dcol;
    if (col >= vpr) {
      col -= vpr;
      ++row;
    }
  }
};

// Largest |bf16| bit pattern (sign cleared): unsigned order puts NaN above Inf above finite.
template <bool VEC>
__device__ uint32_t slice_amax(const QuantParams& p, int64_t lo, int64_t v0, int64_t v1,
                               uint64_t pol) {
  uint32_t m2 = 0;  // two 16-bit maxima side by side (vector path)
  uint32_t m = 0;
  constexpr int kElems = VEC ? 8 : 1;
  const int32_t vpr = p.F / kElems;
  int64_t i = v0 + threadIdx.x;
  if (i < v1) {
    RowWalk w;
    w.init(i, vpr);
    for (; i < v1; i += static_cast<int64_t>(kThreads) * kUnroll) {
      if constexpr (VEC) {
        uint4 v[kUnroll];
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          if (i + static_cast<int64_t>(k) * kThreads < v1) {
            v[k] = ld_keep(p.x + (lo + w.row) * p.stride_x + static_cast<int64_t>(w.col) * 16, pol);
          } else {
            v[k] = make_uint4(0, 0, 0, 0);
          }
          w.step();
        }
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          m2 = __vmaxu2(m2, v[k].x & 0x7fff7fffu);
          m2 = __vmaxu2(m2, v[k].y & 0x7fff7fffu);
          m2 = __vmaxu2(m2, v[k].z & 0x7fff7fffu);
          m2 = __vmaxu2(m2, v[k].w & 0x7fff7fffu);
        }
      } else {
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          if (i + static_cast<int64_t>(k) * kThreads < v1) {
            const uint16_t h = __ldg(reinterpret_cast<const uint16_t*>(
                p.x + (lo + w.row) * p.stride_x + static_cast<int64_t>(w.col) * 2));
            m = max(m, static_cast<uint32_t>(h & 0x7fffu));
          }
          w.step();
        }
      }
    }
  }
  m = max(m, max(m2 & 0xffffu, m2 >> 16));
  return m;
}

template <bool VEC, bool E5M2, bool FAST>
__device__ void slice_quantize(const QuantParams& p, int64_t lo, int64_t v0, int64_t v1,
                               float s) {
  const float y = __frcp_rn(s);
  constexpr int kElems = VEC ? 8 : 1;
  const int32_t vpr = p.F / kElems;
  int64_t i = v0 + threadIdx.x;
  if (i >= v1) return;
  RowWalk w;
  w.init(i, vpr);
  for (; i < v1; i += static_cast<int64_t>(kThreads) * kUnroll) {
    if constexpr (VEC) {
      uint4 v[kUnroll];
      int64_t row[kUnroll];
      int32_t col[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        row[k] = w.row;
        col[k] = w.col;
        if (i + static_cast<int64_t>(k) * kThreads < v1)
          v[k] = __ldcs(reinterpret_cast<const uint4*>(p.x + (lo + w.row) * p.stride_x +
                                                       static_cast<int64_t>(w.col) * 16));
        w.step();
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        if (i + static_cast<int64_t>(k) * kThreads >= v1) break;
        __stcs(reinterpret_cast<uint2*>(p.q + (lo + row[k]) * p.stride_q +
                                        static_cast<int64_t>(col[k]) * 8),
               quant_vec<E5M2, FAST>(v[k], s, y));
      }
    } else {
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        if (i + static_cast<int64_t>(k) * kThreads < v1) {
          const uint32_t h = __ldcs(reinterpret_cast<const unsigned short*>(
              p.x + (lo + w.row) * p.stride_x + static_cast<int64_t>(w.col) * 2));
          const uint32_t c = quant_word<E5M2, FAST>(h | (h << 16), s, y);
          p.q[(lo + w.row) * p.stride_q + w.col] = static_cast<uint8_t>(c & 0xffu);
        }
        w.step();
      }
    }
  }
}

template <bool VEC, bool E5M2>
__global__ void __launch_bounds__(kThreads) vark_quant_kernel(const QuantParams p) {
  __shared__ uint32_t red[kWarps];
  __shared__ float s_scale;
  __shared__ int s_ok;
  const uint64_t pol = l2_policy_evict_last();
  constexpr int kElems = VEC ? 8 : 1;
  const int64_t vpr = p.F / kElems;
  const bool withhold = test_withhold(p);  // failure-detection test hook
  bool first_arrival = true;

  for (int u = 0; u < p.units; ++u) {
    int64_t lo, hi;
    const bool valid = unit_rows(p, u, &lo, &hi);
    if (!valid || hi == lo) {
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (!valid && p.status != nullptr) atomicOr(p.status, GGEMM_VARK_DEV_BAD_OFFS);
        p.scales[u] = 1.0f;
      }
      continue;
    }
    int64_t v0, v1;
    slice_of((hi - lo) * vpr, &v0, &v1);
    // Amax of this CTA's slice of unit u.
    uint32_t m = slice_amax<VEC>(p, lo, v0, v1, pol);
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t mm = 0;
#pragma unroll
      for (int k = 0; k < kWarps; ++k) mm = max(mm, red[k]);
      publish(p, u, mm, withhold && first_arrival);
      first_arrival = false;
      // Quantise the same slice once every CTA has published its amax.
      const bool ok = wait_unit(p, u);
      float s = 1.0f;
      if (ok) {
        s = unit_scale(ld_relaxed_u32(p.ws + 4 + u), p.fmax);
        if (blockIdx.x == 0) p.scales[u] = s;
      }
      s_scale = s;
      s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok) return;
    if (fast_route_ok(s_scale))
      slice_quantize<VEC, E5M2, true>(p, lo, v0, v1, s_scale);
    else
      slice_quantize<VEC, E5M2, false>(p, lo, v0, v1, s_scale);
    __syncthreads();  // red, s_scale and s_ok are rewritten for the next unit
  }
}

// ---------------------------------------------------------------------------------------------
// Bulk-copy kernel (contiguous rows). Every CTA reads its slice of each unit twice: the amax
// warps reduce the slice of unit s (first read, evict-last so that the lines stay in L2), and
// once every CTA has published unit s the quantise warps quantise the same slice (second read,
// evict-first, mostly from L2), while the amax warps already read unit s+1. So HBM serves the
// first reads of one unit while the second reads and the fp8 stores of the previous one go on.
// (Alternatives measured at 4096 x 5760: all of unit u+1 before unit u's quantise pass thrashed
// L2; amax then quantise of the same unit kept L2 but left HBM alternating between reading and
// writing.) Each role has its own ring and producer warp, which issues its chunk copies in the
// role's order, a ring ahead.
// ---------------------------------------------------------------------------------------------

// This CTA's slice of unit w: byte range [b0, b1), whether the unit is valid and non-empty, and
// its cut into n chunks of cb bytes (the last one shorter). The chunks are as equal as 16-byte
// granularity allows: a short last chunk would hold a whole ring stage for few bytes in flight.
struct Slice {
  int64_t b0, b1;
  bool unit_ok;
  int64_t n;
  uint32_t cb;
  __device__ __forceinline__ int64_t chunks() const { return n; }
  __device__ __forceinline__ int64_t chunk_offset(int64_t t) const { return t * cb; }
  __device__ __forceinline__ uint32_t chunk_bytes(int64_t t) const {
    const int64_t rest = b1 - b0 - t * cb;
    return static_cast<uint32_t>(rest < cb ? rest : cb);
  }
};

// Equal chunks of at most CAP bytes over len bytes (len and CAP multiples of 16; CAP is a
// constant, so the divisions are by constants).
template <uint32_t CAP>
__device__ __forceinline__ void cut_slice(Slice& sl) {
  constexpr int64_t cap = CAP;
  const int64_t len = sl.b1 - sl.b0;
  if (len <= 0) {
    sl.n = 0;
    sl.cb = CAP;
    return;
  }
  const int64_t n0 = (len + cap - 1) / cap;
  const int64_t cb = ((len + n0 - 1) / n0 + 15) / 16 * 16;  // <= cap (a multiple of 16)
  sl.cb = static_cast<uint32_t>(cb);
  sl.n = (len + cb - 1) / cb;  // every chunk non-empty
}

// The slice of unit w cut for a ring of CAP-byte chunks (both roles cover the same bytes).
template <uint32_t CAP>
__device__ __forceinline__ Slice slice_info(const QuantParams& p, int w) {
  Slice sl{0, 0, false, 0, CAP};
  if (w < 0 || w >= p.units) return sl;
  int64_t lo, hi;
  if (!unit_rows(p, w, &lo, &hi) || hi == lo) return sl;
  const int64_t vpr = p.F / 8;
  int64_t v0, v1;
  slice_of((hi - lo) * vpr, &v0, &v1);
  sl.b0 = lo * p.stride_x + v0 * 16;
  sl.b1 = lo * p.stride_x + v1 * 16;
  sl.unit_ok = true;
  cut_slice<CAP>(sl);
  return sl;
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, uint64_t limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit) return false;
  }
  return true;
}

// Named barrier over one role's warps (ID 1: amax warps, 2: quantise warps; the producer warps
// never take part), returning the OR of a flag.
template <int ID, int N>
__device__ __forceinline__ bool group_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(ID), "n"(N)
      : "memory");
  return r != 0;
}
template <int ID, int N>
__device__ __forceinline__ void group_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(N) : "memory");
}

// One ring's producer (lane 0 of its warp): every chunk of every unit in order, each into its
// stage once the role's warps have released it; before returning, let the last copy into every
// stage land (the CTA's shared memory must outlive it).
template <uint32_t CAP, int NST>
__device__ void produce(const QuantParams& p, uint32_t stage0, uint64_t* full, uint64_t* empty,
                        uint64_t pol, uint32_t where) {
  int64_t n = 0;
  bool ok = true;
  for (int s = 0; s < p.units && ok; ++s) {
    const Slice sl = slice_info<CAP>(p, s);
    for (int64_t t = 0; t < sl.chunks(); ++t) {
      const int k = static_cast<int>(n % NST);
      if (n >= NST &&
          !wait_bar(smem_u32(empty + k), static_cast<uint32_t>((n / NST - 1) & 1), p.timeout_ns)) {
        report_timeout(p, where);
        ok = false;
        break;
      }
      const uint32_t bytes = sl.chunk_bytes(t);
      const uint32_t bar = smem_u32(full + k);
      mbar_arrive_expect_tx(bar, bytes);
      bulk_load_1d(stage0 + k * CAP, p.x + sl.b0 + sl.chunk_offset(t), bytes, bar, pol);
      ++n;
    }
  }
  for (int64_t c = n > NST ? n - NST : 0; c < n; ++c)
    wait_bar(smem_u32(full + static_cast<int>(c % NST)), static_cast<uint32_t>((c / NST) & 1),
             p.timeout_ns);
}

// Thread 0 of the amax warps: wait until this CTA's quantise warps have finished unit u.
__device__ __forceinline__ bool wait_quantised(const QuantParams& p, const volatile int* q_done,
                                               int u) {
  if (*q_done >= u) return true;
  const uint64_t t0 = globaltimer_ns();
  while (*q_done < u) {
    if (ld_relaxed_u32(p.ws) != 0) return false;  // another CTA gave up
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      report_timeout(p, 0x55000000u | static_cast<uint32_t>(u & 0xffffff));
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// The amax warps (threads [0, WS_AMAX_THREADS)): unit by unit, the amax of this CTA's slice,
// published by thread 0 (which also records invalid or empty units).
__device__ void amax_role(const QuantParams& p, const uint8_t* stages, uint64_t* full,
                          uint64_t* empty, uint32_t* red, const volatile int* q_done) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool withhold = test_withhold(p);
  bool first_arrival = true, fail = false;
  int64_t j = 0;  // chunks consumed
  for (int s = 0; s < p.units; ++s) {
    const Slice a = slice_info<WS_A_CAP>(p, s);
    if (!a.unit_ok && blockIdx.x == 0 && tid == 0) {
      int64_t lo, hi;
      if (!unit_rows(p, s, &lo, &hi) && p.status != nullptr)
        atomicOr(p.status, GGEMM_VARK_DEV_BAD_OFFS);
      p.scales[s] = 1.0f;  // invalid or empty unit
    }
    if (s >= WS_LEAD) {
      bool ok = true;
      if (tid == 0) ok = wait_quantised(p, q_done, s - WS_LEAD);
      fail = group_sync_or<1, WS_AMAX_THREADS>(fail || !ok);
      if (fail) break;
    }
    uint32_t m2 = 0;  // two 16-bit maxima of |bf16| bit patterns side by side
    for (int64_t t = 0; t < a.chunks(); ++t) {
      const int k = static_cast<int>(j % WS_A_STAGES);
      if (!__all_sync(0xffffffffu,
                      wait_bar(smem_u32(full + k), static_cast<uint32_t>((j / WS_A_STAGES) & 1),
                               p.timeout_ns))) {
        fail = true;
        break;
      }
      const uint4* st = reinterpret_cast<const uint4*>(stages + k * WS_A_CAP);
      const uint32_t nv = a.chunk_bytes(t) / 16;
#pragma unroll 4
      for (uint32_t v = tid; v < nv; v += WS_AMAX_THREADS) {
        const uint4 x = st[v];
        m2 = __vmaxu2(m2, x.x & 0x7fff7fffu);
        m2 = __vmaxu2(m2, x.y & 0x7fff7fffu);
        m2 = __vmaxu2(m2, x.z & 0x7fff7fffu);
        m2 = __vmaxu2(m2, x.w & 0x7fff7fffu);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(empty + k));
      ++j;
    }
    if (!a.unit_ok) {
      fail = group_sync_or<1, WS_AMAX_THREADS>(fail);
      if (fail) break;
      continue;
    }
    const uint32_t m = __reduce_max_sync(0xffffffffu, max(m2 & 0xffffu, m2 >> 16));
    if (lane == 0) red[warp] = m;
    fail = group_sync_or<1, WS_AMAX_THREADS>(fail);
    if (fail) break;
    if (tid == 0) {  // the atomics and their fence hold up thread 0 only
      uint32_t mm = 0;
#pragma unroll
      for (int w = 0; w < WS_AMAX_WARPS; ++w) mm = max(mm, red[w]);
      publish(p, s, mm, withhold && first_arrival);
      first_arrival = false;
    }
    group_sync<1, WS_AMAX_THREADS>();  // red[] is rewritten for the next unit
  }
  if (fail && tid == 0) report_timeout(p, 0x52000000u);
}

// The quantise warps (threads [WS_AMAX_THREADS, kQtThreads)): unit by unit, once every CTA has
// published the unit's amax, this CTA's slice in fp8; q_done then records the unit.
template <bool E5M2>
__device__ void quant_role(const QuantParams& p, const uint8_t* stages, uint64_t* full,
                           uint64_t* empty, volatile int* q_done) {
  const int tq = threadIdx.x - WS_AMAX_THREADS, lane = threadIdx.x & 31;
  bool fail = false;
  int64_t j = 0;  // chunks consumed
  for (int s = 0; s < p.units; ++s) {
    const Slice b = slice_info<WS_Q_CAP>(p, s);
    float scale = 1.0f, recip = 1.0f;
    bool fast = true;
    if (b.unit_ok && (b.chunks() > 0 || blockIdx.x == 0)) {
      bool ok = true;
      if (tq == 0) {
        ok = wait_unit(p, s);
        if (ok && blockIdx.x == 0) p.scales[s] = unit_scale(ld_relaxed_u32(p.ws + 4 + s), p.fmax);
      }
      fail = group_sync_or<2, WS_QUANT_THREADS>(fail || !ok);
      if (fail) break;
      scale = unit_scale(ld_relaxed_u32(p.ws + 4 + s), p.fmax);
      recip = __frcp_rn(scale);
      fast = fast_route_ok(scale);
    }
    for (int64_t t = 0; t < b.chunks(); ++t) {
      const int k = static_cast<int>(j % WS_Q_STAGES);
      if (!__all_sync(0xffffffffu,
                      wait_bar(smem_u32(full + k), static_cast<uint32_t>((j / WS_Q_STAGES) & 1),
                               p.timeout_ns))) {
        fail = true;
        break;
      }
      const uint4* st = reinterpret_cast<const uint4*>(stages + k * WS_Q_CAP);
      const uint32_t nv = b.chunk_bytes(t) / 16;
      // contiguous rows: element index = byte offset / 2
      uint2* dst = reinterpret_cast<uint2*>(p.q + (b.b0 + b.chunk_offset(t)) / 2);
      if (fast) {
#pragma unroll 4
        for (uint32_t v = tq; v < nv; v += WS_QUANT_THREADS)
          __stcs(dst + v, quant_vec<E5M2, true>(st[v], scale, recip));
      } else {
        for (uint32_t v = tq; v < nv; v += WS_QUANT_THREADS)
          __stcs(dst + v, quant_vec<E5M2, false>(st[v], scale, recip));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(empty + k));
      ++j;
    }
    fail = group_sync_or<2, WS_QUANT_THREADS>(fail);
    if (fail) break;
    if (tq == 0) *q_done = s;  // every quantise warp is past unit s
  }
  if (fail && tq == 0) report_timeout(p, 0x53000000u);
}

// One CTA per SM (both rings take ~208 KiB): stating it lets ptxas keep the unrolled consumer
// loops in registers.
template <bool E5M2>
__global__ void __launch_bounds__(WS_THREADS, 1) vark_quant_tma_kernel(const QuantParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  uint8_t* stages_a = smem;
  uint8_t* stages_q = smem + WS_A_STAGES * WS_A_CAP;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(stages_q + WS_Q_STAGES * WS_Q_CAP);
  uint64_t* empty_a = full_a + WS_A_STAGES;
  uint64_t* full_q = empty_a + WS_A_STAGES;
  uint64_t* empty_q = full_q + WS_Q_STAGES;
  __shared__ uint32_t red[WS_AMAX_WARPS];
  __shared__ int q_done;  // the last unit this CTA's quantise warps have finished
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int k = 0; k < WS_A_STAGES; ++k) {
      mbar_init(smem_u32(full_a + k), 1);
      mbar_init(smem_u32(empty_a + k), WS_AMAX_WARPS);
    }
    for (int k = 0; k < WS_Q_STAGES; ++k) {
      mbar_init(smem_u32(full_q + k), 1);
      mbar_init(smem_u32(empty_q + k), WS_QUANT_WARPS);
    }
    q_done = -1;
    fence_mbar_init();
  }
  __syncthreads();  // the only barrier over the whole CTA
  if (warp == kQtWarps) {
    if (lane == 0)
      produce<WS_A_CAP, WS_A_STAGES>(p, smem_u32(stages_a), full_a, empty_a,
                                     l2_policy_evict_last(), 0x54000000u);
    return;
  }
  if (warp == kQtWarps + 1) {
    if (lane == 0)
      produce<WS_Q_CAP, WS_Q_STAGES>(p, smem_u32(stages_q), full_q, empty_q,
                                     l2_policy_evict_first(), 0x56000000u);
    return;
  }
  if (warp < WS_AMAX_WARPS)
    amax_role(p, stages_a, full_a, empty_a, red, &q_done);
  else
    quant_role<E5M2>(p, stages_q, full_q, empty_q, &q_done);
}

}  // namespace

size_t quant_workspace_bytes(int32_t units) {
  return 16 + 8 * static_cast<size_t>(units > 0 ? units : 0);
}

// Launch the co-resident quantisation grid. mode 2: bulk-copy kernel (contiguous rows, 16-byte
// aligned x, F % 8 == 0); 1: register-load kernel, 16-byte vectors; 0: register-load kernel, one
// element at a time. The caller has checked the layout for the mode.
cudaError_t quant_launch(const uint8_t* x, uint8_t* q, float* scales, const int64_t* group_offs,
                         int32_t G, int32_t F, int64_t stride_x_bytes, int64_t stride_q_bytes,
                         int32_t fmt, int32_t per_group, int64_t token_limit, void* workspace,
                         uint32_t* status, uint64_t timeout_ns, int mode, int sm_count,
                         cudaStream_t stream) {
  QuantParams p;
  p.x = x;
  p.q = q;
  p.scales = scales;
  p.group_offs = group_offs;
  p.G = G;
  p.per_group = per_group;
  p.units = per_group ? G : 1;
  p.F = F;
  p.stride_x = stride_x_bytes;
  p.stride_q = stride_q_bytes;
  p.token_limit = token_limit;
  p.fmax = fmt == 0 ? 448.0f : 57344.0f;
  p.ws = static_cast<uint32_t*>(workspace);
  p.status = status;
  p.timeout_ns = timeout_ns != 0 ? timeout_ns : kDefaultTimeoutNs;
  cudaError_t e = cudaMemsetAsync(workspace, 0, quant_workspace_bytes(p.units), stream);
  if (e != cudaSuccess) return e;
  const bool e5m2 = fmt == 1;
  const void* fn;
  size_t smem = 0;
  int threads = kThreads;
  if (mode == 2) {
    fn = e5m2 ? reinterpret_cast<const void*>(&vark_quant_tma_kernel<true>)
              : reinterpret_cast<const void*>(&vark_quant_tma_kernel<false>);
    smem = WS_SMEM;
    threads = WS_THREADS;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  } else if (mode == 1) {
    fn = e5m2 ? reinterpret_cast<const void*>(&vark_quant_kernel<true, true>)
              : reinterpret_cast<const void*>(&vark_quant_kernel<true, false>);
  } else {
    fn = e5m2 ? reinterpret_cast<const void*>(&vark_quant_kernel<false, true>)
              : reinterpret_cast<const void*>(&vark_quant_kernel<false, false>);
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  if (per_sm > 4) per_sm = 4;
  void* args[] = {&p};
  return cudaLaunchCooperativeKernel(fn, dim3(per_sm * sm_count), dim3(threads), args, smem,
                                     stream);
}

}  // namespace vark

namespace {

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

extern "C" size_t ggemm_vark_quantize_workspace_bytes(int32_t G) {
  return vark::quant_workspace_bytes(G);
}

extern "C" int ggemm_vark_quantize_fp8(const void* x, void* q, float* scales,
                                       const int64_t* group_offs, int32_t G, int32_t F,
                                       int32_t stride_x, int32_t stride_q, int32_t fmt,
                                       int32_t per_group, int64_t m_total, void* workspace,
                                       void* status, uint64_t timeout_ns, void* stream) {
  if (scales == nullptr || group_offs == nullptr || workspace == nullptr)
    return GGEMM_VARK_EINVAL_PTR;
  if (G < 0 || F <= 0) return GGEMM_VARK_EINVAL_SHAPE;
  if (stride_x < F || stride_q < F) return GGEMM_VARK_EINVAL_STRIDE;
  if ((fmt != 0 && fmt != 1) || (per_group != 0 && per_group != 1) || m_total < -1)
    return GGEMM_VARK_EINVAL_ARG;
  if (!aligned(workspace, 16) || (status != nullptr && !aligned(status, 16)))
    return GGEMM_VARK_EINVAL_ARG;
  if (G == 0) return GGEMM_VARK_OK;
  if (m_total != 0 && (x == nullptr || q == nullptr)) return GGEMM_VARK_EINVAL_PTR;
  if (x == nullptr || q == nullptr) {
    // m_total == 0: no rows; every unit is empty and only the scales are written.
    x = q = workspace;
  }
  if (!aligned(x, 2)) return GGEMM_VARK_EINVAL_ARG;
  uint32_t* dev_status = nullptr;
  int sm_count = 0;
  const int rc = vark::device_status_block(&dev_status, &sm_count);
  if (rc != GGEMM_VARK_OK) return rc;
  uint32_t* st = status != nullptr ? static_cast<uint32_t*>(status) : dev_status;
  const int64_t sx = 2ll * stride_x, sq = stride_q;
  const bool vec = F % 8 == 0 && aligned(x, 16) && sx % 16 == 0 && aligned(q, 8) && sq % 8 == 0;
  const bool contiguous = stride_x == F && stride_q == F;
  const int mode = vec ? (contiguous ? 2 : 1) : 0;
  const int64_t token_limit = m_total >= 0 ? m_total : INT64_MAX;
  const cudaError_t e = vark::quant_launch(
      static_cast<const uint8_t*>(x), static_cast<uint8_t*>(q), scales, group_offs, G, F, sx, sq,
      fmt, per_group, token_limit, workspace, st, timeout_ns, mode, sm_count,
      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return vark::record_cuda_error(e);
  return GGEMM_VARK_OK;
}

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
//  - The second read of a row mostly comes from L2: the distance between the two reads is about
//    one unit (up to ~47 MB at 4096 x 5760 bf16) and B200's L2 is 126 MB. Measured DRAM reads:
//    exactly the input size when a unit's quantise pass directly follows its amax pass, 1.23x
//    the input with the interleaved order below (which keeps HBM reading while stores drain).
//  - Contiguous rows (the usual layout): one producer warp streams the CTA's slices through a
//    ring of shared-memory chunks with 1-D bulk copies (cp.async.bulk), running ahead across the
//    amax/quantise boundary; the 16 consumer warps release chunks through mbarriers and meet at
//    a CTA barrier only a few times per unit. Other layouts (padded rows, unaligned bases,
//    F % 8 != 0) take a register-load kernel with the same schedule and results.
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
// Bulk-copy kernel: kQtThreads consumer threads plus one producer warp, and a ring of QT_STAGES
// chunks of at most QT_CHUNK bytes, one CTA per SM. 64 KB x 3 measured fastest at the gate_up
// shapes: against 32 KB x 3 with two CTAs per SM it takes 11% less time on x [131072, 2880], 13%
// less on dy [131072, 5760] and 8% less on dy under skewed routing (half as many CTAs meet in
// each unit's grid-wide wait, and fewer hand-offs per byte); 48 KB x 4, 56 or 72 KB x 3 and
// 1024 consumer threads were slower, and 96 KB x 2 was faster on x alone but 9% slower on dy.
#ifndef VARK_QT_CONSUMERS
#define VARK_QT_CONSUMERS 512
#endif
constexpr int kQtThreads = VARK_QT_CONSUMERS;  // consumer threads of the bulk-copy kernel
constexpr int kQtWarps = kQtThreads / 32;
static_assert(kQtThreads % 32 == 0 && kQtThreads + 32 <= 1024, "bulk-copy kernel block size");
constexpr int kTmaThreads = kQtThreads + 32;
#ifndef VARK_QT_CHUNK
#define VARK_QT_CHUNK 65536
#endif
#ifndef VARK_QT_STAGES
#define VARK_QT_STAGES 3
#endif
constexpr uint32_t QT_CHUNK = VARK_QT_CHUNK;
static_assert(QT_CHUNK % 16 == 0, "chunk: whole 16-byte vectors");
constexpr int QT_STAGES = VARK_QT_STAGES;
constexpr size_t QT_SMEM = static_cast<size_t>(QT_STAGES) * QT_CHUNK + 2 * QT_STAGES * 8 + 128;
// The same shared memory as a ring of 2 chunks of up to 1.5 x QT_CHUNK. The host takes it when a
// CTA's average slice of a unit fits in two such chunks. At the gate_up shapes x (slices of
// ~159 KB) takes it: 0.299 ms against 0.328 ms with 64 KB x 3, measured in one process; dy
// (~318 KB), for which 96 KB x 2 measured 0.552 ms against 0.499, keeps 64 KB x 3.
// The kernel is instantiated per ring (NS stages of ring_cap<NS>() bytes): the stage index and
// phase of every chunk then come from divisions by a constant.
constexpr int QT_STAGES_WIDE = 2;
template <int NS>
constexpr uint32_t ring_cap() { return static_cast<uint32_t>(QT_STAGES * QT_CHUNK / NS); }
static_assert(ring_cap<QT_STAGES_WIDE>() % 16 == 0 && QT_STAGES_WIDE <= QT_STAGES, "wide ring");

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
// Bulk-copy kernel (contiguous rows). A CTA works through stages: stage 0 reads its slice of
// unit 0 (amax); stage s = 1..U interleaves, chunk by chunk (amax reads QT_LEAD chunks ahead),
// the amax read of its slice of unit s with the quantise read of its slice of unit s-1 (whose scale is known once every CTA has
// published unit s-1). So HBM serves the first reads of one unit while the fp8 stores of the
// previous one stream out, and L2 holds about one unit: the quantise reads of unit s-1 (evict
// first) free the lines the amax reads of unit s fill. (Alternatives measured at 4096 x 5760:
// all of unit u+1 before unit u's quantise pass thrashed L2; amax then quantise of the same unit
// kept L2 but left HBM alternating between reading and writing.) One producer warp issues the
// chunk copies in the same order, QT_STAGES ahead.
// ---------------------------------------------------------------------------------------------

// Order of the chunks within a stage: the amax reads of unit s run QT_LEAD chunks ahead of the
// quantise reads of unit s-1, so the wait for unit s-1's scale overlaps real work (it costs
// QT_LEAD chunks per CTA of extra L2 footprint, ~19 MB over 148 CTAs at 64 KB x 2). The quantise
// pass takes a unit's chunks oldest first; newest first measured 4-11% slower.
#ifndef VARK_QT_LEAD
#define VARK_QT_LEAD 2
#endif
constexpr int64_t QT_LEAD = VARK_QT_LEAD;
__device__ __forceinline__ bool amax_next(int64_t ta, int64_t tb, int64_t na, int64_t nb) {
  return ta < na && (tb == nb || ta < tb + QT_LEAD);
}

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

template <int NS>
__device__ __forceinline__ Slice slice_info(const QuantParams& p, int w) {
  Slice sl{0, 0, false, 0, ring_cap<NS>()};
  if (w < 0 || w >= p.units) return sl;
  int64_t lo, hi;
  if (!unit_rows(p, w, &lo, &hi) || hi == lo) return sl;
  const int64_t vpr = p.F / 8;
  int64_t v0, v1;
  slice_of((hi - lo) * vpr, &v0, &v1);
  sl.b0 = lo * p.stride_x + v0 * 16;
  sl.b1 = lo * p.stride_x + v1 * 16;
  sl.unit_ok = true;
  cut_slice<ring_cap<NS>()>(sl);
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

// Barrier 1 joins the kQtThreads consumer threads only (the producer warp never takes part).
__device__ __forceinline__ bool consumers_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kQtThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kQtThreads) : "memory");
}

// Producer warp, lane 0: issue every chunk in the consumers' order once its stage is free;
// before returning, let the last copy of every stage land (the CTA's shared memory must outlive
// it).
template <int NS>
struct Producer {
  const QuantParams& p;
  uint32_t stage0;
  uint64_t* full;
  uint64_t* empty;
  uint64_t pol_keep, pol_last;
  int64_t n = 0;  // chunks issued
  bool ok = true;
  __device__ __forceinline__ void issue(const Slice& sl, int64_t t, bool first_read) {
    if (!ok) return;
    constexpr int64_t ns = NS;
    const int k = static_cast<int>(n % ns);
    if (n >= ns &&
        !wait_bar(smem_u32(empty + k), static_cast<uint32_t>((n / ns - 1) & 1),
                  p.timeout_ns)) {
      report_timeout(p, 0x53000000u);
      ok = false;
      return;
    }
    const uint32_t bytes = sl.chunk_bytes(t);
    const uint32_t bar = smem_u32(full + k);
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load_1d(stage0 + k * ring_cap<NS>(), p.x + sl.b0 + sl.chunk_offset(t), bytes, bar,
                 first_read ? pol_keep : pol_last);
    ++n;
  }
  __device__ void run() {
    Slice a = slice_info<NS>(p, 0);
    for (int64_t t = 0; t < a.chunks(); ++t) issue(a, t, true);
    for (int s = 1; s <= p.units && ok; ++s) {
      const Slice b = slice_info<NS>(p, s - 1);
      a = slice_info<NS>(p, s);
      const int64_t na = a.chunks(), nb = b.chunks();
      for (int64_t ta = 0, tb = 0; ta < na || tb < nb;) {
        if (amax_next(ta, tb, na, nb))
          issue(a, ta++, true);
        else
          issue(b, tb++, false);
      }
    }
    constexpr int64_t ns = NS;
    for (int64_t c = n > ns ? n - ns : 0; c < n; ++c)
      wait_bar(smem_u32(full + static_cast<int>(c % ns)), static_cast<uint32_t>((c / ns) & 1),
               p.timeout_ns);
  }
};

// Consumer warps (kQtThreads threads): the same chunk order as the producer.
template <bool E5M2, int NS>
struct Consumer {
  const QuantParams& p;
  uint8_t* stages;
  uint64_t* full;
  uint64_t* empty;
  uint32_t* red;       // kQtWarps words
  int lane, warp;
  int64_t j = 0;       // chunks consumed
  bool fail = false;
  bool withhold, first_arrival = true;
  uint32_t m2 = 0;     // running amax (two 16-bit halves) of the current amax slice
  float scale = 1.0f, recip = 1.0f;
  bool fast = true;

  // Wait for chunk j in its stage (warp-uniform verdict); returns the stage or nullptr.
  __device__ __forceinline__ const uint4* acquire(int* k_out) {
    constexpr int64_t ns = NS;
    const int k = static_cast<int>(j % ns);
    *k_out = k;
    if (!__all_sync(0xffffffffu, wait_bar(smem_u32(full + k),
                                          static_cast<uint32_t>((j / ns) & 1),
                                          p.timeout_ns)))
      return nullptr;
    return reinterpret_cast<const uint4*>(stages + k * ring_cap<NS>());
  }
  __device__ __forceinline__ void release(int k) {
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(empty + k));
    ++j;
  }
  __device__ __forceinline__ void amax_chunk(const Slice& sl, int64_t t) {
    if (fail) return;
    int k;
    const uint4* st = acquire(&k);
    if (st == nullptr) {
      fail = true;
      return;
    }
    const uint32_t nv = sl.chunk_bytes(t) / 16;
#pragma unroll 4
    for (uint32_t v = threadIdx.x; v < nv; v += kQtThreads) {
      const uint4 x = st[v];
      m2 = __vmaxu2(m2, x.x & 0x7fff7fffu);
      m2 = __vmaxu2(m2, x.y & 0x7fff7fffu);
      m2 = __vmaxu2(m2, x.z & 0x7fff7fffu);
      m2 = __vmaxu2(m2, x.w & 0x7fff7fffu);
    }
    release(k);
  }
  __device__ __forceinline__ void quant_chunk(const Slice& sl, int64_t t) {
    if (fail) return;
    int k;
    const uint4* st = acquire(&k);
    if (st == nullptr) {
      fail = true;
      return;
    }
    const uint32_t nv = sl.chunk_bytes(t) / 16;
    // contiguous rows: element index = byte offset / 2
    uint2* dst = reinterpret_cast<uint2*>(p.q + (sl.b0 + sl.chunk_offset(t)) / 2);
    if (fast) {
#pragma unroll 4
      for (uint32_t v = threadIdx.x; v < nv; v += kQtThreads)
        __stcs(dst + v, quant_vec<E5M2, true>(st[v], scale, recip));
    } else {
      for (uint32_t v = threadIdx.x; v < nv; v += kQtThreads)
        __stcs(dst + v, quant_vec<E5M2, false>(st[v], scale, recip));
    }
    release(k);
  }
  // All consumers: reduce this CTA's amax of unit u and publish it (thread 0). False on failure.
  __device__ __forceinline__ bool finish_amax(int u) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, max(m2 & 0xffffu, m2 >> 16));
    m2 = 0;
    if (lane == 0) red[warp] = m;
    fail = consumers_sync_or(fail);
    if (fail) return false;
    uint32_t mm = 0;
    if (threadIdx.x == 0) {
#pragma unroll
      for (int k = 0; k < kQtWarps; ++k) mm = max(mm, red[k]);
    }
    consumers_sync();  // red[] may be rewritten after this
    if (threadIdx.x == 0) {  // the atomics and their fence hold up thread 0 only
      publish(p, u, mm, withhold && first_arrival);
      first_arrival = false;
    }
    return true;
  }
  // All consumers: wait until unit w's amax is complete, then set up its scale.
  __device__ __forceinline__ bool get_scale(int w) {
    bool ok = true;
    if (threadIdx.x == 0) {
      ok = wait_unit(p, w);
      if (ok && blockIdx.x == 0)
        p.scales[w] = unit_scale(ld_relaxed_u32(p.ws + 4 + w), p.fmax);
    }
    fail = consumers_sync_or(fail || !ok);
    if (fail) return false;
    scale = unit_scale(ld_relaxed_u32(p.ws + 4 + w), p.fmax);
    recip = __frcp_rn(scale);
    fast = fast_route_ok(scale);
    return true;
  }
  __device__ __forceinline__ void note_unit(int w, const Slice& sl) {
    if (sl.unit_ok || blockIdx.x != 0 || threadIdx.x != 0) return;
    int64_t lo, hi;
    if (!unit_rows(p, w, &lo, &hi) && p.status != nullptr)
      atomicOr(p.status, GGEMM_VARK_DEV_BAD_OFFS);
    p.scales[w] = 1.0f;  // invalid or empty unit
  }
  __device__ __forceinline__ void run() {
    Slice a = slice_info<NS>(p, 0);
    note_unit(0, a);
    for (int64_t t = 0; t < a.chunks(); ++t) amax_chunk(a, t);
    if (a.unit_ok && !finish_amax(0)) return;
    for (int s = 1; s <= p.units; ++s) {
      const Slice b = slice_info<NS>(p, s - 1);
      a = slice_info<NS>(p, s);
      if (s < p.units) note_unit(s, a);
      const bool need_scale = b.unit_ok && (b.b1 > b.b0 || blockIdx.x == 0);
      bool have_scale = false;
      const int64_t na = a.chunks(), nb = b.chunks();
      for (int64_t ta = 0, tb = 0; ta < na || tb < nb;) {
        if (amax_next(ta, tb, na, nb)) {
          amax_chunk(a, ta++);
        } else {
          if (!have_scale) {
            if (!get_scale(s - 1)) return;
            have_scale = true;
          }
          quant_chunk(b, tb++);
        }
      }
      if (need_scale && !have_scale && !get_scale(s - 1)) return;
      if (a.unit_ok && !finish_amax(s)) return;
    }
    fail = consumers_sync_or(fail);
  }
};

template <bool E5M2, int NS>
// One block per SM (the ring takes ~192 KiB): stating it lets ptxas keep the unrolled consumer
// loops in registers (without it, it settled at 56 registers and spilled). The loops unrolled by
// 4, against not unrolled, measured x +1.9 / +2.9%, dy -0.1 / +0.9%, skewed dy +0.9 / +0.6% in two
// one-process A/B runs with bit-identical output; by 8, dy -7%.
__global__ void __launch_bounds__(kTmaThreads, 1) vark_quant_tma_kernel(const QuantParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + QT_STAGES * QT_CHUNK);
  uint64_t* empty = full + QT_STAGES;
  __shared__ uint32_t red[kQtWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int k = 0; k < QT_STAGES; ++k) {
      mbar_init(smem_u32(full + k), 1);
      mbar_init(smem_u32(empty + k), kQtWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();  // the only barrier with the producer warp
  if (warp == kQtWarps) {
    if (lane == 0) {
      Producer<NS> pr{p, smem_u32(smem), full, empty, l2_policy_evict_last(),
                  l2_policy_evict_first()};
      pr.run();
    }
    return;
  }
  Consumer<E5M2, NS> c{p, smem, full, empty, red, lane, warp};
  c.withhold = test_withhold(p);
  c.run();
  if (c.fail && threadIdx.x == 0) report_timeout(p, 0x52000000u);
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
    // Ring: two wide chunks when a CTA's average slice of a unit fits in them (known row count
    // only), else the default ring. Either ring takes ~192 KiB of shared memory: one CTA per SM.
    bool wide = false;
    if (token_limit != INT64_MAX && p.units > 0) {
      const double slice = static_cast<double>(token_limit) * static_cast<double>(stride_x_bytes) /
                           (static_cast<double>(p.units) * sm_count);
      wide = slice <= 2.0 * ring_cap<QT_STAGES_WIDE>();
    }
    if (wide)
      fn = e5m2 ? reinterpret_cast<const void*>(&vark_quant_tma_kernel<true, QT_STAGES_WIDE>)
                : reinterpret_cast<const void*>(&vark_quant_tma_kernel<false, QT_STAGES_WIDE>);
    else
      fn = e5m2 ? reinterpret_cast<const void*>(&vark_quant_tma_kernel<true, QT_STAGES>)
                : reinterpret_cast<const void*>(&vark_quant_tma_kernel<false, QT_STAGES>);
    smem = QT_SMEM;
    threads = kTmaThreads;
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

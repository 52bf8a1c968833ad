/*
 * vark_oracle_c.c - TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Plain-C CPU restatement of the reference's variable-K grouped wgrad, independent of torch:
 *
 *   out[g][m][n] = sL[g] * sR[g] * sum_{t in [off_g, off_{g+1})} LHS[t][m] * RHS[t][n]
 *
 * (ggemm-asm README.md:5,45-48; bench.py:182-193 "dW = lhs^T @ rhs"; bench.py:268 call shape).
 * fp8 codes are decoded from their bit fields per the OCP 8-bit floating point specification
 * (E4M3: bias 7, no infinities, S.1111.111 = NaN; E5M2: bias 15, IEEE-style Inf/NaN), every
 * product and sum is formed in double (an fp8 x fp8 product is exact in double), and the scale
 * is applied after the sum. Strides are in elements, as in the reference's kernel arguments
 * (bench.py:370-374). Also provides round-to-nearest-even fp32 -> bf16.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this file's
 * library (oracle/_build/libvark_oracle.so, built by oracle/Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

double vark_oracle_e4m3fn_to_f64(uint8_t v) {
  const int sign = (v >> 7) & 1;
  const int exp = (v >> 3) & 0xF;
  const int man = v & 0x7;
  double mag;
  if (exp == 0xF && man == 0x7) return NAN;
  if (exp == 0)
    mag = ldexp((double)man, -9); /* man/8 * 2^(1-7) */
  else
    mag = ldexp(1.0 + man / 8.0, exp - 7);
  return sign ? -mag : mag;
}

double vark_oracle_e5m2_to_f64(uint8_t v) {
  const int sign = (v >> 7) & 1;
  const int exp = (v >> 2) & 0x1F;
  const int man = v & 0x3;
  double mag;
  if (exp == 0x1F) {
    if (man != 0) return NAN;
    mag = INFINITY;
  } else if (exp == 0) {
    mag = ldexp((double)man, -16); /* man/4 * 2^(1-15) */
  } else {
    mag = ldexp(1.0 + man / 4.0, exp - 15);
  }
  return sign ? -mag : mag;
}

uint16_t vark_oracle_f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) return (uint16_t)((u >> 16) | 0x40u);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

/* out: double [G][OUT_M][OUT_N] (contiguous). scale_stride 0: scalar scales, 1: per group.
 * Returns 0, or -1 if group_offs is not monotone / negative. */
int vark_oracle_wgrad_f64(const uint8_t* lhs, const uint8_t* rhs, const float* lhs_scale,
                          const float* rhs_scale, int scale_stride, const int64_t* offs, int G,
                          int OUT_M, int OUT_N, int64_t stride_lhs_m, int64_t stride_rhs_m,
                          double* out) {
  double lut_l[256], lut_r[256];
  for (int i = 0; i < 256; ++i) {
    lut_l[i] = vark_oracle_e4m3fn_to_f64((uint8_t)i);
    lut_r[i] = vark_oracle_e5m2_to_f64((uint8_t)i);
  }
  for (int g = 0; g < G; ++g) {
    const int64_t lo = offs[g], hi = offs[g + 1];
    if (lo < 0 || hi < lo) return -1;
    double* o = out + (int64_t)g * OUT_M * OUT_N;
    for (int64_t i = 0; i < (int64_t)OUT_M * OUT_N; ++i) o[i] = 0.0;
    for (int64_t t = lo; t < hi; ++t) {
      const uint8_t* lr = lhs + t * stride_lhs_m;
      const uint8_t* rr = rhs + t * stride_rhs_m;
      for (int m = 0; m < OUT_M; ++m) {
        const double a = lut_l[lr[m]];
        if (a == 0.0) continue;
        double* orow = o + (int64_t)m * OUT_N;
        for (int n = 0; n < OUT_N; ++n) orow[n] += a * lut_r[rr[n]];
      }
    }
    const double s = (double)lhs_scale[(int64_t)g * scale_stride] *
                     (double)rhs_scale[(int64_t)g * scale_stride];
    for (int64_t i = 0; i < (int64_t)OUT_M * OUT_N; ++i) o[i] *= s;
  }
  return 0;
}

/*
 * Exhaustive check of the division method the quantiser uses in place of an IEEE division per
 * element (Markstein's correction step, P. Markstein, "Computation of elementary functions on
 * the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
 *     y = RN(1/b),  q = RN(a*y),  r = RN(a - b*q) (one fma, exact),  q' = RN(q + r*y) (one fma)
 * with a the significand of a bf16 value (k/128, k = 128..255) and b every fp32 in [1, 2).
 * Every step scales exactly by powers of two while the operands and results stay normal, so
 * these 2^30 cases stand for all normal a and b. Returns the number of (a, b) with q' != a/b
 * (the IEEE quotient); the quantiser's tests require 0.
 */
#if defined(__x86_64__) && defined(__GNUC__)
__attribute__((target("fma"))) static long markstein_range_hw(uint32_t lo, uint32_t hi) {
  long bad = 0;
  for (uint32_t bits = lo; bits < hi; ++bits) {
    float b;
    memcpy(&b, &bits, 4);
    const float y = 1.0f / b;
    for (int k = 128; k < 256; ++k) {
      const float a = (float)k * 0.0078125f;
      const float q = a * y;
      const float r = __builtin_fmaf(-b, q, a);
      const float q2 = __builtin_fmaf(r, y, q);
      bad += q2 != a / b;
    }
  }
  return bad;
}
#endif

static long markstein_range_sw(uint32_t lo, uint32_t hi) {
  long bad = 0;
  for (uint32_t bits = lo; bits < hi; ++bits) {
    float b;
    memcpy(&b, &bits, 4);
    const float y = 1.0f / b;
    for (int k = 128; k < 256; ++k) {
      const float a = (float)k * 0.0078125f;
      const float q = a * y;
      const float r = fmaf(-b, q, a);
      const float q2 = fmaf(r, y, q);
      bad += q2 != a / b;
    }
  }
  return bad;
}

/* Mismatches for b with bit patterns in [0x3f800000 + lo, 0x3f800000 + hi), hi <= 2^23. */
long vark_oracle_markstein_mismatches(uint32_t lo, uint32_t hi) {
  if (hi > (1u << 23)) hi = 1u << 23;
#if defined(__x86_64__) && defined(__GNUC__)
  if (__builtin_cpu_supports("fma")) return markstein_range_hw(0x3f800000u + lo, 0x3f800000u + hi);
#endif
  return markstein_range_sw(0x3f800000u + lo, 0x3f800000u + hi);
}

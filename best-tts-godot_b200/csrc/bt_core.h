// bt_core.h -- definitions shared by the host planner and the sm_100a kernels.
//
// numpy-exact float32 math.  The reference computes every hot-path op with
// numpy (tools/ref_runtime.py:446-489), so "identical results" means
// identical to numpy's float32 ufuncs.  numpy 2.x evaluates float32 exp, sin
// and cos with its own SIMD algorithms (Cody-Waite range reduction and short
// polynomials evaluated with fused multiply-adds, published in numpy's
// loops_exponent_log / loops_trigonometric sources), and reduces a contiguous
// float32 axis with its pairwise summation.  The functions below restate
// those published algorithms step by step with explicitly rounded
// operations, so the GPU reproduces numpy bit for bit (the CPU tests compare
// the host build of these same functions with numpy; the GPU tests compare
// the kernels with the oracle).
//
// Every arithmetic step uses an explicitly rounded intrinsic on the device
// (__fadd_rn / __fmul_rn / __fmaf_rn / __fdiv_rn cannot be contracted), and
// the host build is compiled with -ffp-contract=off.
#pragma once
#include <stdint.h>
#include <math.h>

#if defined(__CUDACC__)
#define BT_HD __host__ __device__ __forceinline__
#else
#define BT_HD inline
#endif

#if defined(__CUDA_ARCH__)
#define BT_ADD(a, b) __fadd_rn((a), (b))
#define BT_SUB(a, b) __fsub_rn((a), (b))
#define BT_MUL(a, b) __fmul_rn((a), (b))
#define BT_DIV(a, b) __fdiv_rn((a), (b))
#define BT_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define BT_SQRT(a) __fsqrt_rn(a)
#else
#define BT_ADD(a, b) ((a) + (b))
#define BT_SUB(a, b) ((a) - (b))
#define BT_MUL(a, b) ((a) * (b))
#define BT_DIV(a, b) ((a) / (b))
#define BT_FMA(a, b, c) fmaf((a), (b), (c))
#define BT_SQRT(a) sqrtf(a)
#endif

namespace bt {

BT_HD float bits_f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  union { uint32_t u; float f; } v; v.u = u; return v.f;
#endif
}
BT_HD uint32_t f_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  union { uint32_t u; float f; } v; v.f = f; return v.u;
#endif
}

BT_HD float qnan() { return bits_f(0x7fc00000u); }
BT_HD bool is_nan(float x) { return x != x; }

// 2^e as a float for e in [-126, 127].
BT_HD float pow2i(int e) { return bits_f((uint32_t)(e + 127) << 23); }

// p * 2^k with a single rounding, for p in [0.5, 2) and k in [-152, 128]:
// the first product is exact (normal result), the second rounds once --
// the same result as AVX-512 vscalefps, which numpy's exp uses.
BT_HD float scale_pow2(float p, int k) {
  int k1 = k / 2;
  int k2 = k - k1;
  return BT_MUL(BT_MUL(p, pow2i(k1)), pow2i(k2));
}

#if defined(__CUDACC__)
// The hardware reciprocal approximation (rcp.approx.ftz.f32, relative error
// within about 1 ulp; subnormal operands and results flush to zero).
__device__ __forceinline__ float rcp_approx(float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  return y;
}
// RN(a / b) by Markstein's method: the reciprocal approximation refined by
// one Newton-Raphson step, the quotient a*y corrected by one exact FMA
// residual step (P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; Muller et
// al., Handbook of Floating-Point Arithmetic, the chapter on FMA-based
// division).  Only for operands whose reciprocal, quotient and residual stay
// normal and finite -- every caller bounds its operands -- and every use is
// checked bit for bit against IEEE division over all of its float32 inputs
// (bt_selfcheck).
__device__ __forceinline__ float div_nr(float a, float b) {
  float y = rcp_approx(b);
  const float e = __fmaf_rn(-b, y, 1.0f);
  y = __fmaf_rn(y, e, y);
  const float q = __fmul_rn(a, y);
  const float r = __fmaf_rn(-b, q, a);
  return __fmaf_rn(r, y, q);
}

// 1 / b in double for a float b, within one double ulp of RN64(1 / b):
// the hardware approximation (rcp.approx.ftz.f64) refined by two
// Newton-Raphson steps y += y * (1 - b*y), each with two FMAs -- no call,
// no slow path (b as a double is never subnormal, nor is 1/b).  Zeros and
// infinities, where the steps would give NaN, are set to IEEE's answer.
// Checked against IEEE division on all 2^32 floats (bt_selfcheck).
__device__ __forceinline__ double recip_d(float b) {
  const double d = (double)b;
  double y;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(d));
  double e = __fma_rn(-d, y, 1.0);
  y = __fma_rn(y, e, y);
  e = __fma_rn(-d, y, 1.0);
  y = __fma_rn(y, e, y);
  if (b == 0.0f) y = copysign((double)INFINITY, d);
  if (fabsf(b) == INFINITY) y = copysign(0.0, d);
  return y;
}
// tanh of a float, evaluated in double with no call and no data-dependent
// branch.  With a = |x| (clamped at 9.1) and y = -2a: k = rint(y / ln2),
// r = y - k ln2 (|r| <= ln2 / 2), expm1(r) by its Taylor series to degree 8
// (truncation below 2^-31 relative), expm1(y) = 2^k expm1(r) + (2^k - 1),
// tanh(a) = -expm1(y) / (2 + expm1(y)) with the reciprocal refined by one
// Newton-Raphson step (about 2^-44 from the hardware approximation).  The
// double value errs by less than 2^-30 relative -- a 2^-25 relative error
// already keeps it within half a float ulp -- so its float rounding is
// within one ulp of the correctly rounded tanh (checked
// on all 2^32 inputs by bt_selfcheck; numpy's float32 tanh is itself within
// one ulp of it).  |x| >= 9.1 gives +-1 (tanh rounds to 1 from 9.02 on),
// NaN gives NaN.
__device__ __forceinline__ float tanh_f(float x) {
  const double a = (double)fminf(fabsf(x), 9.1f);
  const double y = -2.0 * a;
  const double kMagic = 6755399441055744.0;   // 1.5 * 2^52: t's low 32 bits hold k
  const double t = __fma_rn(y, 1.4426950408889634, kMagic);
  const double kd = __dsub_rn(t, kMagic);
  const double r = __fma_rn(-kd, 0.6931471805599453, y);
  double p = 2.48015873015873e-05;             // 1/8!
  p = __fma_rn(p, r, 0.0001984126984126984);
  p = __fma_rn(p, r, 0.001388888888888889);
  p = __fma_rn(p, r, 0.008333333333333333);
  p = __fma_rn(p, r, 0.041666666666666664);
  p = __fma_rn(p, r, 0.16666666666666666);
  p = __fma_rn(p, r, 0.5);
  p = __fma_rn(p, r, 1.0);
  p = __dmul_rn(p, r);                         // expm1(r)
  const int k = __double2loint(t);             // in [-27, 0]
  const double s2k = __hiloint2double((1023 + k) << 20, 0);
  const double em = __fma_rn(s2k, p, __dsub_rn(s2k, 1.0));
  const double d = __dadd_rn(2.0, em);
  double w;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(w) : "d"(d));
  w = __fma_rn(w, __fma_rn(-d, w, 1.0), w);
  const float v = copysignf(__double2float_rn(__dmul_rn(-em, w)), x);
  if (x != x) return x;
  return fabsf(x) >= 9.1f ? copysignf(1.0f, x) : v;
}

// Correctly rounded a / b for a divisor shared by many elements: with
// rb = recip_d(b) computed once, RN32(RN64(a * rb)) == RN32(a / b) for all
// float a, b.  (A quotient of two floats that is not a float lies at least
// 2^-49 away (relative) from every float rounding midpoint and is never on
// one; rb errs by at most 2^-52 and the double product adds 2^-53, so it
// rounds to the same float.  Infinities, zeros and NaNs follow IEEE
// division.)
__device__ __forceinline__ float div_by(float a, double rb) {
  return __double2float_rn(__dmul_rn((double)a, rb));
}

// Division of many floats by one divisor b in float32 arithmetic alone
// (Markstein's correction step with the correctly rounded reciprocal):
//   y = RN(1/b) once, then per value  q0 = RN(a y),  r = RN(a - b q0) (an
//   FMA),  q = RN(q0 + r y) (an FMA).
// q == RN(a / b) whenever |a| and |b| lie in the window [2^-60, 2^60): then
// a y, a / b, the residual and every step stay normal, so scaling a or b by
// a power of two scales each step exactly, and the claim reduces to the
// 2^46 pairs of significands in [1, 2) x [1, 2) -- which bt_selfcheck
// (kind 7) checks one by one.  Values outside the window (zeros, subnormals,
// infinities, NaN, huge or tiny values) and divisors outside it take div_by,
// the double-precision path above; callers test the window with
// div_row_outside and recompute those values.  Three float operations per
// value instead of two conversions and a double product.
struct RowDiv {
  float b, y;       // the divisor and RN(1 / b)
  uint32_t span;    // width of the window of |a|'s exponent field; 0 when b lies outside
};
constexpr uint32_t kRowDivLo = 67u << 23;      // 2^-60: biased exponent 67
constexpr uint32_t kRowDivSpan = 120u << 23;   // up to 2^60 (biased exponent 186)
__device__ __forceinline__ bool row_div_in_window(float v) {
  return (f_bits(v) & 0x7f800000u) - kRowDivLo < kRowDivSpan;
}
__device__ __forceinline__ RowDiv row_div(float b) {
  RowDiv d;
  d.b = b;
  d.y = __frcp_rn(b);
  d.span = row_div_in_window(b) ? kRowDivSpan : 0u;
  return d;
}
// the three-operation quotient, valid inside the window
__device__ __forceinline__ float div_row_fast(float a, float b, float y) {
  const float q0 = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(-b, q0, a), y, q0);
}
// whether a lies outside the window (its quotient must come from div_by)
__device__ __forceinline__ bool div_row_outside(float a, const RowDiv& d) {
  return (f_bits(a) & 0x7f800000u) - kRowDivLo >= d.span;
}
#endif

// ---------------------------------------------------------------------------
// exp: numpy's float32 SIMD algorithm (rational minimax on a Cody-Waite
// reduced argument).  x*log2(e) is rounded to an integer quadrant q with the
// 1.5*2^23 trick, r = x - q*ln2 in two fused steps, exp(r) = P5(r)/Q2(r),
// result = that * 2^q.  Overflow above 88.72283935546875 gives +inf,
// underflow at or below -103.97208404541015625 gives 0, NaN gives NaN.
// ---------------------------------------------------------------------------
// IEEE_DIV: the quotient P5/Q2 by IEEE division (the form the self-check
// compares against); otherwise by div_nr on the device (Q2 lies in [0.9,
// 1.1] and P5 in [0.7, 1.5] on the reduced range).
template <bool IEEE_DIV = false>
BT_HD float np_expf_t(float x) {
  const float kXmax = 88.72283935546875f;
  const float kXmin = -103.97208404541015625f;
  if (is_nan(x)) return qnan();
  if (x >= kXmax) return bits_f(0x7f800000u);
  if (x <= kXmin) return 0.0f;
  const float kLog2e = 1.442695040888963407359924681001892137f;
  const float kMagic = 12582912.0f;             // 1.5 * 2^23
  const float kLn2Hi = -6.93145752e-1f;
  const float kLn2Lo = -1.42860677e-6f;
  const float t = BT_ADD(BT_MUL(x, kLog2e), kMagic);
  const float q = BT_SUB(t, kMagic);
  float r = BT_FMA(q, kLn2Hi, x);
  r = BT_FMA(q, kLn2Lo, r);
  float num = BT_FMA(5.082762527590693718096e-04f, r, 6.757896990527504603057e-03f);
  num = BT_FMA(num, r, 5.114512081637298353406e-02f);
  num = BT_FMA(num, r, 2.473615434895520810817e-01f);
  num = BT_FMA(num, r, 7.257664613233124478488e-01f);
  num = BT_FMA(num, r, 9.999999999980870924916e-01f);
  float den = BT_FMA(2.159509375685829852307e-02f, r, -2.742335390411667452936e-01f);
  den = BT_FMA(den, r, 1.0f);
#if defined(__CUDA_ARCH__)
  const float pq = IEEE_DIV ? BT_DIV(num, den) : div_nr(num, den);
#else
  const float pq = BT_DIV(num, den);
#endif
  // For |x| < 86 the quadrant k lies in [-124, 124], so pq * 2^k is normal
  // and exact, and it is pq's bits plus k << 23; bits(t) = 0x4B400000 + k,
  // whose shift by 23 leaves k << 23 (mod 2^32).
  if (!IEEE_DIV && fabsf(x) < 86.0f) return bits_f(f_bits(pq) + (f_bits(t) << 23));
  return scale_pow2(pq, (int)q);
}
BT_HD float np_expf(float x) { return np_expf_t<false>(x); }

// ---------------------------------------------------------------------------
// Double-precision sine / cosine without local memory (the library's own
// implementation; used where numpy leaves its SIMD path -- it calls the C
// library for |x| beyond 117435.992 (sine) / 71476.0625 (cosine) -- and for
// float64 results).  Argument reduction x = q*pi/2 + r:
//   |x| <= 2^20: Cody-Waite with pi/2 split into a 33-bit, a 33-bit and a
//     53-bit part (q*hi and q*mid are exact products);
//   larger |x|: Payne-Hanek -- the 53-bit mantissa times a 160-bit window of
//     the binary expansion of 2/pi, in 32-bit limbs held in named registers.
// sin(r), cos(r) on |r| <= pi/4 by their Taylor series to degree 21 / 22.
// The 2/pi words below are the first 1600 fractional bits of 2/pi, computed
// from Machin's formula pi = 16 atan(1/5) - 4 atan(1/239) at 520 digits.
// ---------------------------------------------------------------------------
#define BT_TWO_OVER_PI_WORDS \
    0xa2f9836eu, 0x4e441529u, 0xfc2757d1u, 0xf534ddc0u, 0xdb629599u, 0x3c439041u, \
    0xfe5163abu, 0xdebbc561u, 0xb7246e3au, 0x424dd2e0u, 0x06492eeau, 0x09d1921cu, \
    0xfe1deb1cu, 0xb129a73eu, 0xe88235f5u, 0x2ebb4484u, 0xe99c7026u, 0xb45f7e41u, \
    0x3991d639u, 0x835339f4u, 0x9c845f8bu, 0xbdf9283bu, 0x1ff897ffu, 0xde05980fu, \
    0xef2f118bu, 0x5a0a6d1fu, 0x6d367ecfu, 0x27cb09b7u, 0x4f463f66u, 0x9e5fea2du, \
    0x7527bac7u, 0xebe5f17bu, 0x3d0739f7u, 0x8a5292eau, 0x6bfb5fb1u, 0x1f8d5d08u, \
    0x56033046u, 0xfc7b6babu, 0xf0cfbc20u, 0x9af4361du, 0xa9e39161u, 0x5ee61b08u, \
    0x6599855fu, 0x14a06840u, 0x8dffd880u, 0x4d732731u, 0x06061556u, 0xca73a8c9u, \
    0x60e27bc0u, 0x8c6b47c4u
constexpr int kTwoOverPiWords = 50;
#if defined(__CUDACC__)
static __constant__ uint32_t kTwoOverPiDev[kTwoOverPiWords] = {BT_TWO_OVER_PI_WORDS};
#endif
static const uint32_t kTwoOverPiHost[kTwoOverPiWords] = {BT_TWO_OVER_PI_WORDS};

BT_HD uint32_t two_over_pi_word(int i) {
  if (i < 0 || i >= kTwoOverPiWords) return 0u;
#if defined(__CUDA_ARCH__)
  return kTwoOverPiDev[i];
#else
  return kTwoOverPiHost[i];
#endif
}

#if defined(__CUDA_ARCH__)
#define BT_DADD(a, b) __dadd_rn((a), (b))
#define BT_DMUL(a, b) __dmul_rn((a), (b))
#define BT_DFMA(a, b, c) __fma_rn((a), (b), (c))
#else
#define BT_DADD(a, b) ((a) + (b))
#define BT_DMUL(a, b) ((a) * (b))
#define BT_DFMA(a, b, c) fma((a), (b), (c))
#endif

BT_HD uint64_t d_bits(double d) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(d);
#else
  union { uint64_t u; double d; } v; v.d = d; return v.u;
#endif
}

// 32-bit limb i of a 224-bit number held in c0..c6.
BT_HD uint64_t limb7(int i, uint64_t c0, uint64_t c1, uint64_t c2, uint64_t c3, uint64_t c4, uint64_t c5,
                     uint64_t c6) {
  switch (i) {
    case 0: return c0; case 1: return c1; case 2: return c2; case 3: return c3;
    case 4: return c4; case 5: return c5; case 6: return c6;
  }
  return 0;
}

// Bits [p, p + 64) of the number held in c0..c6.
BT_HD uint64_t bits64_at(int p, uint64_t c0, uint64_t c1, uint64_t c2, uint64_t c3, uint64_t c4, uint64_t c5,
                         uint64_t c6) {
  const int i = p >> 5, off = p & 31;
  uint64_t v = limb7(i, c0, c1, c2, c3, c4, c5, c6) >> off;
  v |= limb7(i + 1, c0, c1, c2, c3, c4, c5, c6) << (32 - off);
  if (off > 0) v |= limb7(i + 2, c0, c1, c2, c3, c4, c5, c6) << (64 - off);
  return v;
}

// |x| = q*pi/2 + r with |r| <= pi/4 (approximately), for finite |x| > 2^20.
BT_HD double reduce_pio2_large(double ax, int* quad) {
  const uint64_t b = d_bits(ax);
  const int E = (int)((b >> 52) & 0x7ff) - 1023;
  const uint64_t m = (b & ((1ull << 52) - 1)) | (1ull << 52);
  const int e = E - 52;                      // ax = m * 2^e
  const int j0 = (e - 1 > 1) ? e - 1 : 1;    // first bit of 2/pi that matters mod 4
  const int i0 = j0 - 1, wi = i0 >> 5, bo = i0 & 31;
  uint64_t w[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    uint32_t hi = two_over_pi_word(wi + k), lo = two_over_pi_word(wi + k + 1);
    w[k] = bo ? (uint64_t)(uint32_t)((hi << bo) | (lo >> (32 - bo))) : (uint64_t)hi;
  }
  const uint64_t M = 0xffffffffull, ml = m & M, mh = m >> 32;
  const uint64_t a0 = ml * w[4], a1 = ml * w[3], a2 = ml * w[2], a3 = ml * w[1], a4 = ml * w[0];
  const uint64_t b1 = mh * w[4], b2 = mh * w[3], b3 = mh * w[2], b4 = mh * w[1], b5 = mh * w[0];
  uint64_t c0 = a0 & M;
  uint64_t c1 = (a0 >> 32) + (a1 & M) + (b1 & M);
  uint64_t c2 = (a1 >> 32) + (a2 & M) + (b1 >> 32) + (b2 & M);
  uint64_t c3 = (a2 >> 32) + (a3 & M) + (b2 >> 32) + (b3 & M);
  uint64_t c4 = (a3 >> 32) + (a4 & M) + (b3 >> 32) + (b4 & M);
  uint64_t c5 = (a4 >> 32) + (b4 >> 32) + (b5 & M);
  uint64_t c6 = (b5 >> 32);
  c1 += c0 >> 32; c0 &= M;
  c2 += c1 >> 32; c1 &= M;
  c3 += c2 >> 32; c2 &= M;
  c4 += c3 >> 32; c3 &= M;
  c5 += c4 >> 32; c4 &= M;
  c6 += c5 >> 32; c5 &= M;
  const int sh = j0 + 159 - e;               // x*2/pi = P * 2^-sh (mod 4)
  const uint64_t frac = bits64_at(sh - 64, c0, c1, c2, c3, c4, c5, c6);
  int q = (int)(bits64_at(sh, c0, c1, c2, c3, c4, c5, c6) & 3);
  q += (int)(frac >> 63);                    // round to the nearest quadrant
  *quad = q & 3;
  const double f = (double)(int64_t)frac * 5.421010862427522e-20;   // 2^-64
  return BT_DMUL(f, 0x1.921fb54442d18p+0);
}

// Taylor coefficients (-1)^k / (2k+1)! and (-1)^k / (2k)!, correctly rounded.
BT_HD double sin_taylor(double r) {
  const double r2 = BT_DMUL(r, r);
  double p = 0x1.71b8ef6dcf572p-66;          // +1/21!
  p = BT_DFMA(p, r2, -0x1.2f49b46814157p-57);  // -1/19!
  p = BT_DFMA(p, r2, 0x1.952c77030ad4ap-49);   // +1/17!
  p = BT_DFMA(p, r2, -0x1.ae7f3e733b81fp-41);  // -1/15!
  p = BT_DFMA(p, r2, 0x1.6124613a86d09p-33);   // +1/13!
  p = BT_DFMA(p, r2, -0x1.ae64567f544e4p-26);  // -1/11!
  p = BT_DFMA(p, r2, 0x1.71de3a556c734p-19);   // +1/9!
  p = BT_DFMA(p, r2, -0x1.a01a01a01a01ap-13);  // -1/7!
  p = BT_DFMA(p, r2, 0x1.1111111111111p-7);    // +1/5!
  p = BT_DFMA(p, r2, -0x1.5555555555555p-3);   // -1/3!
  return BT_DFMA(BT_DMUL(p, r2), r, r);
}
BT_HD double cos_taylor(double r) {
  const double r2 = BT_DMUL(r, r);
  double p = -0x1.0ce396db7f853p-70;         // -1/22!
  p = BT_DFMA(p, r2, 0x1.e542ba4020225p-62);   // +1/20!
  p = BT_DFMA(p, r2, -0x1.6827863b97d97p-53);  // -1/18!
  p = BT_DFMA(p, r2, 0x1.ae7f3e733b81fp-45);   // +1/16!
  p = BT_DFMA(p, r2, -0x1.93974a8c07c9dp-37);  // -1/14!
  p = BT_DFMA(p, r2, 0x1.1eed8eff8d898p-29);   // +1/12!
  p = BT_DFMA(p, r2, -0x1.27e4fb7789f5cp-22);  // -1/10!
  p = BT_DFMA(p, r2, 0x1.a01a01a01a01ap-16);   // +1/8!
  p = BT_DFMA(p, r2, -0x1.6c16c16c16c17p-10);  // -1/6!
  p = BT_DFMA(p, r2, 0x1.5555555555555p-5);    // +1/4!
  p = BT_DFMA(p, r2, -0.5);                    // -1/2!
  return BT_DFMA(p, r2, 1.0);
}

#if defined(__CUDACC__)
#define BT_COLD static __host__ __device__ __noinline__
#else
#define BT_COLD static inline
#endif

BT_COLD double bt_sincos_d(double x, bool cosine) {
  if (x != x) return x;
  const double ax = fabs(x);
  if (ax == INFINITY) return ax - ax;  // NaN
  int q;
  double r;
  if (ax <= 1048576.0) {
    const double t = BT_DMUL(ax, 0x1.45f306dc9c883p-1);
    const double qd = rint(t);
    r = BT_DFMA(-qd, 0x1.921fb54400000p+0, ax);
    r = BT_DFMA(-qd, 0x1.0b4611a600000p-34, r);
    r = BT_DFMA(-qd, 0x1.3198a2e037073p-69, r);
    q = (int)((int64_t)qd & 3);
  } else {
    r = reduce_pio2_large(ax, &q);
  }
  if (cosine) q += 1;
  double v = (q & 1) ? cos_taylor(r) : sin_taylor(r);
  if (q & 2) v = -v;
  if (!cosine && x < 0) v = -v;
  if (!cosine && x == 0) v = x;   // sin(+-0) = +-0
  return v;
}

// ---------------------------------------------------------------------------
// sin / cos: numpy's float32 SIMD algorithm.  q = round(x * 2/pi) (computed
// as one fused multiply-add with the 1.5*2^23 rounding constant), a
// three-part Cody-Waite reduction r = x - q*pi/2, then the sine polynomial
// (odd, degree 9) or the cosine polynomial (even, degree 8) on r chosen by
// the quadrant, negated in quadrants 2 and 3.  Beyond |x| = 117435.992
// (sine) or 71476.0625 (cosine) numpy falls back to the C library; there
// bt_sincos_d (double precision, rounded to float) stands in for it.
// ---------------------------------------------------------------------------
// NaN and the arguments numpy hands to the C library, kept out of line so
// the common path stays small.
BT_COLD float np_sincosf_big(float x, bool cosine) {
  if (is_nan(x)) return qnan();
  return (float)bt_sincos_d((double)x, cosine);
}

// The quadrant q = t - 1.5*2^23 of t = fma(x, 2/pi, 1.5*2^23) is an integer
// with |q| < 2^22, so t lies in [2^23, 2^24) where its ulp is 1 and the low
// mantissa bits of t are q modulo 2^22: the two low bits of t are q mod 4,
// the same as (int)q & 3 -- read from the bits instead of converting.
BT_HD float np_sincosf(float x, bool cosine) {
  const float lim = cosine ? 71476.0625f : 117435.992f;
  if (!(fabsf(x) <= lim)) return np_sincosf_big(x, cosine);
  const float kTwoOverPi = 0x1.45f306p-1f;
  const float kMagic = 12582912.0f;
  const float t = BT_FMA(x, kTwoOverPi, kMagic);
  const float q = BT_SUB(t, kMagic);
  float r = BT_FMA(q, -0x1.921fb0p+00f, x);
  r = BT_FMA(q, -0x1.5110b4p-22f, r);
  r = BT_FMA(q, -0x1.846988p-48f, r);
  float r2 = BT_MUL(r, r);
  float c = BT_FMA(0x1.98e616p-16f, r2, -0x1.6c06dcp-10f);
  c = BT_FMA(c, r2, 0x1.55553cp-05f);
  c = BT_FMA(c, r2, -0x1.000000p-01f);
  c = BT_FMA(c, r2, 0x1.000000p+00f);
  float s = BT_FMA(0x1.7d3bbcp-19f, r2, -0x1.a06bbap-13f);
  s = BT_FMA(s, r2, 0x1.11119ap-07f);
  s = BT_FMA(s, r2, -0x1.555556p-03f);
  s = BT_FMA(s, r2, 0.0f);
  s = BT_FMA(s, r, r);
  const uint32_t iq = f_bits(t) + (cosine ? 1u : 0u);
  float v = (iq & 1u) ? c : s;
  if (iq & 2u) v = BT_SUB(0.0f, v);
  return v;
}
BT_HD float np_sinf(float x) { return np_sincosf(x, false); }
BT_HD float np_cosf(float x) { return np_sincosf(x, true); }

// Sigmoid exactly as the reference spells it: 1 / (1 + exp(-x))
// (ref_runtime.py:470-471), each step rounded in float32.
// On the device the reciprocal goes through div_nr while 1 + exp(-x) is
// below 2^120 (then 1/d stays far from the subnormal range), else through
// recip_d rounded to float (1/d of a float d is never within 2^-47,
// relative, of a float rounding midpoint, subnormal ones included, and
// recip_d errs by at most 2^-52): no division subroutine call.
template <bool IEEE_DIV = false>
BT_HD float np_sigmoidf_t(float x) {
  const float d = BT_ADD(1.0f, np_expf_t<IEEE_DIV>(-x));
#if defined(__CUDA_ARCH__)
  if (!IEEE_DIV) return d < 0x1p120f ? div_nr(1.0f, d) : __double2float_rn(recip_d(d));
#endif
  return BT_DIV(1.0f, d);
}
BT_HD float np_sigmoidf(float x) { return np_sigmoidf_t<false>(x); }

// ---------------------------------------------------------------------------
// numpy's pairwise summation of a contiguous float32 run (the inner loop of
// np.add.reduce over a contiguous axis): runs of fewer than 8 are summed
// left to right; runs of at most 128 use 8 interleaved accumulators combined
// as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) followed by the remainder left to
// right; longer runs split at n2 = n/2 rounded down to a multiple of 8 and
// add the two halves.  np.sum adds the result to an initial +0.0.
// ---------------------------------------------------------------------------
constexpr int kPwLeaf = 128;

BT_HD int64_t pw_split(int64_t n) {
  int64_t h = n / 2;
  return h - (h % 8);
}

// Depth of the deepest node of the pairwise tree of a run of length n.
inline int pw_depth(int64_t n) {
  if (n <= kPwLeaf) return 0;
  int64_t h = pw_split(n);
  int a = pw_depth(h), b = pw_depth(n - h);
  return 1 + (a > b ? a : b);
}

template <class T, class F>
inline float pw_sum_host(const T* a, int64_t n, F f) {
  if (n < 8) {
    float res = 0.0f;
    for (int64_t i = 0; i < n; ++i) res = BT_ADD(res, f(a[i]));
    return res;
  }
  if (n <= kPwLeaf) {
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = f(a[j]);
    int64_t i = 8;
    for (; i < n - (n % 8); i += 8)
      for (int j = 0; j < 8; ++j) r[j] = BT_ADD(r[j], f(a[i + j]));
    float res = BT_ADD(BT_ADD(BT_ADD(r[0], r[1]), BT_ADD(r[2], r[3])),
                       BT_ADD(BT_ADD(r[4], r[5]), BT_ADD(r[6], r[7])));
    for (; i < n; ++i) res = BT_ADD(res, f(a[i]));
    return res;
  }
  int64_t h = pw_split(n);
  return BT_ADD(pw_sum_host(a, h, f), pw_sum_host(a + h, n - h, f));
}

// numpy's mean of a float32 run: the float32 sum divided by the count in
// double precision (np.mean divides by an intp count, which promotes the
// division to float64) and rounded back to float32.
BT_HD float np_mean_from_sum(float sum, int64_t n) {
  return (float)((double)sum / (double)n);
}

}  // namespace bt

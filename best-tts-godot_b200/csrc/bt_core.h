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

// ---------------------------------------------------------------------------
// exp: numpy's float32 SIMD algorithm (rational minimax on a Cody-Waite
// reduced argument).  x*log2(e) is rounded to an integer quadrant q with the
// 1.5*2^23 trick, r = x - q*ln2 in two fused steps, exp(r) = P5(r)/Q2(r),
// result = that * 2^q.  Overflow above 88.72283935546875 gives +inf,
// underflow at or below -103.97208404541015625 gives 0, NaN gives NaN.
// ---------------------------------------------------------------------------
BT_HD float np_expf(float x) {
  const float kXmax = 88.72283935546875f;
  const float kXmin = -103.97208404541015625f;
  if (is_nan(x)) return qnan();
  if (x >= kXmax) return bits_f(0x7f800000u);
  if (x <= kXmin) return 0.0f;
  const float kLog2e = 1.442695040888963407359924681001892137f;
  const float kMagic = 12582912.0f;             // 1.5 * 2^23
  const float kLn2Hi = -6.93145752e-1f;
  const float kLn2Lo = -1.42860677e-6f;
  float q = BT_ADD(BT_MUL(x, kLog2e), kMagic);
  q = BT_SUB(q, kMagic);
  float r = BT_FMA(q, kLn2Hi, x);
  r = BT_FMA(q, kLn2Lo, r);
  float num = BT_FMA(5.082762527590693718096e-04f, r, 6.757896990527504603057e-03f);
  num = BT_FMA(num, r, 5.114512081637298353406e-02f);
  num = BT_FMA(num, r, 2.473615434895520810817e-01f);
  num = BT_FMA(num, r, 7.257664613233124478488e-01f);
  num = BT_FMA(num, r, 9.999999999980870924916e-01f);
  float den = BT_FMA(2.159509375685829852307e-02f, r, -2.742335390411667452936e-01f);
  den = BT_FMA(den, r, 1.0f);
  return scale_pow2(BT_DIV(num, den), (int)q);
}

// ---------------------------------------------------------------------------
// sin / cos: numpy's float32 SIMD algorithm.  q = round(x * 2/pi) (computed
// as one fused multiply-add with the 1.5*2^23 rounding constant), a
// three-part Cody-Waite reduction r = x - q*pi/2, then the sine polynomial
// (odd, degree 9) or the cosine polynomial (even, degree 8) on r chosen by
// the quadrant, negated in quadrants 2 and 3.  Beyond |x| = 117435.992
// (sine) or 71476.0625 (cosine) numpy falls back to the C library, which
// this code replaces with a double-precision evaluation rounded to float.
// ---------------------------------------------------------------------------
BT_HD float np_sincosf(float x, bool cosine) {
  if (is_nan(x)) return qnan();
  const float lim = cosine ? 71476.0625f : 117435.992f;
  if (!(fabsf(x) <= lim)) {
    double d = (double)x;
    return (float)(cosine ? cos(d) : sin(d));
  }
  const float kTwoOverPi = 0x1.45f306p-1f;
  const float kMagic = 12582912.0f;
  float q = BT_SUB(BT_FMA(x, kTwoOverPi, kMagic), kMagic);
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
  int iq = (int)q + (cosine ? 1 : 0);
  float v = ((iq & 1) == 0) ? s : c;
  if ((iq & 2) == 2) v = BT_SUB(0.0f, v);
  return v;
}
BT_HD float np_sinf(float x) { return np_sincosf(x, false); }
BT_HD float np_cosf(float x) { return np_sincosf(x, true); }

// Sigmoid exactly as the reference spells it: 1 / (1 + exp(-x))
// (ref_runtime.py:470-471), each step rounded in float32.
BT_HD float np_sigmoidf(float x) {
  return BT_DIV(1.0f, BT_ADD(1.0f, np_expf(-x)));
}

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

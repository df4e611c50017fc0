// bt_pk.h -- two-lane (float2) forms of the numpy-exact float32 math, for
// sm_100a kernels.
//
// sm_100 executes add / multiply / fused multiply-add on a pair of floats in
// one instruction (PTX add / mul / fma .rn.f32x2).  Each lane is rounded
// exactly like the scalar __fadd_rn / __fmul_rn / __fmaf_rn, so a function
// below gives, lane by lane, the same bits as its scalar original in
// bt_core.h while issuing half the arithmetic instructions.  Subtraction is
// written as addition of the negated operand, which IEEE 754 defines to be
// the same operation.
#pragma once
#include <cuda_runtime.h>
#include "bt_core.h"

namespace bt {

__device__ __forceinline__ float2 pk(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 pk(float a, float b) { return make_float2(a, b); }

// The packed operations are issued as PTX with an explicit .rn rounding
// modifier.  Even so, the compiler (CUDA 12.9, --fmad=false) fuses a packed
// multiply whose result feeds a packed add into one packed fused
// multiply-add -- one rounding instead of two, which changes results in a few
// percent of cases.  So a sum that takes a packed product as an operand goes
// through pk_add_lanes (two scalar __fadd_rn, never contracted); pk_add is
// only for operands that are not products.
__device__ __forceinline__ float2 pk_add(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// a + b lane by lane with scalar adds: for sums with a packed product as an
// operand (see above).
__device__ __forceinline__ float2 pk_add_lanes(float2 a, float2 b) {
  return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
}
__device__ __forceinline__ float2 pk_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 pk_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// div_row_fast (bt_core.h) on two lanes that share the divisor b:
// nb = (-b, -b), y2 = (RN(1/b), RN(1/b)).  Three packed operations for two
// quotients; the window rules of div_row_fast apply lane by lane.
__device__ __forceinline__ float2 pk_div_row_fast(float2 a, float2 nb, float2 y2) {
  const float2 q0 = pk_mul(a, y2);
  return pk_fma(pk_fma(nb, q0, a), y2, q0);
}

// Both lanes through the scalar function (arguments numpy does not reduce
// itself, and NaN); out of line, it is almost never taken.
template <bool COS, bool SQUARE>
__device__ __noinline__ float2 pk_sincos_big(float2 z) {
  float a = np_sincosf(z.x, COS), b = np_sincosf(z.y, COS);
  if (SQUARE) {
    a = BT_MUL(a, a);
    b = BT_MUL(b, b);
  }
  return make_float2(a, b);
}

// sin (COS false) or cos (COS true) of both lanes, np_sincosf step for step.
// With SQUARE the result is the square as numpy's Pow(., 2) computes it: the
// quadrant's sign flip cannot change a square (0 - v and v square to the
// same float, zeros included), so it is left out.  CHECKED false: the caller
// guarantees |z| <= 117435.992 (sine) or 71476.0625 (cosine) -- numpy's own
// reduction range -- for both lanes, so the out-of-range test is skipped.
template <bool COS, bool SQUARE = false, bool CHECKED = true>
__device__ __forceinline__ float2 pk_np_sincos(float2 z) {
  const float lim = COS ? 71476.0625f : 117435.992f;
  if (CHECKED && (!(fabsf(z.x) <= lim) || !(fabsf(z.y) <= lim))) return pk_sincos_big<COS, SQUARE>(z);
  const float2 t = pk_fma(z, pk(0x1.45f306p-1f), pk(12582912.0f));
  const float2 q = pk_add(t, pk(-12582912.0f));
  float2 r = pk_fma(q, pk(-0x1.921fb0p+00f), z);
  r = pk_fma(q, pk(-0x1.5110b4p-22f), r);
  r = pk_fma(q, pk(-0x1.846988p-48f), r);
  const float2 r2 = pk_mul(r, r);
  float2 c = pk_fma(pk(0x1.98e616p-16f), r2, pk(-0x1.6c06dcp-10f));
  c = pk_fma(c, r2, pk(0x1.55553cp-05f));
  c = pk_fma(c, r2, pk(-0x1.000000p-01f));
  c = pk_fma(c, r2, pk(0x1.000000p+00f));
  float2 s = pk_fma(pk(0x1.7d3bbcp-19f), r2, pk(-0x1.a06bbap-13f));
  s = pk_fma(s, r2, pk(0x1.11119ap-07f));
  s = pk_fma(s, r2, pk(-0x1.555556p-03f));
  s = pk_fma(s, r2, pk(0.0f));
  s = pk_fma(s, r, r);
  // low two bits of t = quadrant mod 4 (see np_sincosf); cosine shifts it by one
  const uint32_t qx = __float_as_uint(t.x) + (COS ? 1u : 0u), qy = __float_as_uint(t.y) + (COS ? 1u : 0u);
  float2 v = make_float2((qx & 1u) ? c.x : s.x, (qy & 1u) ? c.y : s.y);
  if (SQUARE) return pk_mul(v, v);
  if (qx & 2u) v.x = BT_SUB(0.0f, v.x);
  if (qy & 2u) v.y = BT_SUB(0.0f, v.y);
  return v;
}

// a / b of both lanes by div_nr's steps (the reciprocal approximations are
// scalar; the refinement and correction are two-lane).
__device__ __forceinline__ float2 pk_div_nr(float2 a, float2 b) {
  float2 y = make_float2(rcp_approx(b.x), rcp_approx(b.y));
  const float2 nb = pk_mul(b, pk(-1.0f));
  const float2 e = pk_fma(nb, y, pk(1.0f));
  y = pk_fma(y, e, y);
  const float2 q = pk_mul(a, y);
  const float2 r = pk_fma(nb, q, a);
  return pk_fma(r, y, q);
}

// The quotient of numpy's exp, P5(r) / Q2(r), two lanes at a time: the
// hardware reciprocal approximation of Q2 and one FMA residual correction
// of the quotient, with no Newton-Raphson step on the reciprocal.  Not a
// correctly rounded division in general; for exp's own operands (Q2 in
// [0.9, 1.1], P5 in [0.7, 1.5]) it gives the IEEE quotient on every float32
// input, which bt_selfcheck (kind 1) checks over all 2^32 of them.
__device__ __forceinline__ float2 pk_exp_quotient(float2 num, float2 den) {
  const float2 y = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  const float2 q = pk_mul(num, y);
  const float2 r = pk_fma(pk_mul(den, pk(-1.0f)), q, num);
  return pk_fma(r, y, q);
}

// Both lanes through the scalar np_expf (NaN and the saturated ranges; the
// scalar function is short, so it stays inline -- no call, no stack frame).
__device__ __forceinline__ float2 pk_exp_edge(float2 x) { return make_float2(np_expf(x.x), np_expf(x.y)); }

// exp of both lanes, np_expf step for step, for |x| < 86 in both lanes
// (others -- and NaN -- take the scalar function).  The quadrant k is read
// from the bits of t = RN(RN(x * log2e) + 1.5*2^23): t lies in [2^23, 2^24)
// with ulp 1, so bits(t) = 0x4B400000 + k, and since the low nine bits of
// 0x4B400000 are zero, bits(t) << 23 = k << 23 (mod 2^32).  On this range
// k lies in [-124, 124] and P5/Q2 in [0.7, 1.5], so pq * 2^k is normal and
// exact -- numpy's two scaling multiplies round nothing -- and it is formed
// by adding k << 23 to the bits of pq.
// A lane at or below numpy's underflow bound (-103.972..., where np_expf
// returns +0: masked softmax keys, large sigmoid arguments) stays on this
// path too, selecting +0 at the end, so a warp whose rows hold such values
// does not split between the two paths.
constexpr float kExpXmin = -103.97208404541015625f;
// the fast path proper: ux / uy mark lanes at or below kExpXmin, every other
// lane lies in (-86, 86).  A marked lane computes on its own argument
// (infinite or NaN intermediates included: no float operation traps) and
// its result is replaced by +0 at the end.
__device__ __forceinline__ float2 pk_np_exp_core(float2 x, bool ux, bool uy) {
  const float kMagic = 12582912.0f;   // 1.5 * 2^23
  // product then sum: lane by lane (two roundings, see pk_add_lanes)
  const float2 t = pk_add_lanes(pk_mul(x, pk(1.442695040888963407359924681001892137f)), pk(kMagic));
  const float2 q = pk_add(t, pk(-kMagic));
  float2 r = pk_fma(q, pk(-6.93145752e-1f), x);
  r = pk_fma(q, pk(-1.42860677e-6f), r);
  float2 num = pk_fma(pk(5.082762527590693718096e-04f), r, pk(6.757896990527504603057e-03f));
  num = pk_fma(num, r, pk(5.114512081637298353406e-02f));
  num = pk_fma(num, r, pk(2.473615434895520810817e-01f));
  num = pk_fma(num, r, pk(7.257664613233124478488e-01f));
  num = pk_fma(num, r, pk(9.999999999980870924916e-01f));
  float2 den = pk_fma(pk(2.159509375685829852307e-02f), r, pk(-2.742335390411667452936e-01f));
  den = pk_fma(den, r, pk(1.0f));
  const float2 pq = pk_exp_quotient(num, den);
  return make_float2(ux ? 0.0f : __uint_as_float(__float_as_uint(pq.x) + (__float_as_uint(t.x) << 23)),
                     uy ? 0.0f : __uint_as_float(__float_as_uint(pq.y) + (__float_as_uint(t.y) << 23)));
}
__device__ __forceinline__ float2 pk_np_exp(float2 x) {
  const bool ux = x.x <= kExpXmin, uy = x.y <= kExpXmin;
  if (!((fabsf(x.x) < 86.0f || ux) && (fabsf(x.y) < 86.0f || uy))) return pk_exp_edge(x);
  return pk_np_exp_core(x, ux, uy);
}
// pk_np_exp for arguments at most 0 or NaN (softmax's x - max).  The fast
// path takes [-41, 0] and the underflow range; a lane in between (exp from
// about 1.6e-18 down to subnormal) or NaN sends both lanes through the
// scalar function and sets `tiny`: of these exponentials only values of at
// least 2^-60 (or exact zeros) stay inside the window of the float32 row
// division (div_row_fast in bt_core.h).
__device__ __forceinline__ float2 pk_np_exp_nonpos(float2 x, bool& tiny) {
  const bool ux = x.x <= kExpXmin, uy = x.y <= kExpXmin;
  if (!((x.x >= -41.0f || ux) && (x.y >= -41.0f || uy))) {
    tiny = true;
    return pk_exp_edge(x);
  }
  return pk_np_exp_core(x, ux, uy);
}

// 1 / (1 + exp(-x)) of both lanes, np_sigmoidf step for step: the quotient
// through pk_div_nr while both denominators are below 2^120, else lane by
// lane as np_sigmoidf does.
__device__ __forceinline__ float2 pk_np_sigmoid(float2 x) {
  const float2 d = pk_add(pk(1.0f), pk_np_exp(make_float2(-x.x, -x.y)));
  if (d.x < 0x1p120f && d.y < 0x1p120f) return pk_div_nr(pk(1.0f), d);
  return make_float2(d.x < 0x1p120f ? div_nr(1.0f, d.x) : __double2float_rn(recip_d(d.x)),
                     d.y < 0x1p120f ? div_nr(1.0f, d.y) : __double2float_rn(recip_d(d.y)));
}

// sin of both lanes (see pk_np_sincos)
template <bool SQUARE, bool CHECKED = true>
__device__ __forceinline__ float2 pk_np_sin(float2 z) {
  return pk_np_sincos<false, SQUARE, CHECKED>(z);
}

}  // namespace bt

// bt_dq.h -- the per-element arithmetic of DynamicQuantizeLinear
// (tools/ref_runtime.py:106-116), shared by the quantize kernel and the
// exhaustive self-check.
//
//   scale = (hi - lo) / 255 (1 when 0), zp = clip(rint(0 - lo / scale), 0, 255)
//   y     = uint8(clip(rint(x / float32(scale)) + zp, 0, 255))
//
// x / float32(scale) is numpy's correctly rounded float32 quotient q32.
// q8_exact forms it as RN32(RN64(x * recip_d(scale))), exact by the
// midpoint-distance argument of div_by.  q8 takes a float32 shortcut for
// the common case and falls back to q8_exact near the only places where the
// shortcut could differ:
//
//   q0 = RN32(x * r), r = RN32(1 / scale).  |r - 1/s| <= 2^-24 / s, so the
//   exact product is within |q| 2^-24 < ulp(q) of q = x / s, and its rounding
//   adds at most another ulp(q): |q0 - q| < 2 ulp(q).  q32 is within half an
//   ulp of q, so |q32 - q0| < 2.5 ulp(q) <= 2.5 * 2^-15 whenever |q| < 512.
//   rint is constant between consecutive half-integers, hence when q0 is
//   finite, |q0| < 256 and q0 lies more than 2^-13 from every half-integer,
//   rint(q32) = rint(q0).  Everything else (ties and near-ties, NaN,
//   infinities, a reciprocal that overflows) takes q8_exact.
//
// The distance test: k = rint(q0), d = |q0 - k| (exact by Sterbenz's lemma,
// or because k = 0), and the distance to the nearest half-integer is
// |0.5 - d| (exact for d >= 0.25; for d < 0.25 it is above 0.25 either way).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "bt_core.h"

namespace bt {

struct DqParams {
  float scale32;   // float32(scale): the divisor of the element quotients
  float zp;        // zero point, integral in [0, 255]
  float r32;       // RN32(1 / scale32): the shortcut's multiplier
  double rscale;   // recip_d(scale32): the exact path's multiplier
};

// Order-preserving map of non-NaN floats to unsigned integers (the range
// record: [0] = ~ord(min) and [1] = ord(max) by atomicMax, [2] = NaN seen).
__device__ __forceinline__ uint32_t dq_ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float dq_from_ord(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// atomicMax into a range-record word, skipped when the word already holds
// at least v: the words only grow, so the result is the same, and most of a
// large grid's CTAs then issue no atomic on the two contended addresses.
__device__ __forceinline__ void dq_raise(uint32_t* w, uint32_t v) {
  if (v > *(volatile const uint32_t*)w) atomicMax(w, v);
}

__device__ __forceinline__ DqParams dq_params_from(double scale, double z) {
  DqParams p;
  p.scale32 = __double2float_rn(scale);
  p.zp = (float)z;
  p.r32 = __frcp_rn(p.scale32);
  p.rscale = recip_d(p.scale32);
  return p;
}

// scale and zero point from the range record (every CTA, identically)
__device__ __forceinline__ DqParams dq_params(const uint32_t* rec, int64_t n) {
  double lo = 0.0, hi = 0.0;
  if (rec[2] == 0u && n > 0) {
    const float m = dq_from_ord(~rec[0]), M = dq_from_ord(rec[1]);
    if (m < 0.0f) lo = (double)m;     // min(0.0, float(m)) keeps 0.0 unless m < 0
    if (M > 0.0f) hi = (double)M;     // max(0.0, float(M)) keeps 0.0 unless M > 0
  }
  double scale = __ddiv_rn(__dsub_rn(hi, lo), 255.0);
  if (scale == 0.0) scale = 1.0;
  double z = rint(__dsub_rn(0.0, __ddiv_rn(lo, scale)));
  z = z != z ? 0.0 : fmin(fmax(z, 0.0), 255.0);
  return dq_params_from(scale, z);
}

// + zp (exact for |v| < 2^24; beyond that either way saturates), clip, NaN -> 0
__device__ __forceinline__ uint32_t dq_clip(float k, const DqParams& p) {
  const float v = BT_ADD(k, p.zp);
  if (!(v > 0.0f)) return 0u;
  return v >= 255.0f ? 255u : (uint32_t)v;
}

__device__ __forceinline__ uint32_t q8_exact(float x, const DqParams& p) {
  return dq_clip(rintf(div_by(x, p.rscale)), p);
}

__device__ __forceinline__ uint32_t q8(float x, const DqParams& p) {
  const float q0 = BT_MUL(x, p.r32);
  const float k = rintf(q0);
  const float d = fabsf(BT_SUB(q0, k));
  if (fabsf(q0) < 256.0f && fabsf(BT_SUB(0.5f, d)) > 0x1p-13f) return dq_clip(k, p);
  return q8_exact(x, p);
}

}  // namespace bt

// bt_ewmath.h -- per-element device helpers shared by the elementwise engine
// (bt_ew.cu) and the fused chains (bt_chain.cu): loads and stores with
// numpy's conversion semantics, and the float32 op table (each op rounds
// once, numpy's own algorithms for the transcendentals, see bt_core.h).
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>
#include "bt_ops.h"
#include "bt_core.h"

namespace bt {
namespace {

// ---- element load / store with numpy conversion semantics ----------------
template <class CT>
__device__ __forceinline__ CT ld1(const void* p, int dt, int64_t i) {
  switch (dt) {
    case BT_F32: return (CT)__ldg((const float*)p + i);
    case BT_F16: return (CT)__half2float(__ldg((const __half*)p + i));
    case BT_F64: return (CT)__ldg((const double*)p + i);
    case BT_I8: return (CT)(signed char)__ldg((const char*)p + i);
    case BT_U8: return (CT)__ldg((const unsigned char*)p + i);
    case BT_BOOL: return (CT)(__ldg((const unsigned char*)p + i) != 0);
    case BT_I16: return (CT)__ldg((const short*)p + i);
    case BT_U16: return (CT)__ldg((const unsigned short*)p + i);
    case BT_I32: return (CT)__ldg((const int*)p + i);
    case BT_U32: return (CT)__ldg((const unsigned int*)p + i);
    case BT_I64: return (CT)__ldg((const long long*)p + i);
    case BT_U64: return (CT)__ldg((const unsigned long long*)p + i);
  }
  return CT(0);
}

// Float to integer conversion as numpy's C casts compile on x86-64:
// truncation toward zero through a 32-bit (or, for uint32 / int64 / uint64,
// a 64-bit) cvtt, whose out-of-range and NaN result is the "integer
// indefinite" INT_MIN; narrower targets keep the low bits.
__device__ __forceinline__ int32_t cvtt32(double v) {
  if (!(v > -2147483649.0 && v < 2147483648.0)) return INT32_MIN;
  return (int32_t)v;
}
__device__ __forceinline__ int64_t cvtt64(double v) {
  if (!(v > -9223372036854775808.0 && v < 9223372036854775808.0)) return INT64_MIN;
  return (int64_t)v;
}
__device__ __forceinline__ uint64_t cvtt_u64(double v) {
  if (v < 9223372036854775808.0) return (uint64_t)cvtt64(v);
  return (uint64_t)cvtt64(v - 9223372036854775808.0) ^ 0x8000000000000000ull;
}

template <class CT>
__device__ __forceinline__ void st1(void* p, int dt, int64_t i, CT v) {
  constexpr bool kFloat = (CT(0.5) != CT(0));
  switch (dt) {
    case BT_F32: ((float*)p)[i] = (float)v; return;
    case BT_F64: ((double*)p)[i] = (double)v; return;
    case BT_F16: ((__half*)p)[i] = __double2half((double)v); return;
    case BT_BOOL: ((unsigned char*)p)[i] = (v != CT(0)) ? 1 : 0; return;
    default: break;
  }
  if (kFloat) {
    double d = (double)v;
    switch (dt) {
      case BT_I8: ((int8_t*)p)[i] = (int8_t)cvtt32(d); return;
      case BT_U8: ((uint8_t*)p)[i] = (uint8_t)cvtt32(d); return;
      case BT_I16: ((int16_t*)p)[i] = (int16_t)cvtt32(d); return;
      case BT_U16: ((uint16_t*)p)[i] = (uint16_t)cvtt32(d); return;
      case BT_I32: ((int32_t*)p)[i] = cvtt32(d); return;
      case BT_U32: ((uint32_t*)p)[i] = (uint32_t)cvtt64(d); return;
      case BT_I64: ((int64_t*)p)[i] = cvtt64(d); return;
      case BT_U64: ((uint64_t*)p)[i] = cvtt_u64(d); return;
    }
  } else {
    long long w = (long long)v;
    switch (dt) {
      case BT_I8: ((int8_t*)p)[i] = (int8_t)w; return;
      case BT_U8: ((uint8_t*)p)[i] = (uint8_t)w; return;
      case BT_I16: ((int16_t*)p)[i] = (int16_t)w; return;
      case BT_U16: ((uint16_t*)p)[i] = (uint16_t)w; return;
      case BT_I32: ((int32_t*)p)[i] = (int32_t)w; return;
      case BT_U32: ((uint32_t*)p)[i] = (uint32_t)w; return;
      case BT_I64: ((int64_t*)p)[i] = (int64_t)w; return;
      case BT_U64: ((uint64_t*)p)[i] = (uint64_t)w; return;
    }
  }
}

// ---- numpy op semantics per compute type ----------------------------------
// np.maximum / np.minimum: NaN propagates; for equal operands (including
// +0 / -0) the second operand is returned.
template <class T>
__device__ __forceinline__ T np_max(T a, T b) { return (a != a) ? a : ((b != b) ? b : (a > b ? a : b)); }
template <class T>
__device__ __forceinline__ T np_min(T a, T b) { return (a != a) ? a : ((b != b) ? b : (a < b ? a : b)); }

__device__ __forceinline__ float np_powf(float a, float b) {
  if (b == 2.0f) return BT_MUL(a, a);   // numpy's power for exponent 2 is x*x
  return (float)pow((double)a, (double)b);
}

// tanh form of GELU in the reference's evaluation order
// 0.5*x*(1.0 + tanh(k*(x + 0.044715*x*x*x))) (ref_runtime.py:288-293).
__device__ __forceinline__ float np_fast_gelu(float x) {
  const float k = 0.7978845608028654f;
  float a = BT_MUL(0.5f, x);
  float c = BT_MUL(BT_MUL(BT_MUL(0.044715f, x), x), x);
  float f = BT_MUL(k, BT_ADD(x, c));
  float g = (float)tanh((double)f);
  return BT_MUL(a, BT_ADD(1.0f, g));
}

// TRIG false: sine and cosine never reach this call (the vector kernels run
// them in their own specialisations), so their out-of-line fallback is not
// linked into the runtime-op kernels.
template <bool TRIG = true>
__device__ __forceinline__ float apply_f32(int op, float a, float b, float c, float alpha, int n_in) {
  switch (op) {
    case BT_OP_ADD: return BT_ADD(a, b);
    case BT_OP_SUB: return BT_SUB(a, b);
    case BT_OP_MUL: return BT_MUL(a, b);
    case BT_OP_DIV: return BT_DIV(a, b);
    case BT_OP_POW: return np_powf(a, b);
    case BT_OP_SQRT: return BT_SQRT(a);
    case BT_OP_EXP: return np_expf(a);
    case BT_OP_SIN: return TRIG ? np_sinf(a) : a;
    case BT_OP_COS: return TRIG ? np_cosf(a) : a;
    case BT_OP_ATAN: return (float)atan((double)a);
    case BT_OP_TANH: return tanh_f(a);
    case BT_OP_SIGMOID: return np_sigmoidf(a);
    case BT_OP_FLOOR: return floorf(a);
    case BT_OP_ROUND: return rintf(a);
    case BT_OP_LEAKYRELU: return a < 0.0f ? BT_MUL(a, alpha) : a;
    case BT_OP_CLIP: return np_min(np_max(a, b), c);
    case BT_OP_EQUAL: return a == b ? 1.0f : 0.0f;
    case BT_OP_GREATER: return a > b ? 1.0f : 0.0f;
    case BT_OP_LESS: return a < b ? 1.0f : 0.0f;
    case BT_OP_GEQ: return a >= b ? 1.0f : 0.0f;
    case BT_OP_NEG: return -a;
    case BT_OP_ABS: return fabsf(a);
    case BT_OP_LOG: return (float)log((double)a);
    case BT_OP_MIN: return np_min(a, b);
    case BT_OP_MAX: return np_max(a, b);
    case BT_OP_ERF: return (float)erf((double)a);
    case BT_OP_GELU: return np_fast_gelu(n_in > 1 ? BT_ADD(a, b) : a);
    case BT_OP_DEQUANT: return BT_MUL(n_in > 2 ? BT_SUB(a, c) : a, b);
    default: return a;  // CAST_INT / CAST_BOOL / IDENTITY: conversion only
  }
}

}  // namespace
}  // namespace bt

// bt_ew.cu -- broadcast elementwise engine for sm_100a.
//
// One call = one numpy ufunc application (tools/ref_runtime.py:446-503,
// :572-578, :610-611, :631-636).  The host planner (bt_host.cpp) broadcasts
// every operand view to the output shape and merges contiguous axes; the
// launcher then picks one of three kernels:
//   flat  -- one axis, every operand contiguous (stride 1) or a scalar
//            (stride 0): 4-element vector loads/stores (128-bit for fp32),
//            grid-stride over SM-count-multiple grids;
//   rows  -- two axes [R, T] with unit or zero inner strides (per-row scale,
//            per-column bias, full tensors): vectorised along T when every
//            row start is 16-byte aligned;
//   nd    -- any rank up to 8, coordinates unravelled per element.
// Every path rounds each op once in its compute type (no contraction; the
// float32 transcendentals are numpy's own algorithms, see bt_core.h).
#include <cuda_fp16.h>
#include <stdint.h>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"
#include "bt_pk.h"
#include "bt_ewmath.h"

namespace bt {
namespace {

struct Operand {
  const void* p;
  int32_t dt;
  int32_t pad;
  int64_t st[BT_MAX_RANK];
};

struct EwArgs {
  int32_t op, n_in, rank, cdt;
  float alpha;
  int32_t odt;
  int64_t n;
  int64_t shape[BT_MAX_RANK];
  Operand in[3];
  void* out;
  int64_t ost[BT_MAX_RANK];
};

__device__ __forceinline__ double apply_f64(int op, double a, double b, double c, float alpha, int n_in) {
  switch (op) {
    case BT_OP_ADD: return __dadd_rn(a, b);
    case BT_OP_SUB: return __dsub_rn(a, b);
    case BT_OP_MUL: return __dmul_rn(a, b);
    case BT_OP_DIV: return __ddiv_rn(a, b);
    case BT_OP_POW: return b == 2.0 ? __dmul_rn(a, a) : pow(a, b);
    case BT_OP_SQRT: return __dsqrt_rn(a);
    case BT_OP_EXP: return exp(a);
    case BT_OP_SIN: return bt_sincos_d(a, false);
    case BT_OP_COS: return bt_sincos_d(a, true);
    case BT_OP_ATAN: return atan(a);
    case BT_OP_TANH: return tanh(a);
    case BT_OP_SIGMOID: return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-a)));
    case BT_OP_FLOOR: return floor(a);
    case BT_OP_ROUND: return rint(a);
    case BT_OP_LEAKYRELU: return a < 0.0 ? __dmul_rn(a, (double)alpha) : a;
    case BT_OP_CLIP: return np_min(np_max(a, b), c);
    case BT_OP_EQUAL: return a == b ? 1.0 : 0.0;
    case BT_OP_GREATER: return a > b ? 1.0 : 0.0;
    case BT_OP_LESS: return a < b ? 1.0 : 0.0;
    case BT_OP_GEQ: return a >= b ? 1.0 : 0.0;
    case BT_OP_NEG: return -a;
    case BT_OP_ABS: return fabs(a);
    case BT_OP_LOG: return log(a);
    case BT_OP_MIN: return np_min(a, b);
    case BT_OP_MAX: return np_max(a, b);
    case BT_OP_ERF: return erf(a);
    default: return a;
  }
}

__device__ __forceinline__ long long floor_div_i64(long long a, long long b) {
  if (b == 0) return 0;                               // numpy: 0 (and a warning)
  if (a == INT64_MIN && b == -1) return INT64_MIN;    // numpy: overflow -> MIN
  long long q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) q -= 1;
  return q;
}

__device__ __forceinline__ long long apply_i64(int op, long long a, long long b, long long c, float, int) {
  switch (op) {
    case BT_OP_ADD: return (long long)((unsigned long long)a + (unsigned long long)b);
    case BT_OP_SUB: return (long long)((unsigned long long)a - (unsigned long long)b);
    case BT_OP_MUL: return (long long)((unsigned long long)a * (unsigned long long)b);
    case BT_OP_DIV: return floor_div_i64(a, b);
    case BT_OP_CLIP: return a < b ? b : (a > c ? c : a);
    case BT_OP_EQUAL: return a == b;
    case BT_OP_GREATER: return a > b;
    case BT_OP_LESS: return a < b;
    case BT_OP_GEQ: return a >= b;
    case BT_OP_NEG: return (long long)(0ull - (unsigned long long)a);
    case BT_OP_ABS: return a < 0 ? (long long)(0ull - (unsigned long long)a) : a;
    case BT_OP_MIN: return a < b ? a : b;
    case BT_OP_MAX: return a > b ? a : b;
    default: return a;
  }
}

template <class CT> struct Apply;
template <> struct Apply<float> {
  static __device__ __forceinline__ float f(int op, float a, float b, float c, float al, int n) { return apply_f32(op, a, b, c, al, n); }
};
template <> struct Apply<double> {
  static __device__ __forceinline__ double f(int op, double a, double b, double c, float al, int n) { return apply_f64(op, a, b, c, al, n); }
};
template <> struct Apply<long long> {
  static __device__ __forceinline__ long long f(int op, long long a, long long b, long long c, float al, int n) { return apply_i64(op, a, b, c, al, n); }
};

// One output element given the operands' element offsets.
template <class CT>
__device__ __forceinline__ void ew_element(const EwArgs& a, const int64_t* off, int64_t oo) {
  if (a.op == BT_OP_WHERE) {
    bool cond = ld1<double>(a.in[0].p, a.in[0].dt, off[0]) != 0.0;
    int k = cond ? 1 : 2;
    st1<CT>(a.out, a.odt, oo, ld1<CT>(a.in[k].p, a.in[k].dt, off[k]));
    return;
  }
  if (a.op == BT_OP_AND) {
    bool r = ld1<double>(a.in[0].p, a.in[0].dt, off[0]) != 0.0 &&
             ld1<double>(a.in[1].p, a.in[1].dt, off[1]) != 0.0;
    st1<CT>(a.out, a.odt, oo, r ? CT(1) : CT(0));
    return;
  }
  CT x = ld1<CT>(a.in[0].p, a.in[0].dt, off[0]);
  CT y = a.n_in > 1 ? ld1<CT>(a.in[1].p, a.in[1].dt, off[1]) : CT(0);
  CT z = a.n_in > 2 ? ld1<CT>(a.in[2].p, a.in[2].dt, off[2]) : CT(0);
  st1<CT>(a.out, a.odt, oo, Apply<CT>::f(a.op, x, y, z, a.alpha, a.n_in));
}

// ---- kernels ------------------------------------------------------------------
template <class CT>
__global__ void __launch_bounds__(256) ew_nd_kernel(EwArgs a) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    int64_t rem = i, off[3] = {0, 0, 0}, oo = 0;
    for (int d = a.rank - 1; d >= 0; --d) {
      int64_t ext = a.shape[d];
      int64_t c = rem % ext;
      rem /= ext;
      for (int k = 0; k < 3; ++k) off[k] += c * a.in[k].st[d];
      oo += c * a.ost[d];
    }
    ew_element<CT>(a, off, oo);
  }
}

// Flat (rank 1) float32 path: every input is a scalar or a unit-stride run,
// the output is a unit-stride run.  VEC = 4 when every unit-stride operand
// starts on a 4-element boundary of its own type.
// Loads VEC consecutive elements of operand o starting at element `base`
// (VEC = 4: one 128-bit fp32, 64-bit fp16 or 32-bit int8 load).
template <int VEC>
__device__ __forceinline__ void ld_vec(const Operand& o, int64_t base, float* x) {
  if (o.st[0] == 0) {
    const float s = ld1<float>(o.p, o.dt, 0);
#pragma unroll
    for (int j = 0; j < VEC; ++j) x[j] = s;
  } else if (VEC == 4 && o.dt == BT_F32) {
    const float4 f = __ldcs((const float4*)((const float*)o.p + base));
    x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
  } else if (VEC == 4 && o.dt == BT_F16) {
    uint2 u = __ldcs((const uint2*)((const __half*)o.p + base));
    __half2 h0 = *reinterpret_cast<__half2*>(&u.x), h1 = *reinterpret_cast<__half2*>(&u.y);
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    x[0] = f0.x; x[1] = f0.y; x[2] = f1.x; x[3] = f1.y;
  } else if (VEC == 4 && o.dt == BT_I8) {
    const int w = __ldcs((const int*)((const signed char*)o.p + base));
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = (float)(signed char)(w >> (8 * j));
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) x[j] = ld1<float>(o.p, o.dt, base + j);
  }
}

// OP >= 0: the op is fixed at compile time (the switch in apply_f32 folds
// away); OP < 0: the op is read from the arguments.
template <int OP, bool TRIG = true>
__device__ __forceinline__ float apply_op(const EwArgs& a, float x, float y, float z) {
  return apply_f32<TRIG>(OP >= 0 ? OP : a.op, x, y, z, a.alpha, a.n_in);
}

// Four results of one vector (operands k = 0..2, elements j = 0..3).  Sine,
// cosine, exp and sigmoid run two elements per instruction (bt_pk.h); every
// other op goes element by element.
template <int OP>
__device__ __forceinline__ float4 apply_vec4(const EwArgs& a, float4 x, float4 y, float4 z) {
  if (OP == BT_OP_SIN || OP == BT_OP_COS) {
    const float2 lo = pk_np_sincos<OP == BT_OP_COS>(make_float2(x.x, x.y));
    const float2 hi = pk_np_sincos<OP == BT_OP_COS>(make_float2(x.z, x.w));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  if (OP == BT_OP_EXP) {
    const float2 lo = pk_np_exp(make_float2(x.x, x.y)), hi = pk_np_exp(make_float2(x.z, x.w));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  if (OP == BT_OP_SIGMOID) {
    const float2 lo = pk_np_sigmoid(make_float2(x.x, x.y)), hi = pk_np_sigmoid(make_float2(x.z, x.w));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  return make_float4(apply_op<OP>(a, x.x, y.x, z.x), apply_op<OP>(a, x.y, y.y, z.y), apply_op<OP>(a, x.z, y.z, z.z),
                     apply_op<OP>(a, x.w, y.w, z.w));
}
__device__ __forceinline__ float4 f4(const float (&v)[4]) { return make_float4(v[0], v[1], v[2], v[3]); }

template <int VEC>
__global__ void __launch_bounds__(256) ew_flat_kernel(EwArgs a) {
  const int64_t nv = a.n / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // U vectors per thread per iteration, all loads issued before the math.
  constexpr int U = 2;
  for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v0 < nv; v0 += U * stride) {
    float x[U][3][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * stride;
      if (v < nv) {
#pragma unroll
        for (int k = 0; k < 3; ++k)
          if (k < a.n_in) ld_vec<VEC>(a.in[k], v * VEC, x[u][k]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * stride;
      if (v >= nv) break;
      const int64_t base = v * VEC;
      float r[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        r[j] = apply_f32(a.op, x[u][0][j], a.n_in > 1 ? x[u][1][j] : 0.f, a.n_in > 2 ? x[u][2][j] : 0.f, a.alpha,
                         a.n_in);
      if (VEC == 4 && a.odt == BT_F32) {
        __stcs((float4*)((float*)a.out + base), make_float4(r[0], r[1], r[2], r[3]));
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) st1<float>(a.out, a.odt, base + j, r[j]);
      }
    }
  }
  // tail
  const int64_t t0 = nv * VEC;
  const int64_t i = t0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < a.n) {
    int64_t off[3];
    for (int k = 0; k < 3; ++k) off[k] = i * a.in[k].st[0];
    float x0 = ld1<float>(a.in[0].p, a.in[0].dt, off[0]);
    float x1 = a.n_in > 1 ? ld1<float>(a.in[1].p, a.in[1].dt, off[1]) : 0.f;
    float x2 = a.n_in > 2 ? ld1<float>(a.in[2].p, a.in[2].dt, off[2]) : 0.f;
    st1<float>(a.out, a.odt, i, apply_f32(a.op, x0, x1, x2, a.alpha, a.n_in));
  }
}

// The same with the op fixed at compile time (OP >= 0, VEC = 4).  (Tanh
// declares a minimum of one CTA per SM: ptxas then keeps its double
// evaluation in registers; without a minimum it chose fewer and spilled.)
template <int VEC, int OP>
__global__ void __launch_bounds__(256, OP == BT_OP_TANH ? 1 : 0) ew_flat_op_kernel(EwArgs a) {
  constexpr bool kTrig = !(VEC == 4 && OP < 0);   // see apply_f32
  const int64_t nv = a.n / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // U vectors per thread per iteration, all loads issued before the math:
  // four for sin, cos and LeakyRelu, two for the rest (measured per op on
  // the 256 MB sweep), one for Div, where a call to an out-of-line path
  // would otherwise need a stack frame.
  constexpr int U = OP == BT_OP_DIV ? 1 : (OP == BT_OP_SIN || OP == BT_OP_COS || OP == BT_OP_LEAKYRELU) ? 4 : 2;
  for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v0 < nv; v0 += U * stride) {
    float x[U][3][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * stride;
      if (v < nv) {
#pragma unroll
        for (int k = 0; k < 3; ++k)
          if (k < a.n_in) ld_vec<VEC>(a.in[k], v * VEC, x[u][k]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * stride;
      if (v >= nv) break;
      const int64_t base = v * VEC;
      float r[VEC];
      if constexpr (VEC == 4 && OP >= 0) {
        const float4 v4 = apply_vec4<OP>(a, f4(x[u][0]), a.n_in > 1 ? f4(x[u][1]) : make_float4(0.f, 0.f, 0.f, 0.f),
                                         a.n_in > 2 ? f4(x[u][2]) : make_float4(0.f, 0.f, 0.f, 0.f));
        r[0] = v4.x; r[1] = v4.y; r[2] = v4.z; r[3] = v4.w;
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          r[j] = apply_op<OP, kTrig>(a, x[u][0][j], a.n_in > 1 ? x[u][1][j] : 0.f, a.n_in > 2 ? x[u][2][j] : 0.f);
      }
      if (VEC == 4 && a.odt == BT_F32) {
        __stcs((float4*)((float*)a.out + base), make_float4(r[0], r[1], r[2], r[3]));
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) st1<float>(a.out, a.odt, base + j, r[j]);
      }
    }
  }
  // tail
  const int64_t t0 = nv * VEC;
  const int64_t i = t0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < a.n) {
    int64_t off[3];
    for (int k = 0; k < 3; ++k) off[k] = i * a.in[k].st[0];
    float x0 = ld1<float>(a.in[0].p, a.in[0].dt, off[0]);
    float x1 = a.n_in > 1 ? ld1<float>(a.in[1].p, a.in[1].dt, off[1]) : 0.f;
    float x2 = a.n_in > 2 ? ld1<float>(a.in[2].p, a.in[2].dt, off[2]) : 0.f;
    st1<float>(a.out, a.odt, i, apply_op<OP, kTrig>(a, x0, x1, x2));
  }
}

// [R, T] float32 path: operand k's element (r, t) is at r*st0 + t*st1 with
// st1 in {0, 1}; the output is contiguous.  blockIdx.y walks rows.
template <int VEC>
__global__ void __launch_bounds__(256) ew_rows_kernel(EwArgs a) {
  const int64_t R = a.shape[0], T = a.shape[1];
  const int64_t nv = T / VEC;
  for (int64_t r = blockIdx.y; r < R; r += gridDim.y) {
    float rowv[3];
#pragma unroll
    for (int k = 0; k < 3; ++k)
      if (k < a.n_in && a.in[k].st[1] == 0) rowv[k] = ld1<float>(a.in[k].p, a.in[k].dt, r * a.in[k].st[0]);
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = v * VEC;
      float x[3][VEC];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        if (k >= a.n_in) break;
        const Operand& o = a.in[k];
        if (o.st[1] == 0) {
#pragma unroll
          for (int j = 0; j < VEC; ++j) x[k][j] = rowv[k];
        } else if (VEC == 4 && o.dt == BT_F32) {
          float4 f = (o.st[0] == 0) ? __ldg((const float4*)((const float*)o.p + t))
                                    : __ldcs((const float4*)((const float*)o.p + r * o.st[0] + t));
          x[k][0] = f.x; x[k][1] = f.y; x[k][2] = f.z; x[k][3] = f.w;
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) x[k][j] = ld1<float>(o.p, o.dt, r * o.st[0] + t + j);
        }
      }
      float res[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        res[j] = apply_f32(a.op, x[0][j], a.n_in > 1 ? x[1][j] : 0.f, a.n_in > 2 ? x[2][j] : 0.f, a.alpha, a.n_in);
      const int64_t ob = r * a.ost[0] + t;
      if (VEC == 4 && a.odt == BT_F32) {
        __stcs((float4*)((float*)a.out + ob), make_float4(res[0], res[1], res[2], res[3]));
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) st1<float>(a.out, a.odt, ob + j, res[j]);
      }
    }
    // tail of the row
    for (int64_t t = nv * VEC + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T;
         t += (int64_t)gridDim.x * blockDim.x) {
      float x[3] = {0.f, 0.f, 0.f};
      for (int k = 0; k < a.n_in; ++k) x[k] = ld1<float>(a.in[k].p, a.in[k].dt, r * a.in[k].st[0] + t * a.in[k].st[1]);
      st1<float>(a.out, a.odt, r * a.ost[0] + t, apply_f32(a.op, x[0], x[1], x[2], a.alpha, a.n_in));
    }
  }
}

// Inputs of an op with its own compiled kernel: two for the arithmetic
// binaries, one for the rest.
template <int OP>
__host__ __device__ constexpr int fixed_n_in() {
  return (OP == BT_OP_ADD || OP == BT_OP_SUB || OP == BT_OP_MUL || OP == BT_OP_DIV || OP == BT_OP_POW) ? 2 : 1;
}
// Vectors each thread of ew_rows_op_kernel loads before it computes (one
// where a call to an out-of-line path would otherwise need a stack frame;
// Div keeps four: by a row-constant divisor it multiplies by the divisor's
// double reciprocal, and its per-element quotient fits the registers).
template <int OP>
__host__ __device__ constexpr int rows_unroll() {
  return (OP == BT_OP_SIGMOID || OP == BT_OP_GELU || OP == BT_OP_POW) ? 1 : 4;
}

// The same with the op fixed at compile time (OP >= 0, VEC = 4): each thread
// issues the loads of U vectors of a row, then computes and stores them.
template <int VEC, int OP>
__global__ void __launch_bounds__(256) ew_rows_op_kernel(EwArgs a) {
  constexpr bool kTrig = !(VEC == 4 && OP < 0);   // see apply_f32
  constexpr int NIN = fixed_n_in<OP>();
  constexpr int U = rows_unroll<OP>();
  const int64_t R = a.shape[0], T = a.shape[1];
  const int64_t nv = T / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = blockIdx.y; r < R; r += gridDim.y) {
    float rowv[NIN];
#pragma unroll
    for (int k = 0; k < NIN; ++k)
      if (a.in[k].st[1] == 0) rowv[k] = ld1<float>(a.in[k].p, a.in[k].dt, r * a.in[k].st[0]);
    // Div by a divisor constant along the row: its double reciprocal, once
    const bool row_div = OP == BT_OP_DIV && a.in[NIN - 1].st[1] == 0;
    const double rdiv = row_div ? recip_d(rowv[NIN - 1]) : 0.0;
    for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v0 < nv; v0 += U * stride) {
      float x[U][NIN][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t t = (v0 + u * stride) * VEC;
        if (v0 + u * stride >= nv) break;
#pragma unroll
        for (int k = 0; k < NIN; ++k) {
          const Operand& o = a.in[k];
          if (o.st[1] == 0) {
#pragma unroll
            for (int j = 0; j < VEC; ++j) x[u][k][j] = rowv[k];
          } else if (VEC == 4 && o.dt == BT_F32) {
            float4 f = (o.st[0] == 0) ? __ldg((const float4*)((const float*)o.p + t))
                                      : __ldcs((const float4*)((const float*)o.p + r * o.st[0] + t));
            x[u][k][0] = f.x; x[u][k][1] = f.y; x[u][k][2] = f.z; x[u][k][3] = f.w;
          } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) x[u][k][j] = ld1<float>(o.p, o.dt, r * o.st[0] + t + j);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t t = (v0 + u * stride) * VEC;
        if (v0 + u * stride >= nv) break;
        float res[VEC];
        if constexpr (OP == BT_OP_DIV) {
          if (row_div) {
            // the row's divisor is one float: RN32(RN64(x * r)) with r within
            // a double ulp of 1 / b is RN32(x / b) for every float x, b
#pragma unroll
            for (int j = 0; j < VEC; ++j) res[j] = div_by(x[u][0][j], rdiv);
          } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) res[j] = BT_DIV(x[u][0][j], x[u][1][j]);
          }
        } else if constexpr (VEC == 4 && OP >= 0) {
          const float4 v4 = apply_vec4<OP>(a, f4(x[u][0]), NIN > 1 ? f4(x[u][NIN - 1]) : make_float4(0.f, 0.f, 0.f, 0.f),
                                           make_float4(0.f, 0.f, 0.f, 0.f));
          res[0] = v4.x; res[1] = v4.y; res[2] = v4.z; res[3] = v4.w;
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) res[j] = apply_op<OP, kTrig>(a, x[u][0][j], NIN > 1 ? x[u][NIN - 1][j] : 0.f, 0.f);
        }
        const int64_t ob = r * a.ost[0] + t;
        if (VEC == 4 && a.odt == BT_F32) {
          __stcs((float4*)((float*)a.out + ob), make_float4(res[0], res[1], res[2], res[3]));
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) st1<float>(a.out, a.odt, ob + j, res[j]);
        }
      }
    }
    // tail of the row
    for (int64_t t = nv * VEC + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T; t += stride) {
      float x[3] = {0.f, 0.f, 0.f};
      for (int k = 0; k < NIN; ++k) x[k] = ld1<float>(a.in[k].p, a.in[k].dt, r * a.in[k].st[0] + t * a.in[k].st[1]);
      st1<float>(a.out, a.odt, r * a.ost[0] + t, apply_op<OP, kTrig>(a, x[0], x[1], x[2]));
    }
  }
}

// Batched two-dimensional transpose, for IDENTITY copies between equal
// dtypes whose collapsed form is out[b][m][n] (contiguous) =
// in[b * sb + m + n * sn]: the input runs along m, the output along n.
// 32 x 32 tiles pass through shared memory (one padding column against bank
// conflicts), so both the reads (along m) and the writes (along n) are
// coalesced; a strided element-by-element copy would fetch a 32-byte sector
// for every 4-byte read.  W is the element's byte width; bits are copied.
// The grid walks batches (z), pairs of m tiles (y) and n tiles (x) by
// increments, so no thread divides to find its tile; the two tiles of a pair
// are read before either is written.  VEC (4-byte elements, 16-byte aligned
// rows and strides): each thread reads four consecutive m of one column as
// one 128-bit load and writes four consecutive n of one row as one 128-bit
// store; the tile's column (4q + j of row n) and row (4p + i, column m)
// accesses both land on 32 distinct banks.
template <typename W, bool VEC>
__global__ void __launch_bounds__(256) transpose_kernel(const W* in, W* out, int64_t B, int M, int N, int64_t sb,
                                                        int64_t sn) {
  __shared__ W tile[2][32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8 threads
  const int hi = threadIdx.x >> 3, lo = threadIdx.x & 7;    // 32 x 8 threads, 4 values each (VEC)
  // one tile (m0, n0) through tile buffer u, any shape, bounds-checked
  auto one_tile = [&](const W* src, W* dst, int mr, int nr, int u) {
#pragma unroll
    for (int k = ty; k < 32; k += 8)
      if (tx < mr && k < nr) tile[u][k][tx] = src[tx + k * sn];
    __syncthreads();
#pragma unroll
    for (int k = ty; k < 32; k += 8)
      if (k < mr && tx < nr) dst[(int64_t)k * N + tx] = tile[u][tx][k];
  };
  for (int64_t b = blockIdx.z; b < B; b += gridDim.z)
    for (int m0 = blockIdx.y * 64; m0 < M; m0 += gridDim.y * 64)
      for (int n0 = blockIdx.x * 32; n0 < N; n0 += gridDim.x * 32) {
        const W* src = in + b * sb + m0 + (int64_t)n0 * sn;                 // element (m0, n0) of batch b
        W* dst = out + b * (int64_t)M * N + (int64_t)m0 * N + n0;          // element (m0, n0) of the output
        const int nr = N - n0 < 32 ? N - n0 : 32;
        if (VEC && m0 + 64 <= M && nr == 32) {
          // two full tiles, (m0, n0) and (m0 + 32, n0): both 128-bit loads
          // in flight before either tile is stored
          const uint4 v0 = __ldcs(reinterpret_cast<const uint4*>(src + (int64_t)hi * sn + 4 * lo));
          const uint4 v1 = __ldcs(reinterpret_cast<const uint4*>(src + 32 + (int64_t)hi * sn + 4 * lo));
          tile[0][hi][4 * lo] = v0.x;
          tile[0][hi][4 * lo + 1] = v0.y;
          tile[0][hi][4 * lo + 2] = v0.z;
          tile[0][hi][4 * lo + 3] = v0.w;
          tile[1][hi][4 * lo] = v1.x;
          tile[1][hi][4 * lo + 1] = v1.y;
          tile[1][hi][4 * lo + 2] = v1.z;
          tile[1][hi][4 * lo + 3] = v1.w;
          __syncthreads();
#pragma unroll
          for (int u = 0; u < 2; ++u)
            __stcs(reinterpret_cast<uint4*>(dst + (int64_t)(32 * u + hi) * N + 4 * lo),
                   make_uint4(tile[u][4 * lo][hi], tile[u][4 * lo + 1][hi], tile[u][4 * lo + 2][hi],
                              tile[u][4 * lo + 3][hi]));
        } else if (!VEC && m0 + 64 <= M && nr == 32) {
          // two full tiles, no bounds checks
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const W* s0 = src + 32 * u + tx + ty * sn;
#pragma unroll
            for (int k = 0; k < 32; k += 8) tile[u][ty + k][tx] = s0[k * sn];
          }
          __syncthreads();
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            W* d0 = dst + (int64_t)32 * u * N + tx + (int64_t)ty * N;
#pragma unroll
            for (int k = 0; k < 32; k += 8) d0[(int64_t)k * N] = tile[u][tx][ty + k];
          }
        } else {
          // the edges: each of the (at most) two tiles on its own
          const int mr0 = M - m0 < 32 ? M - m0 : 32;
          one_tile(src, dst, mr0, nr, 0);
          if (m0 + 32 < M) {
            const int mr1 = M - m0 - 32 < 32 ? M - m0 - 32 : 32;
            one_tile(src + 32, dst + (int64_t)32 * N, mr1, nr, 1);
          }
        }
        __syncthreads();
      }
}

// ---- launch helpers ---------------------------------------------------------------
int grid_for(int64_t work, int threads) {
  DevInfo di;
  int sms = 148;
  if (dev_info(&di) == BT_OK && di.sm_count > 0) sms = di.sm_count;
  int64_t blocks = (work + threads - 1) / threads;
  int64_t cap = (int64_t)sms * 8;  // 8 resident 256-thread CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// The fp32 ops with their own compiled vector kernels (the decoder stream's
// and the per-op configurations' ops); the rest share the runtime-op kernel.
#define BT_EW_FIXED_OPS(X) \
  X(BT_OP_ADD) X(BT_OP_SUB) X(BT_OP_MUL) X(BT_OP_DIV) X(BT_OP_POW) X(BT_OP_SQRT) X(BT_OP_EXP) X(BT_OP_SIN) \
  X(BT_OP_COS) X(BT_OP_TANH) X(BT_OP_SIGMOID) X(BT_OP_LEAKYRELU) X(BT_OP_GELU) X(BT_OP_IDENTITY)
// the row-broadcast kernels: the same without tanh (see launch_rows4)
#define BT_EW_ROWS_OPS(X) \
  X(BT_OP_ADD) X(BT_OP_SUB) X(BT_OP_MUL) X(BT_OP_DIV) X(BT_OP_POW) X(BT_OP_SQRT) X(BT_OP_EXP) X(BT_OP_SIN) \
  X(BT_OP_COS) X(BT_OP_SIGMOID) X(BT_OP_LEAKYRELU) X(BT_OP_GELU) X(BT_OP_IDENTITY)

void launch_flat4(int op, int grid, int threads, cudaStream_t s, const EwArgs& a) {
  switch (op) {
#define BT_CASE(OPC) \
  case OPC: ew_flat_op_kernel<4, OPC><<<grid, threads, 0, s>>>(a); return;
    BT_EW_FIXED_OPS(BT_CASE)
#undef BT_CASE
    default: ew_flat_kernel<4><<<grid, threads, 0, s>>>(a); return;
  }
}

void launch_rows4(int op, dim3 grid, int threads, cudaStream_t s, const EwArgs& a) {
  // the compiled kernels read exactly fixed_n_in<OP>() operands; tanh (a
  // unary op that reaches this path only for a strided input) keeps the
  // runtime-op kernel, where its double evaluation needs no stack frame
  const bool binary = op == BT_OP_ADD || op == BT_OP_SUB || op == BT_OP_MUL || op == BT_OP_DIV || op == BT_OP_POW;
  if (a.n_in != (binary ? 2 : 1)) op = -1;
  switch (op) {
#define BT_CASE(OPC) \
  case OPC: ew_rows_op_kernel<4, OPC><<<grid, threads, 0, s>>>(a); return;
    BT_EW_ROWS_OPS(BT_CASE)
#undef BT_CASE
    default: ew_rows_kernel<4><<<grid, threads, 0, s>>>(a); return;
  }
}

bool aligned_run(const void* p, int dt, int vec) {
  return ((uintptr_t)p % (uintptr_t)(dtype_size(dt) * vec)) == 0;
}

}  // namespace
}  // namespace bt

using namespace bt;

extern "C" int bt_elementwise(int op, int n_in, const bt_tensor* in, const bt_tensor* out,
                              const bt_ew_attrs* attrs) {
  if (n_in < 1 || n_in > 3) return set_error(BT_EINVAL, "bt_elementwise: n_in %d outside 1..3", n_in);
  if (!in || !out || !attrs) return set_error(BT_EINVAL, "bt_elementwise: null argument");
  const bool known = (op >= 0 && op <= 31) || op == BT_OP_DEQUANT;
  if (!known) return set_error(BT_EINVAL, "bt_elementwise: unknown op code %d", op);
  int rc = check_tensor(out, "out", false);
  if (rc) return rc;
  for (int k = 0; k < n_in; ++k)
    if ((rc = check_tensor(&in[k], "input", false))) return rc;
  const int cdt = attrs->compute_dtype;
  if (!dtype_valid(cdt)) return set_error(BT_EDTYPE, "bt_elementwise: compute dtype %d", cdt);
  if (cdt == BT_F16) return set_error(BT_EDTYPE, "bt_elementwise: fp16 is widened to fp32 before compute");
  const bool float_only = !(op == BT_OP_ADD || op == BT_OP_SUB || op == BT_OP_MUL || op == BT_OP_DIV ||
                            op == BT_OP_CLIP || op == BT_OP_EQUAL || op == BT_OP_GREATER || op == BT_OP_LESS ||
                            op == BT_OP_GEQ || op == BT_OP_AND || op == BT_OP_WHERE || op == BT_OP_NEG ||
                            op == BT_OP_ABS || op == BT_OP_MIN || op == BT_OP_MAX || op == BT_OP_IDENTITY ||
                            op == BT_OP_CAST_INT || op == BT_OP_CAST_BOOL);
  if (float_only && !is_float_dtype(cdt))
    return set_error(BT_EDTYPE, "bt_elementwise: op %d needs a floating compute dtype", op);
  if ((op == BT_OP_GELU || op == BT_OP_DEQUANT) && cdt != BT_F32)
    return set_error(BT_EDTYPE, "bt_elementwise: op %d computes in float32 only", op);
  if (cdt == BT_U64 && op != BT_OP_ADD && op != BT_OP_SUB && op != BT_OP_MUL && op != BT_OP_IDENTITY &&
      op != BT_OP_CAST_INT && op != BT_OP_CAST_BOOL && op != BT_OP_EQUAL)
    return set_error(BT_EUNSUPPORTED, "bt_elementwise: uint64 compute supports add/sub/mul/equal/casts only");

  const bt_tensor* ops[4];
  for (int k = 0; k < n_in; ++k) ops[k] = &in[k];
  ops[n_in] = out;
  BcastPlan p;
  if ((rc = plan_broadcast(n_in + 1, ops, out->shape, out->rank, &p))) return rc;
  if (p.n == 0) return BT_OK;

  EwArgs a{};
  a.op = op; a.n_in = n_in; a.rank = p.rank; a.cdt = cdt; a.alpha = attrs->alpha; a.odt = out->dtype;
  a.n = p.n;
  for (int d = 0; d < p.rank; ++d) a.shape[d] = p.shape[d];
  for (int k = 0; k < 3; ++k) {
    const int src = k < n_in ? k : 0;
    a.in[k].p = in[src].data;
    a.in[k].dt = in[src].dtype;
    for (int d = 0; d < BT_MAX_RANK; ++d) a.in[k].st[d] = (k < n_in && d < p.rank) ? p.st[k][d] : 0;
  }
  a.out = out->data;
  for (int d = 0; d < BT_MAX_RANK; ++d) a.ost[d] = d < p.rank ? p.st[n_in][d] : 0;

  cudaStream_t s = cur_stream();
  const int threads = 256;
  // a transposing copy between equal dtypes: tiled through shared memory
  if (op == BT_OP_IDENTITY && n_in == 1 && in[0].dtype == out->dtype && (p.rank == 2 || p.rank == 3)) {
    const int r = p.rank;
    const int64_t M = p.shape[r - 2], N = p.shape[r - 1], B = r == 3 ? p.shape[0] : 1;
    const bool out_dense = p.st[1][r - 1] == 1 && p.st[1][r - 2] == N && (r == 2 || p.st[1][0] == M * N);
    const int64_t sn = p.st[0][r - 1], sb = r == 3 ? p.st[0][0] : 0;
    if (out_dense && p.st[0][r - 2] == 1 && sn != 1 && M >= 8 && N >= 8 && M < (1ll << 30) && N < (1ll << 30)) {
      // grid: batches in z, m tiles in y, n tiles in x (each CTA walks the
      // rest by increments), about 32 CTAs per SM in all
      const int64_t tm = (M + 63) / 64, tn = (N + 31) / 32;   // tm: pairs of m tiles
      const int64_t gz = B < 65535 ? B : 65535, gy = tm < 65535 ? tm : 65535;
      DevInfo di;
      const int sms = (dev_info(&di) == BT_OK && di.sm_count > 0) ? di.sm_count : 148;
      int64_t gx = ((int64_t)sms * 32 + gy * gz - 1) / (gy * gz);
      if (gx > tn) gx = tn;
      if (gx < 1) gx = 1;
      const dim3 g((unsigned)gx, (unsigned)gy, (unsigned)gz);
      const int Mi = (int)M, Ni = (int)N;
      const bool vec = dtype_size(out->dtype) == 4 && ((uintptr_t)in[0].data & 15) == 0 &&
                       ((uintptr_t)out->data & 15) == 0 && sn % 4 == 0 && sb % 4 == 0 && N % 4 == 0;
      switch (dtype_size(out->dtype)) {
        case 1: transpose_kernel<uint8_t, false><<<g, 256, 0, s>>>((const uint8_t*)in[0].data, (uint8_t*)out->data, B, Mi, Ni, sb, sn); break;
        case 2: transpose_kernel<uint16_t, false><<<g, 256, 0, s>>>((const uint16_t*)in[0].data, (uint16_t*)out->data, B, Mi, Ni, sb, sn); break;
        case 4:
          if (vec) transpose_kernel<uint32_t, true><<<g, 256, 0, s>>>((const uint32_t*)in[0].data, (uint32_t*)out->data, B, Mi, Ni, sb, sn);
          else transpose_kernel<uint32_t, false><<<g, 256, 0, s>>>((const uint32_t*)in[0].data, (uint32_t*)out->data, B, Mi, Ni, sb, sn);
          break;
        default: transpose_kernel<uint64_t, false><<<g, 256, 0, s>>>((const uint64_t*)in[0].data, (uint64_t*)out->data, B, Mi, Ni, sb, sn); break;
      }
      return check_launch("bt_elementwise(transpose)");
    }
  }
  const bool f32_path = (cdt == BT_F32) && op != BT_OP_WHERE && op != BT_OP_AND;
  if (f32_path && p.rank == 1 && a.ost[0] == 1) {
    bool unit = true, vec_ok = aligned_run(out->data, out->dtype, 4);
    for (int k = 0; k < n_in; ++k) {
      if (a.in[k].st[0] != 0 && a.in[k].st[0] != 1) unit = false;
      if (a.in[k].st[0] == 1 && !aligned_run(a.in[k].p, a.in[k].dt, 4)) vec_ok = false;
    }
    if (unit) {
      if (vec_ok) launch_flat4(op, grid_for((a.n + 3) / 4, threads), threads, s, a);
      else ew_flat_kernel<1><<<grid_for(a.n, threads), threads, 0, s>>>(a);
      return check_launch("bt_elementwise(flat)");
    }
  }
  if (f32_path && p.rank == 2 && a.ost[1] == 1) {
    bool ok = true, vec_ok = (p.shape[1] % 4 == 0) && aligned_run(out->data, out->dtype, 4) && (a.ost[0] % 4 == 0);
    for (int k = 0; k < n_in; ++k) {
      if (a.in[k].st[1] != 0 && a.in[k].st[1] != 1) ok = false;
      if (a.in[k].st[1] == 1 && (a.in[k].st[0] % 4 != 0 || !aligned_run(a.in[k].p, a.in[k].dt, 4))) vec_ok = false;
    }
    if (ok) {
      const int vec = vec_ok ? 4 : 1;
      const int unroll = vec_ok ? 4 : 1;   // vectors per thread (ew_rows_op_kernel)
      int64_t per_row = (p.shape[1] / vec + (int64_t)threads * unroll - 1) / ((int64_t)threads * unroll);
      if (per_row < 1) per_row = 1;
      int gy = (int)(p.shape[0] < 65535 ? p.shape[0] : 65535);
      int gx = (int)(per_row > 64 ? 64 : per_row);
      dim3 grid(gx, gy);
      if (vec_ok) launch_rows4(op, grid, threads, s, a);
      else ew_rows_kernel<1><<<grid, threads, 0, s>>>(a);
      return check_launch("bt_elementwise(rows)");
    }
  }
  const int g = grid_for(a.n, threads);
  switch (cdt) {
    case BT_F32: ew_nd_kernel<float><<<g, threads, 0, s>>>(a); break;
    case BT_F64: ew_nd_kernel<double><<<g, threads, 0, s>>>(a); break;
    default: ew_nd_kernel<long long><<<g, threads, 0, s>>>(a); break;
  }
  return check_launch("bt_elementwise(nd)");
}

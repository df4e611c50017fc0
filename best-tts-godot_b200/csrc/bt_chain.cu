// bt_chain.cu -- fused elementwise chains (bt_fused_chain) for sm_100a.
//
// A chain is a short float32 program evaluated per element of the broadcast
// iteration space of its inputs.  The reference runs each op of such a chain
// as its own dispatch with a barrier after it (executor.gd:678-699): Snake is
// five passes over [C, T] (Mul, Sin, Pow 2, Mul, Add), DequantizeLinear and
// the gain Mul that follows it are two (executor.gd:822-827).  Here a chain
// is one pass: every input element read once, at its stored type, and the
// result written once.  Each instruction rounds as the numpy op it stands for
// (ref_runtime.py:446-479, :631-636): float32 in, float32 out, no contraction.
//
// Layout.  The host broadcasts every input to the output shape, drops size-1
// axes and merges the axes that every operand walks contiguously (numpy's
// broadcasting, the rule of ops.gd:62-129).  The last merged axis is the row,
// T values long; the axes before it are walked row by row, each input's row
// offset unravelled once per row.  The output is dense.  Rows are walked by
// blockIdx.y, values within a row by blockIdx.x and the threads, four values
// per vector where every input that varies along the row starts each row on
// a four-value boundary.
//
// Programs.  Chains the library knows (the catalog below) run in kernels
// compiled for that exact program: the instructions are template arguments,
// so every register index is a constant, the op switch folds away and the
// registers are hardware registers.  Any other valid program runs in the
// interpreter kernel, which copies the program into shared memory (reading
// the launch arguments at constant offsets only) and keeps each thread's
// registers in its own column of a shared-memory array.  Neither kernel
// indexes an array in registers or the launch arguments by a value computed
// at run time.
#include <cuda_fp16.h>
#include <stdint.h>
#include <type_traits>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"
#include "bt_ewmath.h"
#include "bt_pk.h"

namespace bt {
namespace {

constexpr int kChainRegs = 16;        // registers a program may name
constexpr int kChainThreads = 256;

struct ChainIn {
  const void* p;
  int32_t dt;
  int32_t pad;
  int64_t inner;                 // stride along the row (elements)
  int64_t st[BT_MAX_RANK];       // strides of the outer axes (elements)
};

struct ChainLaunch {
  int32_t n_in, n_outer, n_instr, out_reg;
  int64_t R, T;                  // rows, values per row
  int64_t outer[BT_MAX_RANK];    // outer extents, row-major
  ChainIn in[BT_CHAIN_MAX_IN];
  float* out;                    // dense [R, T]
  float alpha[BT_CHAIN_MAX_INSTR];
  int32_t code[BT_CHAIN_MAX_INSTR][4];   // op, dst, a, b (interpreter only)
};

// Offsets of row r in the first NIN inputs.  One outer axis (the common
// case after merging) needs no division; otherwise r is unravelled in 32-bit
// arithmetic (the host keeps R below 2^32), which compiles to a short inline
// sequence where 64-bit division would call a subroutine.
template <int NIN>
__device__ __forceinline__ void row_offsets(const ChainLaunch& a, int64_t r, int64_t (&off)[NIN]) {
  if (a.n_outer <= 1) {
#pragma unroll
    for (int k = 0; k < NIN; ++k) off[k] = a.n_outer == 1 ? r * a.in[k].st[0] : 0;
    return;
  }
#pragma unroll
  for (int k = 0; k < NIN; ++k) off[k] = 0;
  uint32_t rem = (uint32_t)r;
#pragma unroll
  for (int d = BT_MAX_RANK - 1; d >= 0; --d) {
    if (d < a.n_outer) {
      const uint32_t e = (uint32_t)a.outer[d];
      const uint32_t c = rem % e;
      rem /= e;
#pragma unroll
      for (int k = 0; k < NIN; ++k) off[k] += (int64_t)c * a.in[k].st[d];
    }
  }
}

// Four consecutive values of input o from element i (i a multiple of four,
// the base 4-element aligned): one 128-bit float32, 64-bit float16 / 16-bit
// or 32-bit 8-bit load.
__device__ __forceinline__ void ld4(const ChainIn& o, int64_t i, float* x) {
  switch (o.dt) {
    case BT_F32: {
      const float4 f = __ldcs((const float4*)((const float*)o.p + i));
      x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
      return;
    }
    case BT_F16: {
      const uint2 u = __ldcs((const uint2*)((const __half*)o.p + i));
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      x[0] = f0.x; x[1] = f0.y; x[2] = f1.x; x[3] = f1.y;
      return;
    }
    case BT_I8: {
      const int w = __ldcs((const int*)((const signed char*)o.p + i));
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = (float)(signed char)(w >> (8 * j));
      return;
    }
    case BT_U8:
    case BT_BOOL: {
      const unsigned w = __ldcs((const unsigned*)((const unsigned char*)o.p + i));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const unsigned b = (w >> (8 * j)) & 0xffu;
        x[j] = o.dt == BT_BOOL ? (b != 0u ? 1.0f : 0.0f) : (float)b;
      }
      return;
    }
    case BT_I16: {
      const uint2 u = __ldcs((const uint2*)((const short*)o.p + i));
      x[0] = (float)(short)(u.x & 0xffffu); x[1] = (float)(short)(u.x >> 16);
      x[2] = (float)(short)(u.y & 0xffffu); x[3] = (float)(short)(u.y >> 16);
      return;
    }
    default: {   // BT_U16
      const uint2 u = __ldcs((const uint2*)((const unsigned short*)o.p + i));
      x[0] = (float)(u.x & 0xffffu); x[1] = (float)(u.x >> 16);
      x[2] = (float)(u.y & 0xffffu); x[3] = (float)(u.y >> 16);
      return;
    }
  }
}

// ---- compiled programs ----------------------------------------------------------
// One instruction: r[DST] = OP(r[A], r[B]) rounded as numpy rounds the op;
// K is its position (its LeakyRelu slope is alpha[K]).
template <int OP, int DST, int A, int B, int K>
struct In {
  static constexpr int op = OP, dst = DST, a = A, b = B;
  template <int NR>
  static __device__ __forceinline__ void run(float (&r)[NR], const ChainLaunch& l) {
    r[DST] = apply_f32<true>(OP, r[A], r[B], 0.0f, l.alpha[K], 2);
  }
};

// A program in single-assignment form: inputs are registers 0..NIN-1, the
// k-th instruction writes register NIN + k, the result is register OUT.
// Unary instructions name their operand twice (b = a).
template <int NIN_, int OUT_, class... Is>
struct Prog {
  static constexpr int NIN = NIN_, OUT = OUT_, N = sizeof...(Is), NREG = NIN_ + sizeof...(Is);
  static __device__ __forceinline__ float eval(float (&r)[NREG], const ChainLaunch& l) {
    (Is::template run<NREG>(r, l), ...);
    return r[OUT_];
  }
  // Whether the canonical program c (single-assignment form) is this one.
  static bool matches(int n_in, int out_reg, int n_instr, const int (*c)[4]) {
    const int ops[] = {Is::op...}, dst[] = {Is::dst...}, as[] = {Is::a...}, bs[] = {Is::b...};
    if (n_in != NIN || out_reg != OUT || n_instr != N) return false;
    for (int i = 0; i < N; ++i)
      if (c[i][0] != ops[i] || c[i][1] != dst[i] || c[i][2] != as[i] || c[i][3] != bs[i]) return false;
    return true;
  }
};

// The catalog.  Input order is the order the runtime passes them in.
// Mul(DequantizeLinear(q, scale), gain): inputs q, scale, gain
// (ref_runtime.py:631-636 then :450-451).
using ProgDequantMul = Prog<3, 4, In<BT_OP_MUL, 3, 0, 1, 0>, In<BT_OP_MUL, 4, 3, 2, 1>>;
// the same with a zero point: inputs q, scale, gain, zp
using ProgDequantZpMul =
    Prog<4, 6, In<BT_OP_SUB, 4, 0, 3, 0>, In<BT_OP_MUL, 5, 4, 1, 1>, In<BT_OP_MUL, 6, 5, 2, 2>>;
// Snake x + inv_alpha * sin(alpha * x) ** 2 in the graph's op order (Mul,
// Sin, Pow, Mul, Add): inputs x, alpha, the exponent (2), inv_alpha
using ProgSnake = Prog<4, 8, In<BT_OP_MUL, 4, 1, 0, 0>, In<BT_OP_SIN, 5, 4, 4, 1>, In<BT_OP_POW, 6, 5, 2, 2>,
                       In<BT_OP_MUL, 7, 3, 6, 3>, In<BT_OP_ADD, 8, 0, 7, 4>>;
// Sigmoid(Add(x, y)): inputs x, y
using ProgAddSigmoid = Prog<2, 3, In<BT_OP_ADD, 2, 0, 1, 0>, In<BT_OP_SIGMOID, 3, 2, 2, 1>>;
// Mul then Add (an affine step, gain * x + shift): inputs x, gain, shift
using ProgMulAdd = Prog<3, 4, In<BT_OP_MUL, 3, 0, 1, 0>, In<BT_OP_ADD, 4, 3, 2, 1>>;
// Add then LeakyRelu (a residual sum feeding an activation): inputs x, y
using ProgAddLeaky = Prog<2, 3, In<BT_OP_ADD, 2, 0, 1, 0>, In<BT_OP_LEAKYRELU, 3, 2, 2, 1>>;
// DequantizeLinear alone (ref_runtime.py:631-636): inputs q, scale
using ProgDequant = Prog<2, 2, In<BT_OP_MUL, 2, 0, 1, 0>>;
// DequantizeLinear with a zero point: inputs q, scale, zp
using ProgDequantZp = Prog<3, 4, In<BT_OP_SUB, 3, 0, 2, 0>, In<BT_OP_MUL, 4, 3, 1, 1>>;

// How a compiled kernel loads input k: SIG holds four bits per input.
// kAny: decided at run time (row-constant or not, any dtype); kRow: the
// input is constant along the row (loaded once per row); kF32 / kF16 / kI8 /
// kU8: varies along the row, unit stride, that dtype (four values per load).
// The host launches a specialised SIG only when the inputs are exactly so.
enum : uint32_t { kAny = 0, kRow = 1, kF32 = 2, kF16 = 3, kI8 = 4, kU8 = 5 };
constexpr uint32_t sig(uint32_t k0, uint32_t k1 = 0, uint32_t k2 = 0, uint32_t k3 = 0) {
  return k0 | (k1 << 4) | (k2 << 8) | (k3 << 12);
}
template <uint32_t SIG, int K>
__host__ __device__ constexpr uint32_t kind_of() { return (SIG >> (4 * K)) & 15u; }
// Snake over a float32 row with per-row alpha, exponent and inv_alpha
constexpr uint32_t kSnakeSig = sig(kF32, kRow, kRow, kRow);
// vectors in flight per thread: eight where a varying input is 8-bit (four
// bytes per vector, so little is in flight otherwise), else four (two for
// the layout-generic kernels, whose every input may vary)
template <uint32_t SIG>
__host__ __device__ constexpr int chain_unroll() {
  return SIG == 0 ? 2 : (kind_of<SIG, 0>() == kI8 || kind_of<SIG, 0>() == kU8) ? 8 : 4;
}

// Input K's VEC values of vector v (row offset off, row constant rowv).
template <uint32_t SIG, int K, int VEC>
__device__ __forceinline__ void load_in(const ChainIn& o, int64_t off, int64_t v, float rowv, float* x) {
  constexpr uint32_t kd = kind_of<SIG, K>();
  if constexpr (kd == kRow) {
    // read from rowv where it is used (see lane_value)
  } else if constexpr (kd == kF32 && VEC == 4) {
    const float4 f = __ldcs((const float4*)((const float*)o.p + off + v * 4));
    x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
  } else if constexpr (kd == kF16 && VEC == 4) {
    const uint2 u = __ldcs((const uint2*)((const __half*)o.p + off + v * 4));
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    x[0] = f0.x; x[1] = f0.y; x[2] = f1.x; x[3] = f1.y;
  } else if constexpr ((kd == kI8 || kd == kU8) && VEC == 4) {
    // the four bytes stay packed in one register until they are used
    x[0] = __int_as_float(__ldcs((const int*)((const signed char*)o.p + off + v * 4)));
  } else {
    if (o.inner == 0) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) x[j] = rowv;
    } else if constexpr (VEC == 4) {
      ld4(o, off + v * 4, x);
    } else {
      x[0] = ld1<float>(o.p, o.dt, off + v * o.inner);
    }
  }
}

// Value j of input k's vector (as load_in left it).
template <uint32_t SIG, int VEC>
__device__ __forceinline__ float lane_value(int k, int j, const float* xk, const float* rowv) {
  const uint32_t kd = (SIG >> (4 * k)) & 15u;   // folds: k and j are unrolled constants
  if (kd == kRow) return rowv[k];
  if (VEC == 4 && kd == kI8) return (float)(signed char)(__float_as_int(xk[0]) >> (8 * j));
  if (VEC == 4 && kd == kU8) return (float)((__float_as_uint(xk[0]) >> (8 * j)) & 0xffu);
  return xk[j];
}

template <uint32_t SIG, int VEC, int K, int NIN>
struct LoadAll {
  static __device__ __forceinline__ void run(const ChainLaunch& a, const int64_t* off, int64_t v, const float* rowv,
                                             float (*x)[VEC]) {
    load_in<SIG, K, VEC>(a.in[K], off[K], v, rowv[K], x[K]);
    LoadAll<SIG, VEC, K + 1, NIN>::run(a, off, v, rowv, x);
  }
};
template <uint32_t SIG, int VEC, int NIN>
struct LoadAll<SIG, VEC, NIN, NIN> {
  static __device__ __forceinline__ void run(const ChainLaunch&, const int64_t*, int64_t, const float*,
                                             float (*)[VEC]) {}
};

// Snake of four values two at a time (bt_pk.h), for rows whose exponent is
// 2: alpha * x, numpy's sine squared as Pow(., 2) squares it, times
// inv_alpha, added to x lane by lane (a packed product feeding a packed add
// may be contracted into one FMA, which would round once instead of twice).
__device__ __forceinline__ void snake4(const float (&x)[4], float al, float ial, float* out) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float2 v = make_float2(x[2 * h], x[2 * h + 1]);
    const float2 s2 = pk_np_sin<true>(pk_mul(pk(al), v));
    const float2 z = pk_add_lanes(v, pk_mul(pk(ial), s2));
    out[2 * h] = z.x;
    out[2 * h + 1] = z.y;
  }
}

// U vectors of VEC values per thread in flight; every load of a vector is
// issued before any of its math.
template <class P, int VEC, int U, uint32_t SIG>
__global__ void __launch_bounds__(kChainThreads, SIG == 0 ? 1 : (U == 4 ? 3 : 4)) chain_prog_kernel(ChainLaunch a) {
  constexpr int NIN = P::NIN;
  const int64_t R = a.R, T = a.T;
  const int64_t nv = T / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = blockIdx.y; r < R; r += gridDim.y) {
    int64_t off[NIN];
    row_offsets<NIN>(a, r, off);
    float rowv[NIN];
#pragma unroll
    for (int k = 0; k < NIN; ++k) rowv[k] = a.in[k].inner == 0 ? ld1<float>(a.in[k].p, a.in[k].dt, off[k]) : 0.0f;
    float* orow = a.out + r * T;
    for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v0 < nv; v0 += U * stride) {
      float x[U][NIN][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t v = v0 + u * stride;
        if (v < nv) LoadAll<SIG, VEC, 0, NIN>::run(a, off, v, rowv, x[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t v = v0 + u * stride;
        if (v >= nv) break;
        float res[VEC];
        auto each = [&]() {
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            float reg[P::NREG];
#pragma unroll
            for (int k = 0; k < NIN; ++k) reg[k] = lane_value<SIG, VEC>(k, j, x[u][k], rowv);
            res[j] = P::eval(reg, a);
          }
        };
        if constexpr (std::is_same<P, ProgSnake>::value && SIG == kSnakeSig && VEC == 4) {
          if (rowv[2] == 2.0f) snake4(x[u][0], rowv[1], rowv[3], res);
          else each();
        } else {
          each();
        }
        if constexpr (VEC == 4) {
          __stcs((float4*)(orow + v * VEC), make_float4(res[0], res[1], res[2], res[3]));
        } else {
          orow[v] = res[0];
        }
      }
    }
    // the row's last T % VEC values
    for (int64_t t = nv * VEC + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T; t += stride) {
      float reg[P::NREG];
#pragma unroll
      for (int k = 0; k < NIN; ++k) reg[k] = ld1<float>(a.in[k].p, a.in[k].dt, off[k] + t * a.in[k].inner);
      orow[t] = P::eval(reg, a);
    }
  }
}

// ---- the interpreter ------------------------------------------------------------
// Register j of thread i lives at regs[j][i]: consecutive threads hit
// consecutive banks whatever the program names.  The row's input offsets
// live in shared memory too (every thread of a CTA works on the same row),
// so that little stays live in registers across the op evaluation.
__global__ void __launch_bounds__(kChainThreads, 4) chain_interp_kernel(ChainLaunch a) {
  __shared__ int4 code[BT_CHAIN_MAX_INSTR];
  __shared__ float alpha[BT_CHAIN_MAX_INSTR];
  __shared__ float regs[kChainRegs][kChainThreads];
  __shared__ int64_t roff[BT_CHAIN_MAX_IN];
  if (threadIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < BT_CHAIN_MAX_INSTR; ++k) {
      code[k] = make_int4(a.code[k][0], a.code[k][1], a.code[k][2], a.code[k][3]);
      alpha[k] = a.alpha[k];
    }
  }
  float* my = &regs[0][threadIdx.x];
  const int64_t R = a.R, T = a.T;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = blockIdx.y; r < R; r += gridDim.y) {
    if (threadIdx.x == 0) {
      int64_t off[BT_CHAIN_MAX_IN];
      row_offsets<BT_CHAIN_MAX_IN>(a, r, off);
#pragma unroll
      for (int k = 0; k < BT_CHAIN_MAX_IN; ++k) roff[k] = off[k];
    }
    __syncthreads();
    float* orow = a.out + r * T;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T; t += stride) {
#pragma unroll
      for (int k = 0; k < BT_CHAIN_MAX_IN; ++k)
        if (k < a.n_in) my[k * kChainThreads] = ld1<float>(a.in[k].p, a.in[k].dt, roff[k] + t * a.in[k].inner);
      const int n_instr = a.n_instr;
      for (int i = 0; i < n_instr; ++i) {
        const int4 c = code[i];
        my[c.y * kChainThreads] =
            apply_f32<true>(c.x, my[c.z * kChainThreads], my[c.w * kChainThreads], 0.0f, alpha[i], 2);
      }
      orow[t] = my[a.out_reg * kChainThreads];
    }
    __syncthreads();   // roff is rewritten for the next row
  }
}

// ---- host side ------------------------------------------------------------------
bool chain_op_ok(int op) {
  switch (op) {
    case BT_OP_ADD: case BT_OP_SUB: case BT_OP_MUL: case BT_OP_DIV: case BT_OP_POW: case BT_OP_SQRT:
    case BT_OP_EXP: case BT_OP_SIN: case BT_OP_COS: case BT_OP_TANH: case BT_OP_SIGMOID: case BT_OP_LEAKYRELU:
    case BT_OP_ERF: case BT_OP_IDENTITY: case BT_OP_NEG: case BT_OP_ABS: case BT_OP_MIN: case BT_OP_MAX:
    case BT_OP_FLOOR: case BT_OP_ROUND: case BT_OP_ATAN:
      return true;
    default:
      return false;
  }
}

bool chain_binary(int op) {
  return op == BT_OP_ADD || op == BT_OP_SUB || op == BT_OP_MUL || op == BT_OP_DIV || op == BT_OP_POW ||
         op == BT_OP_MIN || op == BT_OP_MAX;
}

// Input types whose float32 widening is exact, so that the chain's float32
// arithmetic is the arithmetic numpy does with them next to float32 data.
bool chain_dtype_ok(int dt) {
  return dt == BT_F32 || dt == BT_F16 || dt == BT_I8 || dt == BT_U8 || dt == BT_I16 || dt == BT_U16 ||
         dt == BT_BOOL;
}

// Validates the program and rewrites it in single-assignment form (inputs
// 0..n_in-1, instruction k writes n_in + k; a unary instruction names its
// operand twice) for the catalog match.  A register read before anything was
// written to it is an error.  *out: the result's single-assignment name.
int chain_canon(const bt_chain* prog, int (*canon)[4], int* out, const char* what) {
  const int n_in = prog->n_in, n_instr = prog->n_instr;
  if (n_in < 1 || n_in > BT_CHAIN_MAX_IN)
    return set_error(BT_EINVAL, "%s: n_in %d outside 1..%d", what, n_in, BT_CHAIN_MAX_IN);
  if (n_instr < 0 || n_instr > BT_CHAIN_MAX_INSTR)
    return set_error(BT_EINVAL, "%s: %d instructions (max %d)", what, n_instr, BT_CHAIN_MAX_INSTR);
  if (prog->out_reg < 0 || prog->out_reg >= kChainRegs)
    return set_error(BT_EINVAL, "%s: output register %d", what, prog->out_reg);
  int name[kChainRegs];
  for (int j = 0; j < kChainRegs; ++j) name[j] = j < n_in ? j : -1;
  for (int k = 0; k < n_instr; ++k) {
    const bt_chain_instr& ins = prog->instr[k];
    if (!chain_op_ok(ins.op)) return set_error(BT_EINVAL, "%s: instruction %d has op %d", what, k, ins.op);
    const bool bin = chain_binary(ins.op);
    if (ins.dst < 0 || ins.dst >= kChainRegs || ins.a < 0 || ins.a >= kChainRegs ||
        (bin && (ins.b < 0 || ins.b >= kChainRegs)))
      return set_error(BT_EINVAL, "%s: instruction %d uses a register outside 0..%d", what, k, kChainRegs - 1);
    if (name[ins.a] < 0 || (bin && name[ins.b] < 0))
      return set_error(BT_EINVAL, "%s: instruction %d reads a register nothing wrote", what, k);
    canon[k][0] = ins.op;
    canon[k][1] = n_in + k;
    canon[k][2] = name[ins.a];
    canon[k][3] = bin ? name[ins.b] : name[ins.a];
    name[ins.dst] = n_in + k;
  }
  if (name[prog->out_reg] < 0) return set_error(BT_EINVAL, "%s: the output register is never written", what);
  *out = name[prog->out_reg];
  return BT_OK;
}

// The catalog, in the order bt_chain_kind numbers it, each program with the
// input layouts it has kernels specialised for (the c4 weights: int8 values,
// per-channel scale, gain and zero point; Snake: a float32 row with its
// per-channel constants; the rest: float32 with a same-shape or per-row
// second operand).
#define BT_CHAIN_CATALOG(X)                                                                          \
  X(ProgDequantMul, sig(kI8, kRow, kRow))                                                           \
  X(ProgDequantZpMul, sig(kI8, kRow, kRow, kRow))                                                    \
  X(ProgSnake, sig(kF32, kRow, kRow, kRow))                                                          \
  X(ProgAddSigmoid, sig(kF32, kF32), sig(kF32, kRow))                                                \
  X(ProgMulAdd, sig(kF32, kRow, kRow), sig(kF32, kF32, kF32))                                        \
  X(ProgAddLeaky, sig(kF32, kF32), sig(kF32, kRow))                                                 \
  X(ProgDequant, sig(kI8, kRow))                                                                     \
  X(ProgDequantZp, sig(kI8, kRow, kRow))

// Grid: rows in y, about 16 CTAs per SM in all, at least one per row.
dim3 chain_grid(const ChainLaunch& a, int per_cta, int sms) {
  const int64_t per_row = (a.T + per_cta - 1) / per_cta;
  const int64_t gy = a.R < 65535 ? a.R : 65535;
  const int64_t cap = ((int64_t)sms * 16 + gy - 1) / gy;
  int64_t gx = per_row < cap ? per_row : cap;
  if (gx < 1) gx = 1;
  return dim3((unsigned)gx, (unsigned)gy);
}

// Launches program P: the kernel specialised for the inputs' layout `actual`
// when it is one of P's SIGS, else the one that decides at run time.
template <class P, uint32_t... SIGS>
int launch_prog(const ChainLaunch& a, bool vec, uint32_t actual, int sms, cudaStream_t s) {
  constexpr int U = 2;
  bool done = false;
  if (vec)
    ((!done && actual == SIGS
          ? (chain_prog_kernel<P, 4, chain_unroll<SIGS>(), SIGS>
             <<<chain_grid(a, 4 * chain_unroll<SIGS>() * kChainThreads, sms), kChainThreads, 0, s>>>(a),
             done = true)
          : false),
     ...);
  if (!done) {
    if (vec)
      chain_prog_kernel<P, 4, U, 0><<<chain_grid(a, 4 * U * kChainThreads, sms), kChainThreads, 0, s>>>(a);
    else
      chain_prog_kernel<P, 1, U, 0><<<chain_grid(a, U * kChainThreads, sms), kChainThreads, 0, s>>>(a);
  }
  return check_launch("bt_fused_chain");
}

}  // namespace
}  // namespace bt

using namespace bt;

extern "C" int bt_fused_chain(const bt_chain* prog, const bt_tensor* in, const bt_tensor* out) {
  if (!prog || !in || !out) return set_error(BT_EINVAL, "bt_fused_chain: null argument");
  int canon[BT_CHAIN_MAX_INSTR][4], canon_out = -1;
  int rc = chain_canon(prog, canon, &canon_out, "bt_fused_chain");
  if (rc) return rc;
  const int n_in = prog->n_in, n_instr = prog->n_instr;

  rc = check_tensor(out, "out", false);
  if (rc) return rc;
  if (out->dtype != BT_F32) return set_error(BT_EDTYPE, "bt_fused_chain: the output must be float32");
  if (!is_contiguous(out)) return set_error(BT_EUNSUPPORTED, "bt_fused_chain: the output must be dense (C order)");
  for (int k = 0; k < n_in; ++k) {
    if ((rc = check_tensor(&in[k], "input", false))) return rc;
    if (!chain_dtype_ok(in[k].dtype))
      return set_error(BT_EDTYPE, "bt_fused_chain: input %d has dtype %d (float32, float16, 8/16-bit integers "
                                  "and bool widen exactly to float32)", k, in[k].dtype);
  }

  // broadcast every input to the output shape (stride 0 on broadcast axes)
  const int orank = out->rank;
  int64_t st[BT_CHAIN_MAX_IN][BT_MAX_RANK];
  int64_t n = 1;
  for (int d = 0; d < orank; ++d) n *= out->shape[d];
  if (n == 0) return BT_OK;
  for (int k = 0; k < n_in; ++k) {
    const bt_tensor& t = in[k];
    if (t.rank > orank)
      return set_error(BT_ESHAPE, "bt_fused_chain: input %d has rank %d > output rank %d", k, t.rank, orank);
    const int pad = orank - t.rank;
    for (int d = 0; d < orank; ++d) {
      if (d < pad) { st[k][d] = 0; continue; }
      const int64_t e = t.shape[d - pad];
      if (e == out->shape[d]) st[k][d] = e == 1 ? 0 : t.strides[d - pad];
      else if (e == 1) st[k][d] = 0;
      else return set_error(BT_ESHAPE, "bt_fused_chain: input %d: extent %lld on axis %d does not broadcast to %lld",
                            k, (long long)e, d, (long long)out->shape[d]);
    }
  }
  // drop size-1 axes; merge axis i-1 into i where every input and the dense
  // output step through both contiguously
  int64_t dims[BT_MAX_RANK], cs[BT_CHAIN_MAX_IN][BT_MAX_RANK];
  int r = 0;
  for (int d = 0; d < orank; ++d) {
    if (out->shape[d] == 1) continue;
    dims[r] = out->shape[d];
    for (int k = 0; k < n_in; ++k) cs[k][r] = st[k][d];
    ++r;
  }
  if (r == 0) {
    dims[0] = 1;
    for (int k = 0; k < n_in; ++k) cs[k][0] = 0;
    r = 1;
  }
  for (int i = r - 1; i > 0; --i) {
    bool ok = true;
    for (int k = 0; k < n_in; ++k)
      if (cs[k][i - 1] != cs[k][i] * dims[i]) { ok = false; break; }
    if (!ok) continue;   // (the dense output always merges)
    dims[i - 1] *= dims[i];
    for (int k = 0; k < n_in; ++k) cs[k][i - 1] = cs[k][i];
    for (int j = i; j < r - 1; ++j) {
      dims[j] = dims[j + 1];
      for (int k = 0; k < n_in; ++k) cs[k][j] = cs[k][j + 1];
    }
    --r;
  }

  ChainLaunch a{};
  a.n_in = n_in;
  a.n_instr = n_instr;
  a.out_reg = prog->out_reg;
  a.T = dims[r - 1];
  a.n_outer = r - 1;
  a.R = 1;
  for (int d = 0; d < r - 1; ++d) {
    a.outer[d] = dims[d];
    a.R *= dims[d];
  }
  bool vec = a.T % 4 == 0 && ((uintptr_t)out->data % 16) == 0;
  for (int k = 0; k < n_in; ++k) {
    ChainIn& c = a.in[k];
    c.p = in[k].data;
    c.dt = in[k].dtype;
    c.inner = cs[k][r - 1];
    for (int d = 0; d < r - 1; ++d) c.st[d] = cs[k][d];
    if (c.inner != 0 && c.inner != 1) vec = false;
    if (c.inner == 1) {
      if (((uintptr_t)c.p % (uintptr_t)(4 * dtype_size(c.dt))) != 0) vec = false;
      for (int d = 0; d < r - 1; ++d)
        if (c.st[d] % 4 != 0) vec = false;
    }
  }
  if (a.R >= (int64_t)1 << 32)
    return set_error(BT_ETOOBIG, "bt_fused_chain: %lld rows (at most 2^32 - 1)", (long long)a.R);
  a.out = (float*)out->data;
  for (int k = 0; k < n_instr; ++k) {
    a.alpha[k] = prog->instr[k].alpha;
    a.code[k][0] = prog->instr[k].op;
    a.code[k][1] = prog->instr[k].dst;
    a.code[k][2] = prog->instr[k].a;
    a.code[k][3] = chain_binary(prog->instr[k].op) ? prog->instr[k].b : prog->instr[k].a;
  }

  DevInfo di;
  const int sms = (dev_info(&di) == BT_OK && di.sm_count > 0) ? di.sm_count : 148;
  cudaStream_t s = cur_stream();
  // the inputs' layout, for the specialised kernels
  uint32_t actual = 0;
  for (int k = 0; k < n_in; ++k) {
    uint32_t kd = kAny;
    if (a.in[k].inner == 0) kd = kRow;
    else if (in[k].dtype == BT_F32) kd = kF32;
    else if (in[k].dtype == BT_F16) kd = kF16;
    else if (in[k].dtype == BT_I8) kd = kI8;
    else if (in[k].dtype == BT_U8) kd = kU8;
    actual |= kd << (4 * k);
  }
#define BT_TRY(P, ...) \
  if (P::matches(n_in, canon_out, n_instr, canon)) return launch_prog<P, __VA_ARGS__>(a, vec, actual, sms, s);
  BT_CHAIN_CATALOG(BT_TRY)
#undef BT_TRY
  // any other program: the interpreter, one value per thread and step
  chain_interp_kernel<<<chain_grid(a, kChainThreads, sms), kChainThreads, 0, s>>>(a);
  return check_launch("bt_fused_chain(interpreter)");
}

// Which kernel bt_fused_chain would run for a program: the index of the
// catalog entry it matches (0-based), or BT_CHAIN_INTERPRETER; a negative
// BT_E* code for an invalid program.  Host only.
extern "C" int bt_chain_kind(const bt_chain* prog) {
  if (!prog) return set_error(BT_EINVAL, "bt_chain_kind: null argument");
  int canon[BT_CHAIN_MAX_INSTR][4], o = -1;
  const int rc = chain_canon(prog, canon, &o, "bt_chain_kind");
  if (rc) return rc;
  int idx = 0;
#define BT_KIND(P, ...) \
  if (P::matches(prog->n_in, o, prog->n_instr, canon)) return idx; \
  ++idx;
  BT_CHAIN_CATALOG(BT_KIND)
#undef BT_KIND
  return BT_CHAIN_INTERPRETER;
}

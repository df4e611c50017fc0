// bt_rows.cu -- row kernels for sm_100a: reductions, softmax, (skip) layer
// normalisation and the fused AdaIN1d -> Snake of the Kokoro generator.
//
// Layout: one CTA owns one row of T contiguous fp32 values.  The row is
// staged once from HBM into shared memory (128-bit loads over the 16-byte
// aligned middle of the row, the shared buffer offset so the phases match),
// every statistic is computed from shared memory, and the outputs are
// streamed back with 128-bit stores.  HBM therefore sees each input byte once
// and each output byte once -- the algorithmic minimum -- while the
// statistics keep numpy's exact two-pass order.
//
// numpy order.  np.add.reduce over a contiguous float32 axis is numpy's
// pairwise summation (bt_core.h).  Its tree depends on T only, so each CTA
// first lays the tree out in shared memory (heap numbering: node h has
// children 2h and 2h+1; kind 0 = absent, 1 = leaf of <= 128 values,
// 2 = inner node), then sums all leaves in parallel (8 lanes per leaf, one
// lane per numpy accumulator, combined by shuffles in numpy's bracket order)
// and finally combines the inner nodes level by level.  The result is
// bit-identical to numpy for any T.  Means divide the float32 sum by the
// count in double precision, as np.mean does.
#include <cuda_fp16.h>
#include <stdint.h>
#include <atomic>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"
#include "bt_async.h"
#include "bt_pk.h"
#include <map>
#include <mutex>
#include <vector>

namespace bt {
namespace {

constexpr int kMaxRow = 49152;   // longest row one CTA stages (192 KiB fp32)

// ---- pairwise plan -----------------------------------------------------------
struct PwPlan {
  unsigned char* kind;   // [2 << depth]
  float* hsum;           // [2 << depth]
  int* leaf_off;         // [1 << depth]
  short* leaf_len;
  short* leaf_id;
  int* n_leaf;           // counter in shared memory
  int depth;
};

// Shared-memory bytes the plan of depth D needs (after the row buffer).
__host__ __device__ inline size_t plan_bytes(int D) {
  size_t ids = (size_t)2 << D, leaves = (size_t)1 << D;
  return ids * sizeof(float) + leaves * sizeof(int) + ids + 2 * leaves * sizeof(short) + 16;
}

__device__ inline PwPlan plan_at(unsigned char* base, int D) {
  PwPlan P;
  size_t ids = (size_t)2 << D, leaves = (size_t)1 << D;
  P.hsum = (float*)base;
  P.leaf_off = (int*)(base + ids * sizeof(float));
  P.n_leaf = (int*)(base + ids * sizeof(float) + leaves * sizeof(int));
  P.kind = base + ids * sizeof(float) + leaves * sizeof(int) + 16;
  P.leaf_len = (short*)(P.kind + ids);
  P.leaf_id = P.leaf_len + leaves;
  P.depth = D;
  return P;
}

// Lays out numpy's pairwise tree for a run of n values (whole CTA).
__device__ void pw_build(PwPlan& P, int n) {
  if (threadIdx.x == 0) *P.n_leaf = 0;
  __syncthreads();
  const int ids = 2 << P.depth;
  for (int h = threadIdx.x + 1; h < ids; h += blockDim.x) {
    const int k = 31 - __clz(h);
    int lo = 0, len = n;
    bool exists = true;
    for (int b = k - 1; b >= 0; --b) {
      if (len <= kPwLeaf) { exists = false; break; }
      const int h2 = (int)pw_split(len);
      if ((h >> b) & 1) { lo += h2; len -= h2; } else { len = h2; }
    }
    unsigned char kd = 0;
    if (exists) kd = (len <= kPwLeaf) ? 1 : 2;
    P.kind[h] = kd;
    if (kd == 1) {
      const int pos = atomicAdd(P.n_leaf, 1);
      P.leaf_off[pos] = lo;
      P.leaf_len[pos] = (short)len;
      P.leaf_id[pos] = (short)h;
    }
  }
  __syncthreads();
}

// Element transforms applied while summing: the value itself, or its
// squared deviation from a mean (Sub then Mul, each rounded).
struct PwIdentity {
  __device__ __forceinline__ float operator()(float v) const { return v; }
  __device__ __forceinline__ float2 two(float2 acc, float2 v) const { return pk_add(acc, v); }
};
struct PwSquaredDev {
  float mu;
  __device__ __forceinline__ float operator()(float v) const {
    const float d = BT_SUB(v, mu);
    return BT_MUL(d, d);
  }
  // the product feeds an add: lane by lane (see pk_add_lanes)
  __device__ __forceinline__ float2 two(float2 acc, float2 v) const {
    const float2 d = pk_add(v, pk(-mu));
    return pk_add_lanes(acc, pk_mul(d, d));
  }
};

// numpy's pairwise sum of f(s[0..n)) with the plan in P (whole CTA; every
// thread receives the result).  Two lanes per leaf, each holding four of
// numpy's eight accumulators (lane h owns r[4h..4h+3]); `aligned` means s is
// 16-byte aligned, so every leaf (leaf offsets are multiples of 8) can be read
// with 128-bit shared loads.  The inner nodes are combined by one warp, level
// by level.
template <class F>
__device__ float pw_sum(const float* s, PwPlan& P, F f, bool aligned) {
  const int h = threadIdx.x & 1;
  const int grp = threadIdx.x >> 1, ngrp = blockDim.x >> 1;
  const unsigned pmask = 3u << (threadIdx.x & 30);
  const int nl = *P.n_leaf;
  for (int L = grp; L < nl; L += ngrp) {
    const int off = P.leaf_off[L], len = P.leaf_len[L];
    float res = 0.0f;
    if (len < 8) {
      if (h == 0)
        for (int i = 0; i < len; ++i) res = BT_ADD(res, f(s[off + i]));
    } else {
      const float* q = s + off + 4 * h;
      float r0, r1, r2, r3;
      if (aligned) {
        const float4 v = *(const float4*)q;
        r0 = f(v.x); r1 = f(v.y); r2 = f(v.z); r3 = f(v.w);
      } else {
        r0 = f(q[0]); r1 = f(q[1]); r2 = f(q[2]); r3 = f(q[3]);
      }
      const int full = len & ~7;
      for (int i = 8; i < full; i += 8) {
        if (aligned) {
          const float4 v = *(const float4*)(q + i);
          r0 = BT_ADD(r0, f(v.x)); r1 = BT_ADD(r1, f(v.y)); r2 = BT_ADD(r2, f(v.z)); r3 = BT_ADD(r3, f(v.w));
        } else {
          r0 = BT_ADD(r0, f(q[i])); r1 = BT_ADD(r1, f(q[i + 1]));
          r2 = BT_ADD(r2, f(q[i + 2])); r3 = BT_ADD(r3, f(q[i + 3]));
        }
      }
      // lane 0: (r0+r1)+(r2+r3), lane 1: (r4+r5)+(r6+r7); their sum is numpy's
      // ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) (float addition commutes).
      float t = BT_ADD(BT_ADD(r0, r1), BT_ADD(r2, r3));
      t = BT_ADD(t, __shfl_xor_sync(pmask, t, 1));
      res = t;
      if (h == 0)
        for (int i = full; i < len; ++i) res = BT_ADD(res, f(s[off + i]));
    }
    if (h == 0) P.hsum[P.leaf_id[L]] = res;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    for (int k = P.depth - 1; k >= 0; --k) {
      for (int j = threadIdx.x; j < (1 << k); j += 32) {
        const int hh = (1 << k) + j;
        if (P.kind[hh] == 2) P.hsum[hh] = BT_ADD(P.hsum[2 * hh], P.hsum[2 * hh + 1]);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  const float total = P.hsum[1];
  __syncthreads();  // P may be reused by the caller's next sum
  return total;
}

// np.max-style block maximum (NaN propagates).
__device__ float block_max(const float* s, int n, float* red) {
  float m = -INFINITY;
  bool nan = false;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = s[i];
    if (v != v) nan = true;
    m = fmaxf(m, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    nan |= __shfl_xor_sync(0xffffffffu, (int)nan, o) != 0;
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = nan ? qnan() : m;
  __syncthreads();
  float r = -INFINITY;
  bool rn = false;
  for (int i = 0; i < nw; ++i) { float v = red[i]; if (v != v) rn = true; r = fmaxf(r, v); }
  __syncthreads();
  return rn ? qnan() : r;
}

// ---- row staging --------------------------------------------------------------

// First element index at which g is 16-byte aligned, and the number of
// 4-element vectors after it.
struct RowSplit { int head, nvec; };
__device__ __forceinline__ RowSplit row_split(const float* g, int n) {
  RowSplit r;
  r.head = (4 - phase4(g)) & 3;
  if (r.head > n) r.head = n;
  r.nvec = (n - r.head) / 4;
  return r;
}

// s[i] = g0[i] (+ g1[i] (+ g2[i])) for i < n; optionally also res[i] = s[i].
// s must share g0's 16-byte phase.  Sources with another phase, and the
// residual output when its phase differs, fall back to scalar accesses.
__device__ void stage_row(float* s, const float* g0, const float* g1, const float* g2, int n, float* res) {
  const RowSplit sp = row_split(g0, n);
  const bool v1 = g1 && phase4(g1) == phase4(g0);
  const bool v2 = g2 && phase4(g2) == phase4(g0);
  const bool vr = res && phase4(res) == phase4(g0);
  for (int i = threadIdx.x; i < sp.head; i += blockDim.x) {
    float v = g0[i];
    if (g1) v = BT_ADD(v, g1[i]);
    if (g2) v = BT_ADD(v, g2[i]);
    s[i] = v;
    if (res) res[i] = v;
  }
  for (int q = threadIdx.x; q < sp.nvec; q += blockDim.x) {
    const int i = sp.head + 4 * q;
    float4 v = __ldcs((const float4*)(g0 + i));
    if (g1) {
      float4 w = v1 ? __ldcs((const float4*)(g1 + i)) : make_float4(g1[i], g1[i + 1], g1[i + 2], g1[i + 3]);
      v.x = BT_ADD(v.x, w.x); v.y = BT_ADD(v.y, w.y); v.z = BT_ADD(v.z, w.z); v.w = BT_ADD(v.w, w.w);
    }
    if (g2) {
      float4 w = v2 ? __ldcs((const float4*)(g2 + i)) : make_float4(g2[i], g2[i + 1], g2[i + 2], g2[i + 3]);
      v.x = BT_ADD(v.x, w.x); v.y = BT_ADD(v.y, w.y); v.z = BT_ADD(v.z, w.z); v.w = BT_ADD(v.w, w.w);
    }
    *(float4*)(s + i) = v;
    if (res) {
      if (vr) __stcs((float4*)(res + i), v);
      else { res[i] = v.x; res[i + 1] = v.y; res[i + 2] = v.z; res[i + 3] = v.w; }
    }
  }
  for (int i = sp.head + 4 * sp.nvec + threadIdx.x; i < n; i += blockDim.x) {
    float v = g0[i];
    if (g1) v = BT_ADD(v, g1[i]);
    if (g2) v = BT_ADD(v, g2[i]);
    s[i] = v;
    if (res) res[i] = v;
  }
}

// Shared row buffer aligned to g's 16-byte phase.
__device__ __forceinline__ float* row_buffer(unsigned char* smem, const void* g) {
  return (float*)smem + phase4(g);
}

// Dynamic shared memory layout: [row buffer: n + 4 floats][32 floats][plan].
__host__ __device__ inline size_t row_smem_bytes(int n, int D) {
  size_t rowb = ((size_t)n + 4) * sizeof(float);
  rowb = (rowb + 15) & ~(size_t)15;
  return rowb + 32 * sizeof(float) + plan_bytes(D);
}
__device__ inline float* red_area(unsigned char* smem, int n) {
  size_t rowb = (((size_t)n + 4) * sizeof(float) + 15) & ~(size_t)15;
  return (float*)(smem + rowb);
}
__device__ inline unsigned char* plan_area(unsigned char* smem, int n) {
  return (unsigned char*)(red_area(smem, n) + 32);
}

// ---- kernels ---------------------------------------------------------------------
struct ReduceRowsArgs {
  const void* x;
  int32_t xdt;        // BT_F32 or BT_F16 (widened exactly)
  int32_t mean;
  int32_t n, depth;
  int64_t rows;
  float* out;
};

__global__ void reduce_rows_kernel(ReduceRowsArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = a.n;
  PwPlan P = plan_at(plan_area(smem, n), a.depth);
  pw_build(P, n);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    float* s;
    if (a.xdt == BT_F32) {
      const float* g = (const float*)a.x + row * (int64_t)n;
      s = row_buffer(smem, g);
      stage_row(s, g, nullptr, nullptr, n, nullptr);
    } else {
      const __half* g = (const __half*)a.x + row * (int64_t)n;
      s = (float*)smem;
      for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = __half2float(g[i]);
    }
    __syncthreads();
    const float sum = BT_ADD(0.0f, pw_sum(s, P, PwIdentity(), ((uintptr_t)s & 15) == 0));
    if (threadIdx.x == 0) a.out[row] = a.mean ? np_mean_from_sum(sum, n) : sum;
  }
}

// Reduction of the middle axis of a contiguous [O, R, I] view: numpy adds the
// R slices one after another into the output (its inner loop runs along I).
struct ReduceColsArgs {
  const void* x;
  int32_t xdt;
  int32_t mean;
  int64_t O, R, I;
  float* out;
};
__global__ void reduce_cols_kernel(ReduceColsArgs a) {
  const int64_t total = a.O * a.I;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = idx / a.I, i = idx - o * a.I;
    int64_t p = o * a.R * a.I + i;
    float acc = 0.0f;
    if (a.xdt == BT_F32) {
      const float* x = (const float*)a.x;
      for (int64_t r = 0; r < a.R; ++r, p += a.I) acc = BT_ADD(acc, __ldg(x + p));
    } else {
      const __half* x = (const __half*)a.x;
      for (int64_t r = 0; r < a.R; ++r, p += a.I) acc = BT_ADD(acc, __half2float(x[p]));
    }
    a.out[idx] = a.mean ? np_mean_from_sum(acc, a.R) : acc;
  }
}

// floor(n / d) for a fixed d and every n < 2^32 by a multiply and a shift
// (the round-up method of Granlund and Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1 (below 2^32), floor(n / d) =
// (umulhi(m, n) + n) >> l, the sum formed in 64 bits.
struct FastDiv {
  uint32_t d, m, l;
};
inline FastDiv fast_div_for(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, l};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)__umulhi(f.m, n) + n) >> f.l);
}

struct SoftmaxArgs {
  const float* x;
  const float* mask;                 // may be null
  int32_t n, depth;
  int64_t rows;
  int32_t lead_rank;                 // rank of x's leading (row) axes
  int64_t lead_shape[BT_MAX_RANK];
  int64_t mask_lead_st[BT_MAX_RANK]; // mask stride per leading axis (0 = broadcast)
  int64_t mask_col_st;               // mask stride along the softmax axis (0 or 1)
  int32_t mask_row_const;            // 1: every leading stride is 0 (one mask row for all rows)
  // the leading axes collapsed for the mask row's offset (innermost first;
  // axes of extent 1 dropped, neighbours merged where the mask's strides
  // allow): set for fewer than 2^32 rows, read by the warp-row kernels
  int32_t mnd;
  FastDiv mdiv[BT_MAX_RANK];
  int64_t mst[BT_MAX_RANK];
  float* out;
};

// Offset of row `row`'s mask row (row < 2^32; the collapsed axes above).
__device__ __forceinline__ long long mask_row_offset(const SoftmaxArgs& a, uint32_t row) {
  long long moff = 0;
  uint32_t rem = row;
  for (int d = 0; d < a.mnd; ++d) {
    const uint32_t q = fast_div(rem, a.mdiv[d]);
    moff += (long long)(rem - q * a.mdiv[d].d) * a.mst[d];
    rem = q;
  }
  return moff;
}

__global__ void softmax_rows_kernel(SoftmaxArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = a.n;
  PwPlan P = plan_at(plan_area(smem, n), a.depth);
  float* red = red_area(smem, n);
  pw_build(P, n);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const float* g = a.x + row * (int64_t)n;
    float* s = row_buffer(smem, g);
    stage_row(s, g, nullptr, nullptr, n, nullptr);
    if (a.mask) {
      __syncthreads();
      int64_t rem = row, moff = 0;
      for (int d = a.lead_rank - 1; d >= 0; --d) {
        const int64_t c = rem % a.lead_shape[d];
        rem /= a.lead_shape[d];
        moff += c * a.mask_lead_st[d];
      }
      for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = BT_ADD(s[i], a.mask[moff + i * a.mask_col_st]);
    }
    __syncthreads();
    const float m = block_max(s, n, red);
    for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = np_expf(BT_SUB(s[i], m));
    __syncthreads();
    const float denom = BT_ADD(0.0f, pw_sum(s, P, PwIdentity(), ((uintptr_t)s & 15) == 0));
    const double rd = recip_d(denom);
    float* o = a.out + row * (int64_t)n;
    const RowSplit sp = row_split(o, n);
    const bool vec = phase4(o) == phase4(g);
    if (vec) {
      for (int i = threadIdx.x; i < sp.head; i += blockDim.x) o[i] = div_by(s[i], rd);
      for (int q = threadIdx.x; q < sp.nvec; q += blockDim.x) {
        const int i = sp.head + 4 * q;
        float4 v = *(const float4*)(s + i);
        __stcs((float4*)(o + i), make_float4(div_by(v.x, rd), div_by(v.y, rd), div_by(v.z, rd), div_by(v.w, rd)));
      }
      for (int i = sp.head + 4 * sp.nvec + threadIdx.x; i < n; i += blockDim.x) o[i] = div_by(s[i], rd);
    } else {
      for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = div_by(s[i], rd);
    }
    __syncthreads();
  }
}

struct LayerNormArgs {
  const float* x;
  const float* skip;      // [rows, n] or null
  const float* bias;      // [n] or null (added after skip)
  const void* gamma;      // [n]
  const void* beta;       // [n] or null
  int32_t gdt, bdt;       // dtypes of gamma / beta (F32 or F16)
  int32_t n, depth;
  int64_t rows;
  float eps;
  float* out;
};

__device__ __forceinline__ float ldf(const void* p, int dt, int64_t i) {
  return dt == BT_F16 ? __half2float(((const __half*)p)[i]) : ((const float*)p)[i];
}

__global__ void layernorm_rows_kernel(LayerNormArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = a.n;
  PwPlan P = plan_at(plan_area(smem, n), a.depth);
  pw_build(P, n);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const float* g = a.x + row * (int64_t)n;
    float* s = row_buffer(smem, g);
    stage_row(s, g, a.skip ? a.skip + row * (int64_t)n : nullptr, nullptr, n, nullptr);
    if (a.bias) {
      __syncthreads();
      for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = BT_ADD(s[i], a.bias[i]);
    }
    __syncthreads();
    const bool al = ((uintptr_t)s & 15) == 0;
    const float mu = np_mean_from_sum(BT_ADD(0.0f, pw_sum(s, P, PwIdentity(), al)), n);
    const float var = np_mean_from_sum(BT_ADD(0.0f, pw_sum(s, P, PwSquaredDev{mu}, al)), n);
    const float sd = BT_SQRT(BT_ADD(var, a.eps));
    const double rsd = recip_d(sd);
    float* o = a.out + row * (int64_t)n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float y = BT_MUL(div_by(BT_SUB(s[i], mu), rsd), ldf(a.gamma, a.gdt, i));
      if (a.beta) y = BT_ADD(y, ldf(a.beta, a.bdt, i));
      o[i] = y;
    }
    __syncthreads();
  }
}

struct AdainArgs {
  bt_adain_args p;
  int32_t depth;
  int32_t n;
};

__global__ void adain_snake_kernel(AdainArgs A) {
  extern __shared__ __align__(16) unsigned char smem[];
  // Scalars and per-output pointers are read from the parameter block with
  // compile-time indices (no reference to the parameter block is taken).
  const int n = A.n;
  const int64_t rows = A.p.rows, channels = A.p.channels;
  const int n_src = A.p.n_src, n_out = A.p.n_out, adt = A.p.alpha_dtype;
  const int64_t gstride = A.p.gain_stride, sstride = A.p.shift_stride;
  const float eps = A.p.eps;
  const float* src0 = A.p.src[0];
  const float* src1 = A.p.src[1];
  const float* src2 = A.p.src[2];
  float* resp = A.p.res;
  PwPlan P = plan_at(plan_area(smem, n), A.depth);
  pw_build(P, n);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * (int64_t)n;
    const float* g0 = src0 + base;
    float* s = row_buffer(smem, g0);
    stage_row(s, g0, n_src > 1 ? src1 + base : nullptr, n_src > 2 ? src2 + base : nullptr, n,
              resp ? resp + base : nullptr);
    __syncthreads();
    // ReduceMean -> Sub -> Mul(d, d) -> ReduceMean -> Add eps -> Sqrt
    const bool al = ((uintptr_t)s & 15) == 0;
    const float mu = np_mean_from_sum(BT_ADD(0.0f, pw_sum(s, P, PwIdentity(), al)), n);
    const float var = np_mean_from_sum(BT_ADD(0.0f, pw_sum(s, P, PwSquaredDev{mu}, al)), n);
    const float sd = BT_SQRT(BT_ADD(var, eps));
    const double rsd = recip_d(sd);
    const int64_t c = row % channels, b = row / channels;
    const RowSplit sp = row_split(g0, n);
#pragma unroll
    for (int k = 0; k < BT_ADAIN_MAX_OUT; ++k) {
      if (k >= n_out) break;
      const float gain = A.p.gain[k][b * gstride + c], shift = A.p.shift[k][b * sstride + c];
      const void* alpha_k = A.p.alpha[k];
      const bool snake = alpha_k != nullptr;
      float al = 0.f, ial = 0.f;
      if (snake) {
        al = ldf(alpha_k, adt, c);
        ial = ldf(A.p.inv_alpha[k], adt, c);
      }
      float* o = A.p.out[k] + base;
      // Sub -> Div -> Mul(1+gamma) -> Add(beta) [-> Mul(alpha) -> Sin -> Pow 2 -> Mul(1/alpha) -> Add]
      auto f = [&](float v) -> float {
        float y = BT_ADD(BT_MUL(gain, div_by(BT_SUB(v, mu), rsd)), shift);
        if (!snake) return y;
        const float t = np_sinf(BT_MUL(al, y));
        return BT_ADD(y, BT_MUL(ial, BT_MUL(t, t)));
      };
      if (phase4(o) == phase4(g0)) {
        for (int i = threadIdx.x; i < sp.head; i += blockDim.x) o[i] = f(s[i]);
        for (int q = threadIdx.x; q < sp.nvec; q += blockDim.x) {
          const int i = sp.head + 4 * q;
          const float4 d = *(const float4*)(s + i);
          __stcs((float4*)(o + i), make_float4(f(d.x), f(d.y), f(d.z), f(d.w)));
        }
        for (int i = sp.head + 4 * sp.nvec + threadIdx.x; i < n; i += blockDim.x) o[i] = f(s[i]);
      } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = f(s[i]);
      }
    }
    __syncthreads();
  }
}

struct MeanLeakyArgs {
  const float* a[3];
  const float* b[3];
  int64_t n;
  double rdiv;    // RN64(1 / divisor)
  float slope;
  float* out;
};

__device__ __forceinline__ float mean_leaky(float a0, float b0, float a1, float b1, float a2, float b2,
                                            double rdiv, float slope) {
  float v = BT_ADD(BT_ADD(BT_ADD(a0, b0), BT_ADD(a1, b1)), BT_ADD(a2, b2));
  v = div_by(v, rdiv);
  return v < 0.0f ? BT_MUL(v, slope) : v;
}

__global__ void __launch_bounds__(256) mean_leaky_kernel(MeanLeakyArgs m) {
  const int64_t nv = m.n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const int64_t i = 4 * v;
    float4 x[6];
    x[0] = __ldcs((const float4*)(m.a[0] + i)); x[1] = __ldcs((const float4*)(m.b[0] + i));
    x[2] = __ldcs((const float4*)(m.a[1] + i)); x[3] = __ldcs((const float4*)(m.b[1] + i));
    x[4] = __ldcs((const float4*)(m.a[2] + i)); x[5] = __ldcs((const float4*)(m.b[2] + i));
    float4 r;
    r.x = mean_leaky(x[0].x, x[1].x, x[2].x, x[3].x, x[4].x, x[5].x, m.rdiv, m.slope);
    r.y = mean_leaky(x[0].y, x[1].y, x[2].y, x[3].y, x[4].y, x[5].y, m.rdiv, m.slope);
    r.z = mean_leaky(x[0].z, x[1].z, x[2].z, x[3].z, x[4].z, x[5].z, m.rdiv, m.slope);
    r.w = mean_leaky(x[0].w, x[1].w, x[2].w, x[3].w, x[4].w, x[5].w, m.rdiv, m.slope);
    __stcs((float4*)(m.out + i), r);
  }
  for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m.n; i += stride)
    m.out[i] = mean_leaky(m.a[0][i], m.b[0][i], m.a[1][i], m.b[1][i], m.a[2][i], m.b[2][i], m.rdiv, m.slope);
}

__global__ void mean_leaky_scalar_kernel(MeanLeakyArgs m) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m.n; i += stride)
    m.out[i] = mean_leaky(m.a[0][i], m.b[0][i], m.a[1][i], m.b[1][i], m.a[2][i], m.b[2][i], m.rdiv, m.slope);
}

// ---- launch helpers ----------------------------------------------------------------
constexpr int kMaxDevices = 64;
std::atomic<int> g_smem_ready[kMaxDevices];

int raise_smem_limits() {
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  if (di.device >= kMaxDevices) return set_error(BT_EUNSUPPORTED, "device ordinal %d >= %d", di.device, kMaxDevices);
  if (g_smem_ready[di.device].load()) return BT_OK;
  const void* fns[] = {(const void*)reduce_rows_kernel, (const void*)softmax_rows_kernel,
                       (const void*)layernorm_rows_kernel, (const void*)adain_snake_kernel};
  for (const void* f : fns) {
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, di.max_smem_optin);
    if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  g_smem_ready[di.device].store(1);
  return BT_OK;
}

int row_threads(int n) {
  if (n <= 1024) return 128;
  if (n <= 8192) return 256;
  return 512;
}

int row_launch_check(int n, size_t* smem, int* depth) {
  if (n > kMaxRow)
    return set_error(BT_ETOOBIG, "row of %d values exceeds the %d-value limit of one CTA", n, kMaxRow);
  int rc = raise_smem_limits();
  if (rc) return rc;
  *depth = pw_depth(n);
  *smem = row_smem_bytes(n, *depth);
  DevInfo di;
  dev_info(&di);
  if ((int64_t)*smem > di.max_smem_optin)
    return set_error(BT_ETOOBIG, "row needs %zu bytes of shared memory (device allows %d)", *smem, di.max_smem_optin);
  return BT_OK;
}

int row_grid(int64_t rows) {
  int64_t g = rows < 1 ? 1 : rows;
  if (g > 2147483647) g = 2147483647;
  return (int)g;
}

// ---- warp-per-row kernels --------------------------------------------------
// Rows of at most kWarpRowMax values (softmax over 510 keys, layer norm over
// 768 channels, means over 2048 frames) are too short to keep a CTA busy:
// here one warp owns a row end to end.  It stages the row into its own slice
// of shared memory with cp.async, sums numpy's pairwise tree from a plan the
// host built once per row length (four groups of eight lanes, one leaf per
// group at a time, lane j holding numpy's accumulator j), combines the tree
// in registers (perfect trees) or level by level, and writes the outputs.
// Only warp-level synchronisation; eight independent rows per CTA.
constexpr int kWarpRowMax = 2048;   // -> at most 32 leaves, depth <= 5
constexpr int kWarpLeaves = 32;
constexpr int kWarpHeap = 64;       // heap ids < 2^(D+1) <= 64
constexpr int kWarpsPerCta = 8;

struct WPlan {
  int32_t n, D, n_leaf, perfect;     // perfect: every leaf at depth D
  uint32_t inner[2];                 // bit h: heap node h is an inner node
  uint16_t off[kWarpLeaves];         // leaf offsets, in row order
  uint8_t len[kWarpLeaves];          // leaf lengths (<= 128)
  uint8_t id[kWarpLeaves];           // heap ids (< 64)
};

// The plan as the kernels read it: copied once per CTA into shared memory
// (lane-divergent reads of a kernel parameter array would be serialised).
struct WView {
  const uint16_t* off;
  const uint8_t* len;
  const uint8_t* id;
  const uint32_t* inner;
  int n, D, n_leaf, perfect;
};
struct WShared {
  uint16_t off[kWarpLeaves];
  uint8_t len[kWarpLeaves];
  uint8_t id[kWarpLeaves];
  uint32_t inner[2];
};
__device__ __forceinline__ WView wplan_load(const WPlan& P, WShared& sh) {
  for (int i = threadIdx.x; i < P.n_leaf; i += blockDim.x) {
    sh.off[i] = P.off[i];
    sh.len[i] = P.len[i];
    sh.id[i] = P.id[i];
  }
  if (threadIdx.x < 2) sh.inner[threadIdx.x] = P.inner[threadIdx.x];
  __syncthreads();
  WView v;
  v.off = sh.off; v.len = sh.len; v.id = sh.id; v.inner = sh.inner;
  v.n = P.n; v.D = P.D; v.n_leaf = P.n_leaf; v.perfect = P.perfect;
  return v;
}

// Floats of one warp's shared slice: the heap, then the row (+ 4 for the
// 16-byte phase), rounded to 16 bytes.
__host__ __device__ inline int wrow_stride(int n) { return kWarpHeap + (((n + 4) + 3) & ~3); }

// Root of the pairwise tree whose leaf sums the warp's lanes have written
// into heap (all 32 lanes call; every lane returns the root, and the heap is
// free again on return).
__device__ __forceinline__ float warp_heap_total(const WView& P, float* heap) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  float total;
  if (P.perfect) {
    const int nl = 1 << P.D;                // leaf i sits at heap id nl + i
    total = lane < nl ? heap[nl + lane] : 0.0f;
    for (int m = 1; m < nl; m <<= 1) total = BT_ADD(total, __shfl_xor_sync(0xffffffffu, total, m));
    // with fewer than 32 leaves only lanes < nl hold the root: share lane 0's
    total = __shfl_sync(0xffffffffu, total, 0);
  } else {
    for (int k = P.D - 1; k >= 0; --k) {
      for (int jj = lane; jj < (1 << k); jj += 32) {
        const int h = (1 << k) + jj;
        if ((P.inner[h >> 5] >> (h & 31)) & 1u) heap[h] = BT_ADD(heap[2 * h], heap[2 * h + 1]);
      }
      __syncwarp();
    }
    total = heap[1];
  }
  __syncwarp();                             // the heap is reused by the next sum
  return total;
}

// numpy's pairwise sum of f(row[i]) over the whole row (all 32 lanes call;
// every lane returns the sum, before numpy's "+ 0.0").  A row starting on an
// 8-byte boundary is summed by groups of four lanes, lane j holding numpy's
// accumulators r[2j] and r[2j+1] as one float2 (eight leaves at a time, one
// 64-bit load and one two-lane add per step); otherwise by groups of eight
// lanes, lane j holding r[j].  f.two(acc, v) adds the transformed pair v to
// acc; f(v) transforms one value.
template <class F>
__device__ __forceinline__ float warp_pw_sum(const WView& P, const float* row, float* heap, F f) {
  const int lane = threadIdx.x & 31;
  if (((uintptr_t)row & 7) == 0) {
    const int j = lane & 3, g = lane >> 2;
    const unsigned gmask = 0xfu << (lane & 28);
    for (int L = g; L < P.n_leaf; L += 8) {
      const int off = P.off[L], len = P.len[L];
      const int steps = len >> 3, end = steps << 3;
      const float2* q = reinterpret_cast<const float2*>(row + off + 2 * j);
      float2 acc = pk(-0.0f);               // -0.0 + x == x: acc starts as numpy's r[j] = a[j]
#pragma unroll 4
      for (int m = 0; m < steps; ++m) acc = f.two(acc, q[4 * m]);
      // numpy's bracket ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)); addition commutes
      float t = BT_ADD(acc.x, acc.y);
      t = BT_ADD(t, __shfl_xor_sync(gmask, t, 1));
      t = BT_ADD(t, __shfl_xor_sync(gmask, t, 2));
      if (steps == 0) t = 0.0f;             // a run shorter than 8 is summed from +0.0
      if (len > end) {
        if (j == 0)
          for (int i = end; i < len; ++i) t = BT_ADD(t, f(row[off + i]));
        t = __shfl_sync(gmask, t, 0, 4);
      }
      if (j == 0) heap[P.id[L]] = t;
    }
    return warp_heap_total(P, heap);
  }
  const int j = lane & 7, g = lane >> 3;
  const unsigned gmask = 0xffu << (lane & 24);
  for (int L = g; L < P.n_leaf; L += 4) {
    const int off = P.off[L], len = P.len[L];
    const int steps = len >> 3, end = steps << 3;
    const float* q = row + off + j;
    float acc = -0.0f;
#pragma unroll 4
    for (int m = 0; m < steps; ++m) acc = BT_ADD(acc, f(q[8 * m]));
    acc = BT_ADD(acc, __shfl_xor_sync(gmask, acc, 1));
    acc = BT_ADD(acc, __shfl_xor_sync(gmask, acc, 2));
    acc = BT_ADD(acc, __shfl_xor_sync(gmask, acc, 4));
    if (steps == 0) acc = 0.0f;
    if (len > end) {
      if (j == 0)
        for (int i = end; i < len; ++i) acc = BT_ADD(acc, f(row[off + i]));
      acc = __shfl_sync(gmask, acc, 0, 8);
    }
    if (j == 0) heap[P.id[L]] = acc;
  }
  return warp_heap_total(P, heap);
}

struct WReduceArgs {
  WPlan P;
  const void* x;
  int32_t xdt, mean;
  int64_t rows;
  float* out;
};
struct WSoftmaxArgs {
  WPlan P;
  SoftmaxArgs a;
};
struct WLayerNormArgs {
  WPlan P;
  LayerNormArgs a;
};

// This warp's heap and row slice; the row buffer shares g's 16-byte phase.
struct WSlice {
  float* heap;
  float* slice;
};
__device__ __forceinline__ WSlice warp_slice(unsigned char* smem, int n) {
  WSlice w;
  w.heap = reinterpret_cast<float*>(smem) + (threadIdx.x >> 5) * wrow_stride(n);
  w.slice = w.heap + kWarpHeap;
  return w;
}

// Calls body(row, b) for this warp's rows (one per warp on a full grid, more
// when the grid is smaller) with b = the staged copy of src(row).
template <class Src, class Body>
__device__ __forceinline__ void warp_rows(const WSlice& W, int n, int64_t rows, Src src, Body body) {
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerCta) {
    const float* g = src(row);
    float* b = W.slice + phase4(g);
    stage_floats_async(b, g, n, lane, 32);
    cp_async_wait_all();
    __syncwarp();
    body(row, b);
    __syncwarp();   // the slice is reused by this warp's next row
  }
}

__global__ void __launch_bounds__(256) wrow_reduce_kernel(WReduceArgs A) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ WShared sh;
  const WView P = wplan_load(A.P, sh);
  const int lane = threadIdx.x & 31, n = P.n;
  const WSlice W = warp_slice(smem, n);
  auto finish = [&](int64_t row, const float* b) {
    const float sum = BT_ADD(0.0f, warp_pw_sum(P, b, W.heap, PwIdentity()));
    if (lane == 0) A.out[row] = A.mean ? np_mean_from_sum(sum, n) : sum;
  };
  if (A.xdt == BT_F32) {
    const float* x = (const float*)A.x;
    warp_rows(W, n, A.rows, [&](int64_t row) { return x + row * n; }, finish);
    return;
  }
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5); row < A.rows;
       row += (int64_t)gridDim.x * kWarpsPerCta) {
    const __half* g = (const __half*)A.x + row * n;
    for (int i = lane; i < n; i += 32) W.slice[i] = __half2float(g[i]);
    __syncwarp();
    finish(row, W.slice);
    __syncwarp();
  }
}

// Rows of NL x 128 float32 (1024 or 2048 values), whose pairwise tree is
// perfect with 128-value leaves, summed straight from global memory: lane
// j of group g (four lanes per leaf) holds numpy's accumulators r[2j],
// r[2j+1] of leaves g and g + 8 as float2 and adds step m of each (one
// 8-byte load per leaf and step: a warp load covers eight leaves, 32 bytes
// each), the same additions in the same order as warp_pw_sum's float2 path.
// No shared memory, so occupancy is not bound by staging whole rows.
template <int NL>
__global__ void __launch_bounds__(256) wrow_reduce_direct_kernel(const float* x, int mean, int64_t rows, float* out) {
  constexpr int LPG = NL / 8;   // leaves per lane group
  const int lane = threadIdx.x & 31, g = lane >> 2, j = lane & 3;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerCta) {
    const float2* r = reinterpret_cast<const float2*>(x + row * (int64_t)(NL * 128));
    float2 acc[LPG];
#pragma unroll
    for (int t = 0; t < LPG; ++t) acc[t] = pk(-0.0f);   // -0.0 + x == x: acc starts as numpy's r[j] = a[j]
#pragma unroll
    for (int m = 0; m < 16; ++m)
#pragma unroll
      for (int t = 0; t < LPG; ++t) acc[t] = pk_add(acc[t], __ldcs(r + (g + 8 * t) * 64 + 4 * m + j));
    // numpy's bracket ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) per leaf
    float ls[LPG];
#pragma unroll
    for (int t = 0; t < LPG; ++t) {
      float v = BT_ADD(acc[t].x, acc[t].y);
      v = BT_ADD(v, __shfl_xor_sync(0xffffffffu, v, 1));
      v = BT_ADD(v, __shfl_xor_sync(0xffffffffu, v, 2));
      ls[t] = v;
    }
    // leaf L's sum into lane L, then the perfect tree by xor shuffles (as
    // warp_heap_total sums a perfect tree)
    const float v0 = __shfl_sync(0xffffffffu, ls[0], 4 * (lane & 7));
    const float v1 = __shfl_sync(0xffffffffu, ls[LPG - 1], 4 * (lane & 7));
    float total = lane < 8 ? v0 : (lane < NL ? v1 : 0.0f);
#pragma unroll
    for (int m = 1; m < NL; m <<= 1) total = BT_ADD(total, __shfl_xor_sync(0xffffffffu, total, m));
    if (lane == 0) {
      const float sum = BT_ADD(0.0f, total);
      out[row] = mean ? np_mean_from_sum(sum, NL * 128) : sum;
    }
  }
}

// Writes o[i] = f(b[i]) for the row, 128-bit where o shares g's phase.
template <class F>
__device__ __forceinline__ void warp_write(float* o, const float* b, const float* g, int n, F f) {
  const int lane = threadIdx.x & 31;
  if (phase4(o) == phase4(g)) {
    int head = (4 - phase4(o)) & 3;
    if (head > n) head = n;
    const int nvec = (n - head) >> 2;
    for (int i = lane; i < head; i += 32) o[i] = f(b[i], i);
    for (int q = lane; q < nvec; q += 32) {
      const int i = head + 4 * q;
      const float4 v = *reinterpret_cast<const float4*>(b + i);
      __stcs(reinterpret_cast<float4*>(o + i), make_float4(f(v.x, i), f(v.y, i + 1), f(v.z, i + 2), f(v.w, i + 3)));
    }
    for (int i = head + 4 * nvec + lane; i < n; i += 32) o[i] = f(b[i], i);
  } else {
    for (int i = lane; i < n; i += 32) o[i] = f(b[i], i);
  }
}

__global__ void __launch_bounds__(256) wrow_softmax_kernel(WSoftmaxArgs A) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ WShared sh;
  const WView P = wplan_load(A.P, sh);
  const SoftmaxArgs& a = A.a;
  const int lane = threadIdx.x & 31, n = P.n;
  const WSlice W = warp_slice(smem, n);
  const float* x = a.x;
  warp_rows(W, n, a.rows, [&](int64_t row) { return x + row * (int64_t)n; }, [&](int64_t row, float* b) {
    const float* mr = nullptr;
    if (a.mask) {
      // the mask row of this row (the host sends this kernel fewer than
      // 2^32 rows)
      mr = a.mask + (a.mask_row_const ? 0ll : mask_row_offset(a, (uint32_t)row));
    }
    // the mask Add (when fused) and the row maximum in one pass.  fmaxf
    // skips NaN where np.max returns it, but the row's result is all NaN
    // either way: a NaN element's exp is NaN, so the sum and every quotient
    // are NaN (and with no NaN both maxima are the same float).
    // 128-bit over the slice's aligned interior [head, head + 4 nvec)
    int head = (4 - phase4(b)) & 3;
    if (head > n) head = n;
    const int nvec = (n - head) >> 2, tail0 = head + 4 * nvec;
    const bool mvec = mr && a.mask_col_st == 1 && phase4(mr) == phase4(b);
    float m = -INFINITY;
    if (mr && a.mask_col_st) {
      for (int i = lane; i < n; i += 32) {
        if (mvec && i >= head && i < tail0) continue;
        const float v = BT_ADD(b[i], mr[i * a.mask_col_st]);
        b[i] = v;
        m = fmaxf(m, v);
      }
      if (mvec) {
        for (int q = lane; q < nvec; q += 32) {
          float4 v = *reinterpret_cast<const float4*>(b + head + 4 * q);
          const float4 w = __ldg(reinterpret_cast<const float4*>(mr + head + 4 * q));
          v = make_float4(BT_ADD(v.x, w.x), BT_ADD(v.y, w.y), BT_ADD(v.z, w.z), BT_ADD(v.w, w.w));
          *reinterpret_cast<float4*>(b + head + 4 * q) = v;
          m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
        }
      }
    } else {
      const float mv = mr ? mr[0] : 0.0f;
      for (int i = lane; i < head; i += 32) {
        const float v = mr ? BT_ADD(b[i], mv) : b[i];
        b[i] = v;
        m = fmaxf(m, v);
      }
      for (int q = lane; q < nvec; q += 32) {
        float4 v = *reinterpret_cast<const float4*>(b + head + 4 * q);
        if (mr) {
          v = make_float4(BT_ADD(v.x, mv), BT_ADD(v.y, mv), BT_ADD(v.z, mv), BT_ADD(v.w, mv));
          *reinterpret_cast<float4*>(b + head + 4 * q) = v;
        }
        m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
      }
      for (int i = tail0 + lane; i < n; i += 32) {
        const float v = mr ? BT_ADD(b[i], mv) : b[i];
        b[i] = v;
        m = fmaxf(m, v);
      }
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncwarp();
    // exp(x - max) (x - m == x + (-m)), 128-bit over the interior
    const float2 nm = pk(-m);
    for (int i = lane; i < head; i += 32) b[i] = np_expf(BT_SUB(b[i], m));
    for (int q = lane; q < nvec; q += 32) {
      const float4 v = *reinterpret_cast<const float4*>(b + head + 4 * q);
      const float2 lo = pk_np_exp(pk_add(pk(v.x, v.y), nm)), hi = pk_np_exp(pk_add(pk(v.z, v.w), nm));
      *reinterpret_cast<float4*>(b + head + 4 * q) = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    for (int i = tail0 + lane; i < n; i += 32) b[i] = np_expf(BT_SUB(b[i], m));
    __syncwarp();
    const float denom = BT_ADD(0.0f, warp_pw_sum(P, b, W.heap, PwIdentity()));
    const double rd = recip_d(denom);
    warp_write(a.out + row * (int64_t)n, b, x + row * (int64_t)n, n, [=](float v, int) { return div_by(v, rd); });
  });
}

// ---- register-resident rows -----------------------------------------------------
// Rows of a compile-time length N (softmax over ALBERT's 510-key attention
// rows, layer norm over its 768 channels): one warp per row, the row held in
// registers.  Lane l = 4G + p (group G of four lanes, position p) holds, in
// slot k < NS, the pair of elements 8b + 2p and +1 of block b = NS G + k:
// the eight values of a block sit in the four lanes of one group, two each,
// which is the layout of numpy's eight pairwise accumulators.  numpy's tree
// over the row (pw_split) is unrolled at compile time: a leaf's accumulator
// pairs run down its blocks within a group (one two-lane add per block) and
// hop to the next group with one shuffle; the bracket
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) is two shuffles; the leftover values
// of a leaf are gathered in order.  No shared memory, no loop over leaves,
// no plan: every index is a constant.
__host__ __device__ constexpr int pw_split_c(int n) { return n / 2 - (n / 2) % 8; }

// max of three floats in one instruction (sm_100); NaN operands are skipped
// as fmaxf skips them
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

struct RegIdentity {
  static constexpr bool kPacked = true;
  __device__ __forceinline__ float2 operator()(float2 v) const { return v; }
};
// (v - mu)^2 of both lanes, each step rounded on its own (numpy's x - mu,
// then ** 2, which is x * x)
struct RegSquaredDev {
  static constexpr bool kPacked = false;
  float mu;
  __device__ __forceinline__ float2 operator()(float2 v) const {
    const float dx = BT_SUB(v.x, mu), dy = BT_SUB(v.y, mu);
    return make_float2(BT_MUL(dx, dx), BT_MUL(dy, dy));
  }
};

// numpy's sum of f(values) over the leaf [OFF, OFF + LEN) (OFF a multiple of
// 8), the same value in every lane.
template <int NS, int LEN, int OFF, class F>
__device__ __forceinline__ float reg_leaf_sum(const float2 (&v)[NS], F f) {
  constexpr int b0 = OFF / 8, nb = LEN / 8, R = LEN % 8;
  float res = 0.0f;                       // a run shorter than 8 starts from +0.0
  if constexpr (nb > 0) {
    float2 acc = f(v[b0 % NS]);           // r[j] = a[j] (held by group b0 / NS)
#pragma unroll
    for (int b = b0 + 1; b < b0 + nb; ++b) {
      if (b % NS == 0) {                  // the next block sits in the next group
        acc.x = __shfl_up_sync(0xffffffffu, acc.x, 4);
        acc.y = __shfl_up_sync(0xffffffffu, acc.y, 4);
      }
      const float2 t = f(v[b % NS]);
      // two lanes per add where no product feeds it (a packed product
      // feeding a packed add may be contracted into one FMA)
      acc = F::kPacked ? pk_add(acc, t) : make_float2(BT_ADD(acc.x, t.x), BT_ADD(acc.y, t.y));
    }
    float t = BT_ADD(acc.x, acc.y);
    t = BT_ADD(t, __shfl_xor_sync(0xffffffffu, t, 1));
    t = BT_ADD(t, __shfl_xor_sync(0xffffffffu, t, 2));
    res = __shfl_sync(0xffffffffu, t, 4 * ((b0 + nb - 1) / NS));
  }
  if constexpr (R > 0) {
    constexpr int bR = b0 + nb;
    const float2 w = f(v[bR % NS]);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const float c = (i & 1) ? w.y : w.x;
      res = BT_ADD(res, __shfl_sync(0xffffffffu, c, 4 * (bR / NS) + (i >> 1)));
    }
  }
  return res;
}

// Whether numpy's tree over a row of N values is eight leaves of one lane
// group each (8 NS values, a multiple of 8, starting at group boundaries)
// joined as ((L0+L1)+(L2+L3))+((L4+L5)+(L6+L7)): 768 values (12 slots) are.
template <int NS, int N>
__host__ __device__ constexpr bool group_tree() {
  // (every inner level must split: runs of at most kPwLeaf values are leaves)
  return N == 64 * NS && N / 8 <= kPwLeaf && N / 8 > 8 && N / 4 > kPwLeaf && pw_split_c(N) == N / 2 &&
         pw_split_c(N / 2) == N / 4 && pw_split_c(N / 4) == N / 8;
}

// numpy's sum of f(values) over such a row: each group sums its leaf down
// its slots and brackets it (two shuffles), then three xor shuffles across
// groups join the leaves level by level, in every lane (each float sum
// commutes, so the lanes of both partners get numpy's value).
static_assert(!group_tree<8, 512>(), "512 values: four 128-value leaves");
static_assert(group_tree<12, 768>(), "768 values: eight 96-value leaves");

template <int NS, class F>
__device__ __forceinline__ float reg_group_tree_sum(const float2 (&v)[NS], F f) {
  float2 acc = f(v[0]);
#pragma unroll
  for (int k = 1; k < NS; ++k) {
    const float2 t = f(v[k]);
    acc = F::kPacked ? pk_add(acc, t) : make_float2(BT_ADD(acc.x, t.x), BT_ADD(acc.y, t.y));
  }
  float t = BT_ADD(acc.x, acc.y);
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) t = BT_ADD(t, __shfl_xor_sync(0xffffffffu, t, m));
  return t;
}

template <int NS, int LEN, int OFF, class F>
__device__ __forceinline__ float reg_pw_sum(const float2 (&v)[NS], F f) {
  if constexpr (OFF == 0 && group_tree<NS, LEN>()) {
    return reg_group_tree_sum<NS>(v, f);
  } else if constexpr (LEN <= kPwLeaf) {
    return reg_leaf_sum<NS, LEN, OFF>(v, f);
  } else {
    constexpr int S = pw_split_c(LEN);
    const float l = reg_pw_sum<NS, S, OFF>(v, f);
    const float r = reg_pw_sum<NS, LEN - S, OFF + S>(v, f);
    return BT_ADD(l, r);
  }
}

// Slots per lane for rows of N values.
template <int N>
__host__ __device__ constexpr int reg_slots() { return ((N + 7) / 8 + 7) / 8; }

template <int N>
__global__ void __launch_bounds__(256, 4) wrow_softmax_reg_kernel(SoftmaxArgs a) {
  static_assert(N % 2 == 0 && N >= 2 && N <= 512, "rows of an even length up to 512");
  static_assert(reg_slots<N>() == 8, "eight slots per lane");
  const int lane = threadIdx.x & 31;
  const int e0 = 64 * (lane >> 2) + 2 * (lane & 3);   // element of slot 0
  // a mask shared by every row is read once per CTA, into shared memory in
  // the lanes' order
  __shared__ __align__(16) float2 mk[8][32];
  const bool mconst = a.mask && a.mask_row_const;
  if (mconst) {
    for (int i = threadIdx.x; i < 8 * 32; i += blockDim.x) {
      const int k = i >> 5, l = i & 31;
      const int e = 64 * (l >> 2) + 2 * (l & 3) + 8 * k;
      mk[k][l] = e < N ? make_float2(a.mask[e * a.mask_col_st], a.mask[(e + 1) * a.mask_col_st])
                       : make_float2(0.0f, 0.0f);
    }
    __syncthreads();
  }
  // rows straight into registers, the next row's loads issued before the
  // current row is computed (each lane's eight pairs of both rows in flight)
  const int64_t stride = (int64_t)gridDim.x * kWarpsPerCta;
  int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  float2 nx[8];
  // slots 0-6 lie inside every row of 510 or 512 values (e0 + 48 <= 502);
  // only slot 7 of the last lanes can pass the end
  static_assert(N >= 503, "slots 0-6 in bounds");
  auto load_row = [&](int64_t r) {
    const float2* xr = reinterpret_cast<const float2*>(a.x + r * N + e0);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      nx[k] = (k < 7 || e0 + 8 * k < N) ? __ldcs(xr + 4 * k) : make_float2(-INFINITY, -INFINITY);
  };
  if (row < a.rows) load_row(row);
  for (; row < a.rows; row += stride) {
    float2 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = nx[k];
    if (row + stride < a.rows) load_row(row + stride);
    if (a.mask) {
      if (mconst) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          v[k] = pk_add(v[k], mk[k][lane]);   // (past the row: -inf + 0)
      } else {
        // this row's mask row (the host sends fewer than 2^32 rows), pairs
        // loaded as one 8-byte vector where the row is contiguous and aligned
        const float* mr = a.mask + mask_row_offset(a, (uint32_t)row);
        if (a.mask_col_st == 1 && ((uintptr_t)mr & 7) == 0) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int e = e0 + 8 * k;
            if (k < 7 || e < N) v[k] = pk_add(v[k], __ldg(reinterpret_cast<const float2*>(mr + e)));
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int e = e0 + 8 * k;
            if (k < 7 || e < N) v[k] = pk_add(v[k], make_float2(mr[e * a.mask_col_st], mr[(e + 1) * a.mask_col_st]));
          }
        }
      }
    }
    // row maximum (a NaN anywhere makes the whole row NaN either way, see
    // wrow_softmax_kernel)
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) m = max3f(m, v[k].x, v[k].y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // exp(x - max), two lanes per instruction (x - m == x + (-m), at most 0
    // or NaN)
    const float2 nm = pk(-m);
    bool tiny = false;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      v[k] = pk_np_exp_nonpos(pk_add(v[k], nm), tiny);   // (past the row: exp(-inf) = +0)
    const float total = reg_pw_sum<8, N, 0>(v, RegIdentity());
    const float denom = BT_ADD(0.0f, total);
    // The quotients in float32 (div_row_fast, two lanes at a time).  The
    // denominator lies in [1, 512] (the row's maximum contributes exp(0) = 1)
    // or is NaN, and each value in [2^-60, 1], +0 (0 y = 0, residual +0:
    // exactly +0) or NaN (NaN either way) -- unless the exponential set
    // `tiny`, and then this lane divides in double.
    const float2 nb = pk(-denom), y2 = pk(__frcp_rn(denom));
    float2* orow = reinterpret_cast<float2*>(a.out + row * N + e0);
    if (!tiny) {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < 7 || e0 + 8 * k < N) __stcs(orow + 4 * k, pk_div_row_fast(v[k], nb, y2));
    } else {
      const double rd = recip_d(denom);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < 7 || e0 + 8 * k < N) __stcs(orow + 4 * k, make_float2(div_by(v[k].x, rd), div_by(v[k].y, rd)));
    }
  }
}

// (Skip +) layer norm over rows of N values held in registers (see the
// register-resident rows above): numpy's mean, then the mean of the squared
// deviations, each a pairwise sum unrolled at compile time; the output steps
// Sub -> Div -> Mul(gamma) [-> Add(beta)], each rounded.  CTAs of four
// warps, eight per SM; each warp copies its next row into shared memory
// (cp.async, each lane its own pairs) as soon as the current row is in its
// registers, so the copy runs while the row is computed; gamma, beta and the
// skip bias sit in shared memory in the lanes' own order (float32, read once
// per CTA).
constexpr int kLnWarps = 4;
template <int N>
__global__ void __launch_bounds__(32 * kLnWarps, 8) wrow_layernorm_reg_kernel(LayerNormArgs a) {
  constexpr int NS = reg_slots<N>();
  static_assert(N % 8 == 0 && NS <= 12, "rows of a multiple of 8 values, at most 768");
  __shared__ __align__(16) float2 stage[kLnWarps][NS][32];
  __shared__ __align__(16) float4 sgb[NS][32];   // (gamma pair, beta pair)
  __shared__ __align__(16) float2 sbias[NS][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int e0 = 8 * NS * (lane >> 2) + 2 * (lane & 3);   // element of slot 0
  for (int i = threadIdx.x; i < NS * 32; i += 32 * kLnWarps) {
    const int k = i >> 5, l = i & 31;
    const int e = 8 * NS * (l >> 2) + 2 * (l & 3) + 8 * k;
    float2 g = make_float2(0.0f, 0.0f), be = g, bi = g;
    if (e < N) {
      g = make_float2(ldf(a.gamma, a.gdt, e), ldf(a.gamma, a.gdt, e + 1));
      if (a.beta) be = make_float2(ldf(a.beta, a.bdt, e), ldf(a.beta, a.bdt, e + 1));
      if (a.bias) bi = make_float2(a.bias[e], a.bias[e + 1]);
    }
    sgb[k][l] = make_float4(g.x, g.y, be.x, be.y);
    sbias[k][l] = bi;
  }
  __syncthreads();
  const int64_t step = (int64_t)gridDim.x * kLnWarps;
  auto prefetch = [&](int64_t r) {
    const float* xr = a.x + r * N;
#pragma unroll
    for (int k = 0; k < NS; ++k)
      if (e0 + 8 * k < N) cp_async8(&stage[w][k][lane], xr + e0 + 8 * k);
    cp_async_commit();
  };
  int64_t row = (int64_t)blockIdx.x * kLnWarps + w;
  if (row < a.rows) prefetch(row);
  for (; row < a.rows; row += step) {
    cp_async_wait<0>();                  // this row's copies (this lane's own)
    float2 v[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) v[k] = e0 + 8 * k < N ? stage[w][k][lane] : make_float2(0.0f, 0.0f);
    // the slots are free once read (each lane copies and reads only its own)
    if (row + step < a.rows) prefetch(row + step);
    if (a.skip || a.bias) {
      const float* sk = a.skip ? a.skip + row * N : nullptr;
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const int e = e0 + 8 * k;
        if (e < N) {
          if (sk) {
            const float2 q = __ldcs(reinterpret_cast<const float2*>(sk + e));
            v[k] = make_float2(BT_ADD(v[k].x, q.x), BT_ADD(v[k].y, q.y));
          }
          if (a.bias) v[k] = make_float2(BT_ADD(v[k].x, sbias[k][lane].x), BT_ADD(v[k].y, sbias[k][lane].y));
        }
      }
    }
    const float sum = reg_pw_sum<NS, N, 0>(v, RegIdentity());
    const float mu = np_mean_from_sum(BT_ADD(0.0f, sum), N);
    const float ssq = reg_pw_sum<NS, N, 0>(v, RegSquaredDev{mu});
    const float var = np_mean_from_sum(BT_ADD(0.0f, ssq), N);
    const float sd = BT_SQRT(BT_ADD(var, a.eps));
    // (x - mu) / sd in float32 (div_row_fast, two lanes at a time); a lane
    // holding a deviation outside the window divides all its values in double
    const RowDiv dv = row_div(sd);
    bool outside = false;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      v[k] = make_float2(BT_SUB(v[k].x, mu), BT_SUB(v[k].y, mu));
      if (e0 + 8 * k < N) outside |= div_row_outside(v[k].x, dv) | div_row_outside(v[k].y, dv);
    }
    if (!outside) {
      const float2 nb = pk(-dv.b), y2 = pk(dv.y);
#pragma unroll
      for (int k = 0; k < NS; ++k) v[k] = pk_div_row_fast(v[k], nb, y2);
    } else {
      const double rb = recip_d(sd);   // div_by is exact for every value
#pragma unroll
      for (int k = 0; k < NS; ++k) v[k] = make_float2(div_by(v[k].x, rb), div_by(v[k].y, rb));
    }
    float* orow = a.out + row * N;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const int e = e0 + 8 * k;
      if (e < N) {
        const float4 gb = sgb[k][lane];
        float y0 = BT_MUL(v[k].x, gb.x);
        float y1 = BT_MUL(v[k].y, gb.y);
        if (a.beta) {
          y0 = BT_ADD(y0, gb.z);
          y1 = BT_ADD(y1, gb.w);
        }
        __stcs(reinterpret_cast<float2*>(orow + e), make_float2(y0, y1));
      }
    }
  }
}

__global__ void __launch_bounds__(256) wrow_layernorm_kernel(WLayerNormArgs A) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ WShared sh;
  const WView P = wplan_load(A.P, sh);
  const LayerNormArgs& a = A.a;
  const int lane = threadIdx.x & 31, n = P.n;
  const WSlice W = warp_slice(smem, n);
  const float* x = a.x;
  warp_rows(W, n, a.rows, [&](int64_t row) { return x + row * (int64_t)n; }, [&](int64_t row, float* b) {
    if (a.skip || a.bias) {
      const float* sk = a.skip ? a.skip + row * (int64_t)n : nullptr;
      for (int i = lane; i < n; i += 32) {
        float v = b[i];
        if (sk) v = BT_ADD(v, sk[i]);
        if (a.bias) v = BT_ADD(v, a.bias[i]);
        b[i] = v;
      }
      __syncwarp();
    }
    const float mu = np_mean_from_sum(BT_ADD(0.0f, warp_pw_sum(P, b, W.heap, PwIdentity())), n);
    const float var = np_mean_from_sum(BT_ADD(0.0f, warp_pw_sum(P, b, W.heap, PwSquaredDev{mu})), n);
    const float sd = BT_SQRT(BT_ADD(var, a.eps));
    const double rsd = recip_d(sd);
    float* o = a.out + row * (int64_t)n;
    // Sub -> Div -> Mul(gamma) [-> Add(beta)], each rounded
    auto ln = [&](float v, float g, float be) {
      const float y = BT_MUL(div_by(BT_SUB(v, mu), rsd), g);
      return a.beta ? BT_ADD(y, be) : y;
    };
    const int ph = phase4(b);
    const bool vec = phase4(o) == ph && a.gdt == BT_F32 && phase4(a.gamma) == ph &&
                     (!a.beta || (a.bdt == BT_F32 && phase4(a.beta) == ph));
    if (vec) {
      // 128-bit over the aligned interior; gamma / beta fp32 at the row's phase
      int head = (4 - ph) & 3;
      if (head > n) head = n;
      const int nvec = (n - head) >> 2, tail0 = head + 4 * nvec;
      const float* gm = (const float*)a.gamma;
      const float* bt = (const float*)a.beta;
      for (int i = lane; i < head; i += 32) o[i] = ln(b[i], gm[i], bt ? bt[i] : 0.0f);
      for (int q = lane; q < nvec; q += 32) {
        const int i = head + 4 * q;
        const float4 v = *reinterpret_cast<const float4*>(b + i);
        const float4 g = __ldg(reinterpret_cast<const float4*>(gm + i));
        const float4 be = bt ? __ldg(reinterpret_cast<const float4*>(bt + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        __stcs(reinterpret_cast<float4*>(o + i),
               make_float4(ln(v.x, g.x, be.x), ln(v.y, g.y, be.y), ln(v.z, g.z, be.z), ln(v.w, g.w, be.w)));
      }
      for (int i = tail0 + lane; i < n; i += 32) o[i] = ln(b[i], gm[i], bt ? bt[i] : 0.0f);
    } else {
      for (int i = lane; i < n; i += 32)
        o[i] = ln(b[i], ldf(a.gamma, a.gdt, i), a.beta ? ldf(a.beta, a.bdt, i) : 0.0f);
    }
  });
}

// ---- warp-row host side ------------------------------------------------------
// ---- pairwise plans for rows up to kMaxRow values -------------------------
constexpr int kDirLeaves = 384;     // kMaxRow / 128
constexpr int kDirHeap = 1024;      // heap ids < 2^(D+1), D <= 9

struct DPlan {
  int32_t n, D, n_leaf, perfect;
  uint32_t inner[kDirHeap / 64];    // bit h: heap node h (< 2^D) is an inner node
  uint16_t off[kDirLeaves];
  uint8_t len[kDirLeaves];
  uint16_t id[kDirLeaves];
};
struct DShared {
  uint16_t off[kDirLeaves];
  uint16_t id[kDirLeaves];
  uint8_t len[kDirLeaves];
  uint32_t inner[kDirHeap / 64];
};
// Sum of K consecutive leaf sums p[0..K) in pairwise order.
template <int K>
__device__ __forceinline__ float dir_lane_leaves(const float* p) {
  float v[K];
#pragma unroll
  for (int i = 0; i < K; ++i) v[i] = p[i];
#pragma unroll
  for (int w = K; w > 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w / 2; ++i) v[i] = BT_ADD(v[2 * i], v[2 * i + 1]);
  }
  return v[0];
}

// ---- chunked row sums -----------------------------------------------------
// ReduceSum / ReduceMean of float32 rows longer than a warp's shared-memory
// slice, one warp per row, the row streamed through two buffers of kChunk
// values: while the warp sums the pairwise leaves of one run of whole leaves
// (a chunk), the cp.async copy of the next run -- of this row or of the
// warp's next row -- is in flight.  Copies are coalesced 16-byte transfers;
// the leaves are summed as in warp_pw_sum (four lanes per leaf with float2
// accumulators on 8-byte aligned rows, eight otherwise).
constexpr int kChunk = 1024;

struct CReduceArgs {
  DPlan P;
  uint16_t chunk_leaf[kDirLeaves + 1];   // chunk c holds leaves [chunk_leaf[c], chunk_leaf[c + 1])
  int32_t n_chunk;
  const float* x;
  int32_t mean;
  int64_t rows;
  float* out;
};

// Per-warp shared floats of chunk_reduce_kernel: the heap, then two buffers
// (kChunk values + 4 for the 16-byte phase each).
__host__ __device__ inline int chunk_warp_floats(int D) { return (2 << D) + 2 * (kChunk + 4); }

__global__ void __launch_bounds__(256) chunk_reduce_kernel(CReduceArgs A) {
  extern __shared__ __align__(16) float csm[];
  __shared__ DShared sh;
  __shared__ uint16_t schunk[kDirLeaves + 1];
  for (int i = threadIdx.x; i < A.P.n_leaf; i += blockDim.x) {
    sh.off[i] = A.P.off[i];
    sh.len[i] = A.P.len[i];
    sh.id[i] = A.P.id[i];
  }
  for (int i = threadIdx.x; i <= A.n_chunk; i += blockDim.x) schunk[i] = A.chunk_leaf[i];
  for (int i = threadIdx.x; i < kDirHeap / 64; i += blockDim.x) sh.inner[i] = A.P.inner[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = A.P.n, D = A.P.D, n_leaf = A.P.n_leaf, nch = A.n_chunk;
  const bool perfect = A.P.perfect != 0;
  float* heap = csm + warp * chunk_warp_floats(D);
  float* const buf0 = heap + (2 << D);   // buffer `slot` starts at buf0 + slot * (kChunk + 4)
  const int64_t rstride = (int64_t)gridDim.x * 8;
  int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= A.rows) return;
  auto chunk_lo = [&](int c) { return (int)sh.off[schunk[c]]; };
  auto chunk_hi = [&](int c) { return schunk[c + 1] < n_leaf ? (int)sh.off[schunk[c + 1]] : n; };
  auto issue = [&](int64_t row, int c, int slot) {
    const float* g = A.x + row * n + chunk_lo(c);
    stage_floats_async(buf0 + slot * (kChunk + 4) + phase4(g), g, chunk_hi(c) - chunk_lo(c), lane, 32);
    cp_async_commit();
  };
  issue(r, 0, 0);
  int c = 0, slot = 0;
  while (r < A.rows) {
    int64_t rn = r;
    int cn = c + 1;
    if (cn == nch) {
      cn = 0;
      rn += rstride;
    }
    if (rn < A.rows) issue(rn, cn, slot ^ 1);
    else cp_async_commit();          // an empty group keeps the count
    cp_async_wait<1>();              // this chunk's copies (this lane's)
    __syncwarp();
    const int e0 = chunk_lo(c);
    const float* g = A.x + r * n + e0;
    const float* b = buf0 + slot * (kChunk + 4) + phase4(g);   // b[e - e0]: value e of the row
    const int l0 = schunk[c], l1 = schunk[c + 1];
    if (((uintptr_t)b & 7) == 0) {
      const int j = lane & 3;
      const unsigned gmask = 0xfu << (lane & 28);
      for (int L = l0 + (lane >> 2); L < l1; L += 8) {
        const int off = sh.off[L] - e0, len = sh.len[L];
        const int steps = len >> 3, end = steps << 3;
        const float2* q = reinterpret_cast<const float2*>(b + off + 2 * j);
        float2 acc = pk(-0.0f);      // -0.0 + x == x: acc starts as numpy's r[j] = a[j]
#pragma unroll 4
        for (int m = 0; m < steps; ++m) acc = pk_add(acc, q[4 * m]);
        float t = BT_ADD(acc.x, acc.y);
        t = BT_ADD(t, __shfl_xor_sync(gmask, t, 1));
        t = BT_ADD(t, __shfl_xor_sync(gmask, t, 2));
        if (steps == 0) t = 0.0f;
        if (len > end) {
          if (j == 0)
            for (int i = end; i < len; ++i) t = BT_ADD(t, b[off + i]);
          t = __shfl_sync(gmask, t, 0, 4);
        }
        if (j == 0) heap[sh.id[L]] = t;
      }
    } else {
      const int j = lane & 7;
      const unsigned gmask = 0xffu << (lane & 24);
      for (int L = l0 + (lane >> 3); L < l1; L += 4) {
        const int off = sh.off[L] - e0, len = sh.len[L];
        const int steps = len >> 3, end = steps << 3;
        const float* q = b + off + j;
        float acc = -0.0f;
#pragma unroll 4
        for (int m = 0; m < steps; ++m) acc = BT_ADD(acc, q[8 * m]);
        acc = BT_ADD(acc, __shfl_xor_sync(gmask, acc, 1));
        acc = BT_ADD(acc, __shfl_xor_sync(gmask, acc, 2));
        acc = BT_ADD(acc, __shfl_xor_sync(gmask, acc, 4));
        if (steps == 0) acc = 0.0f;
        if (len > end) {
          if (j == 0)
            for (int i = end; i < len; ++i) acc = BT_ADD(acc, b[off + i]);
          acc = __shfl_sync(gmask, acc, 0, 8);
        }
        if (j == 0) heap[sh.id[L]] = acc;
      }
    }
    __syncwarp();                     // the buffer is refilled two chunks later
    if (c == nch - 1) {
      float total;
      if (perfect && D <= 9) {
        const float* leaf = heap + (1 << D);
        switch (D) {
          case 9: total = dir_lane_leaves<16>(leaf + 16 * lane); break;
          case 8: total = dir_lane_leaves<8>(leaf + 8 * lane); break;
          case 7: total = dir_lane_leaves<4>(leaf + 4 * lane); break;
          case 6: total = dir_lane_leaves<2>(leaf + 2 * lane); break;
          default: total = lane < (1 << D) ? leaf[lane] : 0.0f; break;
        }
        const int levels = D < 5 ? D : 5;
        for (int m = 0; m < levels; ++m) total = BT_ADD(total, __shfl_xor_sync(0xffffffffu, total, 1 << m));
        total = __shfl_sync(0xffffffffu, total, 0);
      } else {
        for (int k = D - 1; k >= 0; --k) {
          for (int jj = lane; jj < (1 << k); jj += 32) {
            const int hh = (1 << k) + jj;
            if ((sh.inner[hh >> 5] >> (hh & 31)) & 1u) heap[hh] = BT_ADD(heap[2 * hh], heap[2 * hh + 1]);
          }
          __syncwarp();
        }
        total = heap[1];
      }
      if (lane == 0) A.out[r] = A.mean ? np_mean_from_sum(BT_ADD(0.0f, total), n) : BT_ADD(0.0f, total);
      __syncwarp();                   // the heap is reused by the next row
    }
    r = rn;
    c = cn;
    slot ^= 1;
  }
  cp_async_wait_all();
}

// Runs of whole leaves spanning at most kChunk values, in row order.
bool chunk_plan(const DPlan& p, uint16_t* chunk_leaf, int* n_chunk) {
  int nc = 0, L = 0;
  while (L < p.n_leaf) {
    if (nc >= kDirLeaves) return false;
    chunk_leaf[nc++] = (uint16_t)L;
    const int start = p.off[L];
    int L1 = L + 1;
    while (L1 < p.n_leaf && (int)p.off[L1] + (int)p.len[L1] - start <= kChunk) ++L1;
    L = L1;
  }
  chunk_leaf[nc] = (uint16_t)p.n_leaf;
  *n_chunk = nc;
  return true;
}

void dplan_node(DPlan& p, int h, int lo, int n, bool& ok) {
  if (n <= kPwLeaf) {
    if (p.n_leaf >= kDirLeaves || h >= kDirHeap) { ok = false; return; }
    p.off[p.n_leaf] = (uint16_t)lo;
    p.len[p.n_leaf] = (uint8_t)n;
    p.id[p.n_leaf] = (uint16_t)h;
    ++p.n_leaf;
    return;
  }
  if (2 * h >= kDirHeap) { ok = false; return; }
  p.inner[h >> 5] |= 1u << (h & 31);
  const int n2 = (int)pw_split(n);
  dplan_node(p, 2 * h, lo, n2, ok);
  dplan_node(p, 2 * h + 1, lo + n2, n - n2, ok);
}

// The pairwise plan of a row of n values for chunk_reduce_kernel (cached).
bool dplan_for(int n, DPlan* out) {
  if (n < 1 || n > kMaxRow) return false;
  static std::mutex mu;
  static std::map<int, DPlan> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(n);
  if (it == cache.end()) {
    DPlan p;
    memset(&p, 0, sizeof(p));
    p.n = n;
    p.D = pw_depth(n);
    bool ok = p.D <= 9;
    if (ok) dplan_node(p, 1, 0, n, ok);
    p.perfect = (ok && p.n_leaf == (1 << p.D)) ? 1 : 0;
    if (!ok) p.n = -1;
    it = cache.emplace(n, p).first;
  }
  if (it->second.n < 0) return false;
  *out = it->second;
  return true;
}

void wplan_node(WPlan& p, int h, int lo, int n, bool& ok) {
  if (n <= kPwLeaf) {
    if (p.n_leaf >= kWarpLeaves || h >= kWarpHeap) { ok = false; return; }
    p.off[p.n_leaf] = (uint16_t)lo;
    p.len[p.n_leaf] = (uint8_t)n;
    p.id[p.n_leaf] = (uint8_t)h;
    ++p.n_leaf;
    return;
  }
  if (h >= kWarpHeap) { ok = false; return; }
  p.inner[h >> 5] |= 1u << (h & 31);
  const int n2 = (int)pw_split(n);
  wplan_node(p, 2 * h, lo, n2, ok);
  wplan_node(p, 2 * h + 1, lo + n2, n - n2, ok);
}

// The pairwise plan of a row of n values for the warp kernels (cached per
// n); false when n is outside their cover.
bool wplan_for(int n, WPlan* out) {
  if (n < 1 || n > kWarpRowMax) return false;
  static std::mutex mu;
  static std::map<int, WPlan> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(n);
  if (it == cache.end()) {
    WPlan p;
    memset(&p, 0, sizeof(p));
    p.n = n;
    p.D = pw_depth(n);
    bool ok = p.D <= 5;
    if (ok) wplan_node(p, 1, 0, n, ok);
    p.perfect = (ok && p.n_leaf == (1 << p.D)) ? 1 : 0;
    if (!ok) p.n = -1;
    it = cache.emplace(n, p).first;
  }
  if (it->second.n < 0) return false;
  *out = it->second;
  return true;
}

std::atomic<int> g_wrow_ready[kMaxDevices];

// Launch geometry of a warp-row kernel: its dynamic shared memory (eight
// slices) and one warp per row.  (A persistent grid with the next row's copy
// in flight measured slower: the second buffer halves the warps per SM.)
// Returns BT_EUNSUPPORTED, without setting an error, when there are too few
// rows to fill the device one warp per row (the CTA-per-row kernels serve
// those).
int wrow_setup(int n, int64_t rows, size_t* smem, int* grid) {
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  if (di.device >= kMaxDevices) return set_error(BT_EUNSUPPORTED, "device ordinal %d >= %d", di.device, kMaxDevices);
  if (rows < 2ll * di.sm_count * kWarpsPerCta) return BT_EUNSUPPORTED;
  if (!g_wrow_ready[di.device].load()) {
    const void* fns[] = {(const void*)wrow_reduce_kernel, (const void*)wrow_softmax_kernel,
                         (const void*)wrow_layernorm_kernel};
    for (const void* f : fns) {
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, f);
      if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
      e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               di.max_smem_optin - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    g_wrow_ready[di.device].store(1);
  }
  *smem = (size_t)kWarpsPerCta * wrow_stride(n) * sizeof(float);
  int64_t g = (rows + kWarpsPerCta - 1) / kWarpsPerCta;
  if (g > 2147483647) g = 2147483647;
  *grid = (int)g;
  return BT_OK;
}

}  // namespace
}  // namespace bt

using namespace bt;

extern "C" int bt_init(int device) {
  if (device >= 0) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  }
  return raise_smem_limits();
}

extern "C" int bt_reduce(int kind, const bt_tensor* x, const int64_t* axes, int n_axes, int keepdims,
                         const bt_tensor* out) {
  if (kind != BT_REDUCE_SUM && kind != BT_REDUCE_MEAN) return set_error(BT_EINVAL, "bt_reduce: kind %d", kind);
  int rc = check_tensor(x, "x", false);
  if (rc) return rc;
  if ((rc = check_tensor(out, "out", false))) return rc;
  if (n_axes < 0 || n_axes > x->rank || (n_axes > 0 && !axes)) return set_error(BT_EINVAL, "bt_reduce: bad axes");
  if (x->dtype != BT_F32 && x->dtype != BT_F16)
    return set_error(BT_EDTYPE, "bt_reduce: input dtype %d (float32/float16 only)", x->dtype);
  if (out->dtype != BT_F32) return set_error(BT_EDTYPE, "bt_reduce: output must be float32");
  if (!is_contiguous(x) || !is_contiguous(out)) return set_error(BT_EUNSUPPORTED, "bt_reduce: contiguous views only");
  bool red[BT_MAX_RANK] = {false};
  for (int i = 0; i < n_axes; ++i) {
    if (axes[i] < 0 || axes[i] >= x->rank) return set_error(BT_EINVAL, "bt_reduce: axis %lld", (long long)axes[i]);
    if (red[axes[i]]) return set_error(BT_EINVAL, "bt_reduce: repeated axis %lld", (long long)axes[i]);
    red[axes[i]] = true;
  }
  // expected output extent
  int64_t expect = 1;
  for (int d = 0; d < x->rank; ++d) if (!red[d]) expect *= x->shape[d];
  if (numel(out) != expect) return set_error(BT_ESHAPE, "bt_reduce: output has %lld elements, expected %lld",
                                             (long long)numel(out), (long long)expect);
  (void)keepdims;
  // Collapse to [O, R, I]: the reduced axes must be one contiguous block
  // (after dropping size-1 axes).
  int first = -1, last = -1;
  for (int d = 0; d < x->rank; ++d) {
    if (x->shape[d] == 1) continue;
    if (red[d]) { if (first < 0) first = d; last = d; }
  }
  int64_t O = 1, R = 1, I = 1;
  for (int d = 0; d < x->rank; ++d) {
    if (x->shape[d] == 1) continue;
    if (first >= 0 && d >= first && d <= last) {
      if (!red[d]) return set_error(BT_EUNSUPPORTED, "bt_reduce: reduced axes must form one contiguous block");
      R *= x->shape[d];
    } else if (first >= 0 && d > last) I *= x->shape[d];
    else O *= x->shape[d];
  }
  if (numel(x) == 0 || expect == 0) {
    if (expect == 0) return BT_OK;
    // empty reduction: sum 0, mean NaN (numpy's 0/0)
    return set_error(BT_EUNSUPPORTED, "bt_reduce: empty reduction is handled by the caller");
  }
  cudaStream_t s = cur_stream();
  if (I == 1 && x->dtype == BT_F32 && R > kWarpRowMax) {
    // rows too long for a warp's shared-memory slice: streamed through two
    // chunk buffers per warp (shorter rows stage whole, which measured
    // faster at 2048 values)
    DPlan dp;
    DevInfo di;
    if ((rc = dev_info(&di))) return rc;
    CReduceArgs ca;   // the kernel parameter block (about 3 KB)
    if (O >= 4ll * di.sm_count && R <= kMaxRow && dplan_for((int)R, &dp) &&
        chunk_plan(dp, ca.chunk_leaf, &ca.n_chunk)) {
      ca.P = dp;
      ca.x = (const float*)x->data;
      ca.mean = kind == BT_REDUCE_MEAN;
      ca.rows = O;
      ca.out = (float*)out->data;
      const size_t smem = (size_t)8 * chunk_warp_floats(dp.D) * sizeof(float);
      static std::atomic<int> attr_done[kMaxDevices];
      if (di.device >= kMaxDevices) return set_error(BT_EUNSUPPORTED, "device ordinal %d", di.device);
      if (!attr_done[di.device].load()) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, chunk_reduce_kernel);
        if (e == cudaSuccess)
          e = cudaFuncSetAttribute(chunk_reduce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   di.max_smem_optin - (int)fa.sharedSizeBytes);
        if (e != cudaSuccess) return set_error(BT_ECUDA, "bt_reduce(chunked rows) attributes: %s", cudaGetErrorString(e));
        attr_done[di.device].store(1);
      }
      int64_t g = (O + 7) / 8;
      if (g > 2147483647) g = 2147483647;
      chunk_reduce_kernel<<<(int)g, 256, smem, s>>>(ca);
      return check_launch("bt_reduce(chunked rows)");
    }
  }
  if (I == 1) {
    WPlan wp;
    if (R <= kWarpRowMax && wplan_for((int)R, &wp)) {
      size_t smem;
      int grid;
      rc = wrow_setup((int)R, O, &smem, &grid);
      if (rc == BT_OK && x->dtype == BT_F32 && wp.perfect && (wp.n_leaf == 8 || wp.n_leaf == 16) &&
          (int64_t)wp.n_leaf * 128 == R && ((uintptr_t)x->data & 7) == 0) {
        // perfect trees of 128-value leaves: straight from global memory
        if (wp.n_leaf == 8)
          wrow_reduce_direct_kernel<8><<<grid, 32 * kWarpsPerCta, 0, s>>>((const float*)x->data, kind == BT_REDUCE_MEAN,
                                                                         O, (float*)out->data);
        else
          wrow_reduce_direct_kernel<16><<<grid, 32 * kWarpsPerCta, 0, s>>>((const float*)x->data, kind == BT_REDUCE_MEAN,
                                                                          O, (float*)out->data);
        return check_launch("bt_reduce(warp rows, direct)");
      }
      if (rc == BT_OK) {
        WReduceArgs a{wp, x->data, x->dtype, kind == BT_REDUCE_MEAN, O, (float*)out->data};
        wrow_reduce_kernel<<<grid, 32 * kWarpsPerCta, smem, s>>>(a);
        return check_launch("bt_reduce(warp rows)");
      }
      if (rc != BT_EUNSUPPORTED) return rc;
    }
    if (R > kMaxRow) return set_error(BT_ETOOBIG, "bt_reduce: reduced run of %lld values exceeds %d", (long long)R, kMaxRow);
    size_t smem;
    int depth;
    if ((rc = row_launch_check((int)R, &smem, &depth))) return rc;
    ReduceRowsArgs a{x->data, x->dtype, kind == BT_REDUCE_MEAN, (int)R, depth, O, (float*)out->data};
    reduce_rows_kernel<<<row_grid(O), row_threads((int)R), smem, s>>>(a);
    return check_launch("bt_reduce(rows)");
  }
  ReduceColsArgs a{x->data, x->dtype, kind == BT_REDUCE_MEAN, O, R, I, (float*)out->data};
  int64_t work = O * I;
  int g = (int)((work + 255) / 256);
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  reduce_cols_kernel<<<g, 256, 0, s>>>(a);
  return check_launch("bt_reduce(cols)");
}

extern "C" int bt_softmax(const bt_tensor* x, const bt_tensor* mask, int axis, const bt_tensor* out) {
  int rc = check_tensor(x, "x", false);
  if (rc) return rc;
  if ((rc = check_tensor(out, "out", false))) return rc;
  if (x->dtype != BT_F32 || out->dtype != BT_F32) return set_error(BT_EDTYPE, "bt_softmax: float32 only");
  if (x->rank < 1) return set_error(BT_ESHAPE, "bt_softmax: rank 0 input");
  if (axis < 0) axis += x->rank;
  if (axis != x->rank - 1) return set_error(BT_EUNSUPPORTED, "bt_softmax: last axis only (got %d)", axis);
  if (!is_contiguous(x) || !is_contiguous(out) || numel(out) != numel(x))
    return set_error(BT_EUNSUPPORTED, "bt_softmax: contiguous x and out of equal size only");
  const int64_t n = x->shape[x->rank - 1];
  const int64_t rows = n ? numel(x) / n : 0;
  if (rows == 0 || n == 0) return BT_OK;
  SoftmaxArgs a{};
  a.x = (const float*)x->data;
  a.out = (float*)out->data;
  a.n = (int)n;
  a.rows = rows;
  a.lead_rank = x->rank - 1;
  for (int d = 0; d < a.lead_rank; ++d) a.lead_shape[d] = x->shape[d];
  if (mask) {
    if ((rc = check_tensor(mask, "mask", false))) return rc;
    if (mask->dtype != BT_F32) return set_error(BT_EDTYPE, "bt_softmax: mask must be float32");
    if (mask->rank > x->rank) return set_error(BT_ESHAPE, "bt_softmax: mask rank exceeds x rank");
    const int pad = x->rank - mask->rank;
    for (int d = 0; d < x->rank; ++d) {
      int64_t e = d < pad ? 1 : mask->shape[d - pad];
      int64_t st = (d < pad || e == 1) ? 0 : mask->strides[d - pad];
      if (e != 1 && e != x->shape[d]) return set_error(BT_ESHAPE, "bt_softmax: mask does not broadcast on axis %d", d);
      if (d < a.lead_rank) a.mask_lead_st[d] = st;
      else a.mask_col_st = st;
    }
    a.mask = (const float*)mask->data;
    a.mask_row_const = 1;
    for (int d = 0; d < a.lead_rank; ++d)
      if (a.mask_lead_st[d] != 0) a.mask_row_const = 0;
    if (rows < (1ll << 32)) {
      // collapse the leading axes for mask_row_offset: an outer axis whose
      // mask stride is the inner one's stride times its extent merges into it
      int64_t ext[BT_MAX_RANK];
      for (int d = a.lead_rank - 1; d >= 0; --d) {
        const int64_t e = a.lead_shape[d], st = a.mask_lead_st[d];
        if (e == 1) continue;
        if (a.mnd > 0 && st == a.mst[a.mnd - 1] * ext[a.mnd - 1]) {
          ext[a.mnd - 1] *= e;
          continue;
        }
        ext[a.mnd] = e;
        a.mst[a.mnd] = st;
        ++a.mnd;
      }
      for (int d = 0; d < a.mnd; ++d) a.mdiv[d] = fast_div_for((uint32_t)ext[d]);
    }
  }
  // rows of 510 / 512 values, 8-byte aligned: held in registers
  if ((n == 510 || n == 512) && rows < (1ll << 32) && ((uintptr_t)x->data & 7) == 0 &&
      ((uintptr_t)out->data & 7) == 0) {
    DevInfo di;
    const int sms = (dev_info(&di) == BT_OK && di.sm_count > 0) ? di.sm_count : 148;
    const int64_t need = (rows + kWarpsPerCta - 1) / kWarpsPerCta;
    const int64_t cap = (int64_t)sms * 8;   // 8 CTAs of 8 warps per SM at most
    const int grid = (int)(need < cap ? need : cap);
    if (n == 510) wrow_softmax_reg_kernel<510><<<grid, 32 * kWarpsPerCta, 0, cur_stream()>>>(a);
    else wrow_softmax_reg_kernel<512><<<grid, 32 * kWarpsPerCta, 0, cur_stream()>>>(a);
    return check_launch("bt_softmax(register rows)");
  }
  WPlan wp;
  if (n <= kWarpRowMax && rows < (1ll << 32) && wplan_for((int)n, &wp)) {
    size_t smem;
    int grid;
    rc = wrow_setup((int)n, rows, &smem, &grid);
    if (rc == BT_OK) {
      WSoftmaxArgs w{wp, a};
      wrow_softmax_kernel<<<grid, 32 * kWarpsPerCta, smem, cur_stream()>>>(w);
      return check_launch("bt_softmax(warp rows)");
    }
    if (rc != BT_EUNSUPPORTED) return rc;
  }
  size_t smem;
  int depth;
  if ((rc = row_launch_check((int)n, &smem, &depth))) return rc;
  a.depth = depth;
  softmax_rows_kernel<<<row_grid(rows), row_threads((int)n), smem, cur_stream()>>>(a);
  return check_launch("bt_softmax");
}

extern "C" int bt_layernorm(const bt_tensor* x, const bt_tensor* skip, const bt_tensor* bias, const bt_tensor* gamma,
                            const bt_tensor* beta, int axis, float eps, const bt_tensor* out) {
  int rc = check_tensor(x, "x", false);
  if (rc) return rc;
  if ((rc = check_tensor(out, "out", false))) return rc;
  if ((rc = check_tensor(gamma, "gamma", false))) return rc;
  if (x->dtype != BT_F32 || out->dtype != BT_F32) return set_error(BT_EDTYPE, "bt_layernorm: float32 x/out only");
  if (!is_contiguous(x) || !is_contiguous(out) || numel(out) != numel(x))
    return set_error(BT_EUNSUPPORTED, "bt_layernorm: contiguous x and out of equal size only");
  if (x->rank < 1) return set_error(BT_ESHAPE, "bt_layernorm: rank 0 input");
  if (axis < 0) axis += x->rank;
  if (axis < 0 || axis >= x->rank) return set_error(BT_EINVAL, "bt_layernorm: axis out of range");
  int64_t n = 1;
  for (int d = axis; d < x->rank; ++d) n *= x->shape[d];
  const int64_t rows = n ? numel(x) / n : 0;
  if (rows == 0 || n == 0) return BT_OK;
  auto check_vec = [&](const bt_tensor* t, const char* name) -> int {
    if ((t->dtype != BT_F32 && t->dtype != BT_F16) || numel(t) != n || !is_contiguous(t))
      return set_error(BT_EUNSUPPORTED, "bt_layernorm: %s must be a contiguous float32/float16 run of %lld values",
                       name, (long long)n);
    return BT_OK;
  };
  if ((rc = check_vec(gamma, "gamma"))) return rc;
  LayerNormArgs a{};
  a.x = (const float*)x->data;
  a.gamma = gamma->data;
  a.gdt = gamma->dtype;
  if (beta) {
    if ((rc = check_tensor(beta, "beta", false)) || (rc = check_vec(beta, "beta"))) return rc;
    a.beta = beta->data;
    a.bdt = beta->dtype;
  }
  if (skip) {
    if ((rc = check_tensor(skip, "skip", false))) return rc;
    if (skip->dtype != BT_F32 || !is_contiguous(skip) || numel(skip) != numel(x))
      return set_error(BT_EUNSUPPORTED, "bt_layernorm: skip must be contiguous float32 shaped like x");
    a.skip = (const float*)skip->data;
  }
  if (bias) {
    if ((rc = check_tensor(bias, "bias", false))) return rc;
    if (bias->dtype != BT_F32 || numel(bias) != n || !is_contiguous(bias))
      return set_error(BT_EUNSUPPORTED, "bt_layernorm: bias must be a contiguous float32 run of %lld values", (long long)n);
    a.bias = (const float*)bias->data;
  }
  a.n = (int)n;
  a.rows = rows;
  a.eps = eps;
  a.out = (float*)out->data;
  WPlan wp;
  if (n <= kWarpRowMax && wplan_for((int)n, &wp)) {
    size_t smem;
    int grid;
    rc = wrow_setup((int)n, rows, &smem, &grid);
    if (rc == BT_OK) {
      // rows of 768 values (ALBERT's hidden size), 8-byte aligned: held in registers
      // (measured against the staged warp kernel on 87381 rows: equal for
      // LayerNormalization, 0.75 against 0.61 of the HBM peak for
      // SkipLayerNormalization)
      if (n == 768 && ((uintptr_t)a.x & 7) == 0 && ((uintptr_t)a.out & 7) == 0 &&
          (!a.skip || ((uintptr_t)a.skip & 7) == 0)) {
        DevInfo di;
        const int sms = (dev_info(&di) == BT_OK && di.sm_count > 0) ? di.sm_count : 148;
        const int64_t need = (rows + kLnWarps - 1) / kLnWarps;
        const int64_t cap = (int64_t)sms * 8;   // eight CTAs of four warps per SM
        wrow_layernorm_reg_kernel<768><<<(int)(need < cap ? need : cap), 32 * kLnWarps, 0, cur_stream()>>>(a);
        return check_launch("bt_layernorm(register rows)");
      }
      WLayerNormArgs w{wp, a};
      wrow_layernorm_kernel<<<grid, 32 * kWarpsPerCta, smem, cur_stream()>>>(w);
      return check_launch("bt_layernorm(warp rows)");
    }
    if (rc != BT_EUNSUPPORTED) return rc;
  }
  size_t smem;
  int depth;
  if (n > kMaxRow) return set_error(BT_ETOOBIG, "bt_layernorm: normalised run of %lld values exceeds %d", (long long)n, kMaxRow);
  if ((rc = row_launch_check((int)n, &smem, &depth))) return rc;
  a.depth = depth;
  layernorm_rows_kernel<<<row_grid(rows), row_threads((int)n), smem, cur_stream()>>>(a);
  return check_launch("bt_layernorm");
}

namespace {

int adain_check(const bt_adain_args* p) {
  if (!p) return set_error(BT_EINVAL, "bt_adain_snake: null argument");
  if (p->rows < 0 || p->cols < 1 || p->channels < 1)
    return set_error(BT_EINVAL, "bt_adain_snake: rows %lld cols %lld channels %lld", (long long)p->rows,
                     (long long)p->cols, (long long)p->channels);
  if (p->n_src < 1 || p->n_src > BT_ADAIN_MAX_SRC || p->n_out < 1 || p->n_out > BT_ADAIN_MAX_OUT)
    return set_error(BT_EINVAL, "bt_adain_snake: n_src %d n_out %d", p->n_src, p->n_out);
  for (int k = 0; k < p->n_src; ++k)
    if (!p->src[k]) return set_error(BT_EINVAL, "bt_adain_snake: src[%d] is null", k);
  for (int k = 0; k < p->n_out; ++k) {
    if (!p->out[k] || !p->gain[k] || !p->shift[k])
      return set_error(BT_EINVAL, "bt_adain_snake: output %d lacks out/gain/shift", k);
    if ((p->alpha[k] == nullptr) != (p->inv_alpha[k] == nullptr))
      return set_error(BT_EINVAL, "bt_adain_snake: output %d has only one of alpha / inv_alpha", k);
  }
  if (p->alpha_dtype != BT_F16 && p->alpha_dtype != BT_F32)
    return set_error(BT_EDTYPE, "bt_adain_snake: alpha dtype %d", p->alpha_dtype);
  if (p->gain_stride < p->channels || p->shift_stride < p->channels)
    return set_error(BT_EINVAL, "bt_adain_snake: gain/shift batch strides (%lld, %lld) below C = %lld",
                     (long long)p->gain_stride, (long long)p->shift_stride, (long long)p->channels);
  return BT_OK;
}

// the one-CTA-per-row kernel
int adain_one_cta(const bt_adain_args* p) {
  if (p->cols > kMaxRow) return set_error(BT_ETOOBIG, "bt_adain_snake: rows of %lld values exceed %d", (long long)p->cols, kMaxRow);
  size_t smem;
  int depth, rc;
  if ((rc = row_launch_check((int)p->cols, &smem, &depth))) return rc;
  AdainArgs A;
  A.p = *p;
  A.depth = depth;
  A.n = (int)p->cols;
  adain_snake_kernel<<<row_grid(p->rows), row_threads((int)p->cols), smem, cur_stream()>>>(A);
  return check_launch("bt_adain_snake");
}

}  // namespace

extern "C" int bt_adain_snake(const bt_adain_args* p) {
  int rc = adain_check(p);
  if (rc) return rc;
  if (p->rows == 0) return BT_OK;
  rc = adain_v3(p);
  if (rc != BT_EUNSUPPORTED) return rc;
  return adain_one_cta(p);
}

extern "C" int bt_adain_snake_range(const bt_adain_args* p, uint32_t* range) {
  int rc = adain_check(p);
  if (rc) return rc;
  if (!range) return set_error(BT_EINVAL, "bt_adain_snake_range: null range records");
  if ((uintptr_t)range & 15) return set_error(BT_EINVAL, "bt_adain_snake_range: range records not 16-byte aligned");
  cudaError_t e = cudaMemsetAsync(range, 0, (size_t)16 * p->n_out, cur_stream());
  if (e != cudaSuccess) return set_error(BT_ECUDA, "bt_adain_snake_range: memset: %s", cudaGetErrorString(e));
  if (p->rows == 0) return BT_OK;
  uint32_t* rec[BT_ADAIN_MAX_OUT];
  for (int k = 0; k < p->n_out; ++k) rec[k] = range + 4 * k;
  rc = adain_v3(p, rec);
  if (rc != BT_EUNSUPPORTED) return rc;
  // outside the cluster kernel: the one-CTA kernel, then a range pass per output
  if ((rc = adain_one_cta(p))) return rc;
  for (int k = 0; k < p->n_out; ++k)
    if ((rc = dq_range_launch(p->out[k], BT_F32, p->rows * p->cols, rec[k]))) return rc;
  return BT_OK;
}

extern "C" int bt_resblock_mean_leaky(const float* const* a, const float* const* b, int64_t n, float divisor,
                                      float slope, float* out) {
  if (!a || !b || !out) return set_error(BT_EINVAL, "bt_resblock_mean_leaky: null argument");
  MeanLeakyArgs m{};
  bool vec = ((uintptr_t)out % 16) == 0;
  for (int k = 0; k < 3; ++k) {
    if (!a[k] || !b[k]) return set_error(BT_EINVAL, "bt_resblock_mean_leaky: null input %d", k);
    m.a[k] = a[k];
    m.b[k] = b[k];
    if ((uintptr_t)a[k] % 16 || (uintptr_t)b[k] % 16) vec = false;
  }
  if (n < 0) return set_error(BT_EINVAL, "bt_resblock_mean_leaky: negative size");
  if (n == 0) return BT_OK;
  m.n = n;
  m.rdiv = 1.0 / (double)divisor;
  m.slope = slope;
  m.out = out;
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  int64_t blocks = ((vec ? n / 4 : n) + 255) / 256;
  int64_t cap = (int64_t)di.sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (vec) mean_leaky_kernel<<<(int)blocks, 256, 0, cur_stream()>>>(m);
  else mean_leaky_scalar_kernel<<<(int)blocks, 256, 0, cur_stream()>>>(m);
  return check_launch("bt_resblock_mean_leaky");
}

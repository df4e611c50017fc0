// bt_adain.cu -- AdaIN1d + Snake with rows split across a thread-block
// cluster (sm_100a).
//
// A row of T values (T up to 49152) is cut at pairwise-tree leaf boundaries
// into `cs` contiguous segments, one per CTA of a cluster of cs CTAs.  Each
// CTA
//   1. stages its segment of every source into shared memory with one bulk
//      (TMA) copy per source, completing on an mbarrier;
//   2. sums its leaves of h = src0 + src1 + src2 (numpy's eight-accumulator
//      leaf sum, two lanes per leaf) and stores each leaf sum into the tree
//      array of every CTA of the cluster with st.async, which completes
//      four bytes on the receiving CTA's mbarrier;
//   3. waits on its own mbarrier for all leaf sums of the row (no cluster
//      barrier), combines the tree (one warp) -> the exact numpy mean; the
//      same for the squared deviations -> the variance;
//   4. writes its segment of the residual (a bulk copy out of shared memory)
//      and of every output.
// HBM sees each input once and each output once.  The pairwise plan (sorted
// leaves, heap ids, inner-node bitmask) depends on T only; the host computes
// it once per T and passes it in the kernel's parameter block, so no CTA
// rebuilds it.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <algorithm>
#include <type_traits>
#include <map>
#include <mutex>
#include <vector>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"
#include "bt_dq.h"
#include "bt_pk.h"
#include "bt_bulk.h"

namespace bt {
namespace cg = cooperative_groups;

namespace {

constexpr int kMaxLeaves = 512;
constexpr int kMaxSlots = 384;
constexpr int kMaxIds = 1024;     // heap ids < 2^(D+1), D <= 9
constexpr int kMaxCluster = 8;
constexpr int kThreads = 256;
constexpr int kMaxT = 49152;

// The pairwise plan of one row length T for a cluster of cs CTAs.  Rank r
// owns the elements [rank_e[r], rank_e[r+1]) -- whole leaves -- and the
// slots [rank_slot[r], rank_slot[r+1]).  A slot is the work of one group of
// eight lanes in a leaf pass: one leaf, or two leaves with the same number of
// 8-element steps, summed side by side in the two halves of a float2.
//   w0: offset of leaf A / 8 (bits 0-12) | offset of leaf B / 8 (13-25),
//       both relative to rank_e[r] (B = A when the slot has one leaf)
//   w1: heap id of A (0-9) | heap id of B (10-19, 0 = none) | steps (20-24)
//       | A's remainder len % 8 (25-27) | B's remainder (28-30)
struct SlotPlan {
  int32_t T, D, cs;
  int32_t perfect;                     // 1: every leaf at depth D (leaf i = heap id 2^D + i)
  int32_t nleaves;                     // leaves of the whole row (every rank's)
  int32_t rank_e[kMaxCluster + 1];
  int32_t rank_slot[kMaxCluster + 1];
  uint32_t inner[kMaxIds / 32];        // bit h: heap node h is an inner node
  uint32_t w0[kMaxSlots];
  uint32_t w1[kMaxSlots];
};

struct AdainArgs {
  SlotPlan P;
  int64_t gain_stride, shift_stride;
  int32_t n_out, alpha_dtype, seg_cap;
  int32_t log2_cs, log2_c, channels32;   // log2_c < 0: channels not a power of two
  float eps;
  double rT;                             // RN64(1 / T)
  const float* src0;
  const float* src1;
  const float* src2;
  float* res;
  const float* gain[BT_ADAIN_MAX_OUT];
  const float* shift[BT_ADAIN_MAX_OUT];
  const void* alpha[BT_ADAIN_MAX_OUT];
  const void* inv_alpha[BT_ADAIN_MAX_OUT];
  float* out[BT_ADAIN_MAX_OUT];
  uint32_t* range[BT_ADAIN_MAX_OUT];     // RANGE kernels: output k's min / max / NaN record
};

__device__ __forceinline__ int phase4(const void* p) { return (int)(((uintptr_t)p >> 2) & 3); }


__device__ __forceinline__ float ldf(const void* p, int dt, int64_t i) {
  return dt == BT_F16 ? __half2float(((const __half*)p)[i]) : ((const float*)p)[i];
}

// Copies n floats g[0..n) into b[0..n) (b shares g's 16-byte phase): the
// aligned interior as one bulk copy completing on `bar` (issued by thread
// 0), the at most six edge elements by plain loads of threads 32-37.
__device__ __forceinline__ void stage_bulk(float* b, const float* g, int n, uint64_t* bar) {
  int head = (4 - phase4(g)) & 3;
  if (head > n) head = n;
  const int nvec = (n - head) >> 2;
  const int tail0 = head + 4 * nvec;
  const int nedge = head + (n - tail0);
  const int t = (int)threadIdx.x - 32;
  if (t >= 0 && t < nedge) {
    const int i = t < head ? t : tail0 + (t - head);
    b[i] = g[i];
  }
  if (threadIdx.x == 0 && nvec > 0) bulk_load(b + head, g + head, 16u * (unsigned)nvec, bar);
}

// Combines the inner nodes of the tree in hs (warp 0, level by level); the
// root hs[1] is the sum.  Only warp 0 returns with a complete tree: callers
// read hs[1] from warp 0 (or after a barrier).
__device__ __forceinline__ void tree_combine(float* hs, const uint32_t* inner, int D) {
  if (threadIdx.x < 32) {
    for (int k = D - 1; k >= 0; --k) {
      for (int j = threadIdx.x; j < (1 << k); j += 32) {
        const int h = (1 << k) + j;
        if ((inner[h >> 5] >> (h & 31)) & 1u) hs[h] = BT_ADD(hs[2 * h], hs[2 * h + 1]);
      }
      __syncwarp();
    }
  }
}

// Sum of K consecutive leaves p[0..K) in pairwise order: (p0+p1), (p2+p3),
// ... then pairs of those, and so on.
template <int K>
__device__ __forceinline__ float lane_leaves(const float* p) {
  float v[K];
  if constexpr (K == 2) {
    const float2 q = *reinterpret_cast<const float2*>(p);
    v[0] = q.x; v[1] = q.y;
  } else {
#pragma unroll
    for (int i = 0; i < K; i += 4) {
      const float4 q = *reinterpret_cast<const float4*>(p + i);
      v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
    }
  }
#pragma unroll
  for (int w = K; w > 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w / 2; ++i) v[i] = BT_ADD(v[2 * i], v[2 * i + 1]);
  }
  return v[0];
}

// Root of the pairwise tree held in hs (call from all 32 lanes of warp 0;
// every lane returns it).  A perfect tree (every leaf at depth D, leaf i at
// heap id 2^D + i) is summed with the same additions as tree_combine but in
// registers: lane l adds its 2^D / 32 consecutive leaves pairwise, then xor
// shuffles join sibling lanes level by level (float addition commutes).
// Other trees go level by level through shared memory.
__device__ __forceinline__ float tree_total(float* hs, const uint32_t* inner, int D, bool perfect) {
  const int lane = threadIdx.x & 31;
  if (perfect && D <= 9) {
    const float* leaf = hs + (1 << D);
    float v;
    int levels = 5;
    switch (D) {
      case 9: v = lane_leaves<16>(leaf + 16 * lane); break;
      case 8: v = lane_leaves<8>(leaf + 8 * lane); break;
      case 7: v = lane_leaves<4>(leaf + 4 * lane); break;
      case 6: v = lane_leaves<2>(leaf + 2 * lane); break;
      default:
        v = lane < (1 << D) ? leaf[lane] : 0.0f;
        levels = D;
        break;
    }
    for (int m = 0; m < levels; ++m) v = BT_ADD(v, __shfl_xor_sync(0xffffffffu, v, 1 << m));
    return v;
  }
  tree_combine(hs, inner, D);
  return hs[1];
}

__device__ __forceinline__ float2 shfl_xor2(unsigned mask, float2 v, int m) {
  return make_float2(__shfl_xor_sync(mask, v.x, m), __shfl_xor_sync(mask, v.y, m));
}

// One leaf-sum pass over this CTA's slots.  Lane j of a slot's group owns
// numpy's accumulator j of both leaves (elements 8m + j), so at every step
// the group reads eight consecutive floats per leaf: the host orders slots so
// that the four groups of a warp start in different 8-bank octets, which
// keeps the reads free of bank conflicts.  The accumulators start at -0.0
// (-0.0 + x == x for every x, so the first add reproduces numpy's r[j] =
// a[j]); lanes then combine them with xor shuffles over lane bits 0, 1, 2 --
// numpy's bracket ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), float addition being
// commutative -- and add the len % 8 remainder left to right (a leaf shorter
// than 8 is the remainder alone, summed from +0.0).  Lanes j < cs store the
// leaf sums into hs[id] of cluster rank j with st.async, each store
// completing 4 bytes on that rank's mbarrier `bar` (hs and bar are this
// CTA's shared addresses; every rank uses the same layout).
//   pass 1 (SQ false): leaf value h = src0 (+ src1 (+ src2)); with NSRC > 1 h
//     is also stored back into b0 for the later passes;
//   pass 2 (SQ true, NSRC 1): (h - mu)^2.
template <int NSRC, bool SQ>
__device__ __forceinline__ void slot_pass(const uint32_t* sw, int ns, float* b0, const float* b1, const float* b2,
                                          float mu, unsigned hs, unsigned bar, int cs) {
  const int j = threadIdx.x & 7;
  const unsigned gmask = 0xffu << (threadIdx.x & 24);
  const float2 nmu = pk(-mu);
  auto lv = [&](int i) -> float {   // one leaf value, scalar (remainders)
    float v = b0[i];
    if (NSRC > 1) v = BT_ADD(v, b1[i]);
    if (NSRC > 2) v = BT_ADD(v, b2[i]);
    if (NSRC > 1 && !SQ) b0[i] = v;
    if (SQ) {
      const float d = BT_SUB(v, mu);
      return BT_MUL(d, d);
    }
    return v;
  };
  for (int s = threadIdx.x >> 3; s < ns; s += kThreads >> 3) {
    const uint32_t w0 = sw[2 * s], w1 = sw[2 * s + 1];
    const int oa = (int)(w0 & 0x1fffu) << 3;
    const int ob = (int)((w0 >> 13) & 0x1fffu) << 3;
    const int steps = (int)((w1 >> 20) & 31u);
    const int end = steps << 3;
    float2 acc = pk(-0.0f);
    float* pa0 = b0 + oa + j;
    float* pb0 = b0 + ob + j;
    const float* pa1 = NSRC > 1 ? b1 + oa + j : nullptr;
    const float* pb1 = NSRC > 1 ? b1 + ob + j : nullptr;
    const float* pa2 = NSRC > 2 ? b2 + oa + j : nullptr;
    const float* pb2 = NSRC > 2 ? b2 + ob + j : nullptr;
#pragma unroll 4
    for (int m = 0; m < steps; ++m) {
      const int i = 8 * m;
      float2 x = pk(pa0[i], pb0[i]);
      if (NSRC > 1) {
        x = pk_add(x, pk(pa1[i], pb1[i]));
        if (NSRC > 2) x = pk_add(x, pk(pa2[i], pb2[i]));
        if (!SQ) {
          pa0[i] = x.x;
          pb0[i] = x.y;
        }
      }
      if (SQ) {
        const float2 d = pk_add(x, nmu);
        acc = pk_add_lanes(acc, pk_mul(d, d));
      } else {
        acc = pk_add(acc, x);
      }
    }
    acc = pk_add(acc, shfl_xor2(gmask, acc, 1));
    acc = pk_add(acc, shfl_xor2(gmask, acc, 2));
    acc = pk_add(acc, shfl_xor2(gmask, acc, 4));
    if (steps == 0) acc = pk(0.0f);
    const int ta = (int)((w1 >> 25) & 7u), tb = (int)((w1 >> 28) & 7u);
    if (ta | tb) {
      // one lane walks the remainders (pass 1 may store h back), then shares
      if (j == 0) {
        for (int t = 0; t < ta; ++t) acc.x = BT_ADD(acc.x, lv(oa + end + t));
        for (int t = 0; t < tb; ++t) acc.y = BT_ADD(acc.y, lv(ob + end + t));
      }
      acc.x = __shfl_sync(gmask, acc.x, 0, 8);
      acc.y = __shfl_sync(gmask, acc.y, 0, 8);
    }
    if (j < cs) {
      const unsigned dst = cluster_addr(hs, (unsigned)j), rbar = cluster_addr(bar, (unsigned)j);
      st_async_f32(dst + 4u * (w1 & 1023u), acc.x, rbar);
      const unsigned idb = (w1 >> 10) & 1023u;
      if (idb) st_async_f32(dst + 4u * idb, acc.y, rbar);
    }
  }
}

// RANGE: also folds every output value into that output's range record
// (DynamicQuantizeLinear of the output then needs no pass of its own over it).
template <int NSRC, bool SNAKE, bool RANGE = false>
__global__ void __launch_bounds__(kThreads, 4) adain_cluster_kernel(AdainArgs A) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float prm[BT_ADAIN_MAX_OUT][4];   // gain, shift, alpha, 1/alpha of this row
  __shared__ float s_mu;                       // mean of this row
  __shared__ double s_rsd;                     // RN64(1 / sd) of this row
  __shared__ int in_range[BT_ADAIN_MAX_OUT];   // output k's sin arguments provably in range
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = A.P.cs;                 // 1, 2, 4 or 8
  const int rank = (int)cluster.block_rank();
  const int row32 = (int)(blockIdx.x >> A.log2_cs);
  const int64_t row = row32;
  const int T = A.P.T;
  const int e0 = A.P.rank_e[rank];
  const int seg = A.P.rank_e[rank + 1] - e0;
  const int sl0 = A.P.rank_slot[rank];
  const int ns = A.P.rank_slot[rank + 1] - sl0;
  const int ids = 2 << A.P.D;

  // shared layout: hs1[ids] hs2[ids] | slot words[2 ns] inner[32] | sources
  float* hs1 = (float*)smem;
  float* hs2 = hs1 + ids;
  uint32_t* sw = (uint32_t*)(hs2 + ids);
  uint32_t* inner = sw + 2 * ns;
  for (int i = threadIdx.x; i < ns; i += kThreads) {
    sw[2 * i] = A.P.w0[sl0 + i];
    sw[2 * i + 1] = A.P.w1[sl0 + i];
  }
  for (int i = threadIdx.x; i < kMaxIds / 32; i += kThreads) inner[i] = A.P.inner[i];
  const int bt = A.log2_c >= 0 ? (row32 >> A.log2_c) : row32 / A.channels32;
  const int c = row32 - bt * A.channels32;
  // sources from the next 16-byte boundary; indexing smem directly (no
  // integer round trip) keeps the pointers in the shared address space
  const int sb_words = (2 * ids + 2 * ns + kMaxIds / 32 + 3) & ~3;
  float* sb = reinterpret_cast<float*>(smem) + sb_words;
  const int64_t gofs = row * (int64_t)T + e0;
  const float* g0 = A.src0 + gofs;
  float* b0 = sb + phase4(g0);
  const float* g1 = NSRC > 1 ? A.src1 + gofs : nullptr;
  const float* g2 = NSRC > 2 ? A.src2 + gofs : nullptr;
  float* b1 = NSRC > 1 ? sb + A.seg_cap + phase4(g1) : nullptr;
  float* b2 = NSRC > 2 ? sb + 2 * A.seg_cap + phase4(g2) : nullptr;

  // the segment of every source by bulk copies completing on one mbarrier;
  // the leaf sums of the two tree passes arrive from every rank by st.async
  // on two more (4 bytes per leaf of the row each, expected from the start)
  __shared__ __align__(8) uint64_t s_bar;
  __shared__ __align__(8) uint64_t s_sum_bar[2];
  if (threadIdx.x == 0) {
    mbar_init(&s_bar, 1);
    mbar_init(&s_sum_bar[0], 1);
    mbar_init(&s_sum_bar[1], 1);
    mbar_arrive_expect_tx(&s_sum_bar[0], 4u * (unsigned)A.P.nleaves);
    mbar_arrive_expect_tx(&s_sum_bar[1], 4u * (unsigned)A.P.nleaves);
    unsigned bytes = 0;
    // announce the bytes before the copies: a copy may complete first
    {
      auto interior = [&](const float* g) {
        int h = (4 - phase4(g)) & 3;
        if (h > seg) h = seg;
        return 16u * (unsigned)((seg - h) >> 2);
      };
      bytes = interior(g0);
      if (NSRC > 1) bytes += interior(g1);
      if (NSRC > 2) bytes += interior(g2);
    }
    mbar_arrive_expect_tx(&s_bar, bytes);
  }
  stage_bulk(b0, g0, seg, &s_bar);
  if (NSRC > 1) stage_bulk(b1, g1, seg, &s_bar);
  if (NSRC > 2) stage_bulk(b2, g2, seg, &s_bar);
  // every CTA of the cluster arrives once its mbarriers are initialised (no
  // release semantics needed beyond the initialisation fence); the wait
  // comes before the first st.async below
  if (cs > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  // the row constants after the copies are issued: their loads overlap the
  // copies instead of delaying them
#pragma unroll
  for (int k = 0; k < BT_ADAIN_MAX_OUT; ++k) {
    if (threadIdx.x == 32 * k && k < A.n_out) {
      prm[k][0] = A.gain[k][bt * A.gain_stride + c];
      prm[k][1] = A.shift[k][bt * A.shift_stride + c];
      if (SNAKE) {
        prm[k][2] = ldf(A.alpha[k], A.alpha_dtype, c);
        prm[k][3] = ldf(A.inv_alpha[k], A.alpha_dtype, c);
      }
    }
  }
  // A CTA barrier for the edge elements, the plan, the row constants and
  // the mbarriers' initialisation; then every thread waits for the bulk
  // copies (a wait that gives up is counted, see bt_bulk.h), and with
  // cs > 1 for every CTA of the cluster to have initialised its mbarriers.
  __syncthreads();
  mbar_wait(&s_bar, 0);
  if (cs > 1) asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");

  // ReduceMean(h).  np.mean: RN32(RN64(sum) / T), computed as
  // RN32(RN64(sum * RN64(1/T))) -- the same float (division by a per-row
  // constant, see div_by).  Warp 0 sums the tree and derives the row
  // scalars; every other warp waits at the CTA barrier.
  slot_pass<NSRC, false>(sw, ns, b0, b1, b2, 0.0f, smem_u32(hs1), smem_u32(&s_sum_bar[0]), cs);
  // pass 1 stored h into b0; the residual's bulk store below reads it
  fence_async_shared();
  __syncthreads();
  int head = (4 - phase4(g0)) & 3;
  if (head > seg) head = seg;
  const int nvec = (seg - head) >> 2;
  float* const rs = A.res ? A.res + gofs : nullptr;
  const bool res_bulk = rs && phase4(rs) == phase4(g0) && nvec > 0;
  if (threadIdx.x < 32) {
    mbar_wait(&s_sum_bar[0], 0);   // every rank's leaf sums
    const float sum = tree_total(hs1, inner, A.P.D, A.P.perfect != 0);
    if (threadIdx.x == 0) s_mu = div_by(BT_ADD(0.0f, sum), A.rT);
  } else if (rs) {
    // the residual h is complete after the first pass: while warp 0 sums
    // the tree, thread 32 stores its aligned interior from shared memory in
    // one bulk copy (b0 is only read from here on; thread 32 waits for the
    // copy before the CTA exits) and the other threads write the edges
    const int t = (int)threadIdx.x - 32;
    constexpr int kW = kThreads - 32;
    if (res_bulk) {
      if (t == 0) {
        bulk_store(rs + head, b0 + head, 16u * (unsigned)nvec);
        bulk_commit();
      }
      for (int i = t; i < head; i += kW) rs[i] = b0[i];
      for (int i = head + 4 * nvec + t; i < seg; i += kW) rs[i] = b0[i];
    } else {
      for (int i = t; i < seg; i += kW) rs[i] = b0[i];
    }
  }
  __syncthreads();
  const float mu = s_mu;
  // Sub, Mul(d, d), ReduceMean, Add eps, Sqrt
  slot_pass<1, true>(sw, ns, b0, nullptr, nullptr, mu, smem_u32(hs2), smem_u32(&s_sum_bar[1]), cs);
  if (threadIdx.x < 32) {
    mbar_wait(&s_sum_bar[1], 0);
    const float ssq = tree_total(hs2, inner, A.P.D, A.P.perfect != 0);
    if (threadIdx.x == 0) {
      const float var = div_by(BT_ADD(0.0f, ssq), A.rT);
      const float sd = BT_SQRT(BT_ADD(var, A.eps));
      const double rsd0 = recip_d(sd);
      s_rsd = rsd0;
      if (SNAKE) {
        // Every |h_i - mu| is at most sqrt(S), S = sum_j (h_j - mu)^2, so
        // |n_i| <= sqrt(S) / sd; the float32 sum of S and each later
        // rounding are far inside the 1 % margins below.  When the bound on
        // |alpha * y| is under half numpy's reduction range, no argument can
        // leave it (NaN or Inf anywhere makes the comparison false and keeps
        // the checks).
        const float nb = BT_MUL(BT_MUL(BT_SQRT(ssq), (float)rsd0), 1.01f);
        for (int k = 0; k < BT_ADAIN_MAX_OUT; ++k) {
          const float zb = BT_MUL(BT_MUL(fabsf(prm[k][2]), BT_ADD(BT_MUL(fabsf(prm[k][0]), nb), fabsf(prm[k][1]))),
                                  1.01f);
          in_range[k] = (k < A.n_out && zb <= 0.5f * 117435.992f) ? 1 : 0;
        }
      }
    }
  }
  __syncthreads();
  const double rsd = s_rsd;

  // the outputs of this segment (coalesced, 128-bit where the phases agree)
  const float2 nmu = pk(-mu);
#pragma unroll
  for (int k = 0; k < BT_ADAIN_MAX_OUT; ++k) {
    if (k >= A.n_out) break;
    const float gain = prm[k][0], shift = prm[k][1];
    const float al = SNAKE ? prm[k][2] : 0.0f, ial = SNAKE ? prm[k][3] : 0.0f;
    // Sub -> Div -> Mul(1 + gamma) -> Add(beta) [-> Mul(alpha) -> Sin -> Pow 2 -> Mul(1/alpha) -> Add]
    auto f = [&](float v) -> float {
      float y = BT_ADD(BT_MUL(gain, div_by(BT_SUB(v, mu), rsd)), shift);
      if (SNAKE) {
        const float t = np_sinf(BT_MUL(al, y));
        y = BT_ADD(y, BT_MUL(ial, BT_MUL(t, t)));
      }
      return y;
    };
    // the same steps on two elements at a time; CHECKED false when the row's
    // bound shows every sin argument in numpy's reduction range
    auto f2 = [&](float2 v, auto checked) -> float2 {
      const float2 a = pk_add(v, nmu);
      const float2 n = pk(div_by(a.x, rsd), div_by(a.y, rsd));
      float2 y = pk_add_lanes(pk_mul(pk(gain), n), pk(shift));
      if (SNAKE)
        y = pk_add_lanes(y, pk_mul(pk(ial), pk_np_sin<true, decltype(checked)::value>(pk_mul(pk(al), y))));
      return y;
    };
    // the range of the values written (RANGE)
    float rlo = INFINITY, rhi = -INFINITY;
    bool rnan = false;
    auto track = [&](float v) {
      if (RANGE) {
        rnan |= v != v;
        rlo = fminf(rlo, v);
        rhi = fmaxf(rhi, v);
      }
    };
    auto vec_loop = [&](float* o, auto checked) {
#pragma unroll 2
      for (int q = threadIdx.x; q < nvec; q += kThreads) {
        const float4 v = *(const float4*)(b0 + head + 4 * q);
        const float2 lo = f2(pk(v.x, v.y), checked), hi = f2(pk(v.z, v.w), checked);
        __stcs((float4*)(o + head + 4 * q), make_float4(lo.x, lo.y, hi.x, hi.y));
        track(lo.x); track(lo.y); track(hi.x); track(hi.y);
      }
    };
    auto put = [&](float* o, int i) {
      const float v = f(b0[i]);
      o[i] = v;
      track(v);
    };
    float* o = A.out[k] + gofs;
    if (phase4(o) == phase4(g0)) {
      if (SNAKE && in_range[k]) vec_loop(o, std::false_type());
      else vec_loop(o, std::true_type());
      for (int i = threadIdx.x; i < head; i += kThreads) put(o, i);
      for (int i = head + 4 * nvec + threadIdx.x; i < seg; i += kThreads) put(o, i);
    } else {
      for (int i = threadIdx.x; i < seg; i += kThreads) put(o, i);
    }
    if (RANGE) {
      // CTA-wide min / max / NaN of this output, one atomic each per CTA
      __shared__ float sr_lo[kThreads / 32], sr_hi[kThreads / 32];
      __shared__ int sr_nan;
      for (int m = 16; m > 0; m >>= 1) {
        rlo = fminf(rlo, __shfl_xor_sync(0xffffffffu, rlo, m));
        rhi = fmaxf(rhi, __shfl_xor_sync(0xffffffffu, rhi, m));
      }
      rnan = __any_sync(0xffffffffu, rnan);
      if (threadIdx.x == 0) sr_nan = 0;
      __syncthreads();
      if ((threadIdx.x & 31) == 0) {
        sr_lo[threadIdx.x >> 5] = rlo;
        sr_hi[threadIdx.x >> 5] = rhi;
        if (rnan) sr_nan = 1;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < kThreads / 32; ++w) {
          rlo = fminf(rlo, sr_lo[w]);
          rhi = fmaxf(rhi, sr_hi[w]);
        }
        uint32_t* rec = A.range[k];
        if (rlo <= rhi) {   // not an all-NaN (or empty) segment
          dq_raise(&rec[0], ~dq_ord(rlo));
          dq_raise(&rec[1], dq_ord(rhi));
        }
        if (sr_nan) atomicOr(&rec[2], 1u);
      }
      __syncthreads();   // the shared words are reused by the next output
    }
  }
  if (res_bulk && threadIdx.x == 32) bulk_wait_all();
}

// ---- host side -------------------------------------------------------------
struct HostPlan {
  int T = 0, D = 0;
  std::vector<int> off, len, id;
  std::vector<uint32_t> inner;
};

void plan_node(HostPlan& p, int h, int lo, int n) {
  if (n <= kPwLeaf) {
    p.off.push_back(lo);
    p.len.push_back(n);
    p.id.push_back(h);
    return;
  }
  p.inner[h >> 5] |= 1u << (h & 31);
  const int n2 = (int)pw_split(n);
  plan_node(p, 2 * h, lo, n2);
  plan_node(p, 2 * h + 1, lo + n2, n - n2);
}

const HostPlan& host_plan(int T) {
  static std::mutex mu;
  static std::map<int, HostPlan> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(T);
  if (it != cache.end()) return it->second;
  HostPlan p;
  p.T = T;
  p.D = pw_depth(T);
  p.inner.assign(kMaxIds / 32, 0u);
  plan_node(p, 1, 0, T);
  return cache.emplace(T, std::move(p)).first->second;
}

// Leaves [first[r], first[r+1]) go to cluster rank r: contiguous runs of
// leaves balanced by element count.  False when cs ranks cannot all get one.
bool rank_split(const HostPlan& hp, int cs, std::vector<int>& first) {
  const int n_leaf = (int)hp.off.size();
  first.assign(cs + 1, 0);
  int r = 0;
  int64_t acc = 0;
  for (int L = 0; L < n_leaf; ++L) {
    acc += hp.len[L];
    if (L == n_leaf - 1 || (acc >= (int64_t)hp.T * (r + 1) / cs && r < cs - 1)) first[++r] = L + 1;
  }
  return r == cs;
}

// The slot plan of one (T, cs), built once and cached.
struct ClusterPlan {
  bool ok = false;
  int max_seg = 0;     // longest rank segment (elements)
  int max_slots = 0;   // most slots of one rank
  SlotPlan P;
};

const ClusterPlan& cluster_plan(int T, int cs) {
  static std::mutex mu;
  static std::map<int64_t, ClusterPlan> cache;
  const HostPlan& hp = host_plan(T);
  std::lock_guard<std::mutex> lk(mu);
  const int64_t key = ((int64_t)T << 4) | cs;
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  ClusterPlan cp;
  memset(&cp.P, 0, sizeof(cp.P));
  cp.P.T = T;
  cp.P.D = hp.D;
  cp.P.cs = cs;
  cp.P.perfect = ((int64_t)hp.off.size() == (1ll << hp.D)) ? 1 : 0;
  cp.P.nleaves = (int32_t)hp.off.size();
  for (int i = 0; i < kMaxIds / 32; ++i) cp.P.inner[i] = hp.inner[i];
  std::vector<int> first;
  bool ok = rank_split(hp, cs, first) && (2 << hp.D) <= kMaxIds;
  int n_slots = 0;
  for (int r = 0; ok && r < cs; ++r) {
    const int lb = first[r], le = first[r + 1];
    const int base = hp.off[lb];
    const int end = (le < (int)hp.off.size()) ? hp.off[le] : T;
    cp.P.rank_e[r] = base;
    cp.P.rank_slot[r] = n_slots;
    if (end - base > cp.max_seg) cp.max_seg = end - base;
    // Pair leaves with the same step count (leaves of one octet first), then
    // arrange the slots in runs of four (one warp) so that the A leaves, and
    // the B leaves, of a run start in different bank octets where possible.
    std::map<int, std::vector<int>> by_steps;
    for (int L = lb; L < le; ++L) by_steps[hp.len[L] / 8].push_back(L);
    struct Slot { int a, b; };
    std::vector<Slot> pool;
    auto oct = [&](int L) { return L < 0 ? -1 : (hp.off[L] / 8) & 3; };
    for (auto& g : by_steps) {
      std::vector<int> v = g.second;
      std::stable_sort(v.begin(), v.end(), [&](int x, int y) { return oct(x) < oct(y); });
      for (size_t i = 0; i < v.size(); i += 2) pool.push_back({v[i], i + 1 < v.size() ? v[i + 1] : -1});
    }
    std::vector<Slot> order;
    std::vector<bool> used(pool.size(), false);
    for (size_t done = 0; done < pool.size();) {
      bool ua[4] = {false, false, false, false}, ub[4] = {false, false, false, false};
      for (int g = 0; g < 4 && done < pool.size(); ++g) {
        int best = -1, best_cost = 1 << 30;
        for (size_t i = 0; i < pool.size(); ++i) {
          if (used[i]) continue;
          const int oa = oct(pool[i].a), ob = oct(pool[i].b);
          const int cost = (ua[oa] ? 1 : 0) + (ob >= 0 && ub[ob] ? 1 : 0);
          if (cost < best_cost) { best_cost = cost; best = (int)i; if (cost == 0) break; }
        }
        used[best] = true;
        ua[oct(pool[best].a)] = true;
        if (pool[best].b >= 0) ub[oct(pool[best].b)] = true;
        order.push_back(pool[best]);
        ++done;
      }
    }
    if (n_slots + (int)order.size() > kMaxSlots) { ok = false; break; }
    for (const Slot& sl : order) {
      const int a = sl.a, b = sl.b >= 0 ? sl.b : sl.a;
      const uint32_t oa = (uint32_t)(hp.off[a] - base) / 8, ob = (uint32_t)(hp.off[b] - base) / 8;
      const uint32_t steps = (uint32_t)hp.len[a] / 8;
      const uint32_t ta = (uint32_t)hp.len[a] % 8, tb = sl.b >= 0 ? (uint32_t)hp.len[b] % 8 : 0u;
      const uint32_t idb = sl.b >= 0 ? (uint32_t)hp.id[b] : 0u;
      if (oa >= 8192 || ob >= 8192 || steps > 16) { ok = false; break; }
      cp.P.w0[n_slots] = oa | (ob << 13);
      cp.P.w1[n_slots] = (uint32_t)hp.id[a] | (idb << 10) | (steps << 20) | (ta << 25) | (tb << 28);
      ++n_slots;
    }
    const int rs = n_slots - cp.P.rank_slot[r];
    if (rs > cp.max_slots) cp.max_slots = rs;
  }
  cp.P.rank_e[cs] = T;
  cp.P.rank_slot[cs] = n_slots;
  // every leaf in exactly one slot: each rank then receives 4 * nleaves
  // bytes of leaf sums per pass, the count its mbarriers expect
  int stored = 0;
  for (int i = 0; ok && i < n_slots; ++i) stored += ((cp.P.w1[i] >> 10) & 1023u) ? 2 : 1;
  if (stored != cp.P.nleaves) ok = false;
  cp.ok = ok;
  return cache.emplace(key, cp).first->second;
}

template <int NSRC, bool SNAKE, bool RANGE>
void* kernel_ptr() { return (void*)adain_cluster_kernel<NSRC, SNAKE, RANGE>; }

template <bool RANGE>
void* pick_kernel_t(int nsrc, bool snake) {
  switch (nsrc * 2 + (snake ? 1 : 0)) {
    case 2: return kernel_ptr<1, false, RANGE>();
    case 3: return kernel_ptr<1, true, RANGE>();
    case 4: return kernel_ptr<2, false, RANGE>();
    case 5: return kernel_ptr<2, true, RANGE>();
    case 6: return kernel_ptr<3, false, RANGE>();
    default: return kernel_ptr<3, true, RANGE>();
  }
}
void* pick_kernel(int nsrc, bool snake, bool range = false) {
  return range ? pick_kernel_t<true>(nsrc, snake) : pick_kernel_t<false>(nsrc, snake);
}

std::mutex g_attr_mu;
bool g_attr_done[64] = {false};
size_t g_dyn_max[64] = {0};

// Raises every variant's dynamic shared-memory limit to what the device
// allows beside the kernel's static shared memory; *dyn_max = the smallest
// such limit over the variants.
int set_attributes(int device, int max_smem, size_t* dyn_max) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (device < 0 || device >= 64) return set_error(BT_EUNSUPPORTED, "device ordinal %d", device);
  if (!g_attr_done[device]) {
    size_t lim = (size_t)max_smem;
    for (int v = 0; v < 12; ++v) {
        const int ns = 1 + v % 3, sn = (v / 3) % 2, rg = v / 6;
        void* fn = pick_kernel(ns, sn != 0, rg != 0);
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, fn);
        if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
        if (fa.sharedSizeBytes >= (size_t)max_smem) return set_error(BT_EUNSUPPORTED, "static shared memory");
        const size_t dyn = (size_t)max_smem - fa.sharedSizeBytes;
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
        if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        if (dyn < lim) lim = dyn;
      }
    g_dyn_max[device] = lim;
    g_attr_done[device] = true;
  }
  *dyn_max = g_dyn_max[device];
  return BT_OK;
}

}  // namespace

// Launches the cluster kernel; returns BT_EUNSUPPORTED when this request is
// outside what it handles (the caller then uses the one-CTA-per-row kernel).
// range (optional): per output, a zeroed 3-word min / max / NaN record that
// the kernel folds the written values into.
int adain_v3(const bt_adain_args* p, uint32_t* const* range) {
  const char* env = getenv("BT_ADAIN_ONE_CTA");
  if (env && env[0] == '1') return BT_EUNSUPPORTED;
  if (p->cols < 1 || p->cols > kMaxT) return BT_EUNSUPPORTED;
  bool snake = p->alpha[0] != nullptr;
  for (int k = 1; k < p->n_out; ++k)
    if ((p->alpha[k] != nullptr) != snake) return BT_EUNSUPPORTED;
  const int T = (int)p->cols;
  const HostPlan& hp = host_plan(T);
  const int n_leaf = (int)hp.off.size();
  if (n_leaf > kMaxLeaves || (2 << hp.D) > kMaxIds) return BT_EUNSUPPORTED;
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  // Smallest cluster whose per-CTA segment of all sources fits ~80 KB.
  const int ids = 2 << hp.D;
  const ClusterPlan* cp = nullptr;
  size_t smem = 0;
  int seg_cap = 0;
  for (int cs = 1; cs <= kMaxCluster; cs *= 2) {
    if (cs > n_leaf) break;
    const ClusterPlan& c = cluster_plan(T, cs);
    if (!c.ok) continue;
    cp = &c;
    seg_cap = ((c.max_seg + 4 + 3) / 4) * 4;
    smem = (size_t)2 * ids * sizeof(float) + (size_t)(2 * c.max_slots + kMaxIds / 32) * sizeof(uint32_t) + 16 +
           (size_t)p->n_src * seg_cap * sizeof(float);
    if (smem <= 80 * 1024) break;
  }
  size_t dyn_max = 0;
  if ((rc = set_attributes(di.device, di.max_smem_optin, &dyn_max))) return rc;
  if (!cp || smem > dyn_max) return BT_EUNSUPPORTED;
  const int cs = cp->P.cs;
  if (p->rows > 0x7fffffff / cs || p->channels > 0x7fffffff) return BT_EUNSUPPORTED;

  AdainArgs A;
  memset(&A, 0, sizeof(A));
  A.P = cp->P;
  A.gain_stride = p->gain_stride;
  A.shift_stride = p->shift_stride;
  A.n_out = p->n_out;
  A.alpha_dtype = p->alpha_dtype;
  A.seg_cap = seg_cap;
  A.log2_cs = cs == 1 ? 0 : cs == 2 ? 1 : cs == 4 ? 2 : 3;
  A.channels32 = (int)p->channels;
  A.log2_c = -1;
  for (int b = 0; b < 31; ++b)
    if ((1ll << b) == p->channels) A.log2_c = b;
  A.eps = p->eps;
  A.rT = 1.0 / (double)T;
  A.src0 = p->src[0];
  A.src1 = p->n_src > 1 ? p->src[1] : nullptr;
  A.src2 = p->n_src > 2 ? p->src[2] : nullptr;
  A.res = p->res;
  for (int k = 0; k < p->n_out; ++k) {
    A.gain[k] = p->gain[k];
    A.shift[k] = p->shift[k];
    A.alpha[k] = p->alpha[k];
    A.inv_alpha[k] = p->inv_alpha[k];
    A.out[k] = p->out[k];
    A.range[k] = range ? range[k] : nullptr;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(p->rows * cs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = cur_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&A};
  cudaError_t e = cudaLaunchKernelExC(&cfg, pick_kernel(p->n_src, snake, range != nullptr), args);
  if (e != cudaSuccess) return set_error(BT_ECUDA, "bt_adain_snake(cluster): %s", cudaGetErrorString(e));
  return check_launch("bt_adain_snake(cluster)");
}

}  // namespace bt

extern "C" int bt_wait_timeouts(uint32_t* count) {
  if (!count) return bt::set_error(BT_EINVAL, "bt_wait_timeouts: null count");
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, bt::g_bulk_timeouts, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(bt::g_bulk_timeouts, &zero, sizeof(zero));
  if (e != cudaSuccess) return bt::set_error(BT_ECUDA, "bt_wait_timeouts: %s", cudaGetErrorString(e));
  *count = v;
  return BT_OK;
}

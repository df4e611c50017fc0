// bt_adain.cu -- AdaIN1d + Snake with rows split across a thread-block
// cluster (sm_100a).
//
// A row of T values (T up to 49152) is cut at pairwise-tree leaf boundaries
// into `cs` contiguous segments, one per CTA of a cluster of cs CTAs.  Each
// CTA
//   1. stages its segment of every source into shared memory with cp.async
//      (16-byte global->shared copies, all in flight at once, no registers);
//   2. sums its leaves of h = src0 + src1 + src2 (numpy's eight-accumulator
//      leaf sum, two lanes per leaf) and writes each leaf sum into the tree
//      array of every CTA of the cluster (distributed shared memory);
//   3. after a cluster barrier, combines the tree (one warp, level by level)
//      -> the exact numpy mean; the same for the squared deviations -> the
//      variance;
//   4. writes its segment of the residual and of every output.
// HBM sees each input once and each output once.  The pairwise plan (sorted
// leaves, heap ids, inner-node bitmask) depends on T only; the host computes
// it once per T and passes it in the kernel's parameter block, so no CTA
// rebuilds it.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <map>
#include <mutex>
#include <vector>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"

namespace bt {
namespace cg = cooperative_groups;

namespace {

constexpr int kMaxLeaves = 512;
constexpr int kMaxIds = 1024;     // heap ids < 2^(D+1), D <= 9
constexpr int kMaxCluster = 8;
constexpr int kThreads = 256;
constexpr int kMaxT = 49152;

struct PlanParams {
  int32_t T, D, n_leaf, cs;
  int32_t rank_leaf[kMaxCluster + 1];   // first leaf of each CTA rank
  uint32_t inner[kMaxIds / 32];        // bit h: heap node h is an inner node
  uint16_t off8[kMaxLeaves];           // leaf offset / 8, leaves sorted by offset
  uint16_t id[kMaxLeaves];             // heap id of the leaf
  uint8_t len[kMaxLeaves];             // leaf length (<= 128)
};

struct AdainV3Args {
  PlanParams P;
  int64_t rows, channels;
  int64_t gain_stride, shift_stride;
  int32_t n_src, n_out, alpha_dtype, seg_cap;
  int32_t log2_cs, log2_c, channels32;   // log2_c < 0: channels not a power of two
  float eps;
  const float* src0;
  const float* src1;
  const float* src2;
  float* res;
  const float* gain[BT_ADAIN_MAX_OUT];
  const float* shift[BT_ADAIN_MAX_OUT];
  const void* alpha[BT_ADAIN_MAX_OUT];
  const void* inv_alpha[BT_ADAIN_MAX_OUT];
  float* out[BT_ADAIN_MAX_OUT];
};

__device__ __forceinline__ int phase4(const void* p) { return (int)(((uintptr_t)p >> 2) & 3); }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ double recip_d(float b) { return __ddiv_rn(1.0, (double)b); }
__device__ __forceinline__ float div_by(float a, double rb) { return __double2float_rn(__dmul_rn((double)a, rb)); }
__device__ __forceinline__ float ldf(const void* p, int dt, int64_t i) {
  return dt == BT_F16 ? __half2float(((const __half*)p)[i]) : ((const float*)p)[i];
}

// Copies n floats g[0..n) into b[0..n) (b shares g's 16-byte phase).
__device__ __forceinline__ void stage_async(float* b, const float* g, int n) {
  int head = (4 - phase4(g)) & 3;
  if (head > n) head = n;
  const int nvec = (n - head) >> 2;
  for (int q = threadIdx.x; q < nvec; q += blockDim.x) cp_async16(b + head + 4 * q, g + head + 4 * q);
  for (int i = threadIdx.x; i < head; i += blockDim.x) b[i] = g[i];
  for (int i = head + 4 * nvec + threadIdx.x; i < n; i += blockDim.x) b[i] = g[i];
}

// This CTA's slice of the pairwise plan, copied from the parameter block
// into shared memory (leaf reads are lane-divergent; shared memory serves
// them in parallel, the constant bank would serialise them).
struct SPlan {
  int* off;        // local leaf offsets (relative to the segment start)
  int* len;
  int* id;
  uint32_t* inner;
  int nl;          // leaves of this CTA
  int D;
};

// Combines the inner nodes of the tree in hs (warp 0, level by level); the
// root hs[1] is the sum.  Only warp 0 returns with a complete tree: callers
// read hs[1] from warp 0 (or after a barrier).
__device__ __forceinline__ void tree_combine(float* hs, const SPlan& S) {
  if (threadIdx.x < 32) {
    for (int k = S.D - 1; k >= 0; --k) {
      for (int j = threadIdx.x; j < (1 << k); j += 32) {
        const int h = (1 << k) + j;
        if ((S.inner[h >> 5] >> (h & 31)) & 1u) hs[h] = BT_ADD(hs[2 * h], hs[2 * h + 1]);
      }
      __syncwarp();
    }
  }
}

template <int NSRC, bool SQ>
__device__ __forceinline__ float leaf_value(float* b0, const float* b1, const float* b2, int i, float mu,
                                            bool store) {
  float v = b0[i];
  if (NSRC > 1) v = BT_ADD(v, b1[i]);
  if (NSRC > 2) v = BT_ADD(v, b2[i]);
  if (NSRC > 1 && store) b0[i] = v;
  if (SQ) {
    const float d = BT_SUB(v, mu);
    return BT_MUL(d, d);
  }
  return v;
}

// Sums this CTA's leaves and writes each leaf sum into hs[id] of every CTA of
// the cluster.  LPL lanes per leaf (2, 4 or 8) each own 8 / LPL of numpy's
// eight accumulators (lane j owns r[j*A .. j*A + A - 1], A = 8 / LPL); the
// accumulators are combined in numpy's bracket order
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) -- inside the lane first, then across
// lanes with xor shuffles (float addition commutes).  NSRC > 1 in the first
// pass also stores h = src0 + src1 (+ src2) back into b0.
template <int NSRC, bool SQ, int LPL>
__device__ __forceinline__ void leaf_pass(const SPlan& S, float* b0, const float* b1, const float* b2, float mu,
                                          float* hs, cg::cluster_group& cluster, int cs) {
  constexpr int APL = 8 / LPL;
  const int j = threadIdx.x & (LPL - 1);
  const unsigned gmask = ((1u << LPL) - 1u) << (threadIdx.x & 31 & ~(LPL - 1));
  const bool store = (NSRC > 1) && !SQ;
  auto lv = [&](int i) -> float { return leaf_value<NSRC, SQ>(b0, b1, b2, i, mu, store); };
  for (int L = threadIdx.x / LPL; L < S.nl; L += blockDim.x / LPL) {
    const int off = S.off[L];
    const int len = S.len[L];
    float res = 0.0f;
    if (len < 8) {
      if (j == 0)
        for (int i = 0; i < len; ++i) res = BT_ADD(res, lv(off + i));
    } else {
      const int o = off + j * APL;
      float r[APL];
#pragma unroll
      for (int a = 0; a < APL; ++a) r[a] = lv(o + a);
      const int full = len & ~7;
      for (int i = 8; i < full; i += 8) {
#pragma unroll
        for (int a = 0; a < APL; ++a) r[a] = BT_ADD(r[a], lv(o + i + a));
      }
      float t;
      if (APL == 4) t = BT_ADD(BT_ADD(r[0], r[1]), BT_ADD(r[2 % APL], r[3 % APL]));
      else if (APL == 2) t = BT_ADD(r[0], r[1 % APL]);
      else t = r[0];
#pragma unroll
      for (int m = 1; m < LPL; m <<= 1) t = BT_ADD(t, __shfl_xor_sync(gmask, t, m));
      res = t;
      if (j == 0)
        for (int i = full; i < len; ++i) res = BT_ADD(res, lv(off + i));
    }
    if (j == 0) {
      const int id = S.id[L];
      for (int rr = 0; rr < cs; ++rr) cluster.map_shared_rank(hs, rr)[id] = res;
    }
  }
}

template <int NSRC, bool SNAKE, int LPL>
__global__ void __launch_bounds__(kThreads, 4) adain_v3_kernel(AdainV3Args A) {
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = A.P.cs;                 // 1, 2, 4 or 8
  const int rank = (int)cluster.block_rank();
  const int row32 = (int)(blockIdx.x >> A.log2_cs);
  const int64_t row = row32;
  const int T = A.P.T;
  const int lb = A.P.rank_leaf[rank], le = A.P.rank_leaf[rank + 1];
  const int e0 = 8 * (int)A.P.off8[lb];
  const int e1 = 8 * (int)A.P.off8[le - 1] + (int)A.P.len[le - 1];
  const int seg = e1 - e0;
  const int ids = 2 << A.P.D;
  const int nl = le - lb;

  // shared layout: hs1[ids] hs2[ids] | off[nl] len[nl] id[nl] inner[32] | sources
  float* hs1 = (float*)smem;
  float* hs2 = hs1 + ids;
  SPlan S;
  S.off = (int*)(hs2 + ids);
  S.len = S.off + nl;
  S.id = S.len + nl;
  S.inner = (uint32_t*)(S.id + nl);
  S.nl = nl;
  S.D = A.P.D;
  for (int L = threadIdx.x; L < nl; L += blockDim.x) {
    S.off[L] = 8 * (int)A.P.off8[lb + L] - e0;
    S.len[L] = (int)A.P.len[lb + L];
    S.id[L] = (int)A.P.id[lb + L];
  }
  for (int j = threadIdx.x; j < kMaxIds / 32; j += blockDim.x) S.inner[j] = A.P.inner[j];
  float* sb = (float*)(((uintptr_t)(S.inner + kMaxIds / 32) + 15) & ~(uintptr_t)15);
  const int64_t gofs = row * (int64_t)T + e0;
  const float* g0 = A.src0 + gofs;
  float* b0 = sb + phase4(g0);
  const float* g1 = NSRC > 1 ? A.src1 + gofs : nullptr;
  const float* g2 = NSRC > 2 ? A.src2 + gofs : nullptr;
  float* b1 = NSRC > 1 ? sb + A.seg_cap + phase4(g1) : nullptr;
  float* b2 = NSRC > 2 ? sb + 2 * A.seg_cap + phase4(g2) : nullptr;

  stage_async(b0, g0, seg);
  if (NSRC > 1) stage_async(b1, g1, seg);
  if (NSRC > 2) stage_async(b2, g2, seg);
  cp_async_wait_all();
  // Also guarantees every CTA of the cluster runs before any distributed
  // shared-memory write below.
  cluster.sync();

  // Per-row scalars are derived once (thread 0) and read back by all threads:
  // scal[0] = mu, scal[1] = 1/sd in double precision (two floats' worth).
  __shared__ double scal[2];
  // ReduceMean(h)
  leaf_pass<NSRC, false, LPL>(S, b0, b1, b2, 0.0f, hs1, cluster, cs);
  cluster.sync();
  tree_combine(hs1, S);
  if (threadIdx.x == 0) scal[0] = (double)np_mean_from_sum(BT_ADD(0.0f, hs1[1]), T);
  __syncthreads();
  const float mu = (float)scal[0];
  // Sub, Mul(d, d), ReduceMean, Add eps, Sqrt
  leaf_pass<1, true, LPL>(S, b0, nullptr, nullptr, mu, hs2, cluster, cs);
  cluster.sync();
  tree_combine(hs2, S);
  if (threadIdx.x == 0) {
    const float var = np_mean_from_sum(BT_ADD(0.0f, hs2[1]), T);
    const float sd = BT_SQRT(BT_ADD(var, A.eps));
    scal[1] = recip_d(sd);
  }
  __syncthreads();
  const double rsd = scal[1];

  // residual h and the outputs of this segment (coalesced, 128-bit where the
  // phases agree)
  int head = (4 - phase4(g0)) & 3;
  if (head > seg) head = seg;
  const int nvec = (seg - head) >> 2;
  if (A.res) {
    float* r = A.res + gofs;
    if (phase4(r) == phase4(g0)) {
      for (int q = threadIdx.x; q < nvec; q += blockDim.x)
        __stcs((float4*)(r + head + 4 * q), *(const float4*)(b0 + head + 4 * q));
      for (int i = threadIdx.x; i < head; i += blockDim.x) r[i] = b0[i];
      for (int i = head + 4 * nvec + threadIdx.x; i < seg; i += blockDim.x) r[i] = b0[i];
    } else {
      for (int i = threadIdx.x; i < seg; i += blockDim.x) r[i] = b0[i];
    }
  }
  const int bt = A.log2_c >= 0 ? (row32 >> A.log2_c) : row32 / A.channels32;
  const int c = row32 - bt * A.channels32;
#pragma unroll
  for (int k = 0; k < BT_ADAIN_MAX_OUT; ++k) {
    if (k >= A.n_out) break;
    const float gain = A.gain[k][bt * A.gain_stride + c];
    const float shift = A.shift[k][bt * A.shift_stride + c];
    float al = 0.0f, ial = 0.0f;
    if (SNAKE) {
      al = ldf(A.alpha[k], A.alpha_dtype, c);
      ial = ldf(A.inv_alpha[k], A.alpha_dtype, c);
    }
    // Sub -> Div -> Mul(1 + gamma) -> Add(beta) [-> Mul(alpha) -> Sin -> Pow 2 -> Mul(1/alpha) -> Add]
    auto f = [&](float v) -> float {
      float y = BT_ADD(BT_MUL(gain, div_by(BT_SUB(v, mu), rsd)), shift);
      if (SNAKE) {
        const float t = np_sinf(BT_MUL(al, y));
        y = BT_ADD(y, BT_MUL(ial, BT_MUL(t, t)));
      }
      return y;
    };
    float* o = A.out[k] + gofs;
    if (phase4(o) == phase4(g0)) {
      for (int q = threadIdx.x; q < nvec; q += blockDim.x) {
        const float4 v = *(const float4*)(b0 + head + 4 * q);
        __stcs((float4*)(o + head + 4 * q), make_float4(f(v.x), f(v.y), f(v.z), f(v.w)));
      }
      for (int i = threadIdx.x; i < head; i += blockDim.x) o[i] = f(b0[i]);
      for (int i = head + 4 * nvec + threadIdx.x; i < seg; i += blockDim.x) o[i] = f(b0[i]);
    } else {
      for (int i = threadIdx.x; i < seg; i += blockDim.x) o[i] = f(b0[i]);
    }
  }
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

template <int NSRC, bool SNAKE, int LPL>
void* kernel_ptr() { return (void*)adain_v3_kernel<NSRC, SNAKE, LPL>; }

template <int LPL>
void* pick_kernel_lpl(int nsrc, bool snake) {
  switch (nsrc * 2 + (snake ? 1 : 0)) {
    case 2: return kernel_ptr<1, false, LPL>();
    case 3: return kernel_ptr<1, true, LPL>();
    case 4: return kernel_ptr<2, false, LPL>();
    case 5: return kernel_ptr<2, true, LPL>();
    case 6: return kernel_ptr<3, false, LPL>();
    default: return kernel_ptr<3, true, LPL>();
  }
}

void* pick_kernel(int nsrc, bool snake, int lpl) {
  if (lpl == 2) return pick_kernel_lpl<2>(nsrc, snake);
  if (lpl == 4) return pick_kernel_lpl<4>(nsrc, snake);
  return pick_kernel_lpl<8>(nsrc, snake);
}

std::mutex g_attr_mu;
bool g_attr_done[64] = {false};

int set_attributes(int device, int max_smem) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (device < 0 || device >= 64) return set_error(BT_EUNSUPPORTED, "device ordinal %d", device);
  if (g_attr_done[device]) return BT_OK;
  for (int lpl = 2; lpl <= 8; lpl *= 2)
    for (int ns = 1; ns <= 3; ++ns)
      for (int sn = 0; sn < 2; ++sn) {
        cudaError_t e = cudaFuncSetAttribute(pick_kernel(ns, sn != 0, lpl),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e != cudaSuccess) return set_error(BT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      }
  g_attr_done[device] = true;
  return BT_OK;
}

}  // namespace

// Launches the cluster kernel; returns BT_EUNSUPPORTED when this request is
// outside what it handles (the caller then uses the one-CTA-per-row kernel).
int adain_v3(const bt_adain_args* p) {
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
  int cs = 1;
  size_t smem = 0;
  int seg_cap = 0;
  for (cs = 1; cs <= kMaxCluster; cs *= 2) {
    if (cs > n_leaf) return BT_EUNSUPPORTED;
    // balance leaves by element count
    int max_seg = 0, r = 0, start = 0, acc = 0;
    for (int L = 0; L < n_leaf; ++L) {
      acc += hp.len[L];
      const bool last = L == n_leaf - 1;
      if (last || (acc >= (int64_t)T * (r + 1) / cs && r < cs - 1)) {
        const int seg = hp.off[L] + hp.len[L] - hp.off[start];
        if (seg > max_seg) max_seg = seg;
        start = L + 1;
        ++r;
      }
    }
    if (r != cs) continue;
    seg_cap = ((max_seg + 4 + 3) / 4) * 4;
    smem = (size_t)2 * ids * sizeof(float) + (size_t)3 * n_leaf * sizeof(int) + (kMaxIds / 32) * 4 + 16 +
           (size_t)p->n_src * seg_cap * sizeof(float);
    if (smem <= 80 * 1024 || cs == kMaxCluster) break;
  }
  if (cs > kMaxCluster || smem > (size_t)di.max_smem_optin) return BT_EUNSUPPORTED;

  AdainV3Args A;
  memset(&A, 0, sizeof(A));
  A.P.T = T;
  A.P.D = hp.D;
  A.P.n_leaf = n_leaf;
  A.P.cs = cs;
  for (int i = 0; i < kMaxIds / 32; ++i) A.P.inner[i] = hp.inner[i];
  for (int L = 0; L < n_leaf; ++L) {
    A.P.off8[L] = (uint16_t)(hp.off[L] / 8);
    A.P.id[L] = (uint16_t)hp.id[L];
    A.P.len[L] = (uint8_t)hp.len[L];
  }
  {
    int r = 0, acc = 0;
    A.P.rank_leaf[0] = 0;
    for (int L = 0; L < n_leaf; ++L) {
      acc += hp.len[L];
      if (L == n_leaf - 1 || (acc >= (int64_t)T * (r + 1) / cs && r < cs - 1)) A.P.rank_leaf[++r] = L + 1;
    }
    if (r != cs) return BT_EUNSUPPORTED;
  }
  A.rows = p->rows;
  A.channels = p->channels;
  A.gain_stride = p->gain_stride;
  A.shift_stride = p->shift_stride;
  A.n_src = p->n_src;
  A.n_out = p->n_out;
  A.alpha_dtype = p->alpha_dtype;
  A.seg_cap = seg_cap;
  A.log2_cs = cs == 1 ? 0 : cs == 2 ? 1 : cs == 4 ? 2 : 3;
  if (p->rows > 0x7fffffff / cs || p->channels > 0x7fffffff) return BT_EUNSUPPORTED;
  A.channels32 = (int)p->channels;
  A.log2_c = -1;
  for (int b = 0; b < 31; ++b)
    if ((1ll << b) == p->channels) A.log2_c = b;
  int max_nl = 0;
  for (int r = 0; r < cs; ++r) {
    const int nl = A.P.rank_leaf[r + 1] - A.P.rank_leaf[r];
    if (nl > max_nl) max_nl = nl;
  }
  // lanes per leaf: enough leaves in flight to occupy the CTA
  const int lpl = (max_nl * 8 <= kThreads) ? 8 : (max_nl * 4 <= kThreads) ? 4 : 2;
  A.eps = p->eps;
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
  }
  if ((rc = set_attributes(di.device, di.max_smem_optin))) return rc;

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
  cudaError_t e = cudaLaunchKernelExC(&cfg, pick_kernel(p->n_src, snake, lpl), args);
  if (e != cudaSuccess) return set_error(BT_ECUDA, "bt_adain_snake(cluster): %s", cudaGetErrorString(e));
  return check_launch("bt_adain_snake(cluster)");
}

}  // namespace bt

// bt_quant.cu -- DynamicQuantizeLinear as the reference's numpy op computes
// it (tools/ref_runtime.py:106-116, dispatched at :625-630):
//
//   lo = min(0, float(min x)), hi = max(0, float(max x))     Python floats
//   scale = (hi - lo) / 255, or 1 when that is 0              double
//   zp = clip(rint(0 - lo / scale), 0, 255)                   double
//   y = uint8(clip(rint(x / scale) + zp, 0, 255))             x / scale in float32:
//       numpy 2 turns the Python-float scale into the array's float32
//
// Two kernels over one 12-byte scratch record per (device, stream): the first
// reduces min, max and "NaN seen" into it with atomics (values mapped to
// order-preserving integers, all identities 0, so one memset clears it); the
// second has every CTA derive scale and zero point from the record -- the
// same double arithmetic in every CTA, so all agree -- and quantizes 16
// values per thread (four 128-bit loads, one 128-bit store), each by a
// float32 shortcut that falls back to the exact double quotient near the
// half-integers where the two could differ (bt_dq.h).  CTA 0 writes
// the scale and zero-point outputs.  A NaN anywhere makes numpy's min and max
// NaN, which Python's min(0.0, nan) and max(0.0, nan) turn into 0: scale 1,
// zero point 0; the NaN elements themselves become 0 here (numpy's cast of
// NaN to uint8 is platform-defined; 0 on x86-64).  Aligned float32 inputs
// of up to 2^17 values (most of the model's quantised activations) take one
// launch of one thread-block cluster instead, which holds x in registers,
// combines the range in distributed shared memory and needs neither the
// scratch record nor its memset.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <map>
#include <mutex>
#include <utility>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"
#include "bt_dq.h"

namespace bt {
namespace {

namespace cg = cooperative_groups;
constexpr int kThreads = 256;

// scratch[0] = ~ord(min) (atomicMax), scratch[1] = ord(max), scratch[2] = NaN seen
template <typename T>
__device__ __forceinline__ float ldx(const T* x, int64_t i) {
  if constexpr (sizeof(T) == 2) return __half2float(x[i]);
  else return x[i];
}

template <typename T>
__global__ void __launch_bounds__(kThreads) dq_range_kernel(const T* x, int64_t n, uint32_t* scratch) {
  float lo = INFINITY, hi = -INFINITY;
  bool nan = false;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i0 = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if constexpr (sizeof(T) == 4) {
    // 128-bit loads when x is 16-byte aligned
    if (((uintptr_t)x & 15) == 0) {
      const int64_t nv = n >> 2;
      const float4* xv = reinterpret_cast<const float4*>(x);
      auto take = [&](const float4 f) {
        nan |= (f.x != f.x) | (f.y != f.y) | (f.z != f.z) | (f.w != f.w);
        lo = fminf(lo, fminf(fminf(f.x, f.y), fminf(f.z, f.w)));
        hi = fmaxf(hi, fmaxf(fmaxf(f.x, f.y), fmaxf(f.z, f.w)));
      };
      int64_t v = i0;
      // four vectors in flight per thread
      for (; v + 3 * stride < nv; v += 4 * stride) {
        const float4 f0 = __ldcs(xv + v), f1 = __ldcs(xv + v + stride);
        const float4 f2 = __ldcs(xv + v + 2 * stride), f3 = __ldcs(xv + v + 3 * stride);
        take(f0); take(f1); take(f2); take(f3);
      }
      for (; v < nv; v += stride) take(__ldcs(xv + v));
      // the n % 4 tail: threads of CTA 0
      i0 = (blockIdx.x == 0 && threadIdx.x < (n & 3)) ? (nv << 2) + threadIdx.x : n;
    }
  }
  for (int64_t i = i0; i < n; i += stride) {
    const float v = ldx(x, i);
    nan |= v != v;
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  nan = __any_sync(0xffffffffu, nan);
  __shared__ float slo[kThreads / 32], shi[kThreads / 32];
  __shared__ int snan;
  if (threadIdx.x == 0) snan = 0;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    slo[threadIdx.x >> 5] = lo;
    shi[threadIdx.x >> 5] = hi;
    if (nan) snan = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kThreads / 32; ++w) {
      lo = fminf(lo, slo[w]);
      hi = fmaxf(hi, shi[w]);
    }
    // an all-NaN share leaves lo = +inf, hi = -inf: the identities
    if (lo <= hi) {
      dq_raise(&scratch[0], ~dq_ord(lo));
      dq_raise(&scratch[1], dq_ord(hi));
    }
    if (snan) atomicOr(&scratch[2], 1u);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) dq_quantize_kernel(const T* x, int64_t n, const uint32_t* scratch,
                                                               uint8_t* y, float* scale_out, uint8_t* zp_out) {
  __shared__ DqParams sp;
  if (threadIdx.x == 0) sp = dq_params(scratch, n);
  __syncthreads();
  const DqParams p = sp;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *scale_out = p.scale32;
    *zp_out = (uint8_t)p.zp;
  }
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t done = 0;
  if constexpr (sizeof(T) == 4) {
    if (((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0) {
      // 16 values per thread: four 128-bit loads, one 128-bit store
      const int64_t ng = n >> 4;
      for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < ng; g += stride) {
        const float4* src = reinterpret_cast<const float4*>(x) + 4 * g;
        float4 f[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) f[k] = __ldcs(src + k);
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          w[k] = q8(f[k].x, p) | (q8(f[k].y, p) << 8) | (q8(f[k].z, p) << 16) | (q8(f[k].w, p) << 24);
        __stcs(reinterpret_cast<uint4*>(y) + g, make_uint4(w[0], w[1], w[2], w[3]));
      }
      done = ng << 4;
    }
  }
  for (int64_t i = done + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
    y[i] = (uint8_t)q8(ldx(x, i), p);
}

// Small inputs: one launch of one cluster of kSmallCtas CTAs, x read once,
// no scratch.  For float32 x on a 16-byte boundary of up to kSmallMax values
// every thread loads its (at most kSmallVec) float4 groups into registers
// at once, the CTA reduces them to a record in its shared memory (the
// integer forms of the range record above), and after a cluster barrier
// every CTA combines the kSmallCtas records through distributed shared
// memory, derives scale and zero point as dq_quantize_kernel does and
// quantizes the values it holds.  The second barrier keeps every CTA's
// record alive until all have read it.
constexpr int kSmallCtas = 8;
constexpr int kSmallThreads = 512;
constexpr int kSmallVec = 8;
constexpr int64_t kSmallMax = (int64_t)kSmallCtas * kSmallThreads * kSmallVec * 4;   // 2^17 values

__global__ void __cluster_dims__(kSmallCtas, 1, 1) __launch_bounds__(kSmallThreads, 1)
    dq_cluster_kernel(const float* x, int64_t n, uint8_t* y, float* scale_out, uint8_t* zp_out) {
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  __shared__ uint32_t part[3];
  __shared__ float slo[kSmallThreads / 32], shi[kSmallThreads / 32];
  __shared__ int snan;
  __shared__ DqParams sp;
  const int t0 = rank * kSmallThreads + (int)threadIdx.x;
  constexpr int stride = kSmallCtas * kSmallThreads;
  const int nv = (int)(n >> 2);
  const float4* xv = reinterpret_cast<const float4*>(x);
  float4 v[kSmallVec];
#pragma unroll
  for (int k = 0; k < kSmallVec; ++k) {
    const int q = t0 + k * stride;
    if (q < nv) v[k] = __ldcs(xv + q);
  }
  // the n % 4 tail: threads 0..2 of CTA 0
  const int tail = (rank == 0 && (int)threadIdx.x < (int)(n & 3)) ? (int)(nv << 2) + (int)threadIdx.x : -1;
  const float tv = tail >= 0 ? x[tail] : 0.0f;
  float lo = INFINITY, hi = -INFINITY;
  bool nan = false;
  auto take = [&](float f) {
    nan |= f != f;
    lo = fminf(lo, f);
    hi = fmaxf(hi, f);
  };
#pragma unroll
  for (int k = 0; k < kSmallVec; ++k)
    if (t0 + k * stride < nv) {
      take(v[k].x); take(v[k].y); take(v[k].z); take(v[k].w);
    }
  if (tail >= 0) take(tv);
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  nan = __any_sync(0xffffffffu, nan);
  if (threadIdx.x == 0) snan = 0;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    slo[threadIdx.x >> 5] = lo;
    shi[threadIdx.x >> 5] = hi;
    if (nan) snan = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kSmallThreads / 32; ++w) {
      lo = fminf(lo, slo[w]);
      hi = fmaxf(hi, shi[w]);
    }
    part[0] = lo <= hi ? ~dq_ord(lo) : 0u;   // an all-NaN share keeps the identities
    part[1] = lo <= hi ? dq_ord(hi) : 0u;
    part[2] = snan ? 1u : 0u;
  }
  cluster.sync();
  if (threadIdx.x < 32) {
    // lane r reads CTA r's record; max / or across the lanes
    uint32_t rec[3] = {0u, 0u, 0u};
    if (threadIdx.x < kSmallCtas) {
      const uint32_t* q = cluster.map_shared_rank(part, (int)threadIdx.x);
      rec[0] = q[0];
      rec[1] = q[1];
      rec[2] = q[2];
    }
    for (int o = kSmallCtas / 2; o > 0; o >>= 1) {
      rec[0] = max(rec[0], __shfl_xor_sync(0xffffffffu, rec[0], o));
      rec[1] = max(rec[1], __shfl_xor_sync(0xffffffffu, rec[1], o));
      rec[2] |= __shfl_xor_sync(0xffffffffu, rec[2], o);
    }
    if (threadIdx.x == 0) {
      sp = dq_params(rec, n);
      if (rank == 0) {
        *scale_out = sp.scale32;
        *zp_out = (uint8_t)sp.zp;
      }
    }
  }
  cluster.sync();
  const DqParams p = sp;
  uint32_t* yw = reinterpret_cast<uint32_t*>(y);
#pragma unroll
  for (int k = 0; k < kSmallVec; ++k) {
    const int q = t0 + k * stride;
    if (q < nv) __stcs(yw + q, q8(v[k].x, p) | (q8(v[k].y, p) << 8) | (q8(v[k].z, p) << 16) | (q8(v[k].w, p) << 24));
  }
  if (tail >= 0) y[tail] = (uint8_t)q8(tv, p);
}

// One 16-byte scratch record per (device, stream), allocated on first use.
int scratch_for(int device, cudaStream_t s, uint32_t** out) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, uint32_t*> records;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(device, s);
  auto it = records.find(key);
  if (it == records.end()) {
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, 16);
    if (e != cudaSuccess) return set_error(BT_ECUDA, "bt_dynamic_quantize: scratch cudaMalloc: %s", cudaGetErrorString(e));
    it = records.emplace(key, (uint32_t*)p).first;
  }
  *out = it->second;
  return BT_OK;
}

}  // namespace

// The quantize pass over a filled range record.
int dq_quantize_launch(const bt_tensor* x, const bt_tensor* y, float* scale_out, uint8_t* zp_out,
                       const uint32_t* rec, const char* what) {
  const int64_t n = numel(x);
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  int64_t blocks = (n + kThreads * 16 - 1) / (kThreads * 16);
  const int64_t cap = (int64_t)di.sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  cudaStream_t s = cur_stream();
  if (x->dtype == BT_F32)
    dq_quantize_kernel<float><<<(int)blocks, kThreads, 0, s>>>((const float*)x->data, n, rec, (uint8_t*)y->data,
                                                               scale_out, zp_out);
  else
    dq_quantize_kernel<__half><<<(int)blocks, kThreads, 0, s>>>((const __half*)x->data, n, rec, (uint8_t*)y->data,
                                                                scale_out, zp_out);
  return check_launch(what);
}

// Shared by bt_dynamic_quantize and its no-allocation variant: the launches
// over a given scratch record.
int dynamic_quantize_run(const bt_tensor* x, const bt_tensor* y, float* scale_out, uint8_t* zp_out,
                         uint32_t* scratch) {
  const int64_t n = numel(x);
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  cudaStream_t s = cur_stream();
  if (n <= kSmallMax && x->dtype == BT_F32 && ((uintptr_t)x->data & 15) == 0 && ((uintptr_t)y->data & 3) == 0) {
    // one cluster, one launch, the scratch record unused
    dq_cluster_kernel<<<kSmallCtas, kSmallThreads, 0, s>>>((const float*)x->data, n, (uint8_t*)y->data, scale_out,
                                                           zp_out);
    return check_launch("bt_dynamic_quantize");
  }
  cudaError_t e = cudaMemsetAsync(scratch, 0, 12, s);
  if (e != cudaSuccess) return set_error(BT_ECUDA, "bt_dynamic_quantize: memset: %s", cudaGetErrorString(e));
  int64_t blocks = (n + kThreads * 16 - 1) / (kThreads * 16);
  const int64_t cap = (int64_t)di.sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (x->dtype == BT_F32) dq_range_kernel<float><<<(int)blocks, kThreads, 0, s>>>((const float*)x->data, n, scratch);
  else dq_range_kernel<__half><<<(int)blocks, kThreads, 0, s>>>((const __half*)x->data, n, scratch);
  return dq_quantize_launch(x, y, scale_out, zp_out, scratch, "bt_dynamic_quantize");
}

int dq_range_launch(const void* x, int32_t dtype, int64_t n, uint32_t* rec) {
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  int64_t blocks = (n + kThreads * 16 - 1) / (kThreads * 16);
  const int64_t cap = (int64_t)di.sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (dtype == BT_F32) dq_range_kernel<float><<<(int)blocks, kThreads, 0, cur_stream()>>>((const float*)x, n, rec);
  else dq_range_kernel<__half><<<(int)blocks, kThreads, 0, cur_stream()>>>((const __half*)x, n, rec);
  return check_launch("dq_range");
}

int dynamic_quantize_check(const bt_tensor* x, const bt_tensor* y, const float* scale_out, const uint8_t* zp_out,
                           const char* what) {
  int rc = check_tensor(x, "x", false);
  if (rc) return rc;
  if ((rc = check_tensor(y, "y", false))) return rc;
  if (!scale_out || !zp_out) return set_error(BT_EINVAL, "%s: null scale or zero-point output", what);
  if (x->dtype != BT_F32 && x->dtype != BT_F16) return set_error(BT_EDTYPE, "%s: x must be float32 or float16", what);
  if (y->dtype != BT_U8) return set_error(BT_EDTYPE, "%s: y must be uint8", what);
  if (!is_contiguous(x) || !is_contiguous(y) || numel(x) != numel(y))
    return set_error(BT_EUNSUPPORTED, "%s: contiguous x and y of equal size only", what);
  if (numel(x) == 0) return set_error(BT_ESHAPE, "%s: empty input (numpy's min of an empty array raises)", what);
  return BT_OK;
}

}  // namespace bt

using namespace bt;

extern "C" int bt_dynamic_quantize(const bt_tensor* x, const bt_tensor* y, float* scale_out, uint8_t* zp_out) {
  int rc = dynamic_quantize_check(x, y, scale_out, zp_out, "bt_dynamic_quantize");
  if (rc) return rc;
  DevInfo di;
  if ((rc = dev_info(&di))) return rc;
  uint32_t* scratch = nullptr;
  if ((rc = scratch_for(di.device, cur_stream(), &scratch))) return rc;
  return dynamic_quantize_run(x, y, scale_out, zp_out, scratch);
}

// ---- DynamicQuantizeLinear without any device allocation --------------------
// Some callers of this library cannot allocate device memory while they run:
// an engine that gives each plugin only the buffers from its own pool,
// sized once at start-up; a serving process whose memory budget is fixed
// before the first request; a real-time audio or game loop, where a
// cudaMalloc can synchronise the device or fail under memory pressure in the
// middle of a frame.  bt_dynamic_quantize keeps its range record in memory it
// allocates on first use; this variant keeps it in the file-scope array
// below instead, which every device that loads the library holds until the
// process exits.  The array holds 256 bytes; a call uses one 16-byte range
// record whatever the size of x.  All calls on a device share the record:
// calls whose work overlaps on the GPU (different streams, or host threads
// racing) corrupt each other's range.
namespace bt {
namespace {

constexpr size_t kNoAllocScratchBytes = 256;
constexpr size_t kRangeRecordBytes = 16;
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocScratchBytes / sizeof(uint32_t)];
// A call needs one range record whatever the size of x, so no request can
// exceed the array: the limit is a build-time fact, not a run-time check.
static_assert(kRangeRecordBytes <= kNoAllocScratchBytes, "the range record must fit the static scratch array");

// The device address of g_noalloc_scratch on the current device, looked up
// with cudaGetSymbolAddress by the first call on each device (in host code the
// array's name stands for a host-side shadow, not for device memory).
int noalloc_scratch(int device, uint32_t** out) {
  static std::mutex mu;
  static std::map<int, uint32_t*> addr;
  std::lock_guard<std::mutex> lk(mu);
  auto it = addr.find(device);
  if (it == addr.end()) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_error(BT_ECUDA, "bt_dynamic_quantize_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    it = addr.emplace(device, (uint32_t*)p).first;
  }
  *out = it->second;
  return BT_OK;
}

}  // namespace
}  // namespace bt

extern "C" int bt_dynamic_quantize_noalloc(const bt_tensor* x, const bt_tensor* y, float* scale_out,
                                           uint8_t* zp_out) {
  int rc = dynamic_quantize_check(x, y, scale_out, zp_out, "bt_dynamic_quantize_noalloc");
  if (rc) return rc;
  DevInfo di;
  if ((rc = dev_info(&di))) return rc;
  uint32_t* scratch = nullptr;
  if ((rc = noalloc_scratch(di.device, &scratch))) return rc;
  return dynamic_quantize_run(x, y, scale_out, zp_out, scratch);
}

// ---- DynamicQuantizeLinear over a range its producer recorded ----------------
// bt_adain_snake_range folds each output's values into a range record as it
// writes them; the quantization of that output then only needs the second
// pass.  The record is the one the range kernel above fills, so the results
// are those of bt_dynamic_quantize bit for bit.
extern "C" int bt_dynamic_quantize_ranged(const bt_tensor* x, const bt_tensor* y, float* scale_out, uint8_t* zp_out,
                                          const uint32_t* range) {
  int rc = dynamic_quantize_check(x, y, scale_out, zp_out, "bt_dynamic_quantize_ranged");
  if (rc) return rc;
  if (!range) return set_error(BT_EINVAL, "bt_dynamic_quantize_ranged: null range record");
  return dq_quantize_launch(x, y, scale_out, zp_out, range, "bt_dynamic_quantize_ranged");
}

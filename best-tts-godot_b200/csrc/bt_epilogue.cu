// bt_epilogue.cu -- the integer convolution epilogue of the quantised
// generator, fused: the nodes that follow each ConvInteger in the packed
// graph, as the reference's op table evaluates them one by one
// (ref_runtime.py:446-455 for Add / Mul / Div, :458-466 Floor, :572-578
// Cast with fp16 targets elided to fp32):
//
//   s    = x_scale * float32(w_scale)                 float32 scalar
//   bq   = int32(floor(float32(bias) / s))            one per channel
//   out  = float32(acc + bq[c]) * s                   acc int32 [B, C, T]
//
// int32 addition wraps (numpy int32 arithmetic); int32 -> float32 rounds to
// nearest even; a floor outside the int32 range (or NaN) casts to INT32_MIN,
// numpy's result on x86-64.  The division bias / s is formed as
// RN32(RN64(bias * recip_d(s))), the correctly rounded quotient.  One pass:
// 128-bit int32 loads and float32 stores over each (b, c) row, the row's bq
// formed once per thread.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"

namespace bt {
namespace {

struct EpiArgs {
  const int32_t* acc;
  float* out;
  const void* bias;
  const float* x_scale;
  const void* w_scale;
  int32_t bias_dt, w_dt;
  int64_t rows, C, T;
};

__device__ __forceinline__ float ld_f(const void* p, int dt, int64_t i) {
  return dt == BT_F16 ? __half2float(((const __half*)p)[i]) : ((const float*)p)[i];
}

// numpy's float32 -> int32 cast on x86-64: truncation, INT32_MIN outside the
// range (the value here is already integral)
__device__ __forceinline__ int32_t np_f2i(float v) {
  return (v >= -2147483648.0f && v < 2147483648.0f) ? (int32_t)v : INT32_MIN;
}

__device__ __forceinline__ float epi(int32_t a, int32_t bq, float s) {
  return BT_MUL(__int2float_rn((int32_t)((uint32_t)a + (uint32_t)bq)), s);
}

__global__ void __launch_bounds__(256) conv_epilogue_kernel(EpiArgs A) {
  const float s = BT_MUL(*A.x_scale, ld_f(A.w_scale, A.w_dt, 0));
  const double rs = recip_d(s);
  const int64_t T = A.T;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = blockIdx.y; r < A.rows; r += gridDim.y) {
    const int64_t c = r % A.C;
    const int32_t bq = np_f2i(floorf(div_by(ld_f(A.bias, A.bias_dt, c), rs)));
    const int32_t* a = A.acc + r * T;
    float* o = A.out + r * T;
    // the 16-byte aligned interior as int4 -> float4
    int64_t head = (int64_t)((16 - ((uintptr_t)a & 15)) & 15) / 4;
    if (head > T) head = T;
    const bool vec = (((uintptr_t)a - (uintptr_t)o) & 15) == 0;
    if (!vec) head = T;
    const int64_t nv = (T - head) >> 2;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += stride) {
      const int4 v = __ldcs(reinterpret_cast<const int4*>(a + head) + q);
      __stcs(reinterpret_cast<float4*>(o + head) + q, make_float4(epi(v.x, bq, s), epi(v.y, bq, s),
                                                                  epi(v.z, bq, s), epi(v.w, bq, s)));
    }
    // the ragged ends (all of the row when input and output phases differ)
    const int64_t tail0 = head + 4 * nv;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < head + (T - tail0); i += stride) {
      const int64_t j = i < head ? i : tail0 + (i - head);
      o[j] = epi(a[j], bq, s);
    }
  }
}

}  // namespace
}  // namespace bt

using namespace bt;

extern "C" int bt_conv_int_epilogue(const bt_tensor* acc, const bt_tensor* bias, const bt_tensor* x_scale,
                                    const bt_tensor* w_scale, const bt_tensor* out) {
  int rc = check_tensor(acc, "acc", false);
  if (rc) return rc;
  if ((rc = check_tensor(bias, "bias", false))) return rc;
  if ((rc = check_tensor(x_scale, "x_scale", false))) return rc;
  if ((rc = check_tensor(w_scale, "w_scale", false))) return rc;
  if ((rc = check_tensor(out, "out", false))) return rc;
  if (acc->dtype != BT_I32 || out->dtype != BT_F32)
    return set_error(BT_EDTYPE, "bt_conv_int_epilogue: acc must be int32 and out float32");
  if (x_scale->dtype != BT_F32 || numel(x_scale) != 1)
    return set_error(BT_EDTYPE, "bt_conv_int_epilogue: x_scale must be one float32");
  if ((w_scale->dtype != BT_F32 && w_scale->dtype != BT_F16) || numel(w_scale) != 1)
    return set_error(BT_EDTYPE, "bt_conv_int_epilogue: w_scale must be one float16 / float32");
  if (bias->dtype != BT_F32 && bias->dtype != BT_F16)
    return set_error(BT_EDTYPE, "bt_conv_int_epilogue: bias must be float16 / float32");
  if (acc->rank != 3 || !is_contiguous(acc) || !is_contiguous(out) || numel(out) != numel(acc) ||
      !is_contiguous(bias) || numel(bias) != acc->shape[1])
    return set_error(BT_ESHAPE, "bt_conv_int_epilogue: acc [B, C, T] contiguous, bias [C], out like acc");
  const int64_t rows = acc->shape[0] * acc->shape[1], T = acc->shape[2];
  if (rows == 0 || T == 0) return BT_OK;
  EpiArgs A{(const int32_t*)acc->data, (float*)out->data, bias->data, (const float*)x_scale->data, w_scale->data,
            bias->dtype, w_scale->dtype, rows, acc->shape[1], T};
  const int threads = 256;
  int64_t gx = ((T + 3) / 4 + threads * 2 - 1) / (threads * 2);
  if (gx < 1) gx = 1;
  if (gx > 64) gx = 64;
  const int gy = (int)(rows < 65535 ? rows : 65535);
  conv_epilogue_kernel<<<dim3((unsigned)gx, (unsigned)gy), threads, 0, cur_stream()>>>(A);
  return check_launch("bt_conv_int_epilogue");
}

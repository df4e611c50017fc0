// bt_selfcheck.cu -- exhaustive device checks of the library's own float32
// math: the fast division inside exp and sigmoid, the double reciprocal
// and the float32 quotients behind division by a per-row constant, tanh,
// and DynamicQuantizeLinear's float32 shortcut (bt_selfcheck in bt_ops.h).
#include <cuda_runtime.h>
#include <stdint.h>
#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"
#include "bt_pk.h"
#include "bt_dq.h"

namespace bt {
namespace {

// Same bits, or both NaN (payloads are not compared: numpy's and the parity
// tests' convention).
__device__ __forceinline__ bool same_bits(float a, float b) {
  return __float_as_uint(a) == __float_as_uint(b) || (a != a && b != b);
}

// the (scale, zero point) pairs of kind 6
__constant__ double c_dq_scale[8] = {1.0, 0.0173, 3.0 / 255.0, 0x1.fffffep-1, 1e-30, 0x1p-140, 2.6e36, 0x1.000002p+3};
__constant__ double c_dq_zp[8] = {0.0, 128.0, 255.0, 3.0, 0.0, 17.0, 255.0, 200.0};

__global__ void __launch_bounds__(256) selfcheck_kernel(int kind, uint32_t first, uint64_t count,
                                                        unsigned long long* mismatches) {
  unsigned long long bad = 0;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
    const float x = __uint_as_float((uint32_t)(first + i));
    switch (kind) {
      case 0:
        bad += same_bits(np_expf_t<false>(x), np_expf_t<true>(x)) ? 0 : 1;
        break;
      case 1: {
        const float2 e = pk_np_exp(make_float2(x, -x));
        bad += same_bits(e.x, np_expf_t<true>(x)) ? 0 : 1;
        bad += same_bits(e.y, np_expf_t<true>(-x)) ? 0 : 1;
        break;
      }
      case 2:
        bad += same_bits(np_sigmoidf_t<false>(x), np_sigmoidf_t<true>(x)) ? 0 : 1;
        break;
      case 5: {
        // within one float ulp of the correctly rounded tanh (the double
        // library tanh rounded to float); NaN for NaN
        const float g = tanh_f(x), w = __double2float_rn(tanh((double)x));
        const int gi = (int)__float_as_uint(g), wi = (int)__float_as_uint(w);
        const bool ok = (g != g && w != w) || gi == wi || ((gi ^ wi) >= 0 && (gi - wi == 1 || wi - gi == 1));
        bad += ok ? 0 : 1;
        break;
      }
      case 4: {
        const float2 g = pk_np_sigmoid(make_float2(x, -x));
        bad += same_bits(g.x, np_sigmoidf_t<true>(x)) ? 0 : 1;
        bad += same_bits(g.y, np_sigmoidf_t<true>(-x)) ? 0 : 1;
        break;
      }
      case 6: {
        // DynamicQuantizeLinear's float32 shortcut against its exact double
        // path, at scales that put every quotient regime in reach: unit
        // (ties at every half-integer), ordinary, the smallest and largest
        // scales a float32 range gives, a scale whose reciprocal rounds
        // across a binade, and zero points at both ends
#pragma unroll 1
        for (int j = 0; j < 8; ++j) {
          const DqParams p = dq_params_from(c_dq_scale[j], c_dq_zp[j]);
          bad += q8(x, p) == q8_exact(x, p) ? 0 : 1;
        }
        break;
      }
      default: {
        // within one double ulp of IEEE's 1/x; NaN for NaN
        const double y = recip_d(x), z = __ddiv_rn(1.0, (double)x);
        const long long dy = __double_as_longlong(y), dz = __double_as_longlong(z);
        const bool ok = (y != y && z != z) || dy == dz ||
                        (((dy ^ dz) >= 0) && (dy - dz == 1 || dz - dy == 1) && fabs(z) != INFINITY && z != 0.0);
        bad += ok ? 0 : 1;
        break;
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// kind 7: division by a row constant in float32 (div_row_fast) for the
// divisor significands first .. first + count - 1 in [1, 2), each against
// all 2^23 dividend significands in [1, 2).  q is RN(a / b) iff the residual
// a - b q lies strictly inside half the gap around q (a quotient of floats is
// never a rounding midpoint, so there are no ties): for the correctly rounded
// q that residual is a float, which one FMA computes exactly; for any other q
// the exact residual lies beyond the bound, and so does its rounding.  Below
// a power of two the gap is half as wide.
__global__ void __launch_bounds__(256) rowdiv_check_kernel(uint32_t first, uint32_t count,
                                                           unsigned long long* mismatches) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  unsigned long long bad = 0;
  if (t < count) {
    const float b = bits_f(0x3f800000u | (first + t));
    const float y = __frcp_rn(b);
#pragma unroll 4
    for (uint32_t m = 0; m < (1u << 23); ++m) {
      const float a = bits_f(0x3f800000u | m);
      const float q = div_row_fast(a, b, y);
      const uint32_t qb = f_bits(q);
      const float h = __fmul_rn(b, bits_f((qb & 0x7f800000u) - (24u << 23)));   // b ulp(q) / 2
      const float r = __fmaf_rn(-b, q, a);
      const bool ok = r >= 0.0f ? r < h : -r < ((qb & 0x7fffffu) ? h : __fmul_rn(0.5f, h));
      bad += ok ? 0 : 1;
    }
  }
  for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

}  // namespace
}  // namespace bt

using namespace bt;

extern "C" int bt_selfcheck(int kind, uint32_t first, uint64_t count, unsigned long long* mismatches) {
  if (kind < 0 || kind > 7) return set_error(BT_EINVAL, "bt_selfcheck: kind %d", kind);
  if (!mismatches) return set_error(BT_EINVAL, "bt_selfcheck: null counter");
  if (kind == 7) {
    if (count > (1ull << 23) || (uint64_t)first + count > (1ull << 23))
      return set_error(BT_EINVAL, "bt_selfcheck: divisor significands past 2^23");
    if (count == 0) return BT_OK;
    const uint32_t n = (uint32_t)count;
    rowdiv_check_kernel<<<(n + 255) / 256, 256, 0, cur_stream()>>>(first, n, mismatches);
    return check_launch("bt_selfcheck");
  }
  if (count > (1ull << 32) || (uint64_t)first + count > (1ull << 32))
    return set_error(BT_EINVAL, "bt_selfcheck: range past 2^32 bit patterns");
  if (count == 0) return BT_OK;
  DevInfo di;
  int rc = dev_info(&di);
  if (rc) return rc;
  selfcheck_kernel<<<di.sm_count * 8, 256, 0, cur_stream()>>>(kind, first, count, mismatches);
  return check_launch("bt_selfcheck");
}

// bt_host.cpp -- host-only parts of the C ABI: error state, stream, device
// properties, tensor checks, the broadcast/collapse planner and the host
// evaluation of the library's float32 math (for CPU tests).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <mutex>
#include <vector>
#include <cuda_runtime.h>

#include "bt_ops.h"
#include "bt_internal.h"
#include "bt_core.h"

namespace bt {

namespace {
thread_local char g_err[1024] = "";
thread_local cudaStream_t g_stream = nullptr;
std::mutex g_dev_mu;
std::vector<DevInfo> g_dev;  // indexed by device ordinal
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

cudaStream_t cur_stream() { return g_stream; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(BT_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return BT_OK;
}

int dev_info(DevInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_error(BT_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if ((int)g_dev.size() <= dev) g_dev.resize(dev + 1);
  DevInfo& d = g_dev[dev];
  if (d.device < 0) {
    int v = 0;
    if ((e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return set_error(BT_ECUDA, "device attribute: %s", cudaGetErrorString(e));
    d.sm_count = v;
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.max_smem_optin = v;
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    d.max_threads_per_sm = v;
    d.device = dev;
  }
  *out = d;
  return BT_OK;
}

int dtype_size(int dt) {
  switch (dt) {
    case BT_BOOL: case BT_I8: case BT_U8: return 1;
    case BT_I16: case BT_U16: case BT_F16: return 2;
    case BT_I32: case BT_U32: case BT_F32: return 4;
    case BT_I64: case BT_U64: case BT_F64: return 8;
  }
  return 0;
}
bool dtype_valid(int dt) { return dtype_size(dt) > 0; }
bool is_float_dtype(int dt) { return dt == BT_F16 || dt == BT_F32 || dt == BT_F64; }

int check_tensor(const bt_tensor* t, const char* name, bool allow_null_data) {
  if (!t) return set_error(BT_EINVAL, "%s: null tensor descriptor", name);
  if (!dtype_valid(t->dtype)) return set_error(BT_EDTYPE, "%s: unknown dtype code %d", name, t->dtype);
  if (t->rank < 0 || t->rank > BT_MAX_RANK)
    return set_error(BT_ESHAPE, "%s: rank %d outside 0..%d", name, t->rank, BT_MAX_RANK);
  int64_t n = 1;
  for (int d = 0; d < t->rank; ++d) {
    if (t->shape[d] < 0) return set_error(BT_ESHAPE, "%s: negative extent on axis %d", name, d);
    n *= t->shape[d];
  }
  if (!t->data && n > 0 && !allow_null_data)
    return set_error(BT_EINVAL, "%s: null data pointer", name);
  return BT_OK;
}

int64_t numel(const bt_tensor* t) {
  int64_t n = 1;
  for (int d = 0; d < t->rank; ++d) n *= t->shape[d];
  return n;
}

bool is_contiguous(const bt_tensor* t) {
  int64_t acc = 1;
  for (int d = t->rank - 1; d >= 0; --d) {
    if (t->shape[d] != 1 && t->strides[d] != acc) return false;
    acc *= t->shape[d];
  }
  return true;
}

int plan_broadcast(int n_ops, const bt_tensor* const* ops, const int64_t* out_shape,
                   int out_rank, BcastPlan* p) {
  if (n_ops < 1 || n_ops > 4) return set_error(BT_EINVAL, "planner: %d operands", n_ops);
  if (out_rank < 0 || out_rank > BT_MAX_RANK)
    return set_error(BT_ESHAPE, "planner: output rank %d", out_rank);
  // Right-align every operand to the output and give broadcast axes stride 0
  // (the behaviour of ops.gd:62-77, with arbitrary input strides).
  int64_t st[4][BT_MAX_RANK];
  for (int k = 0; k < n_ops; ++k) {
    const bt_tensor* t = ops[k];
    if (t->rank > out_rank)
      return set_error(BT_ESHAPE, "operand %d has rank %d > output rank %d", k, t->rank, out_rank);
    int pad = out_rank - t->rank;
    for (int i = 0; i < out_rank; ++i) {
      if (i < pad) { st[k][i] = 0; continue; }
      int64_t d = t->shape[i - pad];
      if (d == out_shape[i]) st[k][i] = (d == 1) ? 0 : t->strides[i - pad];
      else if (d == 1) st[k][i] = 0;
      else
        return set_error(BT_ESHAPE, "operand %d: extent %lld on axis %d does not broadcast to %lld",
                         k, (long long)d, i, (long long)out_shape[i]);
    }
  }
  // Drop size-1 axes, then merge axis i-1 into i whenever every operand steps
  // through them contiguously: st[i-1] == st[i] * dims[i] (ops.gd:85-129).
  int64_t dims[BT_MAX_RANK];
  int64_t cs[4][BT_MAX_RANK];
  int r = 0;
  int64_t n = 1;
  for (int i = 0; i < out_rank; ++i) {
    n *= out_shape[i];
    if (out_shape[i] == 1) continue;
    dims[r] = out_shape[i];
    for (int k = 0; k < n_ops; ++k) cs[k][r] = st[k][i];
    ++r;
  }
  for (int i = r - 1; i > 0; --i) {
    bool ok = true;
    for (int k = 0; k < n_ops; ++k)
      if (cs[k][i - 1] != cs[k][i] * dims[i]) { ok = false; break; }
    if (!ok) continue;
    dims[i - 1] *= dims[i];
    for (int k = 0; k < n_ops; ++k) cs[k][i - 1] = cs[k][i];
    for (int j = i; j < r - 1; ++j) {
      dims[j] = dims[j + 1];
      for (int k = 0; k < n_ops; ++k) cs[k][j] = cs[k][j + 1];
    }
    --r;
  }
  if (r == 0) {
    dims[0] = 1;
    for (int k = 0; k < n_ops; ++k) cs[k][0] = 0;
    r = 1;
  }
  p->rank = r;
  p->n = n;
  for (int i = 0; i < r; ++i) {
    p->shape[i] = dims[i];
    for (int k = 0; k < n_ops; ++k) p->st[k][i] = cs[k][i];
  }
  return BT_OK;
}

}  // namespace bt

using namespace bt;

extern "C" {

int bt_abi_version(void) { return BT_ABI_VERSION; }

const char* bt_last_error(void) { return g_err; }

int bt_set_stream(void* stream) {
  g_stream = (cudaStream_t)stream;
  return BT_OK;
}

int bt_sync(void) {
  cudaError_t e = cudaStreamSynchronize(g_stream);
  if (e != cudaSuccess) return set_error(BT_ECUDA, "stream synchronize: %s", cudaGetErrorString(e));
  return BT_OK;
}

int bt_plan_broadcast(int n_ops, const bt_tensor* ops, const int64_t* out_shape, int out_rank,
                      int* rank_out, int64_t* shape_out, int64_t* strides_out) {
  if (!ops || !rank_out || !shape_out || !strides_out || (!out_shape && out_rank > 0))
    return set_error(BT_EINVAL, "bt_plan_broadcast: null argument");
  if (n_ops < 1 || n_ops > 4) return set_error(BT_EINVAL, "bt_plan_broadcast: n_ops %d", n_ops);
  const bt_tensor* ptrs[4];
  for (int k = 0; k < n_ops; ++k) {
    int rc = check_tensor(&ops[k], "operand", true);
    if (rc) return rc;
    ptrs[k] = &ops[k];
  }
  BcastPlan p;
  int rc = plan_broadcast(n_ops, ptrs, out_shape, out_rank, &p);
  if (rc) return rc;
  *rank_out = p.rank;
  for (int i = 0; i < p.rank; ++i) shape_out[i] = p.shape[i];
  for (int k = 0; k < n_ops; ++k)
    for (int i = 0; i < BT_MAX_RANK; ++i) strides_out[k * BT_MAX_RANK + i] = i < p.rank ? p.st[k][i] : 0;
  return BT_OK;
}

int bt_host_math(int kind, const float* in, float* out, int64_t n) {
  if ((!in || !out) && n > 0) return set_error(BT_EINVAL, "bt_host_math: null buffer");
  switch (kind) {
    case 0: for (int64_t i = 0; i < n; ++i) out[i] = np_expf(in[i]); break;
    case 1: for (int64_t i = 0; i < n; ++i) out[i] = np_sinf(in[i]); break;
    case 2: for (int64_t i = 0; i < n; ++i) out[i] = np_cosf(in[i]); break;
    case 3: for (int64_t i = 0; i < n; ++i) out[i] = np_sigmoidf(in[i]); break;
    case 4: out[0] = BT_ADD(0.0f, pw_sum_host(in, n, [](float v) { return v; })); break;
    default: return set_error(BT_EINVAL, "bt_host_math: unknown kind %d", kind);
  }
  return BT_OK;
}

}  // extern "C"

// bt_internal.h -- host-side plumbing shared by the library's translation
// units: error reporting, the per-thread stream, device properties, tensor
// validation and the broadcast planner's result type.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>
#include "bt_ops.h"

namespace bt {

// Records a message for bt_last_error() on the calling thread; returns code.
int set_error(int code, const char* fmt, ...);
// Stream chosen with bt_set_stream() on the calling thread.
cudaStream_t cur_stream();
// Converts a pending CUDA error (launch failure) into BT_ECUDA.
int check_launch(const char* what);

struct DevInfo {
  int device = -1;
  int sm_count = 0;
  int max_smem_optin = 0;   // bytes per block with the opt-in attribute
  int max_threads_per_sm = 0;
};
// Properties of the calling thread's current device (cached).
int dev_info(DevInfo* out);

int dtype_size(int dt);
bool dtype_valid(int dt);
bool is_float_dtype(int dt);
// Validates pointer, dtype and rank of a tensor view; name is used in errors.
int check_tensor(const bt_tensor* t, const char* name, bool allow_null_data);
int64_t numel(const bt_tensor* t);
bool is_contiguous(const bt_tensor* t);

// Result of broadcasting n operand views to an output shape and merging the
// axes every operand walks contiguously.
struct BcastPlan {
  int rank = 0;                       // >= 1
  int64_t shape[BT_MAX_RANK];
  int64_t st[4][BT_MAX_RANK];         // per operand (inputs..., output last)
  int64_t n = 0;                      // total elements
};
// ops[0..n_ops) are the operands (inputs then output); all broadcast to
// out_shape (rank out_rank).
int plan_broadcast(int n_ops, const bt_tensor* const* ops,
                   const int64_t* out_shape, int out_rank, BcastPlan* p);

// AdaIN1d + Snake with rows split across a thread-block cluster (bt_adain.cu).
// Returns BT_EUNSUPPORTED, without setting an error, for requests it does
// not cover; bt_adain_snake then uses the one-CTA-per-row kernel.  range
// (may be null): per output a zeroed 3-word record ([0] = ~ord(min) and
// [1] = ord(max), both by atomicMax, [2] = NaN seen) that the kernel folds
// every written value into -- the record dq_range_launch fills.
int adain_v3(const bt_adain_args* p, uint32_t* const* range = nullptr);

// The range pass of DynamicQuantizeLinear (bt_quant.cu) over n contiguous
// values of x (float32 or float16) into a zeroed 3-word record, on the
// current stream.
int dq_range_launch(const void* x, int32_t dtype, int64_t n, uint32_t* rec);

}  // namespace bt

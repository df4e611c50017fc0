/*
 * bt_ops.h -- C ABI of the B200 (sm_100a) tensor-op library for the best-tts
 * hot path: the elementwise, broadcast, reduction and dequantize ops that the
 * best-tts graph executor dispatches for Kokoro-82M.
 *
 * Every entry point replaces one reference interface, cited beside it as
 * "replaces:" with file:line into studio-ransom/best-tts-godot:
 *   - the numpy op table  tools/ref_runtime.py  RefRuntime.dispatch (:428-668),
 *   - the GDScript executor's GPU dispatchers   runtime/executor.gd,
 *   - the GLSL kernels                          kernels/*.glsl.
 *
 * Conventions
 *   - Plain C: pointers, sizes, ints.  No exceptions cross the ABI.
 *   - Every function returns 0 on success or a negative BT_E* code, and then
 *     bt_last_error() holds a message for the calling thread.
 *   - The caller owns all device memory.  Tensors are described by bt_tensor
 *     views: element strides (0 = broadcast along that axis), rank <= 8.
 *   - Arithmetic follows the reference's numpy semantics: fp16 operands are
 *     widened to fp32 before use (ref_runtime.py:49-51), broadcasting is
 *     numpy's right-aligned rule, the output's dtype is the caller's choice
 *     (numpy's result type) and each op rounds once, in its own dtype.
 *   - Launches are asynchronous on the stream set with bt_set_stream() for
 *     the calling thread (default: the legacy default stream) and on the
 *     calling thread's current CUDA device.
 *   - Entry points marked "host only" touch no GPU and may be called on a
 *     machine without one.
 *   - Device addresses the library caches per device (the scratch records of
 *     bt_dynamic_quantize and bt_dynamic_quantize_noalloc) belong to the
 *     device's primary context: the library must not be used across a
 *     cudaDeviceReset of a device it has run on.
 */
#ifndef BT_OPS_H
#define BT_OPS_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BT_ABI_VERSION 1
#define BT_MAX_RANK 8

/* ---- status codes ------------------------------------------------------ */
#define BT_OK            0
#define BT_EINVAL      (-1)   /* bad argument (null pointer, bad code, ...)  */
#define BT_ESHAPE      (-2)   /* shapes do not broadcast / do not match      */
#define BT_EDTYPE      (-3)   /* dtype combination not supported             */
#define BT_ECUDA       (-4)   /* a CUDA runtime call failed                  */
#define BT_EUNSUPPORTED (-5)  /* valid request outside what is implemented   */
#define BT_ETOOBIG     (-6)   /* size beyond a documented limit              */

/* ---- element types (numpy dtypes) -------------------------------------- */
typedef enum bt_dtype {
  BT_BOOL = 0, BT_I8 = 1, BT_U8 = 2, BT_I16 = 3, BT_U16 = 4, BT_I32 = 5,
  BT_U32 = 6, BT_I64 = 7, BT_U64 = 8, BT_F16 = 9, BT_F32 = 10, BT_F64 = 11
} bt_dtype;

/* A strided view of device memory.  `data` points at element [0,...,0]. */
typedef struct bt_tensor {
  void*   data;
  int32_t dtype;                 /* bt_dtype */
  int32_t rank;                  /* 0 .. BT_MAX_RANK */
  int64_t shape[BT_MAX_RANK];
  int64_t strides[BT_MAX_RANK];  /* in elements; 0 means broadcast */
} bt_tensor;

/* ---- elementwise op codes ----------------------------------------------
 * Codes 0-31 keep the numbering of the reference's op table
 * (runtime/ops.gd:12-19, kernels/elementwise.glsl:43-74) so a reference-side
 * binding can pass its own codes.  CAST_INT / CAST_BOOL / IDENTITY all mean
 * "convert the (fp16-widened) input to the output's dtype" here, because the
 * output descriptor carries the target type. */
typedef enum bt_op {
  BT_OP_ADD = 0, BT_OP_SUB = 1, BT_OP_MUL = 2, BT_OP_DIV = 3, BT_OP_POW = 4,
  BT_OP_SQRT = 5, BT_OP_EXP = 6, BT_OP_SIN = 7, BT_OP_COS = 8, BT_OP_ATAN = 9,
  BT_OP_TANH = 10, BT_OP_SIGMOID = 11, BT_OP_FLOOR = 12, BT_OP_ROUND = 13,
  BT_OP_LEAKYRELU = 14, BT_OP_CLIP = 15, BT_OP_EQUAL = 16, BT_OP_GREATER = 17,
  BT_OP_LESS = 18, BT_OP_GEQ = 19, BT_OP_AND = 20, BT_OP_WHERE = 21,
  BT_OP_CAST_INT = 22, BT_OP_CAST_BOOL = 23, BT_OP_IDENTITY = 24,
  BT_OP_NEG = 25, BT_OP_ABS = 26, BT_OP_LOG = 27, BT_OP_MIN = 28,
  BT_OP_MAX = 29, BT_OP_ERF = 30, BT_OP_GELU = 31,
  /* codes beyond the reference's table */
  BT_OP_DEQUANT = 40   /* (in0 - in2) * in1, in2 optional (DequantizeLinear) */
} bt_op;

/* Attributes of an elementwise call. */
typedef struct bt_ew_attrs {
  int32_t compute_dtype;   /* dtype the op computes in (numpy result type of
                              the widened inputs; BT_F32, BT_F64 or an
                              integer type).  For comparisons: the promoted
                              type of the operands. */
  float   alpha;           /* LeakyRelu slope, applied as float32 */
} bt_ew_attrs;

/* ---- set-up ------------------------------------------------------------ */
int         bt_abi_version(void);                 /* host only */
const char* bt_last_error(void);                  /* host only */
/* Caches the device's properties and raises the shared-memory limits of the
 * row kernels.  Call once per device (the calling thread's current device is
 * used if `device` < 0). */
int         bt_init(int device);
/* Stream for subsequent launches from the calling thread (cudaStream_t). */
int         bt_set_stream(void* stream);
/* Waits for the calling thread's stream; reports asynchronous faults. */
int         bt_sync(void);

/* ---- elementwise -------------------------------------------------------
 * out = op(in[0], in[1], in[2]) with numpy broadcasting of every input view
 * to out->shape.
 * replaces: ref_runtime.py:446-503 (Add..Where), :572-578 (Cast), :610-611
 *           (FastGelu), :631-636 (DequantizeLinear);
 *           executor.gd:678-699 (_ew), :733-827 (_run_gpu op mapping);
 *           kernels/elementwise.glsl:91-163; kernels/misc.glsl:47-66
 *           (MODE_UNPACK_F16 / MODE_DEQUANT_I8). */
int bt_elementwise(int op, int n_in, const bt_tensor* in, const bt_tensor* out,
                   const bt_ew_attrs* attrs);

/* Fused elementwise chain: a short register program evaluated per element of
 * the broadcast iteration space of its inputs, in one pass (every input read
 * once at its stored type, the float32 result written once).  Inputs are
 * widened to float32 into registers r0..r(n_in-1); instruction k computes
 * dst = op(a, b) in float32, rounding once as the numpy op it stands for
 * would (no contraction); the result is register `out_reg`.  Input dtypes:
 * float32, float16, int8, uint8, int16, uint16, bool (their float32 widening
 * is exact, so float32 arithmetic is numpy's arithmetic next to float32
 * data).  The output is dense float32 of the broadcast shape.  A register
 * read before it was written, an unknown op or a bad register index is
 * BT_EINVAL; more than 2^32 - 1 rows (all axes but the last merged one) is
 * BT_ETOOBIG.
 * Programs of the built-in catalog (bt_chain_kind) run in kernels compiled
 * for them; every other valid program runs in an interpreter kernel (the
 * same results, more instructions per value).
 * replaces: chains of ref_runtime.py:446-479 dispatches such as Snake
 *           (Mul, Sin, Pow 2, Mul, Add) and DequantizeLinear + gain Mul
 *           (:631-636, :450-451), each of which the reference executes as a
 *           separate dispatch with a barrier (executor.gd:678-699, the
 *           two-dispatch DequantizeLinear at :822-827). */
#define BT_CHAIN_MAX_INSTR 16
#define BT_CHAIN_MAX_IN 6
typedef struct bt_chain_instr {
  int32_t op;        /* bt_op among ADD SUB MUL DIV POW SQRT EXP SIN COS TANH
                        SIGMOID LEAKYRELU ERF IDENTITY NEG ABS MIN MAX FLOOR
                        ROUND ATAN */
  int32_t dst, a, b; /* register indices 0..15 (b unused by unary ops) */
  float   alpha;     /* LeakyRelu slope */
} bt_chain_instr;
typedef struct bt_chain {
  int32_t n_in;
  int32_t n_instr;
  int32_t out_reg;
  bt_chain_instr instr[BT_CHAIN_MAX_INSTR];
} bt_chain;
int bt_fused_chain(const bt_chain* prog, const bt_tensor* in,
                   const bt_tensor* out);
/* Which kernel bt_fused_chain runs for `prog` (host only): the index of the
 * catalog entry it matches once its registers are renamed to
 * single-assignment form, BT_CHAIN_INTERPRETER for the interpreter, or a
 * negative BT_E* code for an invalid program.  Catalog, in order, with the
 * inputs in the order given:
 *   0 Mul(DequantizeLinear(q, scale), gain)             inputs q, scale, gain
 *   1 Mul(DequantizeLinear(q, scale, zp), gain)         inputs q, scale, gain, zp
 *   2 Snake x + inv_alpha * sin(alpha * x) ** p          inputs x, alpha, p, inv_alpha
 *     (the graph's Mul, Sin, Pow, Mul, Add)
 *   3 Sigmoid(Add(x, y))                                inputs x, y
 *   4 Add(Mul(x, g), b)                                 inputs x, g, b
 *   5 LeakyRelu(Add(x, y))                              inputs x, y
 *   6 DequantizeLinear(q, scale) (a Mul)                inputs q, scale
 *   7 DequantizeLinear(q, scale, zp)                    inputs q, scale, zp
 * replaces: nothing in the reference (a query about this library's own
 *           kernels). */
#define BT_CHAIN_INTERPRETER 64
int bt_chain_kind(const bt_chain* prog);

/* ---- reductions --------------------------------------------------------
 * kind: 0 = ReduceSum, 1 = ReduceMean.  `axes` are normalised axes of x
 * (sorted, distinct, >= 0); out has x's shape with the reduced axes removed
 * (keepdims = 0) or set to 1 (keepdims = 1).  fp32 sums follow numpy's
 * pairwise order over a contiguous reduced block and its sequential order
 * over an outer reduced axis, so results are bit-identical to numpy.
 * replaces: ref_runtime.py:589-598; executor.gd:942-974 (_run_reduce);
 *           kernels/reduce.glsl:30-61. */
#define BT_REDUCE_SUM 0
#define BT_REDUCE_MEAN 1
int bt_reduce(int kind, const bt_tensor* x, const int64_t* axes, int n_axes,
              int keepdims, const bt_tensor* out);

/* ---- softmax -----------------------------------------------------------
 * out = softmax(x + mask) along `axis` (mask optional, broadcast to x),
 * in numpy's order: max, exp(x - max), pairwise sum, divide.
 * replaces: ref_runtime.py:269-273 + :599-600 (and the Add of the attention
 *           mask that precedes it, :446-447); executor.gd:887-903;
 *           kernels/softmax.glsl:26-61. */
int bt_softmax(const bt_tensor* x, const bt_tensor* mask, int axis,
               const bt_tensor* out);

/* ---- layer normalisation -----------------------------------------------
 * out = LN(x [+ skip [+ bias]]) over the axes from `axis` to the last, with
 * gamma (required) and beta (optional); eps is applied as float32.  skip/bias
 * NULL gives LayerNormalization, non-NULL gives SkipLayerNormalization.
 * replaces: ref_runtime.py:276-285 + :601-609; executor.gd:906-939;
 *           kernels/layernorm.glsl:35-75. */
int bt_layernorm(const bt_tensor* x, const bt_tensor* skip,
                 const bt_tensor* bias, const bt_tensor* gamma,
                 const bt_tensor* beta, int axis, float eps,
                 const bt_tensor* out);

/* ---- AdaIN1d + Snake (row-fused) ----------------------------------------
 * For rows r of a [R, T] view (R = batch * channels, T contiguous):
 *   h      = src0 [+ src1 [+ src2]]          (fp32, left to right)
 *   if res != NULL: res = h                  (residual written once)
 *   n      = (h - mean(h)) / sqrt(mean((h - mean)^2) + eps)
 *   y_k    = gain_k[r] * n + shift_k[r]      for each output k < n_out
 *   out_k  = y_k + inv_alpha_k[c] * sin(alpha_k[c] * y_k)^2   (snake)
 *            or y_k when alpha_k == NULL
 * which is the op chain the packed Kokoro graph runs per AdaIN1d + Snake
 * (ReduceMean, Sub, Mul, ReduceMean, Add eps, Sqrt, Div, Mul, Add, then Mul,
 * Sin, Pow 2, Mul, Add), rounded op by op.  Row r is (batch b, channel c)
 * with b = r / C, c = r % C; gain_k / shift_k are fp32 [B, C] views read at
 * b * param_stride + c (gain_stride / shift_stride elements between batch
 * entries, e.g. 2C for the halves of an fc output [B, 2C]); alpha /
 * inv_alpha are [C] (fp16 or fp32).
 * Up to three outputs share one normalisation: the graph computes the
 * instance norm of x once for the three resblocks that read the same x.
 * replaces: the ReduceMean/Sub/.../Add chains that executor.gd:678-699 and
 *           :942-974 dispatch one op at a time (ref_runtime.py:446-479,
 *           :589-598 per op). */
#define BT_ADAIN_MAX_SRC 3
#define BT_ADAIN_MAX_OUT 3
typedef struct bt_adain_args {
  int64_t rows, cols, channels;          /* R, T, C */
  int32_t n_src, n_out;
  const float* src[BT_ADAIN_MAX_SRC];    /* [R, T] fp32, contiguous */
  float*       res;                      /* [R, T] fp32 or NULL */
  float        eps;                      /* as float32 */
  int64_t      gain_stride, shift_stride;/* batch strides of gain / shift */
  const float* gain[BT_ADAIN_MAX_OUT];   /* [B, C] fp32 views */
  const float* shift[BT_ADAIN_MAX_OUT];
  const void*  alpha[BT_ADAIN_MAX_OUT];  /* [C] or NULL (no snake) */
  const void*  inv_alpha[BT_ADAIN_MAX_OUT];
  int32_t      alpha_dtype;              /* BT_F16 or BT_F32 */
  float*       out[BT_ADAIN_MAX_OUT];    /* [R, T] fp32 */
} bt_adain_args;
int bt_adain_snake(const bt_adain_args* a);
/* bt_adain_snake whose outputs go on to a DynamicQuantizeLinear (the input
 * quantisation of the ConvInteger that reads each Snake output in the int8
 * generator): the same outputs, bit for bit, and in the same pass output k's
 * values folded into the range record range + 4 * k, which
 * bt_dynamic_quantize_ranged then consumes.  range: device memory, 16-byte
 * aligned, 16 bytes per output; this call zeroes the records first.  Where
 * the cluster kernel does not apply it runs a separate range pass per output
 * instead, with the same records as the result.
 * replaces: the minmax dispatch of executor.gd:1224-1230 (its pass over the
 *           Snake output) for each quantised conv input. */
int bt_adain_snake_range(const bt_adain_args* a, uint32_t* range);
/* The number of bounded waits on bulk (TMA) copies in bt_adain_snake /
 * bt_adain_snake_range kernels that gave up since the last call (each such
 * wait records itself and lets its kernel run on with unfinished data, so a
 * copy that never lands cannot hang the GPU); the count is then reset.
 * Synchronous (waits for the device).  *count == 0 after a run means every
 * copy completed.  No counterpart in the reference. */
int bt_wait_timeouts(uint32_t* count);

/* ---- residual mean + LeakyRelu (end of a generator stage) ---------------
 * out = leaky((((a0 + b0) + (a1 + b1)) + (a2 + b2)) / 3, slope) elementwise
 * over n fp32 elements: the last residual Add of each of the three resblocks,
 * the two Adds and the Div by 3 of the resblock mean, and the LeakyRelu that
 * starts the next stage (or ends the generator), rounded op by op.
 * replaces: the Add/Add/Div/LeakyRelu dispatches of executor.gd:678-699 at
 * the end of each generator stage (ref_runtime.py:446-455, :476-479). */
int bt_resblock_mean_leaky(const float* const* a, const float* const* b,
                           int64_t n, float divisor, float slope, float* out);

/* ---- DynamicQuantizeLinear ------------------------------------------------
 * y = uint8(clip(rint(x / scale) + zp, 0, 255)) over the n values of x
 * (float32 or float16, contiguous; y uint8 of the same size), with
 *   lo = min(0, min x), hi = max(0, max x), scale = (hi - lo) / 255 in
 *   double (1 when 0), zp = clip(rint(-lo / scale), 0, 255) in double,
 * and x / scale formed in float32 (numpy 2 casts the Python-float scale to
 * the array's dtype).  rint rounds half to even.  *scale_out (float32) and
 * *zp_out (uint8) are device scalars.  A NaN in x gives scale 1, zero point
 * 0 and 0 at the NaN elements (numpy's uint8 cast of NaN on x86-64).  An
 * empty x is an error (numpy's min of an empty array raises).  Uses a
 * 16-byte scratch record per (device, stream), allocated by the first call
 * on that pair: make that call before capturing the stream in a graph.
 * replaces: ref_runtime.py:106-116 and :625-630; the minmax / quantize
 * dispatch pair of executor.gd:1194-1240 (minmax.glsl, quantize.glsl). */
int bt_dynamic_quantize(const bt_tensor* x, const bt_tensor* y, float* scale_out,
                        uint8_t* zp_out);
/* The same results as bt_dynamic_quantize for callers that cannot allocate
 * device memory at run time (an engine that hands plugins only buffers from
 * its own pool, a serving process with a fixed memory budget, a real-time
 * loop where an allocation could stall or fail mid-frame): it allocates
 * nothing.  Its 16-byte range record lives in a 256-byte static device array
 * that every device loading the library keeps until exit; a call needs that
 * one record whatever the size of x, so no input is too large for it (the
 * library checks this when it is built).  The first call on a device looks
 * up the array's device address: make it before any stream capture.  All
 * calls on a device share the record, so calls that overlap on the GPU race.
 * No counterpart in the reference: the reference's executor always allocates
 * its min/max scratch (executor.gd:1201-1206). */
int bt_dynamic_quantize_noalloc(const bt_tensor* x, const bt_tensor* y,
                                float* scale_out, uint8_t* zp_out);
/* bt_dynamic_quantize of an x whose range record its producer already wrote
 * (bt_adain_snake_range): only the quantize pass runs, results identical to
 * bt_dynamic_quantize's.  range points at the 16-byte record of x, left
 * unchanged.
 * replaces: the quantize dispatch of executor.gd:1232-1238 after a fused
 *           minmax. */
int bt_dynamic_quantize_ranged(const bt_tensor* x, const bt_tensor* y,
                               float* scale_out, uint8_t* zp_out,
                               const uint32_t* range);

/* ---- integer convolution epilogue ----------------------------------------
 * The nodes after each ConvInteger of the quantised generator in one pass:
 *   s   = x_scale * float32(w_scale)          (DynamicQuantizeLinear's scale
 *                                              times the weight scale)
 *   bq  = int32(floor(float32(bias) / s))     per channel
 *   out = float32(acc + bq[c]) * s            acc int32 [B, C, T] -> float32
 * each step rounded as numpy rounds the reference's op-by-op chain: int32
 * addition wraps, int32 -> float32 rounds to nearest even, a floor outside
 * the int32 range (or NaN) becomes INT32_MIN (numpy's cast on x86-64).
 * x_scale: one float32; w_scale: one float16 / float32; bias [C] float16 /
 * float32; all device memory.
 * replaces: the Cast / Mul / Div / Floor / Cast / Reshape / Add / Cast / Mul
 * nodes after each ConvInteger (ref_runtime.py:446-455, :572-578 per node;
 * one executor.gd:678-699 dispatch each). */
int bt_conv_int_epilogue(const bt_tensor* acc, const bt_tensor* bias,
                         const bt_tensor* x_scale, const bt_tensor* w_scale,
                         const bt_tensor* out);

/* ---- host-only helpers (no GPU) ------------------------------------------ */
/* Broadcast-and-collapse planner used by bt_elementwise: merges adjacent axes
 * that every operand walks contiguously and drops size-1 axes (the behaviour
 * of runtime/ops.gd:62-129).  Writes the collapsed rank, shape and the
 * collapsed strides of the n_ops operands (operand k's strides at
 * strides_out[k * BT_MAX_RANK + d]).  replaces: ops.gd:45-129. */
int bt_plan_broadcast(int n_ops, const bt_tensor* ops, const int64_t* out_shape,
                      int out_rank, int* rank_out, int64_t* shape_out,
                      int64_t* strides_out);
/* Evaluates the library's float32 math routines on the host, element by
 * element, so CPU tests can compare them with numpy.  kind: 0 exp, 1 sin,
 * 2 cos, 3 sigmoid, 4 pairwise row sum (n values -> out[0]). */
int bt_host_math(int kind, const float* in, float* out, int64_t n);

/* ---- device self-check ----------------------------------------------------
 * Evaluates the device float32 routine `kind` on every input whose bit
 * pattern lies in first .. first + count - 1 (count up to 2^32) and adds to
 * *mismatches (a device counter the caller allocates and zeroes) the number
 * of inputs whose result differs in any bit from the same routine with its
 * quotient computed by IEEE division (two NaNs count as equal).  kind: 0 exp, 1 exp two lanes at a
 * time (each input paired with its negation), 2 sigmoid, 3 the double
 * reciprocal behind division by a per-row constant (softmax, layer and
 * instance norms), which must lie within one double ulp of IEEE's 1/x and
 * equal it on zeros, infinities and NaN, 4 sigmoid two lanes at a time
 * (each input paired with its negation), 5 tanh, which counts as a mismatch
 * only when it is more than one float ulp from the correctly rounded tanh,
 * 6 DynamicQuantizeLinear's float32 shortcut against its exact double path
 * at eight built-in (scale, zero point) pairs (a mismatch per differing
 * pair), 7 division by a per-row constant in float32 arithmetic (the
 * reciprocal's product corrected by one FMA residual step) against the
 * correctly rounded quotient: for kind 7 first .. first + count - 1 (up to
 * 2^23) are divisor significands, each checked against all 2^23 dividend
 * significands (all 2^46 pairs take about half a minute).  Asynchronous on
 * the set stream.
 * No counterpart in the reference: over all 2^32 inputs it shows that the
 * library's fast division gives the IEEE quotient, hence numpy's result,
 * in every use. */
int bt_selfcheck(int kind, uint32_t first, uint64_t count,
                 unsigned long long* mismatches);

#ifdef __cplusplus
}
#endif
#endif /* BT_OPS_H */

"""Drop-in op table for the best-tts hot path on B200.

``BtRuntime.dispatch(op, node_input, node_output, at, env)`` has the signature
and the semantics of the reference's ``RefRuntime.dispatch``
(tools/ref_runtime.py:428-668): ``env`` maps tensor names to arrays, an empty
input name means "absent" (ref_runtime.py:436-439), single-output ops store
``env[node_output[0]]`` (ref_runtime.py:668), ``Split`` stores each named
output (ref_runtime.py:536-547) and an op outside the table raises
``NotImplementedError`` (ref_runtime.py:665-666).

The difference is where the arrays live: values in ``env`` are CUDA tensors
(torch is used only to own device memory and streams) and every op runs as a
hand-written sm_100a kernel behind the C ABI of ``libbt_ops.so``.  numpy
arrays found in ``env`` (constants, initializers) are copied to the device on
first use and cached; the caller's ``env`` entries are never replaced.

Memory layout follows numpy too, because numpy's summation order depends on
it: ``Transpose`` returns a permuted view (ref_runtime.py:517-518 returns
``np.transpose``'s view), element-wise results are allocated in numpy's
order 'K' (the axis order numpy's iterator picks from the operands'
strides), uploads keep a numpy array's axis order, and a reduction over a
view sums in the order numpy's iterator walks that view (pairwise along the
innermost axis in memory, slice after slice along outer ones).

Result dtypes and shapes follow numpy exactly: they are obtained by applying
the same numpy expression to zero-size arrays of the operands' dtypes, and
numpy's broadcasting rule.  Errors numpy would raise (bad broadcast, bad
dtype) surface as the same exceptions before any launch; a status from the
library raises ``BtError`` (a RuntimeError).
"""
import ctypes
import functools
import weakref

import numpy as np
import torch

from . import _lib
from ._lib import OP, check, load, make_tensor

ONNX_TO_NUMPY = {
    1: np.float32, 2: np.uint8, 3: np.int8, 4: np.uint16, 5: np.int16,
    6: np.int32, 7: np.int64, 9: np.bool_, 10: np.float16, 11: np.float64,
    12: np.uint32, 13: np.uint64,
}

TORCH_TO_NP = {
    torch.bool: np.bool_, torch.int8: np.int8, torch.uint8: np.uint8, torch.int16: np.int16,
    torch.int32: np.int32, torch.int64: np.int64, torch.float16: np.float16,
    torch.float32: np.float32, torch.float64: np.float64,
}
NP_TO_TORCH = {np.dtype(v): k for k, v in TORCH_TO_NP.items()}
TORCH_TO_BT = {k: _lib.NP_TO_BT[np.dtype(v)] for k, v in TORCH_TO_NP.items()}
for _name in ("uint16", "uint32", "uint64"):
    if hasattr(torch, _name):
        TORCH_TO_NP[getattr(torch, _name)] = getattr(np, _name)
        NP_TO_TORCH[np.dtype(getattr(np, _name))] = getattr(torch, _name)

UNARY = {"Sqrt": "SQRT", "Exp": "EXP", "Sin": "SIN", "Cos": "COS", "Atan": "ATAN",
         "Tanh": "TANH", "Sigmoid": "SIGMOID", "Floor": "FLOOR", "Round": "ROUND", "Erf": "ERF"}
# numpy expressions of the reference (ref_runtime.py:458-489) used only on
# zero-size arrays, to learn numpy's result dtype.
_UNARY_NP = {"Sqrt": np.sqrt, "Exp": np.exp, "Sin": np.sin, "Cos": np.cos, "Atan": np.arctan,
             "Tanh": np.tanh, "Sigmoid": lambda v: 1.0 / (1.0 + np.exp(-v)), "Floor": np.floor,
             "Round": np.rint, "Erf": None}
COMPARE = {"Greater": "GREATER", "Less": "LESS", "GreaterOrEqual": "GEQ"}
_BINARY = {"Add": "ADD", "Sub": "SUB", "Mul": "MUL", "Div": "DIV", "Pow": "POW"}
_F16_TWO = np.array(2.0, dtype=np.float16)   # the Snake exponent constant of the graph
_SAME = object()   # a cached Cast whose result is its input
OP_NAMES = {v: k for k, v in OP.items()}


def as_cuda_device(device):
    """torch.device for an ordinal, a torch.device or None (current device)."""
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    if isinstance(device, torch.device):
        return device if device.index is not None else torch.device("cuda", torch.cuda.current_device())
    return torch.device("cuda", int(device))


_NP_OF_TORCH = {k: np.dtype(v) for k, v in TORCH_TO_NP.items()}


def np_dtype(t):
    return _NP_OF_TORCH[t.dtype]


_F16 = np.dtype(np.float16)
_F32 = np.dtype(np.float32)


def _wide(dt):
    """fp16 is widened to fp32 before compute (ref_runtime.py:49-51)."""
    return _F32 if dt == _F16 else np.dtype(dt)


@functools.lru_cache(maxsize=4096)
def _bshape(*shapes):
    """numpy's broadcast shape of the given shapes (cached: the same node
    shapes recur for every utterance)."""
    return np.broadcast_shapes(*shapes)


def _probe(dt):
    return np.empty((0,), dtype=dt)


@functools.lru_cache(maxsize=256)
def _ew_attrs(compute_dt, alpha):
    """The attribute block of a launch (shared: the library only reads it)."""
    return _lib.BtEwAttrs(_lib.NP_TO_BT[compute_dt], float(np.float32(alpha)))


@functools.lru_cache(maxsize=4096)
def _binary_result(op, a, b):
    """numpy's result dtype of the binary op on arrays of dtypes a, b."""
    if op == "Div" and a.kind in "iu" and b.kind in "iu":
        return np.floor_divide(_probe(a), _probe(b)).dtype   # ref :452-455
    f = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Div": np.true_divide, "Pow": np.power}[op]
    return f(_probe(a), _probe(b)).dtype


def _raw_stream(device_index):
    """The current CUDA stream of a device as an integer handle."""
    return torch.cuda.current_stream(device_index).cuda_stream


try:   # torch's own fast accessor of the same handle, where this torch has it
    _fast = torch._C._cuda_getCurrentRawStream
    _raw_stream = lambda device_index: _fast(device_index)   # noqa: E731
except AttributeError:
    pass


_I64x8 = ctypes.c_int64 * 8


def tensor_desc(t):
    """BtTensor view of a CUDA tensor (element strides, arbitrary layout)."""
    shape = t.shape
    if len(shape) > 8:
        raise ValueError(f"rank {len(shape)} exceeds 8")
    return _lib.BtTensor(t.data_ptr(), TORCH_TO_BT[t.dtype], len(shape), _I64x8(*shape), _I64x8(*t.stride()))


class BtRuntime:
    """Op-table interpreter whose arithmetic runs on the GPU (see module doc)."""

    HOT_OPS = ("Add", "Sub", "Mul", "Div", "Pow", "Sqrt", "Exp", "Sin", "Cos", "Atan", "Tanh",
               "Sigmoid", "Floor", "Round", "Erf", "LeakyRelu", "Clip", "Equal", "Greater", "Less",
               "GreaterOrEqual", "And", "Where", "Cast", "ReduceMean", "ReduceSum", "Softmax",
               "LayerNormalization", "SkipLayerNormalization", "FastGelu", "DequantizeLinear",
               "DynamicQuantizeLinear", "Split", "Reshape", "Unsqueeze", "Squeeze", "Transpose", "Concat",
               "Slice", "Expand")

    def __init__(self, device=None):
        if not torch.cuda.is_available():
            raise RuntimeError("BtRuntime needs a CUDA device (there is no CPU fallback)")
        self.device = as_cuda_device(device)
        self.lib = load()
        with torch.cuda.device(self.device):
            check(self.lib.bt_init(self.device.index), "bt_init")
        self._index = self.device.index
        self._consts = {}
        self._ew_plans = {}
        self._node_plans = {}   # node signature -> launch plan (see dispatch)
        self._scalars = {}
        self.launches = 0

    # ---- device values ---------------------------------------------------------
    def to_device(self, v):
        """CUDA tensor for an env value (numpy arrays are uploaded once and cached)."""
        if isinstance(v, torch.Tensor):
            if not v.is_cuda:
                v = v.to(self.device)
            return v
        a = np.asarray(v)
        key = id(v)
        hit = self._consts.get(key)
        if hit is not None and hit[0]() is v:
            return hit[1]
        if a.ndim > 1 and not a.flags.c_contiguous:
            # keep the array's axis order in memory (a later reduction sums
            # in that order): upload the dense order-'K' copy, then permute
            dense = np.array(a, order="K", copy=True)
            order = _k_order([dense], dense.shape)
            phys = np.ascontiguousarray(dense.transpose(order))
            t = torch.from_numpy(phys).to(self.device).permute(_inverse(order))
        else:
            # (np.ascontiguousarray makes 0-d arrays 1-d: keep the shape)
            t = torch.from_numpy(np.ascontiguousarray(a).reshape(a.shape)).to(self.device)
        try:
            self._consts[key] = (weakref.ref(v), t)
            # the device copy lives as long as the array: a long run that
            # uploads many host results does not accumulate them
            weakref.finalize(v, self._consts.pop, key, None)
        except TypeError:
            pass
        return t

    def _empty(self, shape, dt):
        return torch.empty(tuple(int(s) for s in shape), dtype=NP_TO_TORCH[np.dtype(dt)], device=self.device)

    def _stream(self):
        """Points the library at this thread's current CUDA stream (set on
        every launch: other callers on the thread may have set another)."""
        check(self.lib.bt_set_stream(_raw_stream(self.device.index)), "bt_set_stream")

    # ---- kernels ------------------------------------------------------------------
    def elementwise(self, opname, inputs, out_shape, out_dt, compute_dt, alpha=0.0):
        """One element-wise launch.  Everything but the data pointers depends
        only on the inputs' dtypes, shapes and strides, so it is prepared once
        per such signature (numpy's result layout, the descriptors, the
        attribute block) and reused: a call then allocates the result, writes
        the pointers into the prepared descriptors and launches."""
        return self._launch_plan(self._ew_plan(opname, inputs, out_shape, out_dt, compute_dt, alpha), inputs)

    def _ew_plan(self, opname, inputs, out_shape, out_dt, compute_dt, alpha=0.0):
        """The prepared launch of one element-wise signature (cached)."""
        key = (opname, tuple(out_shape), out_dt, compute_dt, alpha,
               tuple((t.dtype, t.shape, t.stride()) for t in inputs))
        plan = self._ew_plans.get(key)
        if plan is None:
            plan = self._ew_prepare(opname, inputs, out_shape, out_dt, compute_dt, alpha)
            if len(self._ew_plans) >= 8192:
                self._ew_plans.clear()
            self._ew_plans[key] = plan
        return plan

    def _launch_plan(self, plan, inputs):
        """Allocates the result of a prepared launch, writes the data
        pointers into its descriptors and launches it."""
        alloc_shape, tdt, back, code, descs, od, attrs, numel = plan
        out = torch.empty(alloc_shape, dtype=tdt, device=self.device)
        if numel:
            for i, t in enumerate(inputs):
                descs[i].data = t.data_ptr()
            od.data = out.data_ptr()
            lib = self.lib
            lib.bt_set_stream(_raw_stream(self._index))   # always BT_OK
            rc = lib.bt_elementwise(code, len(inputs), descs, od, attrs)
            if rc:
                check(rc, f"bt_elementwise({OP_NAMES.get(code, code)})")
            self.launches += 1
        return out if back is None else out.permute(back)

    def _remember(self, key, plan):
        """Caches the launch plan of a node signature (dispatch's fast path)."""
        if len(self._node_plans) >= 8192:
            self._node_plans.clear()
        self._node_plans[key] = plan

    def _ew_prepare(self, opname, inputs, out_shape, out_dt, compute_dt, alpha):
        out_shape = tuple(int(v) for v in out_shape)
        back = None
        if any(not t.is_contiguous() for t in inputs):
            order = _k_order(inputs, out_shape)
            if not _is_identity(order):
                # numpy allocates the result in this axis order: run the
                # kernel on the permuted views (contiguous output) and hand
                # back the logical view
                nd = len(out_shape)
                inputs = [t.view((1,) * (nd - t.dim()) + tuple(t.shape)).permute(order) for t in inputs]
                out_shape = tuple(out_shape[a] for a in order)
                back = _inverse(order)
        tdt = NP_TO_TORCH[np.dtype(out_dt)]
        numel = int(np.prod(out_shape, dtype=np.int64)) if out_shape else 1
        descs = (_lib.BtTensor * len(inputs))(*[tensor_desc(t) for t in inputs])
        strides, acc = [], 1
        for d in reversed(out_shape):
            strides.append(acc)
            acc *= d
        od = make_tensor(0, np.dtype(out_dt), out_shape, tuple(reversed(strides)))
        attrs = _ew_attrs(np.dtype(compute_dt), float(alpha))
        return out_shape, tdt, back, OP[opname], descs, od, attrs, numel

    # ---- data movement: strided copies through the IDENTITY kernel ----------------
    @staticmethod
    def _copy_compute(dt):
        """A compute dtype in which IDENTITY copies dt exactly (float32 keeps
        the vector paths for fp32 / fp16 data)."""
        dt = np.dtype(dt)
        if dt.kind == "f":
            return np.float64 if dt == np.float64 else np.float32
        return np.uint64 if dt == np.uint64 else np.int64

    def _copy_desc(self, src_desc, src_dt, out):
        """IDENTITY from a source descriptor (any strides, negative ones
        included) into the tensor view `out`, converting to out's dtype."""
        if out.numel() == 0:
            return out
        descs = (_lib.BtTensor * 1)(src_desc)
        cdt = self._copy_compute(np.result_type(src_dt, np_dtype(out)))
        attrs = _lib.BtEwAttrs(_lib.NP_TO_BT[np.dtype(cdt)], 0.0)
        self._stream()
        check(self.lib.bt_elementwise(OP["IDENTITY"], 1, descs, tensor_desc(out), attrs), "bt_elementwise(copy)")
        self.launches += 1
        return out

    def _materialize(self, view):
        """Contiguous copy of a torch view (permuted, expanded, narrowed)."""
        out = self._empty(tuple(view.shape), np_dtype(view))
        return self._copy_desc(tensor_desc(view), np_dtype(view), out)

    def transpose(self, x, perm):
        nd = x.dim()
        perm = list(range(nd))[::-1] if perm is None else [int(p) % max(nd, 1) for p in perm]
        return self._materialize(x.permute(perm))

    def concat(self, vals, axis):
        if any(np_dtype(v) == np.float16 for v in vals):                # ref :531-535
            vals = [self._widen(v) for v in vals]
        nd = vals[0].dim()
        axis = int(axis)
        if not -nd <= axis < nd:
            raise np.exceptions.AxisError(axis, nd)
        axis %= nd
        for v in vals[1:]:
            if v.dim() != nd or any(v.shape[d] != vals[0].shape[d] for d in range(nd) if d != axis):
                raise ValueError("all the input array dimensions except for the concatenation axis must match exactly")
        dt = np.result_type(*[np_dtype(v) for v in vals])
        shape = list(vals[0].shape)
        shape[axis] = sum(int(v.shape[axis]) for v in vals)
        out = self._empty(shape, dt)
        off = 0
        for v in vals:
            n = int(v.shape[axis])
            if n:
                self._copy_desc(tensor_desc(v), np_dtype(v), out.narrow(axis, off, n))
            off += n
        return out

    def slice(self, x, starts, ends, axes=None, steps=None):
        """ref_runtime.py:307-325: clamp each (start, end) as the reference
        does, then apply Python slice semantics (a clamped end of -1 means the
        last element), and copy the strided view -- negative steps give
        negative strides, which the copy kernel reads directly."""
        starts, ends = _host_ints(starts), _host_ints(ends)
        axes = list(range(len(starts))) if axes is None else _host_ints(axes)
        steps = [1] * len(starts) if steps is None else _host_ints(steps)
        nd = x.dim()
        shape, strides, offset = list(x.shape), list(x.stride()), 0
        for s_, e_, a, st in zip(starts, ends, axes, steps):
            a, s_, e_, st = int(a) % nd, int(s_), int(e_), int(st)
            dim = int(x.shape[a])
            lo, hi = (0, dim) if st > 0 else (-1, dim - 1)
            s_ = min(max(s_ + dim if s_ < 0 else s_, lo), hi)
            e_ = min(max(e_ + dim if e_ < 0 else e_, lo), hi)
            start, stop, step = slice(s_, e_, st).indices(dim)
            shape[a] = len(range(start, stop, step))
            offset += start * strides[a]
            strides[a] *= step
        dt = np_dtype(x)
        # numpy's slice is a view in x's axis order: copy into that order
        _, order = self._physical(x)
        out = self._empty([shape[a] for a in order], dt).permute(_inverse(order))
        if out.numel() == 0:
            return out
        src = make_tensor(x.data_ptr() + offset * x.element_size(), dt, shape, strides)
        return self._copy_desc(src, dt, out)

    def expand(self, x, shape):
        shape = np.broadcast_shapes(tuple(x.shape), tuple(int(v) for v in shape))
        xv = x.reshape((1,) * (len(shape) - x.dim()) + tuple(x.shape)).expand(shape)
        return self._materialize(xv)

    def _widen(self, t):
        """fp16 tensor -> fp32 copy (kernel), other dtypes unchanged."""
        if t.dtype == torch.float16:
            return self.elementwise("IDENTITY", [t], t.shape, np.float32, np.float32)
        return t

    def _contig(self, t):
        """C-contiguous copy of a view (the copy kernel), t itself when it is one."""
        return t if t.is_contiguous() else self._materialize(t)

    def _physical(self, x):
        """(phys, order): x's axes in its memory order (numpy's order 'K'),
        phys = x.permute(order), a C-contiguous tensor when x is a dense
        view; order is the identity for C-contiguous x."""
        if x.is_contiguous():
            return x, list(range(x.dim()))
        order = _k_order([x], tuple(x.shape))
        return x.permute(order), order

    # ---- the op table -----------------------------------------------------------------
    def dispatch(self, op, node_input, node_output, at, env):
        # The most frequent nodes (binary and unary element-wise ops, Cast)
        # first, without the helpers below: once a node signature -- the op
        # and each device input's dtype, shape and strides -- has run, its
        # launch plan (numpy's result dtype and layout included) is cached,
        # and the node costs a lookup, the result's allocation and the launch.
        if op in _BINARY:
            x, y = env[node_input[0]], env[node_input[1]]
            cached = type(x) is torch.Tensor and type(y) is torch.Tensor and x.is_cuda and y.is_cuda
            if cached:
                key = (op, x.dtype, x.shape, x.stride(), y.dtype, y.shape, y.stride())
                plan = self._node_plans.get(key)
                if plan is not None:
                    env[node_output[0]] = self._launch_plan(plan, (x, y))
                    return
            if not isinstance(x, torch.Tensor) or not x.is_cuda:
                x = self.to_device(x)
            if not isinstance(y, torch.Tensor) or not y.is_cuda:
                y = self.to_device(y)
            a, b = _wide(_NP_OF_TORCH[x.dtype]), _wide(_NP_OF_TORCH[y.dtype])
            dt = _binary_result(op, a, b)
            if op == "Pow" and dt.kind != "f":
                raise NotImplementedError("integer Pow is not on the GPU path")
            plan = self._ew_plan(_BINARY[op], [x, y], _bshape(tuple(x.shape), tuple(y.shape)), dt, self._compute(dt))
            if cached:
                self._remember(key, plan)
            env[node_output[0]] = self._launch_plan(plan, (x, y))
            return
        if op in UNARY:
            x = env[node_input[0]]
            cached = type(x) is torch.Tensor and x.is_cuda
            if cached:
                key = (op, x.dtype, x.shape, x.stride())
                plan = self._node_plans.get(key)
                if plan is not None:
                    env[node_output[0]] = self._launch_plan(plan, (x,))
                    return
            x = self.to_device(x)
            a = _wide(np_dtype(x))
            if op == "Erf":
                dt = np.dtype(np.float32) if a == np.float32 else np.dtype(np.float64)
                if a.kind not in "fiub":
                    raise TypeError(f"Erf of {a}")
            else:
                dt = _UNARY_NP[op](_probe(a)).dtype
            plan = self._ew_plan(UNARY[op], [x], x.shape, dt, self._compute(dt))
            if cached:
                self._remember(key, plan)
            env[node_output[0]] = self._launch_plan(plan, (x,))
            return
        if op == "Cast":                                        # ref :572-578
            x = env[node_input[0]]
            cached = type(x) is torch.Tensor and x.is_cuda
            if cached:
                key = (op, at["to"], x.dtype, x.shape, x.stride())
                plan = self._node_plans.get(key)
                if plan is not None:
                    env[node_output[0]] = x if plan is _SAME else self._launch_plan(plan, (x,))
                    return
            x = self.to_device(x)
            target = np.dtype(ONNX_TO_NUMPY[at["to"]])
            if target == np.float16:
                target = np.dtype(np.float32)
            if np_dtype(x) == target and self._physical(x)[0].is_contiguous():
                # astype to the dtype x already has: numpy copies the same
                # values in the same axis order, and graph values are never
                # written after they are made, so x itself serves (half of
                # the model's Casts are float32 -> float32 once fp16 targets
                # are elided, one before every DynamicQuantizeLinear)
                plan, out = _SAME, x
            else:
                src = _wide(np_dtype(x))
                plan = self._ew_plan("IDENTITY", [x], x.shape, target, self._cast_compute(src, target))
                out = self._launch_plan(plan, (x,))
            if cached:
                self._remember(key, plan)
            env[node_output[0]] = out
            return
        if op in ("ReduceMean", "ReduceSum"):                 # ref :589-598
            x = env[node_input[0]]
            ax = env[node_input[1]] if len(node_input) > 1 and node_input[1] else at.get("axes")
            if type(x) is torch.Tensor and x.is_cuda and not isinstance(ax, torch.Tensor):
                akey = None if ax is None else tuple(np.asarray(ax).reshape(-1).tolist())
                key = (op, akey, at.get("keepdims", 1), at.get("noop_with_empty_axes", 0), x.dtype, x.shape,
                       x.stride())
                plan = self._node_plans.get(key)
                if plan is None:
                    plan = self._reduce_plan(op, x, akey, at)
                    if plan is not None:
                        self._remember(key, plan)
                if plan is not None:
                    env[node_output[0]] = self._run_reduce_plan(plan, x)
                    return
        if op == "Concat":                                    # ref :531-535
            # (host values -- the model's shape arithmetic -- are uploaded once
            # and cached by to_device)
            vals = [self.to_device(env[i]) for i in node_input if i]
            if vals and all(type(v) is torch.Tensor for v in vals):
                key = (op, at["axis"], tuple((v.dtype, v.shape, v.stride()) for v in vals))
                plan = self._node_plans.get(key)
                if plan is None:
                    plan = self._concat_plan(vals, at["axis"])
                    if plan is not None:
                        self._remember(key, plan)
                if plan is not None:
                    env[node_output[0]] = self._run_concat_plan(plan, vals)
                    return

        def arg(i, default=None):
            if i >= len(node_input) or not node_input[i]:
                return default
            return env[node_input[i]]

        def dev(i):
            v = arg(i)
            return None if v is None else self.to_device(v)

        if op in ("Add", "Sub", "Mul", "Div", "Pow"):
            x, y = dev(0), dev(1)
            a, b = _wide(np_dtype(x)), _wide(np_dtype(y))
            shape = _bshape(tuple(x.shape), tuple(y.shape))
            dt = _binary_result(op, a, b)
            if op == "Pow" and dt.kind != "f":
                raise NotImplementedError("integer Pow is not on the GPU path")
            name = {"Add": "ADD", "Sub": "SUB", "Mul": "MUL", "Div": "DIV", "Pow": "POW"}[op]
            out = self.elementwise(name, [x, y], shape, dt, self._compute(dt))
        elif op == "LeakyRelu":
            x = dev(0)
            a = _wide(np_dtype(x))
            v = _probe(a)
            dt = np.where(v < 0, v * np.float32(at.get("alpha", 0.01)), v).dtype   # ref :476-479
            out = self.elementwise("LEAKYRELU", [x], x.shape, dt, self._compute(dt),
                                   alpha=np.float32(at.get("alpha", 0.01)))
        elif op == "Clip":
            x, lo, hi = dev(0), dev(1), dev(2)
            v = _probe(_wide(np_dtype(x)))
            if lo is not None:
                v = np.maximum(v, _probe(_wide(np_dtype(lo))))
            if hi is not None:
                v = np.minimum(v, _probe(_wide(np_dtype(hi))))
            dt = v.dtype
            if lo is None and hi is None:
                out = self.elementwise("IDENTITY", [x], x.shape, dt, self._cast_compute(np_dtype(x), dt))
            else:
                lo = lo if lo is not None else self._bound(dt, low=True)
                hi = hi if hi is not None else self._bound(dt, low=False)
                shape = np.broadcast_shapes(tuple(x.shape), tuple(lo.shape), tuple(hi.shape))
                out = self.elementwise("CLIP", [x, lo, hi], shape, dt, self._compute(dt))
        elif op == "Equal":
            x, y = dev(0), dev(1)
            ct = np.result_type(np_dtype(x), np_dtype(y))
            shape = np.broadcast_shapes(tuple(x.shape), tuple(y.shape))
            out = self.elementwise("EQUAL", [x, y], shape, np.bool_, self._compute(_wide(ct)))
        elif op in COMPARE:
            x, y = dev(0), dev(1)
            ct = np.result_type(_wide(np_dtype(x)), _wide(np_dtype(y)))
            shape = np.broadcast_shapes(tuple(x.shape), tuple(y.shape))
            out = self.elementwise(COMPARE[op], [x, y], shape, np.bool_, self._compute(ct))
        elif op == "And":
            x, y = dev(0), dev(1)
            shape = np.broadcast_shapes(tuple(x.shape), tuple(y.shape))
            out = self.elementwise("AND", [x, y], shape, np.bool_, np.float64)
        elif op == "Where":
            c, x, y = dev(0), dev(1), dev(2)
            dt = np.where(_probe(np.bool_), _probe(np_dtype(x)), _probe(np_dtype(y))).dtype
            shape = np.broadcast_shapes(tuple(c.shape), tuple(x.shape), tuple(y.shape))
            out = self.elementwise("WHERE", [c, x, y], shape, dt, self._cast_compute_where(dt))
        elif op == "DequantizeLinear":                          # ref :631-636
            q, scale, zp = dev(0), dev(1), dev(2)
            out = self.dequantize(q, scale, zp)
        elif op == "DynamicQuantizeLinear":                     # ref :106-116, :625-630
            x = dev(0)
            if np_dtype(x) not in (np.float32, np.float16):
                x = self._as_f32(x)
            for name, v in zip(node_output, self.dynamic_quantize(x)):
                if name:
                    env[name] = v
            return
        elif op == "FastGelu":                                  # ref :610-611
            x, b = dev(0), dev(1)
            x = self._as_f32(x)
            ins = [x] + ([self._as_f32(b)] if b is not None else [])
            shape = np.broadcast_shapes(*[tuple(t.shape) for t in ins])
            out = self.elementwise("GELU", ins, shape, np.float32, np.float32)
        elif op in ("ReduceMean", "ReduceSum"):                 # ref :589-598
            axes = arg(1) if len(node_input) > 1 else at.get("axes")
            out = self._reduce(op, dev(0), axes, at)
        elif op == "Softmax":                                   # ref :599-600
            x = self._as_f32(dev(0))
            out = self.softmax(x, None, int(at.get("axis", -1)))
        elif op == "LayerNormalization":                        # ref :601-603
            out = self.layernorm(dev(0), None, None, dev(1), dev(2), int(at.get("axis", -1)),
                                 at.get("epsilon", 1e-5))
        elif op == "SkipLayerNormalization":                    # ref :604-609
            out = self.layernorm(dev(0), dev(1), dev(4), dev(2), dev(3), -1, at.get("epsilon", 1e-12))
        elif op == "Split":                                     # ref :536-547 (views)
            x = dev(0)
            axis = int(at.get("axis", 0)) % max(1, x.dim())
            sizes = arg(1)
            if sizes is None:
                parts = np.array_split(np.empty(x.shape[axis], np.int8), len(node_output))
                sizes = [len(p) for p in parts]
            else:
                sizes = [int(s) for s in np.asarray(sizes if not isinstance(sizes, torch.Tensor)
                                                    else sizes.cpu().numpy()).reshape(-1)]
            for name, p in zip(node_output, torch.split(x, sizes, dim=axis)):
                if name:
                    env[name] = p
            return
        elif op == "Transpose":                                 # ref :517-518 (view)
            x = dev(0)
            perm = at.get("perm")
            nd = x.dim()
            out = x.permute(list(range(nd))[::-1] if perm is None else [int(v) % max(nd, 1) for v in perm])
        elif op == "Concat":                                    # ref :531-535
            out = self.concat([self.to_device(env[i]) for i in node_input if i], at["axis"])
        elif op == "Slice":                                     # ref :548-549, :307-325
            out = self.slice(dev(0), arg(1), arg(2), arg(3), arg(4))
        elif op == "Expand":                                    # ref :553-555
            out = self.expand(dev(0), _host_ints(arg(1)))
        elif op == "Reshape":                                   # ref :511-516 (view)
            x = dev(0)
            shape = [int(s) for s in _host_ints(arg(1))]
            if not at.get("allowzero", 0):
                shape = [x.shape[i] if s == 0 else s for i, s in enumerate(shape)]
            # a view where numpy's reshape gives one, else numpy's C-order copy
            try:
                out = x.view(shape)
            except RuntimeError:
                out = self._materialize(x).view(shape)
        elif op == "Unsqueeze":                                 # ref :519-523 (view)
            x = dev(0)
            axes = arg(1) if len(node_input) > 1 else at.get("axes")
            out = x
            for a in sorted(int(v) for v in _host_ints(axes)):
                out = out.unsqueeze(a)
        elif op == "Squeeze":                                   # ref :524-530 (view)
            x = dev(0)
            axes = arg(1) if len(node_input) > 1 else at.get("axes")
            if axes is None:
                out = x.reshape([s for s in x.shape if s != 1])
            else:
                out = x
                for a in sorted((int(v) % x.dim() for v in _host_ints(axes)), reverse=True):
                    if out.shape[a] != 1:
                        raise ValueError("cannot select an axis to squeeze out which has size not equal to one")
                    out = out.squeeze(a)
        else:
            raise NotImplementedError(f"{op} ({node_output}) is not on the B200 path")
        env[node_output[0]] = out

    def run_nodes(self, nodes, env, fuse=False, keep=()):
        """Executes ``(op, inputs, outputs, attrs)`` nodes in order, wrapping
        failures like the reference's drivers (ref_runtime.py:398-403).

        fuse: runs of nodes that form a known chain (Snake, DequantizeLinear
        then Mul, Add then Sigmoid / LeakyRelu, Mul then Add; chains.plan)
        run as one bt_fused_chain launch each, with identical results; their
        intermediate values are then not stored in ``env``.  A value read by
        more than one node, or named in ``keep``, is never fused away."""
        groups = {}
        skip = set()
        if fuse:
            from . import chains
            for g in chains.plan(nodes, keep):
                groups[g.last] = g
                skip.update(g.nodes)
        for i, (op, ins, outs, at) in enumerate(nodes):
            try:
                g = groups.get(i)
                if g is not None:
                    vals = [env[n] if n else None for n in g.inputs]
                    dts = [np_dtype(v) if isinstance(v, torch.Tensor) else np.asarray(v).dtype for v in vals]
                    ins_dev = [self.to_device(v) for v in vals] if g.inputs_ok(dts) else None
                    # (a view input would give numpy's result its own axis
                    # order, which later reductions follow: node by node then)
                    if ins_dev is not None and all(t.is_contiguous() for t in ins_dev):
                        env[g.output] = self.chain(g.prog(), ins_dev)
                        continue
                    for j in g.nodes:   # not a float32 chain: node by node
                        jop, jins, jouts, jat = nodes[j]
                        self.dispatch(jop, list(jins), list(jouts), dict(jat or {}), env)
                    continue
                if i in skip:
                    continue
                self.dispatch(op, list(ins), list(outs), dict(at or {}), env)
            except Exception as exc:
                raise RuntimeError(f"{op} {list(outs)} failed: {exc}") from exc
        return env

    def capture_nodes(self, nodes, env, warmup=1):
        """The node list as one CUDA graph (see CapturedNodes): for a serving
        loop that runs the same node sequence on inputs of the same shapes,
        the per-node host work of ``dispatch`` is paid once, at capture."""
        return CapturedNodes(self, nodes, env, warmup)

    # ---- helpers --------------------------------------------------------------------------
    @staticmethod
    @functools.lru_cache(maxsize=64)
    def _compute(dt):
        dt = np.dtype(dt)
        if dt == np.float16:
            return np.dtype(np.float32)
        if dt.kind == "f":
            return dt
        if dt.kind == "b":
            return np.dtype(np.int64)
        return np.dtype(np.uint64) if dt == np.uint64 else np.dtype(np.int64)

    @staticmethod
    def _cast_compute(src, dst):
        src, dst = np.dtype(src), np.dtype(dst)
        if src.kind in "iub" and dst.kind in "iub":
            return np.dtype(np.int64)
        if src.kind in "iub" and dst.kind == "f":
            return np.dtype(np.int64)
        if src.kind == "f" and dst == np.float32:
            # float16 widens exactly and float64 rounds once (the load's
            # conversion) -- the same float32 as numpy's astype
            return np.dtype(np.float32)
        return np.dtype(np.float64)

    def _cast_compute_where(self, dt):
        return np.dtype(np.float64) if np.dtype(dt).kind == "f" else np.dtype(np.int64)

    def _bound(self, dt, low):
        dt = np.dtype(dt)
        if dt.kind == "f":
            v = -np.inf if low else np.inf
        elif dt.kind == "b":
            v = False if low else True
        else:
            info = np.iinfo(dt)
            v = info.min if low else info.max
        return self._scalar(v, dt)

    def _scalar(self, value, dt):
        """A 0-d device constant, uploaded once per (value, dtype): no host
        copy inside a captured node list."""
        key = (np.dtype(dt).str, np.array(value, dtype=dt).tobytes())
        t = self._scalars.get(key)
        if t is None:
            t = self._scalars[key] = torch.tensor(np.array(value, dtype=dt)).to(self.device)
        return t

    def dynamic_quantize(self, x, range=None):
        """DynamicQuantizeLinear of a float32 / float16 tensor
        (bt_dynamic_quantize): (y uint8 of x's shape, scale float32 0-d,
        zero point uint8 0-d).  range: x's range record as its producer
        wrote it (adain_snake(..., ranges=)); only the quantize pass runs
        then (bt_dynamic_quantize_ranged)."""
        x = self._contig(x)
        y = self._empty(tuple(x.shape), np.uint8)
        sc = self._empty((), np.float32)
        zp = self._empty((), np.uint8)
        self._stream()
        if range is None:
            check(self.lib.bt_dynamic_quantize(tensor_desc(x), tensor_desc(y), sc.data_ptr(), zp.data_ptr()),
                  "bt_dynamic_quantize")
            self.launches += 2
        else:
            check(self.lib.bt_dynamic_quantize_ranged(tensor_desc(x), tensor_desc(y), sc.data_ptr(), zp.data_ptr(),
                                                      range.data_ptr()), "bt_dynamic_quantize_ranged")
            self.launches += 1
        return y, sc, zp

    def conv_int_epilogue(self, acc, bias, x_scale, w_scale):
        """The integer convolution epilogue in one kernel (bt_conv_int_epilogue):
        float32(acc + int32(floor(bias / s))) * s with s = x_scale * w_scale,
        acc int32 [B, C, T], bias [C]; returns float32 [B, C, T]."""
        acc, bias = self._contig(acc), self._contig(bias)
        out = self._empty(tuple(acc.shape), np.float32)
        self._stream()
        check(self.lib.bt_conv_int_epilogue(tensor_desc(acc), tensor_desc(bias), tensor_desc(x_scale),
                                            tensor_desc(w_scale), tensor_desc(out)), "bt_conv_int_epilogue")
        self.launches += 1
        return out

    def _as_f32(self, t):
        dt = np_dtype(t)
        if dt == np.float32:
            return t
        return self.elementwise("IDENTITY", [t], t.shape, np.float32, self._cast_compute(dt, np.float32))

    def _reduce(self, op, x, axes_in, at):
        x = self._widen(x)
        keep = bool(at.get("keepdims", 1))
        if axes_in is None:
            if at.get("noop_with_empty_axes", 0):
                return x
            axes = tuple(range(x.dim()))
        else:
            axes = tuple(int(a) for a in _host_ints(axes_in))
            if len(axes) == 0:
                return x
        nd = x.dim()
        for a in axes:
            if not -nd <= a < nd:
                raise np.exceptions.AxisError(a, nd)
        norm = sorted(set(a % nd for a in axes))
        if len(norm) != len(axes):
            raise ValueError("duplicate value in 'axis'")
        dt = np_dtype(x)
        if dt != np.float32:
            raise NotImplementedError(f"{op} of {dt} is not on the GPU path (float32/float16 only)")
        if not x.is_contiguous():
            # numpy walks a view in its memory order: reduce the dense
            # physical tensor over the same axes and view the result back
            phys, order = self._physical(x)
            if not _is_identity(order):
                if not phys.is_contiguous():
                    raise NotImplementedError(f"{op} of a permuted view with gaps is not on the GPU path")
                r = self._reduce(op, phys, sorted(order.index(a) for a in norm), {"keepdims": 1})
                r = r.permute(_inverse(order))
                return r if keep else r.squeeze(tuple(norm))
            # C order with gaps (a slice): numpy cannot merge the axes of a
            # reduced block across a gap, so its pairwise runs would be shorter
            for blk in _axis_blocks(norm, x.shape):
                big = [a for a in blk if x.shape[a] != 1]
                for a, b in zip(big, big[1:]):
                    if x.stride(a) != x.stride(b) * x.shape[b]:
                        raise NotImplementedError(f"{op} over axes {axes} of a strided view is not on the GPU path")
        x = self._contig(x)
        kind = 1 if op == "ReduceMean" else 0
        out_shape = [1 if i in norm else s for i, s in enumerate(x.shape)] if keep else \
            [s for i, s in enumerate(x.shape) if i not in norm]
        if x.numel() == 0 or any(x.shape[i] == 0 for i in norm):
            fill = 0.0 if kind == 0 else float("nan")
            return torch.full(out_shape, fill, dtype=torch.float32, device=self.device)
        # numpy reduces one contiguous block of axes in a single pass:
        # pairwise over the block when it is innermost, slice after slice
        # (lexicographic order) otherwise.  Two blocks whose inner block is
        # innermost are the pairwise row sums added slice after slice over
        # the outer block, which is two passes here.  Other axis sets would
        # interleave the outer chains differently and are not on the GPU path.
        blocks = _axis_blocks(norm, x.shape)
        if len(blocks) == 1:
            return self._reduce_block(x, blocks[0], kind).reshape(out_shape)
        innermost = all(s == 1 for s in x.shape[blocks[1][-1] + 1:])
        if len(blocks) == 2 and innermost:
            rows = self._reduce_block(x, blocks[1], 0)
            total = self._reduce_block(rows, blocks[0], 0)
            if kind == 1:
                count = int(np.prod([x.shape[i] for i in norm]))
                total = self._mean_from_sum(total, count)
            return total.reshape(out_shape)
        raise NotImplementedError(f"{op} over axes {axes} of shape {tuple(x.shape)} is not on the GPU path")

    def _reduce_block(self, x, blk, kind):
        """Reduces the contiguous axis block ``blk`` of x with keepdims=1."""
        n_axes = len(blk)
        axes = (ctypes_i64 * n_axes)(*blk)
        out_shape = [1 if i in blk else s for i, s in enumerate(x.shape)]
        out = self._empty(out_shape, np.float32)
        self._stream()
        check(self.lib.bt_reduce(kind, tensor_desc(x), axes, n_axes, 1, tensor_desc(out)), "bt_reduce")
        self.launches += 1
        return out

    def _reduce_plan(self, op, x, axes, at):
        """The cached launch of a reduction in its common form: a dense
        float32 tensor reduced over one contiguous block of axes (one
        bt_reduce launch, as _reduce runs it).  None for every other case,
        which _reduce handles (and where it raises, it raises there)."""
        if np_dtype(x) != np.float32 or not x.is_contiguous() or x.numel() == 0:
            return None
        nd = x.dim()
        if axes is None:
            if at.get("noop_with_empty_axes", 0):
                return None
            axes = tuple(range(nd))
        if len(axes) == 0 or any(not -nd <= a < nd for a in axes):
            return None
        norm = sorted(set(int(a) % nd for a in axes))
        if len(norm) != len(axes) or any(x.shape[i] == 0 for i in norm):
            return None
        blocks = _axis_blocks(norm, x.shape)
        if len(blocks) != 1:
            return None
        blk = blocks[0]
        keep = bool(at.get("keepdims", 1))
        kshape = tuple(1 if i in blk else int(s) for i, s in enumerate(x.shape))
        out_shape = tuple(1 if i in norm else int(s) for i, s in enumerate(x.shape)) if keep else \
            tuple(int(s) for i, s in enumerate(x.shape) if i not in norm)
        strides, acc = [], 1
        for d in reversed(kshape):
            strides.append(acc)
            acc *= d
        od = make_tensor(0, np.dtype(np.float32), kshape, tuple(reversed(strides)))
        return (1 if op == "ReduceMean" else 0, (ctypes_i64 * len(blk))(*blk), len(blk), tensor_desc(x), od, kshape,
                out_shape)

    def _run_reduce_plan(self, plan, x):
        kind, axes, n_axes, xd, od, kshape, out_shape = plan
        out = torch.empty(kshape, dtype=torch.float32, device=self.device)
        xd.data = x.data_ptr()
        od.data = out.data_ptr()
        lib = self.lib
        lib.bt_set_stream(_raw_stream(self._index))   # always BT_OK
        rc = lib.bt_reduce(kind, xd, axes, n_axes, 1, od)
        if rc:
            check(rc, "bt_reduce")
        self.launches += 1
        return out.reshape(out_shape)

    def _concat_plan(self, vals, axis):
        """The cached launches of a Concat whose inputs need no widening:
        the result's layout and, per non-empty input, the copy into its
        slice (descriptors prepared once).  None for every other case, which
        concat handles (and where it raises, it raises there)."""
        if any(v.dtype == torch.float16 for v in vals):
            return None
        nd = vals[0].dim()
        axis = int(axis)
        if not -nd <= axis < nd:
            return None
        axis %= nd
        for v in vals[1:]:
            if v.dim() != nd or any(v.shape[d] != vals[0].shape[d] for d in range(nd) if d != axis):
                return None
        dt = np.result_type(*[np_dtype(v) for v in vals])
        shape = [int(s) for s in vals[0].shape]
        shape[axis] = sum(int(v.shape[axis]) for v in vals)
        strides, acc = [], 1
        for d in reversed(shape):
            strides.append(acc)
            acc *= d
        strides = tuple(reversed(strides))
        item = np.dtype(dt).itemsize
        copies, off = [], 0
        for i, v in enumerate(vals):
            n = int(v.shape[axis])
            if n:
                part = list(shape)
                part[axis] = n
                cdt = self._copy_compute(np.result_type(np_dtype(v), dt))
                copies.append((i, (_lib.BtTensor * 1)(tensor_desc(v)), make_tensor(0, np.dtype(dt), part, strides),
                               _lib.BtEwAttrs(_lib.NP_TO_BT[np.dtype(cdt)], 0.0), off * strides[axis] * item))
            off += n
        return tuple(shape), NP_TO_TORCH[np.dtype(dt)], copies

    def _run_concat_plan(self, plan, vals):
        shape, tdt, copies = plan
        out = torch.empty(shape, dtype=tdt, device=self.device)
        if copies:
            base = out.data_ptr()
            lib = self.lib
            lib.bt_set_stream(_raw_stream(self._index))   # always BT_OK
            for i, descs, od, attrs, offb in copies:
                descs[0].data = vals[i].data_ptr()
                od.data = base + offb
                rc = lib.bt_elementwise(OP["IDENTITY"], 1, descs, od, attrs)
                if rc:
                    check(rc, "bt_elementwise(concat)")
                self.launches += 1
        return out

    def _mean_from_sum(self, s, count):
        # np.mean divides the float32 sum by an intp count: float64 division,
        # rounded to float32.
        c = self._scalar(count, np.int64)
        return self.elementwise("DIV", [s, c], s.shape, np.float32, np.float64)

    def softmax(self, x, mask, axis):
        if mask is None and not x.is_contiguous():
            # numpy sums along the axis pairwise when it is innermost in
            # memory: run the kernel on the physical order, view it back
            nd = x.dim()
            if axis < -nd or axis >= max(nd, 1):
                raise np.exceptions.AxisError(axis, nd)
            phys, order = self._physical(x)
            if order[-1] != axis % nd:
                raise NotImplementedError("Softmax along an axis that is not innermost in memory is not on the GPU path")
            return self.softmax(self._contig(phys), None, -1).permute(_inverse(order))
        x = self._contig(x)
        out = self._empty(x.shape, np.float32)
        if out.numel() == 0:
            return out
        nd = x.dim()
        if axis < -nd or axis >= max(nd, 1):
            raise np.exceptions.AxisError(axis, nd)
        self._stream()
        check(self.lib.bt_softmax(tensor_desc(x), tensor_desc(mask) if mask is not None else None, axis,
                                  tensor_desc(out)), "bt_softmax")
        self.launches += 1
        return out

    def layernorm(self, x, skip, bias, gamma, beta, axis, eps):
        if any(t is not None and not t.is_contiguous() for t in (x, skip, bias)):
            return self._layernorm_view(x, skip, bias, gamma, beta, axis, eps)
        x = self._contig(self._as_f32(x))
        if skip is not None:
            skip = self._contig(self._as_f32(skip))
            if tuple(skip.shape) != tuple(x.shape):
                raise NotImplementedError("SkipLayerNormalization with a broadcast skip is not on the GPU path")
        if bias is not None:
            bias = self._contig(self._as_f32(bias))
        nd = x.dim()
        ax = axis % nd
        trailing = tuple(x.shape[ax:])
        gamma = self._fit_param(gamma, trailing)
        beta = self._fit_param(beta, trailing) if beta is not None else None
        if bias is not None:
            bias = self._fit_param(bias, trailing)
        out = self._empty(x.shape, np.float32)
        if out.numel() == 0:
            return out
        self._stream()
        check(self.lib.bt_layernorm(tensor_desc(x), tensor_desc(skip) if skip is not None else None,
                                    tensor_desc(bias) if bias is not None else None, tensor_desc(gamma),
                                    tensor_desc(beta) if beta is not None else None, axis,
                                    float(np.float32(eps)), tensor_desc(out)), "bt_layernorm")
        self.launches += 1
        return out

    def _layernorm_view(self, x, skip, bias, gamma, beta, axis, eps):
        """(Skip)LayerNormalization of views, in the order numpy walks them.
        SkipLayerNormalization first forms s = x + skip (+ bias) as the
        reference does (ref_runtime.py:604-609).  When the normalised axes
        are innermost in memory, in order, the fused kernel runs on the
        physical tensor (numpy's row sums are pairwise there too); otherwise
        op_layernorm (ref_runtime.py:276-285) runs one numpy op at a time on
        the physical order, where numpy's sums run slice after slice."""
        f32 = np.float32
        x = self._as_f32(x)
        if skip is not None:
            skip = self._as_f32(skip)
            x = self.elementwise("ADD", [x, skip], np.broadcast_shapes(tuple(x.shape), tuple(skip.shape)), f32, f32)
            if bias is not None:
                bias = self._as_f32(bias)
                x = self.elementwise("ADD", [x, bias], np.broadcast_shapes(tuple(x.shape), tuple(bias.shape)), f32, f32)
        nd = x.dim()
        ax = axis % nd
        tail = list(range(ax, nd))
        phys, order = self._physical(x)
        if not phys.is_contiguous():
            raise NotImplementedError("LayerNormalization of a strided view is not on the GPU path")
        inv = _inverse(order)
        if order[nd - len(tail):] == tail:
            return self.layernorm(phys, None, None, gamma, beta, -len(tail), eps).permute(inv)
        trailing = tuple(x.shape[ax:])
        paxes = sorted(order.index(a) for a in tail)
        mu = self._reduce("ReduceMean", phys, paxes, {"keepdims": 1})
        d = self.elementwise("SUB", [phys, mu], phys.shape, f32, f32)
        var = self._reduce("ReduceMean", self.elementwise("MUL", [d, d], d.shape, f32, f32), paxes, {"keepdims": 1})
        e = self._scalar(np.float32(eps), np.float32)
        sd = self.elementwise("SQRT", [self.elementwise("ADD", [var, e], var.shape, f32, f32)], var.shape, f32, f32)
        y = self.elementwise("DIV", [d, sd], d.shape, f32, f32)

        def param(p):
            p = self._contig(self._as_f32(self._fit_param(p, trailing)))
            return p.view((1,) * ax + trailing).permute(order)

        y = self.elementwise("MUL", [y, param(gamma)], y.shape, f32, f32)
        if beta is not None:
            y = self.elementwise("ADD", [y, param(beta)], y.shape, f32, f32)
        return y.permute(inv)

    # ---- fused entry points (beyond the one-op-per-node table) ---------------------
    def chain(self, prog, inputs, out_shape=None):
        """Runs a bt_chain register program (float32, see bt_fused_chain)
        over CUDA tensors broadcast to out_shape (default: their broadcast
        shape); one launch, a dense float32 result."""
        if out_shape is None:
            out_shape = np.broadcast_shapes(*[tuple(t.shape) for t in inputs])
        out = self._empty(out_shape, np.float32)
        if out.numel() == 0:
            return out
        descs = (_lib.BtTensor * len(inputs))(*[tensor_desc(t) for t in inputs])
        self._stream()
        check(self.lib.bt_fused_chain(ctypes.byref(prog), descs, tensor_desc(out)), "bt_fused_chain")
        self.launches += 1
        return out

    def dequant_mul(self, q, scale, zero_point, gain):
        """Mul(DequantizeLinear(q, scale, zero_point), gain): the c4 weight
        path, rounded like the two reference ops (ref_runtime.py:631-636
        then :450-451).  One pass reading the int8 weights (bt_fused_chain)
        where the two ops compute in float32: q and zero point int8 / uint8,
        scale and gain float32 / float16; otherwise the two ops one after
        the other."""
        from . import chains
        g = chains.FusedGroup(0, 1, "dequant_mul", [], "", quant=(0, 3))
        ins = [q, scale, gain] + ([zero_point] if zero_point is not None else [])
        if g.inputs_ok([np_dtype(t) for t in ins]):
            return self.chain(chains.dequant_mul_program(zero_point is not None), ins)
        ins = [q, scale] + ([zero_point] if zero_point is not None else [])
        shape = np.broadcast_shapes(*[tuple(t.shape) for t in ins])
        d = self.elementwise("DEQUANT", ins, shape, np.float32, np.float32)
        shape2 = np.broadcast_shapes(shape, tuple(gain.shape))
        return self.elementwise("MUL", [d, self._as_f32(gain)], shape2, np.float32, np.float32)

    def dequantize(self, q, scale, zero_point=None):
        """DequantizeLinear (ref_runtime.py:631-636): (q - zero_point) *
        scale in float32.  8-bit q and zero point with a float32 / float16
        scale run as one chain pass (bt_fused_chain, the 8-bit values read
        packed); other dtypes on the element-wise DEQUANT op."""
        from . import chains
        ins = [q, scale] + ([zero_point] if zero_point is not None else [])
        g = chains.FusedGroup(0, 0, "dequant", [], "", quant=(0, 2))
        if g.inputs_ok([np_dtype(t) for t in ins]):
            return self.chain(chains.dequant_program(zero_point is not None), ins)
        shape = np.broadcast_shapes(*[tuple(t.shape) for t in ins])
        return self.elementwise("DEQUANT", ins, shape, np.float32, np.float32)

    def snake(self, x, alpha, inv_alpha, power=None):
        """Snake x + inv_alpha * sin(alpha * x) ** power as the graph spells
        it (Mul, Sin, Pow, Mul, Add; power defaults to the graph's float16
        2.0), in one pass (bt_fused_chain); float32 / float16 inputs."""
        from . import chains
        if power is None:
            power = self.to_device(_F16_TWO)
        return self.chain(chains.snake_program(), [x, alpha, power, inv_alpha])

    def adain_snake(self, srcs, gain, shift, eps, alpha=None, inv_alpha=None, res=None, outs=None,
                    ranges=None):
        """Row-fused AdaIN1d (+ Snake) of [B, C, T] float32 tensors (see
        bt_adain_snake in bt_ops.h).  gain / shift are [B, C] float32 views
        with unit channel stride; alpha / inv_alpha [C] (fp16 or fp32).
        ranges: an int32 device tensor of 4 words per output; when given,
        bt_adain_snake_range also records each output's value range there
        for dynamic_quantize(out, range=ranges[k])."""
        x0 = srcs[0]
        B, Cc, T = x0.shape
        a = _lib.BtAdainArgs()
        a.rows, a.cols, a.channels = B * Cc, T, Cc
        a.n_src = len(srcs)
        for i, s in enumerate(srcs):
            assert s.is_contiguous() and s.dtype == torch.float32 and tuple(s.shape) == (B, Cc, T)
            a.src[i] = s.data_ptr()
        a.res = res.data_ptr() if res is not None else None
        a.eps = float(np.float32(eps))
        gains = gain if isinstance(gain, (list, tuple)) else [gain]
        shifts = shift if isinstance(shift, (list, tuple)) else [shift]
        alphas = alpha if isinstance(alpha, (list, tuple)) else [alpha] * len(gains)
        invs = inv_alpha if isinstance(inv_alpha, (list, tuple)) else [inv_alpha] * len(gains)
        a.n_out = len(gains)
        a.gain_stride = gains[0].stride(0)
        a.shift_stride = shifts[0].stride(0)
        a.alpha_dtype = _lib.BT_F16
        if outs is None:
            outs = [self._empty((B, Cc, T), np.float32) for _ in gains]
        for i in range(len(gains)):
            assert gains[i].stride(-1) == 1 and shifts[i].stride(-1) == 1
            assert gains[i].stride(0) == a.gain_stride and shifts[i].stride(0) == a.shift_stride
            a.gain[i] = gains[i].data_ptr()
            a.shift[i] = shifts[i].data_ptr()
            if alphas[i] is not None:
                a.alpha_dtype = _lib.NP_TO_BT[np_dtype(alphas[i])]
                a.alpha[i] = alphas[i].data_ptr()
                a.inv_alpha[i] = invs[i].data_ptr()
            a.out[i] = outs[i].data_ptr()
        self._stream()
        if ranges is None:
            check(self.lib.bt_adain_snake(ctypes.byref(a)), "bt_adain_snake")
        else:
            assert ranges.is_contiguous() and ranges.numel() >= 4 * len(gains) and ranges.element_size() == 4
            check(self.lib.bt_adain_snake_range(ctypes.byref(a), ranges.data_ptr()), "bt_adain_snake_range")
        self.launches += 1
        return outs

    def range_records(self, n):
        """Device storage for n range records (bt_adain_snake_range)."""
        return torch.empty((n, 4), dtype=torch.int32, device=self.device)

    def _fit_param(self, p, trailing):
        """gamma/beta as a contiguous run over the normalised axes (broadcast
        materialised by a kernel when needed)."""
        if tuple(p.shape) == trailing and p.is_contiguous():
            return p
        shape = np.broadcast_shapes(tuple(p.shape), trailing)
        if shape != trailing:
            raise ValueError(f"parameter of shape {tuple(p.shape)} does not broadcast to {trailing}")
        dt = np_dtype(p)
        return self.elementwise("IDENTITY", [p], trailing, dt if dt.kind == "f" else np.float32,
                                np.float64)


def _axis_blocks(axes, shape):
    """Groups sorted axes into runs that are contiguous once size-1 axes are ignored."""
    blocks = []
    for a in axes:
        if blocks:
            prev = blocks[-1][-1]
            if all(shape[i] == 1 for i in range(prev + 1, a)):
                blocks[-1].append(a)
                continue
        blocks.append([a])
    return blocks


def _host_ints(v):
    if v is None:
        return []
    if isinstance(v, torch.Tensor):
        v = v.detach().cpu().numpy()
    return np.asarray(v).reshape(-1).tolist()


def _layout(t):
    """(shape, strides in bytes) of a torch tensor or numpy array."""
    if isinstance(t, torch.Tensor):
        return tuple(t.shape), tuple(st * t.element_size() for st in t.stride())
    a = np.asarray(t)
    return a.shape, a.strides


def _k_order(operands, out_shape):
    """The axis order numpy's iterator picks for order 'K' over these operands
    broadcast to out_shape (nditer's best-axis-ordering pass): a stable
    insertion sort of the axes by stride, smallest first, in which each
    operand with nonzero strides on both axes of a pair votes and C order
    wins conflicts; broadcast and size-1 axes have stride 0 and do not vote.
    Returns logical axes, outermost first (C order is range(nd))."""
    nd = len(out_shape)
    st = []
    for t in operands:
        shape, strides = _layout(t)
        pad = nd - len(shape)
        st.append([0 if i < pad or shape[i - pad] == 1 or out_shape[i] == 1 else strides[i - pad]
                   for i in range(nd)])
    perm = list(range(nd))[::-1]          # iterator position 0 = innermost
    for i0 in range(1, nd):
        ax0, ipos = perm[i0], i0
        for i1 in range(i0 - 1, -1, -1):
            ax1 = perm[i1]
            ambig, swap = True, False
            for s_ in st:
                if s_[ax0] != 0 and s_[ax1] != 0:
                    if abs(s_[ax1]) <= abs(s_[ax0]):
                        swap = False
                    elif ambig:
                        swap = True
                    ambig = False
            if not ambig:
                if swap:
                    ipos = i1
                else:
                    break
        if ipos != i0:
            perm.insert(ipos, perm.pop(i0))
    return perm[::-1]


def _inverse(perm):
    inv = [0] * len(perm)
    for i, p in enumerate(perm):
        inv[p] = i
    return inv


def _is_identity(perm):
    return all(i == p for i, p in enumerate(perm))


ctypes_i64 = ctypes.c_int64


class CapturedNodes:
    """A node list recorded once as a CUDA graph and replayed.

    The list runs ``warmup`` times on a side stream first (numpy constants
    are uploaded and per-stream scratch allocated there), then once more
    under graph capture on the same stream.  ``env`` after capture holds the
    graph's tensors: write new input values into them in place
    (``cap.env[name].copy_(...)``) and ``replay()``; outputs are overwritten
    in place on every replay.  Every node must keep its work on the device:
    a node that needs a value on the host (a shape given as a CUDA tensor,
    for instance) makes the capture fail."""

    def __init__(self, rt, nodes, env, warmup=1):
        self.rt = rt
        self.stream = torch.cuda.Stream(rt.device)
        self.stream.wait_stream(torch.cuda.current_stream(rt.device))
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                rt.run_nodes(nodes, dict(env))
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        self.env = dict(env)
        with torch.cuda.graph(self.graph, stream=self.stream):
            rt.run_nodes(nodes, self.env)

    def replay(self):
        """Runs the recorded launches on the current stream; returns env."""
        self.graph.replay()
        return self.env

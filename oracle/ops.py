"""numpy restatement of the reference op table for the hot path (test oracle).

Reference: ``tools/ref_runtime.py`` of studio-ransom/best-tts-godot.  The
op-table call is ``dispatch(op, node_input, node_output, at, env)``
(ref_runtime.py:428): ``env`` maps tensor names to arrays, an empty input name
means "absent" (ref_runtime.py:436-439), single-output ops store their result
in ``env[node_output[0]]`` (ref_runtime.py:668) and multi-output ops store each
named output themselves (ref_runtime.py:544-547).  Unknown ops raise
``NotImplementedError`` (ref_runtime.py:665-666).

This module is test infrastructure; see the package docstring.
"""
import numpy as np

# ONNX TensorProto element type -> numpy dtype (ref_runtime.py:24-28).
ONNX_TO_NUMPY = {
    1: np.float32, 2: np.uint8, 3: np.int8, 4: np.uint16, 5: np.int16,
    6: np.int32, 7: np.int64, 9: np.bool_, 10: np.float16, 11: np.float64,
    12: np.uint32, 13: np.uint64,
}


def upcast(a):
    """fp16 storage is widened to fp32 before any arithmetic (ref_runtime.py:49-51)."""
    return a.astype(np.float32) if a.dtype == np.float16 else a


def _is_int(a):
    return np.issubdtype(a.dtype, np.integer)


def _div(a, b):
    # ref_runtime.py:452-455: integer / integer is floor division, anything
    # else is true division on the (fp16-widened) operands.
    a, b = upcast(a), upcast(b)
    if _is_int(a) and _is_int(b):
        return np.floor_divide(a, b)
    return np.true_divide(a, b)


def _sigmoid(v):
    # ref_runtime.py:470-471 spells the logistic as 1 / (1 + exp(-v)) with
    # Python-float constants, so every step rounds in the operand's type.
    return 1.0 / (1.0 + np.exp(-v))


def _leaky(v, at):
    # ref_runtime.py:476-479: slope defaults to 0.01 and is applied as float32.
    slope = np.float32(at.get("alpha", 0.01))
    return np.where(v < 0, v * slope, v)


def _softmax(x, axis):
    # ref_runtime.py:269-273: shift by the max along the axis, exponentiate,
    # divide by the sum along the same axis.
    x = upcast(x).astype(np.float32)
    shifted = x - x.max(axis=axis, keepdims=True)
    num = np.exp(shifted)
    return num / num.sum(axis=axis, keepdims=True)


def _layernorm(x, gamma, beta, axis, eps):
    # ref_runtime.py:276-285: two-pass mean / centred variance over every axis
    # from `axis` to the last, divide by sqrt(var + eps), scale, optional shift.
    x = upcast(x).astype(np.float32)
    first = axis if axis >= 0 else x.ndim + axis
    red = tuple(range(first, x.ndim))
    mu = x.mean(axis=red, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=red, keepdims=True)
    y = (x - mu) / np.sqrt(var + eps)
    y = y * upcast(gamma).astype(np.float32)
    if beta is not None:
        y = y + upcast(beta).astype(np.float32)
    return y


def _fast_gelu(x, bias):
    # ref_runtime.py:288-293: optional bias add, then the tanh form of GELU.
    x = upcast(x).astype(np.float32)
    if bias is not None:
        x = x + upcast(bias).astype(np.float32)
    k = np.float32(0.7978845608028654)
    return 0.5 * x * (1.0 + np.tanh(k * (x + 0.044715 * x * x * x)))


def _reduce(op, x, axes_in, at):
    # ref_runtime.py:589-598: axes come from input 1 (opset 18) or the `axes`
    # attribute; no axes means "all axes" unless noop_with_empty_axes is set,
    # in which case the input passes through unchanged.
    v = upcast(x)
    keep = bool(at.get("keepdims", 1))
    if axes_in is None:
        axes = None if not at.get("noop_with_empty_axes", 0) else ()
    else:
        axes = tuple(int(a) for a in np.asarray(axes_in).reshape(-1))
    if axes == ():
        return v
    fn = np.mean if op == "ReduceMean" else np.sum
    return fn(v, axis=axes, keepdims=keep)


def _cast(x, at):
    # ref_runtime.py:572-578: a cast to float16 is elided (the result stays
    # fp32, as ORT's CPU provider does); any other target is a numpy astype of
    # the fp16-widened input.
    target = ONNX_TO_NUMPY[at["to"]]
    if target == np.float16:
        target = np.float32
    return upcast(x).astype(target)


def _dequantize(q, scale, zero_point):
    # ref_runtime.py:631-636: widen the quantized values to fp32, subtract the
    # zero point (also widened) when present, multiply by the scale.  Plain
    # numpy broadcasting; the ONNX `axis` attribute is not consulted.
    v = q.astype(np.float32)
    if zero_point is not None:
        v = v - np.asarray(zero_point).astype(np.float32)
    return v * upcast(scale).astype(np.float32)


def _dynamic_quantize(x):
    # ref_runtime.py:106-116 (dispatched at :625-630).  The float32 range is
    # widened to Python floats and always includes 0; scale and zero point
    # are Python-float (double) arithmetic; the element quotient x / scale
    # divides a float32 array by a Python float, which numpy 2 evaluates in
    # float32, and adding the float64 zero point promotes to float64 before
    # the clip and the uint8 cast.  Three outputs: y, scale as float32, zero
    # point as uint8.
    x = upcast(x).astype(np.float32)
    lo = min(0.0, float(x.min()))
    hi = max(0.0, float(x.max()))
    scale = (hi - lo) / 255.0
    if scale == 0:
        scale = 1.0
    zp = np.clip(np.rint(0.0 - lo / scale), 0.0, 255.0)
    q = np.rint(x / scale)                   # float32
    y = np.clip(q + zp, 0.0, 255.0).astype(np.uint8)
    return y, np.float32(scale), np.uint8(zp)


def _slice(x, starts, ends, axes, steps):
    # ref_runtime.py:307-325 (dispatched at :548-549): each (start, end) is
    # made non-negative by adding the extent, then clamped to [0, dim] for a
    # positive step and to [-1, dim - 1] for a negative one, and handed to a
    # Python slice.  A clamped end of -1 therefore means "the last element"
    # to numpy -- so a full reversal comes out empty, as in the reference.
    starts = np.asarray(starts).reshape(-1)
    ends = np.asarray(ends).reshape(-1)
    axes = list(range(len(starts))) if axes is None else np.asarray(axes).reshape(-1)
    steps = [1] * len(starts) if steps is None else np.asarray(steps).reshape(-1)
    index = [slice(None)] * x.ndim
    for s, e, a, st in zip(starts, ends, axes, steps):
        a, s, e, st = int(a) % x.ndim, int(s), int(e), int(st)
        dim = x.shape[a]
        lo, hi = (0, dim) if st > 0 else (-1, dim - 1)
        s = min(max(s + dim if s < 0 else s, lo), hi)
        e = min(max(e + dim if e < 0 else e, lo), hi)
        index[a] = slice(s, e, st)
    return x[tuple(index)]


def _concat(vals, axis):
    # ref_runtime.py:531-535: any fp16 input widens every input to fp32
    if any(v.dtype == np.float16 for v in vals):
        vals = [upcast(v) for v in vals]
    return np.concatenate(vals, axis=axis)


class OracleRuntime:
    """Op-table interpreter with the reference's ``dispatch`` signature."""

    # Ops the oracle restates.  Everything else raises NotImplementedError,
    # exactly as the reference does for an op it does not know.
    UNARY = {
        "Sqrt": np.sqrt, "Exp": np.exp, "Sin": np.sin, "Cos": np.cos,
        "Atan": np.arctan, "Tanh": np.tanh, "Sigmoid": _sigmoid,
        "Floor": np.floor, "Round": np.rint,
    }

    def dispatch(self, op, node_input, node_output, at, env):
        def arg(i, default=None):
            if i >= len(node_input) or not node_input[i]:
                return default
            return env[node_input[i]]

        x, y = arg(0), arg(1)

        if op in ("Add", "Sub", "Mul"):                       # ref :446-451
            f = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply}[op]
            out = f(upcast(x), upcast(y))
        elif op == "Div":                                     # ref :452-455
            out = _div(x, y)
        elif op == "Pow":                                     # ref :456-457
            out = np.power(upcast(x), upcast(y))
        elif op in self.UNARY:                                # ref :458-475
            out = self.UNARY[op](upcast(x))
        elif op == "LeakyRelu":                               # ref :476-479
            out = _leaky(upcast(x), at)
        elif op == "Clip":                                    # ref :480-486
            out = upcast(x)
            lo, hi = arg(1), arg(2)
            if lo is not None:
                out = np.maximum(out, upcast(lo))
            if hi is not None:
                out = np.minimum(out, upcast(hi))
        elif op == "Erf":                                     # ref :487-489
            from scipy.special import erf
            out = erf(upcast(x))
        elif op == "Equal":                                   # ref :492-493
            out = np.equal(x, y)
        elif op in ("Greater", "Less", "GreaterOrEqual"):     # ref :494-499
            f = {"Greater": np.greater, "Less": np.less,
                 "GreaterOrEqual": np.greater_equal}[op]
            out = f(upcast(x), upcast(y))
        elif op == "And":                                     # ref :500-501
            out = np.logical_and(x, y)
        elif op == "Where":                                   # ref :502-503
            out = np.where(x, y, arg(2))
        elif op == "Cast":                                    # ref :572-578
            out = _cast(x, at)
        elif op in ("ReduceMean", "ReduceSum"):               # ref :589-598
            axes = arg(1) if len(node_input) > 1 else at.get("axes")
            out = _reduce(op, x, axes, at)
        elif op == "Softmax":                                 # ref :599-600
            out = _softmax(x, at.get("axis", -1))
        elif op == "LayerNormalization":                      # ref :601-603
            out = _layernorm(x, y, arg(2), at.get("axis", -1),
                             at.get("epsilon", 1e-5))
        elif op == "SkipLayerNormalization":                  # ref :604-609
            s = upcast(x) + upcast(y)
            if arg(4) is not None:
                s = s + upcast(arg(4))
            out = _layernorm(s, arg(2), arg(3), -1, at.get("epsilon", 1e-12))
        elif op == "FastGelu":                                # ref :610-611
            out = _fast_gelu(x, y)
        elif op == "DequantizeLinear":                        # ref :631-636
            out = _dequantize(x, y, arg(2))
        elif op == "DynamicQuantizeLinear":                   # ref :625-630
            for name, v in zip(node_output, _dynamic_quantize(x)):
                if name:
                    env[name] = v
            return
        # -- view ops that the decoder-stage stream threads between the math
        elif op == "Split":                                   # ref :536-547
            axis = at.get("axis", 0)
            sizes = arg(1)
            if sizes is None:
                parts = np.array_split(x, len(node_output), axis=axis)
            else:
                cuts = np.cumsum([int(s) for s in sizes])[:-1]
                parts = np.split(x, cuts, axis=axis)
            for name, p in zip(node_output, parts):
                if name:
                    env[name] = p
            return
        elif op == "Transpose":                               # ref :517-518
            out = np.transpose(x, at.get("perm"))
        elif op == "Concat":                                  # ref :531-535
            out = _concat([env[i] for i in node_input if i], at["axis"])
        elif op == "Slice":                                   # ref :548-549
            out = _slice(x, arg(1), arg(2), arg(3), arg(4))
        elif op == "Expand":                                  # ref :553-555
            shape = np.broadcast_shapes(x.shape, tuple(int(v) for v in np.asarray(y).reshape(-1)))
            out = np.broadcast_to(x, shape).copy()
        elif op == "Reshape":                                 # ref :511-516
            shape = [int(s) for s in np.asarray(y).reshape(-1)]
            if not at.get("allowzero", 0):
                shape = [x.shape[i] if s == 0 else s for i, s in enumerate(shape)]
            out = x.reshape(shape)
        elif op == "Unsqueeze":                               # ref :519-523
            axes = arg(1) if len(node_input) > 1 else at.get("axes")
            out = x
            for a in sorted(int(v) for v in np.asarray(axes).reshape(-1)):
                out = np.expand_dims(out, a)
        elif op == "Squeeze":                                 # ref :524-530
            axes = arg(1) if len(node_input) > 1 else at.get("axes")
            if axes is None:
                out = np.squeeze(x)
            else:
                out = np.squeeze(x, tuple(int(v) for v in np.asarray(axes).reshape(-1)))
        else:
            raise NotImplementedError(f"{op} ({node_output})")
        env[node_output[0]] = out

    def run_nodes(self, nodes, env):
        """Execute a list of ``(op, inputs, outputs, attrs)`` nodes in order,
        wrapping failures the way the reference's drivers do
        (ref_runtime.py:398-403, kpk_runtime.py:77-80)."""
        for op, ins, outs, at in nodes:
            try:
                self.dispatch(op, list(ins), list(outs), dict(at or {}), env)
            except Exception as exc:
                raise RuntimeError(f"{op} {list(outs)} failed: {exc}") from exc
        return env


def run_nodes_streaming(rt, nodes, env, keep=()):
    """Runs nodes like ``OracleRuntime.run_nodes`` but drops every tensor
    after its last use (names in ``keep`` survive).  The arithmetic is
    unchanged; this only bounds host memory for long streams (the CPU
    baseline of the 24001-sample decoder stage)."""
    last = {}
    for i, (op, ins, outs, at) in enumerate(nodes):
        for n in ins:
            if n:
                last[n] = i
    keep = set(keep)
    for i, (op, ins, outs, at) in enumerate(nodes):
        rt.dispatch(op, list(ins), list(outs), dict(at or {}), env)
        for n in ins:
            if n and last.get(n) == i and n not in keep and n in env:
                del env[n]
    return env

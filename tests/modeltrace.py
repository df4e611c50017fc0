"""The real-model node trace (tests/golden/model_trace.*): loading, attribute
decoding, synthetic inputs for a node signature, and the per-op tolerance.

The packed model stores tensor-valued attributes as ``{"__t": code, "v":
values, "s": shape}`` with the dtype codes of kpk_runtime.py:20-23; they are
decoded the way PackedModel.run decodes them (kpk_runtime.py:65-69)."""
import json
import os

import numpy as np

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KPK_DTYPES = {0: np.float32, 1: np.int8, 2: np.uint8, 3: np.int32, 4: np.int64, 5: np.bool_, 6: np.float16}


def load_meta():
    with open(os.path.join(GOLD, "model_trace.json")) as f:
        return json.load(f)


def load_arrays():
    with np.load(os.path.join(GOLD, "model_trace.npz")) as z:
        return {k: z[k] for k in z.files}


def attrs(raw):
    out = {}
    for k, v in (raw or {}).items():
        if isinstance(v, dict) and "__t" in v:
            v = np.array(v["v"], dtype=KPK_DTYPES[v["__t"]]).reshape(v["s"])
        out[k] = v
    return out


def sampled_env(node, arrays):
    """The reference's own input arrays of a sampled node."""
    pos = node["pos"]
    return {name: np.array(arrays[f"n{pos}/in{j}"], copy=True)
            for j, name in enumerate(node["inputs"]) if name}


def sampled_outputs(node, arrays):
    pos = node["pos"]
    return {name: arrays[f"n{pos}/out{j}"] for j, name in enumerate(node["outputs"])
            if name and f"n{pos}/out{j}" in arrays}


def synthetic_node(sig, seed):
    """A node with the signature's op, attributes, dtypes and shapes: inputs
    of at most 64 elements keep their recorded values (axes, shapes, split
    sizes, exponents, constants), larger ones are seeded random data."""
    rng = np.random.default_rng(seed)
    names, env = [], {}
    for j, s in enumerate(sig["inputs"]):
        if s is None:
            names.append("")
            continue
        name = f"x{j}"
        names.append(name)
        dt, shape = np.dtype(s["dtype"]), tuple(s["shape"])
        if "values" in s:
            a = np.array(s["values"], dtype=dt).reshape(shape)
        elif dt.kind == "f":
            a = (rng.standard_normal(shape) * 2).astype(dt)
        elif dt.kind == "b":
            a = rng.random(shape) < 0.5
        elif dt.kind in "iu":
            info = np.iinfo(dt)
            lo, hi = max(int(info.min), -1000), min(int(info.max), 1000)
            a = rng.integers(lo, hi + 1, shape).astype(dt)
        else:
            raise TypeError(dt)
        env[name] = a
    outs = [f"y{i}" for i in range(sig["n_out"])]
    return (sig["op"], names, outs, attrs(sig["attrs"])), env


def tolerance(op, ins, want):
    """0 = bit-exact, an int = ulps, "close" = FastGelu's relative bound.
    Tanh / Atan / Erf and Pow with exponents other than 2 come from numpy's
    vendor routines (<= 2 ulp); float64 results of integer inputs likewise;
    Sin / Cos beyond numpy's SIMD range from the C library (<= 1 ulp)."""
    if op == "FastGelu":
        return "close"
    if op in ("Tanh", "Atan", "Erf"):
        return 2
    if op == "Pow":
        e = np.asarray(ins[1]) if len(ins) > 1 else None
        return 0 if e is not None and e.size == 1 and float(e.reshape(-1)[0]) == 2.0 else 2
    if want.dtype == np.float64 and op != "Sqrt" and any(np.asarray(a).dtype.kind in "iub" for a in ins):
        return 2
    if op in ("Sin", "Cos"):
        lim = 117435.992 if op == "Sin" else 71476.0625
        x = np.asarray(ins[0], np.float64)
        return 1 if np.any(~(np.abs(x) <= lim)) else 0
    return 0


def compare(got, want, tol, what):
    from parity import assert_same, assert_ulp
    if tol == "close":
        assert got.dtype == want.dtype and got.shape == want.shape, what
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6, err_msg=what)
    elif tol == 0:
        assert_same(got, want, what)
    else:
        assert_ulp(got, want, tol, what)

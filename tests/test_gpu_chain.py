"""Fused elementwise chains on the GPU (bt_fused_chain) against the oracle's
op-by-op chain: the c4 weight path Mul(DequantizeLinear(W), gain) in one
launch at both BASELINE shapes, standalone Snake, Add -> Sigmoid, Add ->
LeakyRelu, Mul -> Add, each over row-broadcast, same-shape, float16,
misaligned and strided inputs; random programs through the interpreter; and
the node-list fusion pass of BtRuntime.run_nodes.  Bit-exact wherever every
op of the chain is (BASELINE: dequant and arithmetic bit-exact; the
transcendentals here are numpy's own algorithms, also bit-exact); tanh,
atan, erf and general powers within 2 ulp."""
import warnings

import numpy as np
import pytest
import torch

from oracle import OracleRuntime
from parity import assert_same, assert_ulp

pytestmark = pytest.mark.gpu


def dev(a):
    a = np.asarray(a)
    return torch.from_numpy(np.ascontiguousarray(a).reshape(a.shape)).cuda()


def host(t):
    return t.cpu().numpy()


def oracle_nodes(nodes, env, out):
    env = dict(env)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, env)
    return env[out]


@pytest.fixture(scope="module")
def rt(gpu_runtime):
    return gpu_runtime


# ---- c4: DequantizeLinear then the gain Mul -------------------------------------------
@pytest.mark.parametrize("shape", [(512, 512, 3), (256, 256, 7)])
@pytest.mark.parametrize("zp_kind", ["none", "zero", "nonzero"])
def test_c4_dequant_gain_one_launch(rt, shape, zp_kind):
    from bt_b200 import configs
    c = configs.c4_dequant(shape=shape)
    C = shape[0]
    rng = np.random.default_rng(3)
    zp = {"none": None, "zero": np.zeros((C, 1, 1), np.int8),
          "nonzero": rng.integers(-20, 21, (C, 1, 1)).astype(np.int8)}[zp_kind]
    env = {"W": c["W"], "scale": c["scale"], "gain": c["gain"]}
    ins = ["W", "scale"]
    if zp is not None:
        env["zp"] = zp
        ins.append("zp")
    want = oracle_nodes([("DequantizeLinear", ins, ["d"], {}), ("Mul", ["d", "gain"], ["y"], {})], env, "y")
    l0 = rt.launches
    got = rt.dequant_mul(dev(c["W"]), dev(c["scale"]), dev(zp) if zp is not None else None, dev(c["gain"]))
    assert rt.launches - l0 == 1
    assert_same(host(got), want, f"dequant x gain {shape} zp={zp_kind}")


def test_dequant_gain_variants(rt):
    """float16 gain and scale, a per-tensor scale, a misaligned weight view
    (the scalar path) and uint8 weights with a zero point."""
    rng = np.random.default_rng(4)
    W = rng.integers(-127, 128, (96, 40, 5)).astype(np.int8)
    s16 = rng.uniform(1e-3, 2e-2, (96, 1, 1)).astype(np.float16)
    g16 = rng.uniform(0.5, 1.5, (96, 1, 1)).astype(np.float16)
    cases = [
        ({"W": W, "s": s16, "g": g16}, ["W", "s"]),
        ({"W": W, "s": np.float32(0.013).reshape(()), "g": rng.uniform(0.5, 1.5, (96, 1, 1)).astype(np.float32)},
         ["W", "s"]),
        ({"W": rng.integers(0, 256, (96, 40, 5)).astype(np.uint8), "s": s16, "g": g16,
          "z": rng.integers(100, 156, (96, 1, 1)).astype(np.uint8)}, ["W", "s", "z"]),
    ]
    for env, ins in cases:
        want = oracle_nodes([("DequantizeLinear", ins, ["d"], {}), ("Mul", ["d", "g"], ["y"], {})], env, "y")
        got = rt.dequant_mul(dev(env["W"]), dev(env["s"]), dev(env["z"]) if "z" in env else None, dev(env["g"]))
        assert_same(host(got), want, f"dequant x gain {[env[k].dtype for k in ins]}")
    # misaligned: the weights start one byte into a buffer
    base = dev(np.concatenate([np.zeros(1, np.int8), W.reshape(-1)]))
    Wv = base[1:].view(96, 40, 5)
    want = oracle_nodes([("DequantizeLinear", ["W", "s"], ["d"], {}), ("Mul", ["d", "g"], ["y"], {})],
                        {"W": W, "s": s16, "g": g16}, "y")
    assert_same(host(rt.dequant_mul(Wv, dev(s16), None, dev(g16))), want, "misaligned weights")


# ---- Snake --------------------------------------------------------------------------
def _snake_nodes():
    return [("Mul", ["alpha", "x"], ["t"], {}), ("Sin", ["t"], ["s"], {}), ("Pow", ["s", "two"], ["p"], {}),
            ("Mul", ["inv", "p"], ["q"], {}), ("Add", ["x", "q"], ["z"], {})]


@pytest.mark.parametrize("shape", [(2, 256, 4000), (3, 128, 4001), (1, 64, 37)])
def test_snake_chain(rt, shape):
    rng = np.random.default_rng(5)
    B, C, T = shape
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    x.reshape(-1)[:16] = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e30, -1e30, 2e5, -2e5, 117435.99, 1e-40, 7e4,
                          3.4e38, -5e4, 1.5e5, 9e5]
    alpha = rng.uniform(0.5, 1.5, (1, C, 1)).astype(np.float16)
    inv = (1.0 / alpha.astype(np.float64)).astype(np.float16)
    two = np.array(2.0, np.float16)
    env = {"x": x, "alpha": alpha, "inv": inv, "two": two}
    want = oracle_nodes(_snake_nodes(), env, "z")
    l0 = rt.launches
    got = rt.snake(dev(x), dev(alpha), dev(inv), dev(two))
    assert rt.launches - l0 == 1
    assert_same(host(got), want, f"snake {shape}")


def test_snake_strided_and_general_power(rt):
    """A transposed view of x (non-unit stride along the row: the scalar
    path) and an exponent other than 2 (np.power in double, within 2 ulp)."""
    rng = np.random.default_rng(6)
    xt = (rng.standard_normal((300, 2, 64)) * 2).astype(np.float32)     # stored [T, B, C]
    x = np.transpose(xt, (1, 2, 0))                                       # viewed [B, C, T]
    alpha = rng.uniform(0.5, 1.5, (1, 64, 1)).astype(np.float32)
    inv = (1.0 / alpha).astype(np.float32)
    two = np.array(2.0, np.float16)
    want = oracle_nodes(_snake_nodes(), {"x": x, "alpha": alpha, "inv": inv, "two": two}, "z")
    got = rt.snake(dev(xt).permute(1, 2, 0), dev(alpha), dev(inv), dev(two))
    assert_same(host(got), want, "snake over a transposed view")
    p = np.array(1.5, np.float32)
    want = oracle_nodes(_snake_nodes(), {"x": x, "alpha": alpha, "inv": inv, "two": p}, "z")
    got = rt.snake(dev(xt).permute(1, 2, 0), dev(alpha), dev(inv), dev(p))
    assert_ulp(host(got), want, 2, "snake with power 1.5")


# ---- two-op chains ------------------------------------------------------------------
@pytest.mark.parametrize("kind", ["add_sigmoid", "add_leaky", "mul_add"])
@pytest.mark.parametrize("layout", ["same", "row", "f16", "odd"])
def test_two_op_chains(rt, kind, layout):
    from bt_b200 import chains
    rng = np.random.default_rng(7)
    shape = (4, 96, 250) if layout != "odd" else (5, 33, 77)
    x = (rng.standard_normal(shape) * 4).astype(np.float32)
    other_shape = shape if layout in ("same", "odd") else (shape[0], shape[1], 1)
    y = (rng.standard_normal(other_shape) * 4).astype(np.float16 if layout == "f16" else np.float32)
    b = (rng.standard_normal((1, shape[1], 1))).astype(np.float32)
    if kind == "add_sigmoid":
        nodes, env, ins, prog = ([("Add", ["x", "y"], ["s"], {}), ("Sigmoid", ["s"], ["z"], {})],
                                 {"x": x, "y": y}, [x, y], chains.add_unary_program("SIGMOID"))
    elif kind == "add_leaky":
        nodes, env, ins, prog = ([("Add", ["x", "y"], ["s"], {}), ("LeakyRelu", ["s"], ["z"], {"alpha": 0.1})],
                                 {"x": x, "y": y}, [x, y], chains.add_unary_program("LEAKYRELU", 0.1))
    else:
        nodes, env, ins, prog = ([("Mul", ["x", "y"], ["m"], {}), ("Add", ["m", "b"], ["z"], {})],
                                 {"x": x, "y": y, "b": b}, [x, y, b], chains.mul_add_program())
    want = oracle_nodes(nodes, env, "z")
    got = rt.chain(prog, [dev(v) for v in ins])
    assert_same(host(got), want, f"{kind} {layout}")


# ---- the interpreter ----------------------------------------------------------------
_EXACT = ["ADD", "SUB", "MUL", "DIV", "SQRT", "EXP", "SIN", "COS", "SIGMOID", "LEAKYRELU", "NEG", "ABS",
          "MIN", "MAX", "FLOOR", "ROUND", "IDENTITY", "POW2"]


def _np_op(op, a, b, alpha):
    """numpy float32 semantics of one chain instruction (the reference's
    expressions, ref_runtime.py:446-479)."""
    env = {"a": a, "b": b}
    onnx = {"ADD": "Add", "SUB": "Sub", "MUL": "Mul", "DIV": "Div", "POW": "Pow", "SQRT": "Sqrt", "EXP": "Exp",
            "SIN": "Sin", "COS": "Cos", "TANH": "Tanh", "SIGMOID": "Sigmoid", "ERF": "Erf", "ATAN": "Atan",
            "FLOOR": "Floor", "ROUND": "Round"}
    with np.errstate(all="ignore"):
        if op == "LEAKYRELU":
            return oracle_nodes([("LeakyRelu", ["a"], ["o"], {"alpha": alpha})], env, "o")
        if op in onnx:
            ins = ["a", "b"] if op in ("ADD", "SUB", "MUL", "DIV", "POW") else ["a"]
            return oracle_nodes([(onnx[op], ins, ["o"], {})], env, "o").astype(np.float32)
        if op == "NEG":
            return np.negative(a)
        if op == "ABS":
            return np.abs(a)
        if op == "MIN":
            return np.minimum(a, b)
        if op == "MAX":
            return np.maximum(a, b)
        return a.astype(np.float32)   # IDENTITY


def _random_program(rng, n_in, n_instr, ops):
    from bt_b200 import chains
    code, written = [], list(range(n_in))
    for _ in range(n_instr):
        op = ops[rng.integers(len(ops))]
        a = int(rng.choice(written))
        b = int(rng.choice(written))
        dst = int(rng.integers(0, 15))
        if dst >= n_in - 1:
            dst += 1                                     # the last input keeps its 2.0
        if op == "POW2":
            code.append(("POW", dst, a, n_in - 1))      # the last input holds 2.0
        else:
            code.append((op, dst, a, b, 0.2))
        if dst not in written:
            written.append(dst)
    out = code[-1][1]
    return chains.program(n_in, code, out), code, out


def _run_np(code, n_in, inputs, out):
    regs = {j: inputs[j] for j in range(n_in)}
    for op, d, a, b, *al in code:
        name = "POW" if op == "POW" else op
        regs[d] = _np_op(name, regs[a], regs[b], al[0] if al else 0.2)
    return regs[out]


@pytest.mark.parametrize("seed", range(12))
def test_interpreter_random_programs_exact(rt, lib, seed):
    import ctypes
    rng = np.random.default_rng(100 + seed)
    n_in = int(rng.integers(2, 7))
    shape = (3, 40, 123)
    inputs = []
    for j in range(n_in - 1):
        shp = [shape, (3, 40, 1), (1, 40, 123), (123,), ()][j % 5]
        a = (rng.standard_normal(shp) * 3).astype(np.float16 if j == 2 else np.float32)
        inputs.append(np.asarray(a))
    inputs.append(np.array(2.0, np.float32))
    prog, code, out = _random_program(rng, n_in, int(rng.integers(1, 10)), _EXACT)
    kind = lib.bt_chain_kind(ctypes.byref(prog))
    assert kind == 64 or 0 <= kind < 8
    # numpy broadcasts inside each op, as the reference's graph does (a 0-d
    # exponent of 2 takes numpy's squaring path, which the kernels match)
    want = np.ascontiguousarray(np.broadcast_to(_run_np(code, n_in, [v.astype(np.float32) for v in inputs], out),
                                                shape))
    got = rt.chain(prog, [dev(v) for v in inputs], shape)
    assert_same(host(got), np.ascontiguousarray(want).astype(np.float32), f"program {code}")


@pytest.mark.parametrize("op", ["TANH", "ATAN", "ERF", "POW"])
def test_interpreter_ulp_ops(rt, op):
    from bt_b200 import chains
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((64, 500)) * 2).astype(np.float32)
    if op == "POW":
        x = np.abs(x)
        p = np.array(1.7, np.float32)
        prog = chains.program(2, [("POW", 2, 0, 1)], 2)
        got = rt.chain(prog, [dev(x), dev(p)])
        want = _np_op("POW", x, p, 0.0)
    else:
        prog = chains.program(1, [(op, 1, 0, 0), ("ADD", 2, 1, 0)], 2)
        got = rt.chain(prog, [dev(x)])
        want = _np_op("ADD", _np_op(op, x, x, 0.0), x, 0.0)
    assert_ulp(host(got), want, 2, op)


# ---- the node-list fusion pass ------------------------------------------------------
def test_run_nodes_fuses_known_chains(rt):
    """The c5 stream's Snake chains and a dequant + gain fuse into one launch
    each; results equal the unfused run bit for bit; kept and multiply-read
    values are never fused away."""
    from bt_b200 import chains
    from bt_b200.decoder import build_stream
    import cases as C
    S = build_stream(1, t0=8)
    env0 = C.c5_small_inputs(S, seed=11)
    keep = set(S.stage_outputs())
    groups = chains.plan(S.nodes, keep)
    assert sum(g.kind == "snake" for g in groups) == 48
    denv = {k: (dev(v) if isinstance(v, np.ndarray) and v.ndim > 0 else v) for k, v in env0.items()}
    plain = rt.run_nodes(S.nodes, dict(denv))
    l0 = rt.launches
    fused = rt.run_nodes(S.nodes, dict(denv), fuse=True, keep=keep)
    fused_launches = rt.launches - l0
    l0 = rt.launches
    rt.run_nodes(S.nodes, dict(denv))
    assert fused_launches < rt.launches - l0 - 4 * 48 + 1
    for name in keep:
        assert_same(host(fused[name]), host(plain[name]), name)
    # a value that must survive is not fused away
    g0 = groups[0]
    inner = S.nodes[g0.nodes[0]][2][0]
    kept = rt.run_nodes(S.nodes, dict(denv), fuse=True, keep=keep | {inner})
    assert inner in kept


@pytest.mark.parametrize("case", ["i8", "i8_zp", "u8_zp_f16scale", "per_tensor", "i32"])
def test_dequantize_linear_alone(rt, case):
    """DequantizeLinear through dispatch: 8-bit inputs take one chain pass,
    int32 inputs the element-wise DEQUANT op; numpy's bits either way."""
    rng = np.random.default_rng(11)
    C = 64
    q = rng.integers(-127, 128, (C, 48, 7)).astype(np.int8)
    sc = rng.uniform(1e-3, 2e-2, (C, 1, 1)).astype(np.float32)
    zp = None
    if case == "i8_zp":
        zp = rng.integers(-9, 10, (C, 1, 1)).astype(np.int8)
    elif case == "u8_zp_f16scale":
        q = rng.integers(0, 256, (C, 48, 7)).astype(np.uint8)
        sc = sc.astype(np.float16)
        zp = rng.integers(100, 156, (C, 1, 1)).astype(np.uint8)
    elif case == "per_tensor":
        sc = np.array(0.0123, np.float32)
    elif case == "i32":
        q = rng.integers(-10 ** 6, 10 ** 6, (C, 48, 7)).astype(np.int32)
    env = {"q": q, "s": sc}
    ins = ["q", "s"]
    if zp is not None:
        env["z"] = zp
        ins.append("z")
    want = oracle_nodes([("DequantizeLinear", ins, ["y"], {})], env, "y")
    denv = {k: dev(v) for k, v in env.items()}
    l0 = rt.launches
    rt.dispatch("DequantizeLinear", ins, ["y"], {}, denv)
    assert rt.launches - l0 == 1
    assert_same(host(denv["y"]), want, f"DequantizeLinear {case}")

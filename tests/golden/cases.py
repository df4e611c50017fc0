"""Parity cases for the hot path, shared by make_golden.py and the tests.

A case is a list of op-table nodes ``(op, inputs, outputs, attrs)`` plus the
arrays its inputs name.  ``make_golden.py`` runs every case through the
reference interpreter itself (tools/ref_runtime.py) and stores the outputs;
the CPU tests run the oracle on the same inputs and the GPU tests run
``BtRuntime`` (and the fused kernels) on them.  All inputs are regenerated
deterministically from the seeds below (np.random.default_rng), and the
fixture stores a SHA-256 of every input so a change in generation is caught.

Sources of the literal cases:
  * tests/test_gpu_elementwise.gd:31-40, :165-181 of the reference (its GPU
    kernel unit test: shapes, the LeakyRelu alpha=0.2 vector and the Where
    vector with their expected values);
  * BASELINE configs c1-c5 at reduced sizes;
  * edge values numpy defines (NaN, +-inf, +-0, subnormals, overflow).
"""
import numpy as np

F32, F16, F64 = np.float32, np.float16, np.float64
SPECIAL = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e-40, 1e-38, 3.0e38, -3.0e38,
                    88.0, 89.0, -87.0, -104.0, -150.0, 1.0, -1.0, 0.5, 2.0, 1e4, -1e4,
                    117435.99, 117436.0, 71476.0, 71477.0, 3e5, -2.5e6], F32)


class Case:
    def __init__(self, name, nodes, env, outputs=None, expect=None):
        self.name = name
        self.nodes = nodes
        self.env = env
        self.outputs = outputs or [nodes[-1][2][0]]
        self.expect = expect or {}   # literal expected values from the reference's own tests


def _u(rng, shape, lo=0.5, hi=3.5):
    return rng.uniform(lo, hi, shape).astype(F32)


def _n(rng, shape, scale=1.0, dt=F32):
    return (rng.standard_normal(shape) * scale).astype(dt)


def cases():
    out = []
    rng = np.random.default_rng(1234)

    # -- the reference's GPU kernel test (tests/test_gpu_elementwise.gd:31-40)
    for name, op, ash, bsh in [("gd_mul_bcast", "Mul", (2, 3, 4), (3, 1)),
                               ("gd_add_scalar", "Add", (5, 7), ()),
                               ("gd_sub_equal", "Sub", (4, 6), (4, 6)),
                               ("gd_div_outer", "Div", (2, 1, 5), (2, 4, 5))]:
        out.append(Case(name, [(op, ["a", "b"], ["y"], {})], {"a": _u(rng, ash), "b": _u(rng, bsh)}))
    for name, op, sh in [("gd_sqrt", "Sqrt", (3, 9)), ("gd_sigmoid", "Sigmoid", (64,)),
                         ("gd_floor", "Floor", (17,))]:
        out.append(Case(name, [(op, ["a"], ["y"], {})], {"a": _u(rng, sh)}))
    leaky_in = np.array([-2.0, -0.5, 0.0, 0.5, 2.0], F32)
    out.append(Case("gd_leaky", [("LeakyRelu", ["a"], ["y"], {"alpha": 0.2})], {"a": leaky_in},
                    expect={"y": np.where(leaky_in < 0, leaky_in * np.float32(0.2), leaky_in)}))
    out.append(Case("gd_where", [("Where", ["c", "x", "z"], ["y"], {})],
                    {"c": np.array([1, 0, 1, 0], F32), "x": np.array([10, 20, 30, 40], F32),
                     "z": np.array([-1], F32)},
                    expect={"y": np.array([10, -1, 30, -1], F32)}))

    # -- c1 at reduced size: broadcast Add / Mul, then unary ops on the result
    x, b = _n(rng, (1, 64, 128)), _n(rng, (1, 64, 1))
    for op in ("Add", "Mul", "Sub", "Div", "Pow"):
        env = {"x": x, "b": b if op != "Pow" else np.array(2.0, F16)}
        out.append(Case(f"c1_{op.lower()}", [(op, ["x", "b"], ["y"], {})], env))
    y = (x + b).astype(F32)
    for op in ("Sigmoid", "Tanh", "Exp", "Sin", "Cos", "Atan", "Erf", "Floor", "Round"):
        out.append(Case(f"c1_{op.lower()}", [(op, ["y"], ["o"], {})], {"y": y * F32(4.0)}))
    out.append(Case("c1_sqrt", [("Sqrt", ["y"], ["o"], {})], {"y": np.abs(y)}))
    out.append(Case("c1_leaky02", [("LeakyRelu", ["y"], ["o"], {"alpha": 0.2})], {"y": y}))
    out.append(Case("c1_leaky_default", [("LeakyRelu", ["y"], ["o"], {})], {"y": y}))
    # wide-range transcendental inputs (numpy's SIMD paths and their fallbacks)
    wide = np.concatenate([_n(rng, (4096,), 30.0), rng.uniform(-2e5, 2e5, 4096).astype(F32), SPECIAL])
    for op in ("Exp", "Sin", "Cos", "Sigmoid", "Tanh", "Sqrt", "Floor", "Round", "Atan", "Erf"):
        out.append(Case(f"wide_{op.lower()}", [(op, ["w"], ["o"], {})], {"w": wide}))

    # -- broadcasting patterns (numpy's right-aligned rule, stride-0 axes)
    shapes = [((3, 1, 5), (1, 4, 1)), ((2, 3, 4, 5), (5,)), ((6,), (2, 1, 6)), ((), (3, 2)),
              ((2, 1, 3, 1, 2), (1, 4, 1, 5, 1)), ((1, 1, 1), (7, 1, 9)), ((4, 1), (4, 1)),
              ((2, 3, 2, 1, 2, 1), (3, 1, 2, 2, 1))]
    for i, (a_sh, b_sh) in enumerate(shapes):
        env = {"a": _n(rng, a_sh), "b": _n(rng, b_sh)}
        for op in ("Add", "Mul", "Div"):
            out.append(Case(f"bcast{i}_{op.lower()}", [(op, ["a", "b"], ["y"], {})], env))

    # -- dtype mixes (fp16 widened first; numpy promotion otherwise)
    dt_pairs = [(F16, F32), (F16, F16), (np.int8, F32), (np.int32, F32), (np.int64, np.int64),
                (np.int32, np.int32), (np.uint8, np.int8), (np.bool_, np.bool_), (F64, F32),
                (np.int64, F16), (np.uint8, F16)]
    for i, (da, db) in enumerate(dt_pairs):
        def mk(dt, shape):
            if np.dtype(dt).kind == "f":
                return _n(rng, shape, 3.0, dt)
            if dt == np.bool_:
                return rng.integers(0, 2, shape).astype(np.bool_)
            info = np.iinfo(dt)
            return rng.integers(max(info.min, -50), min(info.max, 50) + 1, shape).astype(dt)
        env = {"a": mk(da, (3, 8)), "b": mk(db, (8,))}
        if np.dtype(db).kind in "iu":
            env["b"] = np.where(env["b"] == 0, 1, env["b"]).astype(db)
        ops = ("Add", "Mul", "Div", "Sub") if da != np.bool_ else ("Add", "Mul")
        for op in ops:
            out.append(Case(f"dtype{i}_{op.lower()}", [(op, ["a", "b"], ["y"], {})], env))
    ia = rng.integers(-20, 21, (40,)).astype(np.int32)
    ib = rng.integers(1, 7, (40,)).astype(np.int32) * np.where(rng.integers(0, 2, 40) == 0, -1, 1).astype(np.int32)
    out.append(Case("int_floordiv", [("Div", ["a", "b"], ["y"], {})], {"a": ia, "b": ib}))
    for op in ("Sqrt", "Exp", "Sigmoid", "Sin"):
        out.append(Case(f"int_{op.lower()}", [(op, ["a"], ["y"], {})], {"a": np.abs(ia)}))
    out.append(Case("int_leaky", [("LeakyRelu", ["a"], ["y"], {"alpha": 0.2})], {"a": ia}))
    out.append(Case("f16_leaky", [("LeakyRelu", ["a"], ["y"], {"alpha": 0.2})], {"a": _n(rng, (50,), 2.0, F16)}))

    # -- special values through the arithmetic
    sp = SPECIAL
    spb = np.roll(SPECIAL, 5)
    for op in ("Add", "Sub", "Mul", "Div", "Pow"):
        out.append(Case(f"special_{op.lower()}", [(op, ["a", "b"], ["y"], {})], {"a": sp, "b": spb}))
    out.append(Case("special_leaky", [("LeakyRelu", ["a"], ["y"], {"alpha": 0.01})], {"a": sp}))
    xs = _n(rng, (200,), 2.0)
    for e in (2.0, 3.0, 0.5, -1.0, 0.0):
        out.append(Case(f"pow_{e}", [("Pow", ["a", "e"], ["y"], {})], {"a": xs, "e": np.array(e, F16)}))

    # -- Cast (ref_runtime.py:572-578)
    cf = np.concatenate([_n(rng, (64,), 100.0), np.array([0.5, -0.5, 1.5, -1.5, 2.5, 127.9, -128.9, 0.0, -0.0],
                                                          F32)])
    # (float -> narrow int casts are kept in range: outside it C leaves them undefined)
    in_range = {2: np.clip(np.abs(cf), 0, 255), 3: np.clip(cf, -128, 127)}
    for to in (1, 2, 3, 5, 6, 7, 9, 10, 11):
        out.append(Case(f"cast_f32_to_{to}", [("Cast", ["a"], ["y"], {"to": to})], {"a": in_range.get(to, cf)}))
    out.append(Case("cast_f16_to_f32", [("Cast", ["a"], ["y"], {"to": 1})], {"a": _n(rng, (300,), 0.05, F16)}))
    out.append(Case("cast_i32_to_f32", [("Cast", ["a"], ["y"], {"to": 1})],
                    {"a": rng.integers(-2**31, 2**31, (100,), dtype=np.int64).astype(np.int32)}))
    out.append(Case("cast_i64_to_f32", [("Cast", ["a"], ["y"], {"to": 1})],
                    {"a": rng.integers(-2**62, 2**62, (100,), dtype=np.int64)}))
    out.append(Case("cast_bool_to_f32", [("Cast", ["a"], ["y"], {"to": 1})],
                    {"a": rng.integers(0, 2, (30,)).astype(np.bool_)}))
    out.append(Case("cast_i64_to_i32", [("Cast", ["a"], ["y"], {"to": 6})],
                    {"a": rng.integers(-2**40, 2**40, (100,), dtype=np.int64)}))

    # -- Clip / comparisons / logic / Where
    cx = np.concatenate([_n(rng, (40,), 3.0), np.array([np.nan, -0.0, 0.0, np.inf], F32)])
    lo, hi = np.array(-1.0, F32), np.array(1.5, F16)
    out.append(Case("clip_both", [("Clip", ["x", "lo", "hi"], ["y"], {})], {"x": cx, "lo": lo, "hi": hi}))
    out.append(Case("clip_lo", [("Clip", ["x", "lo"], ["y"], {})], {"x": cx, "lo": lo}))
    out.append(Case("clip_hi", [("Clip", ["x", "", "hi"], ["y"], {})], {"x": cx, "hi": hi}))
    out.append(Case("clip_none", [("Clip", ["x"], ["y"], {})], {"x": cx}))
    ca, cb = _n(rng, (4, 6)), _n(rng, (6,))
    cb[::2] = ca[0, ::2]
    for op in ("Equal", "Greater", "Less", "GreaterOrEqual"):
        out.append(Case(f"cmp_{op.lower()}", [(op, ["a", "b"], ["y"], {})], {"a": ca, "b": cb}))
    out.append(Case("cmp_equal_int", [("Equal", ["a", "b"], ["y"], {})],
                    {"a": rng.integers(0, 3, (10,)).astype(np.int64), "b": np.array([1], np.int64)}))
    out.append(Case("cmp_greater_f16", [("Greater", ["a", "b"], ["y"], {})],
                    {"a": _n(rng, (3, 5), 1.0, F16), "b": np.array(0.0, F16)}))
    out.append(Case("logic_and", [("And", ["a", "b"], ["y"], {})],
                    {"a": rng.integers(0, 2, (4, 5)).astype(np.bool_), "b": rng.integers(0, 2, (5,)).astype(np.bool_)}))
    out.append(Case("where_bcast", [("Where", ["c", "x", "z"], ["y"], {})],
                    {"c": rng.integers(0, 2, (3, 1, 4)).astype(np.bool_), "x": _n(rng, (5, 4)),
                     "z": np.array(7.0, F16)}))
    out.append(Case("where_int", [("Where", ["c", "x", "z"], ["y"], {})],
                    {"c": rng.integers(0, 2, (6,)).astype(np.bool_), "x": np.arange(6, dtype=np.int64),
                     "z": np.array(-1, np.int32)}))

    # -- DequantizeLinear (ref_runtime.py:631-636) and c4 dequant * gain
    for i, (qdt, zp, sc_shape, sc_dt) in enumerate([(np.int8, None, (16, 1, 1), F32),
                                                    (np.uint8, np.array(128, np.uint8), (), F32),
                                                    (np.int8, "chan", (16, 1, 1), F16),
                                                    (np.int8, np.array(0, np.int8), (16, 1, 1), F32)]):
        q = rng.integers(np.iinfo(qdt).min, np.iinfo(qdt).max + 1, (16, 16, 3)).astype(qdt)
        env = {"q": q, "s": rng.uniform(1e-3, 2e-2, sc_shape).astype(sc_dt),
               "g": rng.uniform(0.5, 1.5, (16, 1, 1)).astype(F32)}
        ins = ["q", "s"]
        if zp is not None:
            env["z"] = rng.integers(-3, 4, (16, 1, 1)).astype(np.int8) if isinstance(zp, str) else zp
            ins.append("z")
        out.append(Case(f"dequant{i}", [("DequantizeLinear", ins, ["d"], {"axis": 0}),
                                        ("Mul", ["d", "g"], ["y"], {})], env, outputs=["d", "y"]))

    # -- reductions (ref_runtime.py:589-598)
    r3 = _n(rng, (4, 5, 300), 2.0)
    red = [("last", r3, [2], 1), ("last_nokeep", r3, [-1], 0), ("middle", r3, [1], 1),
           ("first", r3, [0], 0), ("outer_block", r3, [0, 1], 1), ("two_block", r3, [0, 2], 1),
           ("trailing_block", r3, [1, 2], 0), ("all", r3, None, 1), ("all_nokeep", r3, None, 0)]
    for name, arr, axes, keep in red:
        for op in ("ReduceMean", "ReduceSum"):
            env = {"x": arr}
            ins = ["x"]
            if axes is not None:
                env["ax"] = np.array(axes, np.int64)
                ins.append("ax")
            out.append(Case(f"red_{name}_{op.lower()}", [(op, ins, ["y"], {"keepdims": keep})], env))
    out.append(Case("red_attr_axes", [("ReduceMean", ["x"], ["y"], {"axes": [2], "keepdims": 1})], {"x": r3}))
    out.append(Case("red_noop", [("ReduceSum", ["x", "ax"], ["y"], {"noop_with_empty_axes": 1})],
                    {"x": r3, "ax": np.array([], np.int64)}))
    out.append(Case("red_f16", [("ReduceMean", ["x", "ax"], ["y"], {})],
                    {"x": _n(rng, (3, 200), 1.0, F16), "ax": np.array([1], np.int64)}))
    for n in (1, 7, 8, 9, 127, 128, 129, 136, 255, 256, 1000, 2048, 4000, 24001):
        out.append(Case(f"red_len{n}", [("ReduceMean", ["x", "ax"], ["y"], {}),
                                        ("ReduceSum", ["x", "ax"], ["z"], {})],
                        {"x": _n(rng, (3, n), 3.0), "ax": np.array([-1], np.int64)}, outputs=["y", "z"]))
    edge = np.zeros((5, 40), F32)
    edge[0] = -0.0
    edge[1, 3] = np.nan
    edge[2, 7] = np.inf
    edge[3, 2], edge[3, 9] = np.inf, -np.inf
    edge[4] = 1e-41
    out.append(Case("red_edges", [("ReduceSum", ["x", "ax"], ["y"], {}), ("ReduceMean", ["x", "ax"], ["z"], {})],
                    {"x": edge, "ax": np.array([1], np.int64)}, outputs=["y", "z"]))

    # -- softmax (ref_runtime.py:269-273) and c3 at reduced size (mask Add first)
    out.append(Case("softmax_basic", [("Softmax", ["x"], ["y"], {"axis": -1})], {"x": _n(rng, (2, 3, 7, 50), 2.0)}))
    sx = _n(rng, (4, 100), 30.0)
    sx[0, :3] = -np.inf
    sx[1, :] = -np.inf
    sx[2, 5] = np.inf
    out.append(Case("softmax_edges", [("Softmax", ["x"], ["y"], {})], {"x": sx}))
    mask = np.zeros((1, 1, 1, 40), F32)
    mask[..., -7:] = -1e4
    out.append(Case("c3_small", [("Add", ["x", "m"], ["s"], {}), ("Softmax", ["s"], ["y"], {"axis": -1})],
                    {"x": _n(rng, (1, 2, 40, 40), 2.0), "m": mask}, outputs=["s", "y"]))
    for n in (1, 8, 129, 510, 1000):
        out.append(Case(f"softmax_len{n}", [("Softmax", ["x"], ["y"], {})], {"x": _n(rng, (3, n), 2.0)}))

    # -- layer norms (ref_runtime.py:276-285, :601-609)
    lx = _n(rng, (2, 10, 48))
    g32, b32 = rng.uniform(0.5, 1.5, (48,)).astype(F32), _n(rng, (48,), 0.1)
    out.append(Case("ln_basic", [("LayerNormalization", ["x", "g", "b"], ["y"], {"axis": -1, "epsilon": 1e-5})],
                    {"x": lx, "g": g32, "b": b32}))
    out.append(Case("ln_f16_params", [("LayerNormalization", ["x", "g", "b"], ["y"], {"epsilon": 1e-12})],
                    {"x": lx, "g": g32.astype(F16), "b": b32.astype(F16)}))
    out.append(Case("ln_nobias", [("LayerNormalization", ["x", "g"], ["y"], {"epsilon": 1e-5})], {"x": lx, "g": g32}))
    out.append(Case("ln_axis_m2", [("LayerNormalization", ["x", "g", "b"], ["y"], {"axis": -2, "epsilon": 1e-5})],
                    {"x": lx, "g": _n(rng, (10, 48)), "b": _n(rng, (48,))}))
    const_rows = np.full((3, 64), 0.25, F32)
    const_rows[1] += np.float32(1e-7) * np.arange(64, dtype=F32)
    out.append(Case("ln_const_rows", [("LayerNormalization", ["x", "g"], ["y"], {"epsilon": 1e-12})],
                    {"x": const_rows, "g": np.ones(64, F32)}))
    out.append(Case("ln_c2_small", [("LayerNormalization", ["x", "g", "b"], ["y"], {"epsilon": 1e-12})],
                    {"x": _n(rng, (1, 51, 768)), "g": rng.uniform(0.5, 1.5, (768,)).astype(F32),
                     "b": _n(rng, (768,), 0.1)}))
    sk = _n(rng, (2, 10, 48))
    out.append(Case("skipln_bias", [("SkipLayerNormalization", ["x", "s", "g", "b", "bias"], ["y"], {})],
                    {"x": lx, "s": sk, "g": g32, "b": b32, "bias": _n(rng, (48,))}))
    out.append(Case("skipln_nobias", [("SkipLayerNormalization", ["x", "s", "g", "b"], ["y"], {"epsilon": 1e-5})],
                    {"x": lx, "s": sk, "g": g32, "b": b32}))
    out.append(Case("fastgelu_bias", [("FastGelu", ["x", "b"], ["y"], {})], {"x": _n(rng, (6, 32), 2.0),
                                                                             "b": _n(rng, (32,))}))
    out.append(Case("fastgelu", [("FastGelu", ["x"], ["y"], {})], {"x": _n(rng, (6, 32), 2.0)}))

    # -- AdaIN and Snake as the graph spells them (one node per op)
    ax = np.array([2], np.int64)
    h = _n(rng, (2, 8, 100), 2.0)
    fc = _n(rng, (2, 16, 1))
    alpha = rng.uniform(0.5, 1.5, (1, 8, 1)).astype(F16)
    env = {"h": h, "fc": fc, "ax": ax, "eps": np.array(1e-5, F16), "one": np.array(1.0, F16),
           "two": np.array(2.0, F16), "alpha": alpha, "inv": (1.0 / alpha.astype(F64)).astype(F16),
           "split": np.array([8, 8], np.int64)}
    nodes = [("Split", ["fc", "split"], ["gamma", "beta"], {"axis": 1}),
             ("Add", ["gamma", "one"], ["gain"], {}),
             ("ReduceMean", ["h", "ax"], ["mu"], {"keepdims": 1}), ("Sub", ["h", "mu"], ["d"], {}),
             ("Mul", ["d", "d"], ["d2"], {}), ("ReduceMean", ["d2", "ax"], ["var"], {"keepdims": 1}),
             ("Add", ["var", "eps"], ["ve"], {}), ("Sqrt", ["ve"], ["sd"], {}), ("Div", ["d", "sd"], ["n"], {}),
             ("Mul", ["gain", "n"], ["m"], {}), ("Add", ["m", "beta"], ["a"], {}),
             ("Mul", ["alpha", "a"], ["t"], {}), ("Sin", ["t"], ["s"], {}), ("Pow", ["s", "two"], ["p"], {}),
             ("Mul", ["inv", "p"], ["q"], {}), ("Add", ["a", "q"], ["z"], {})]
    out.append(Case("adain_snake_chain", nodes, env, outputs=["a", "z"]))

    # -- DynamicQuantizeLinear (ref :106-116): mixed signs, one sign only, all
    # zeros, fp16 input, a range of exactly 255 (scale 1, so x / scale hits
    # rint's halfway cases), one value, the float32 extremes
    dq = [("dq_mixed", _n(rng, (2, 64, 50), 2.0)),
          ("dq_positive", _u(rng, (3, 40))),
          ("dq_negative", -_u(rng, (3, 40))),
          ("dq_zeros", np.zeros((5, 7), F32)),
          ("dq_f16", _n(rng, (4, 33), 3.0, F16)),
          ("dq_ties", np.array([0.0, 255.0, 0.5, 1.5, 2.5, 3.5, 254.5, -0.0, 100.49999, 7.5], F32)),
          ("dq_single", np.array([3.7], F32)),
          ("dq_extremes", np.array([3.0e38, -3.0e38, 1.0, -1.0, 0.0, 1e-30], F32))]
    for name, v in dq:
        out.append(Case(name, [("DynamicQuantizeLinear", ["x"], ["y", "sc", "zp"], {})], {"x": v},
                        outputs=["y", "sc", "zp"]))

    # -- the integer convolution epilogue as the packed graph spells it after
    # each generator ConvInteger: bias scale from the activation and weight
    # scales, the bias quantised to int32, the int32 Add, the (elided) cast to
    # fp16 and the rescale
    def conv_epilogue(acc, bias, xs, ws):
        nodes = [("Cast", ["xs"], ["xs16"], {"to": 10}), ("Mul", ["xs16", "ws"], ["s"], {}),
                 ("Div", ["bias", "s"], ["bt"], {}), ("Floor", ["bt"], ["bf"], {}),
                 ("Cast", ["bf"], ["bq"], {"to": 6}), ("Reshape", ["bq", "shp"], ["bqr"], {}),
                 ("Add", ["acc", "bqr"], ["sum"], {}), ("Cast", ["sum"], ["sumf"], {"to": 10}),
                 ("Mul", ["sumf", "s"], ["y"], {})]
        env = {"acc": acc, "bias": bias, "xs": xs, "ws": ws, "shp": np.array([1, -1, 1], np.int64)}
        return nodes, env
    acc = rng.integers(-(1 << 22), 1 << 22, (2, 16, 37)).astype(np.int32)
    acc[0, 3, :4] = [2147483647, 2147483600, -2147483648, -2147483000]      # int32 wrap-around
    for name, bias, xs, ws in [
            ("conv_epi_f16", _n(rng, (16,), 0.2, F16), np.float32(0.0137), np.float16(0.0021)),
            ("conv_epi_f32", _n(rng, (16,), 0.5), np.float32(0.21), np.float32(3.1e-4)),
            ("conv_epi_tiny_scale", _n(rng, (16,), 10.0, F16), np.float32(1e-6), np.float16(1e-4))]:
        nodes, env = conv_epilogue(acc, bias, np.array(xs, F32), np.array(ws))
        out.append(Case(name, nodes, env, outputs=["s", "bq", "y"]))

    # -- data movement (ref :517-555): transposes, concatenation (with the
    # fp16 widening and integer promotion), slices with negative indices and
    # steps (including the reference's empty full reversal), expand
    t4 = _n(rng, (2, 3, 5, 7))
    for name, perm in [("tr_last2", [0, 1, 3, 2]), ("tr_rotate", [3, 0, 1, 2]), ("tr_default", None)]:
        at = {} if perm is None else {"perm": perm}
        out.append(Case(name, [("Transpose", ["x"], ["y"], at)], {"x": t4}))
    out.append(Case("tr_int64", [("Transpose", ["x"], ["y"], {"perm": [1, 0]})],
                    {"x": rng.integers(-9, 9, (6, 11)).astype(np.int64)}))
    out.append(Case("concat_axis1", [("Concat", ["a", "b", "c"], ["y"], {"axis": 1})],
                    {"a": _n(rng, (2, 3, 4)), "b": _n(rng, (2, 5, 4)), "c": _n(rng, (2, 1, 4))}))
    out.append(Case("concat_f16_mix", [("Concat", ["a", "b"], ["y"], {"axis": -1})],
                    {"a": _n(rng, (3, 4), dt=F16), "b": _n(rng, (3, 2))}))
    out.append(Case("concat_int_promote", [("Concat", ["a", "b"], ["y"], {"axis": 0})],
                    {"a": rng.integers(-5, 5, (2, 3)).astype(np.int32),
                     "b": rng.integers(-5, 5, (1, 3)).astype(np.int64)}))
    s3 = _n(rng, (4, 9, 10))
    i64 = lambda *v: np.array(v, np.int64)   # noqa: E731
    for name, ins in [("slice_basic", (i64(1, 2), i64(3, 8), i64(0, 2), None)),
                      ("slice_neg", (i64(-3), i64(-1), i64(1), None)),
                      ("slice_step", (i64(0, 1), i64(9, 10), i64(1, 2), i64(2, 3))),
                      ("slice_back", (i64(8), i64(1), i64(1), i64(-2))),
                      ("slice_reverse_all", (i64(-1), i64(-(1 << 62)), i64(2), i64(-1))),
                      ("slice_clamp", (i64(-100), i64(100), i64(0), None))]:
        env = {"x": s3, "st": ins[0], "en": ins[1], "ax": ins[2]}
        names = ["x", "st", "en", "ax"]
        if ins[3] is not None:
            env["sp"] = ins[3]
            names.append("sp")
        out.append(Case(name, [("Slice", names, ["y"], {})], env))
    out.append(Case("expand_rank", [("Expand", ["x", "shp"], ["y"], {})],
                    {"x": _n(rng, (3, 1)), "shp": i64(2, 1, 5)}))
    out.append(Case("expand_f16", [("Expand", ["x", "shp"], ["y"], {})],
                    {"x": _n(rng, (1, 4), dt=F16), "shp": i64(3, 4)}))
    return out


def c5_small_inputs(stream, seed=7):
    """Host inputs of a small c5 stream: features, fc outputs and conv
    stand-ins, all ~ N(0,1) from np.random.default_rng(seed) in sorted-name
    order."""
    rng = np.random.default_rng(seed)
    env = {}
    for name in sorted(stream.inputs):
        shape, dt, kind = stream.inputs[name]
        env[name] = rng.standard_normal(shape, dtype=np.float32)
    env.update({k: v for k, v in stream.consts.items()})
    return env

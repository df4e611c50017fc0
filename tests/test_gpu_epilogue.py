"""The fused integer convolution epilogue (bt_conv_int_epilogue) against the
reference's op-by-op chain: the golden fixtures the reference itself produced
(tests/golden, cases conv_epi_*) and the oracle on larger seeded inputs --
stage-0 and stage-1 generator shapes, int32 wrap-around, a bias whose
quotient leaves the int32 range, float16 and float32 bias / weight scale,
rows whose start is not 16-byte aligned.  Bit-exact."""
import os
import warnings

import numpy as np
import pytest
import torch

import cases as C
from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_ops.npz")


def _fused(rt, env):
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()   # noqa: E731
    y = rt.conv_int_epilogue(d(env["acc"]), d(env["bias"]), d(env["xs"]), d(env["ws"]))
    torch.cuda.synchronize()
    return y


def test_fused_epilogue_matches_reference_golden(gpu_runtime):
    gold = np.load(GOLDEN)
    cs = [c for c in C.cases() if c.name.startswith("conv_epi")]
    assert len(cs) == 3
    for c in cs:
        assert_same(_fused(gpu_runtime, c.env), gold[f"{c.name}/y"], c.name)


def test_op_by_op_matches_reference_golden(gpu_runtime):
    """The same chain through the op table (one kernel per node), s and bq too."""
    gold = np.load(GOLDEN)
    for c in [c for c in C.cases() if c.name.startswith("conv_epi")]:
        env = dict(c.env)
        gpu_runtime.run_nodes(c.nodes, env)
        torch.cuda.synchronize()
        for o in ("s", "bq", "y"):
            assert_same(env[o], gold[f"{c.name}/{o}"], f"{c.name}/{o}")


@pytest.mark.parametrize("B,Cc,T,bdt,wdt", [(2, 256, 4000, np.float16, np.float16), (1, 128, 24001, np.float32, np.float16),
                                            (3, 5, 1, np.float16, np.float32), (2, 7, 13, np.float32, np.float32)])
def test_fused_epilogue_matches_oracle(gpu_runtime, B, Cc, T, bdt, wdt):
    rng = np.random.default_rng(B * 1000 + T)
    acc = rng.integers(-(1 << 24), 1 << 24, (B, Cc, T)).astype(np.int32)
    acc.reshape(-1)[:3] = [2147483647, -2147483648, 2147483000]
    bias = (rng.standard_normal(Cc) * 0.3).astype(bdt)
    bias[0] = 60000.0 if bdt == np.float16 else 3.0e9    # quotient past the int32 range
    xs, ws = np.array(0.0173, np.float32), np.array(0.0021, wdt)
    env = {"acc": acc, "bias": bias, "xs": xs, "ws": ws, "shp": np.array([1, -1, 1], np.int64)}
    nodes = [("Cast", ["xs"], ["xs16"], {"to": 10}), ("Mul", ["xs16", "ws"], ["s"], {}),
             ("Div", ["bias", "s"], ["bt"], {}), ("Floor", ["bt"], ["bf"], {}),
             ("Cast", ["bf"], ["bq"], {"to": 6}), ("Reshape", ["bq", "shp"], ["bqr"], {}),
             ("Add", ["acc", "bqr"], ["sum"], {}), ("Cast", ["sum"], ["sumf"], {"to": 10}),
             ("Mul", ["sumf", "s"], ["y"], {})]
    want = dict(env)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, want)
    assert_same(_fused(gpu_runtime, env), want["y"], f"B={B} C={Cc} T={T}")


def test_unaligned_rows(gpu_runtime):
    """T = 4001: successive rows start at every 4-byte phase."""
    rng = np.random.default_rng(77)
    env = {"acc": rng.integers(-(1 << 20), 1 << 20, (1, 8, 4001)).astype(np.int32),
           "bias": rng.standard_normal(8).astype(np.float16), "xs": np.array(0.02, np.float32),
           "ws": np.array(0.003, np.float16)}
    s = np.float32(env["xs"] * np.float32(env["ws"]))
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        bq = np.floor(env["bias"].astype(np.float32) / s).astype(np.int32)
        want = ((env["acc"] + bq.reshape(1, -1, 1)).astype(np.float32) * s).astype(np.float32)
    assert_same(_fused(gpu_runtime, env), want, "unaligned rows")

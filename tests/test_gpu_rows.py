"""Row ops at row counts that take the warp-per-row kernels (at least
2 x SMs x 8 rows), across row lengths with remainders, runs shorter than 8,
perfect and non-perfect pairwise trees and the 2048-value limit; bit-exact
against the oracle through the op table."""
import warnings

import numpy as np
import pytest

from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu

ROWS = 2500
LENGTHS = [5, 8, 100, 510, 768, 777, 1024, 2047, 2048]


def _run_both(rt, nodes, env):
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        want = OracleRuntime().run_nodes(nodes, dict(env))
    got = dict(env)
    rt.run_nodes(nodes, got)
    return got, want


@pytest.mark.parametrize("n", LENGTHS)
def test_warp_rows_reduce(gpu_runtime, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((ROWS, n)) * 3).astype(np.float32)
    x[7, n // 2] = np.nan
    env = {"x": x, "ax": np.array([-1], np.int64), "xh": x.astype(np.float16)}
    nodes = [("ReduceMean", ["x", "ax"], ["m"], {"keepdims": 1}), ("ReduceSum", ["x", "ax"], ["s"], {"keepdims": 0}),
             ("ReduceMean", ["xh", "ax"], ["mh"], {"keepdims": 1})]
    got, want = _run_both(gpu_runtime, nodes, env)
    for k in ("m", "s", "mh"):
        assert_same(got[k], want[k], f"{k} n={n}")


@pytest.mark.parametrize("n", [3001, 4096, 8192, 24001, 49152])
def test_long_rows_reduce(gpu_runtime, n):
    """Rows longer than the warp-staged kernels take, read straight from
    global memory by the warp-per-row sum (odd lengths: unaligned rows)."""
    rng = np.random.default_rng(300 + n)
    rows = 2400
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    x[11, n // 3] = np.inf
    env = {"x": x, "ax": np.array([1], np.int64)}
    nodes = [("ReduceMean", ["x", "ax"], ["m"], {"keepdims": 1}), ("ReduceSum", ["x", "ax"], ["s"], {"keepdims": 0})]
    got, want = _run_both(gpu_runtime, nodes, env)
    for k in ("m", "s"):
        assert_same(got[k], want[k], f"{k} n={n}")


@pytest.mark.parametrize("n", LENGTHS)
def test_warp_rows_softmax(gpu_runtime, n):
    rng = np.random.default_rng(100 + n)
    x = (rng.standard_normal((ROWS // 10, 10, n)) * 2).astype(np.float32)
    mask = np.zeros((1, 1, n), np.float32)
    mask[..., -max(1, n // 7):] = -1e4
    x[3, 4, 0] = np.inf
    env = {"x": x, "mask": mask}
    nodes = [("Add", ["x", "mask"], ["s"], {}), ("Softmax", ["s"], ["y"], {"axis": -1}),
             ("Softmax", ["x"], ["y2"], {"axis": -1})]
    got, want = _run_both(gpu_runtime, nodes, env)
    assert_same(got["y"], want["y"], f"masked softmax n={n}")
    assert_same(got["y2"], want["y2"], f"softmax n={n}")


@pytest.mark.parametrize("n", LENGTHS)
def test_warp_rows_layernorm(gpu_runtime, n):
    rng = np.random.default_rng(200 + n)
    x = rng.standard_normal((ROWS, n)).astype(np.float32)
    skip = rng.standard_normal((ROWS, n)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, n).astype(np.float16)
    beta = (rng.standard_normal(n) * 0.1).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    env = {"x": x, "skip": skip, "g": gamma, "b": beta, "bias": bias, "g32": gamma.astype(np.float32)}
    nodes = [("LayerNormalization", ["x", "g", "b"], ["y"], {"epsilon": 1e-5, "axis": -1}),
             ("SkipLayerNormalization", ["x", "skip", "g", "b", "bias"], ["z"], {"epsilon": 1e-12}),
             ("LayerNormalization", ["x", "g32", "b"], ["y32"], {"epsilon": 1e-5, "axis": -1}),
             ("LayerNormalization", ["x", "g32"], ["y32n"], {"epsilon": 1e-5, "axis": -1})]
    got, want = _run_both(gpu_runtime, nodes, env)
    assert_same(got["y"], want["y"], f"layernorm n={n}")
    assert_same(got["z"], want["z"], f"skip layernorm n={n}")
    assert_same(got["y32"], want["y32"], f"layernorm fp32 gamma/beta n={n}")
    assert_same(got["y32n"], want["y32n"], f"layernorm fp32 gamma, no beta n={n}")


@pytest.mark.parametrize("n", [1024, 2048])
def test_perfect_rows_direct_and_fallback(gpu_runtime, n):
    """Rows of 1024 / 2048 values (perfect trees of 128-value leaves) summed
    straight from global memory, on a [B, C, T] tensor like BASELINE's c2;
    a base one element off an 8-byte boundary takes the staged kernel. Both
    equal numpy bit for bit."""
    import torch
    rng = np.random.default_rng(n + 1)
    x = (rng.standard_normal((4, 700, n)) * 2 + 0.3).astype(np.float32)
    env = {"x": x, "ax": np.array([2], np.int64)}
    nodes = [("ReduceMean", ["x", "ax"], ["m"], {"keepdims": 1}), ("ReduceSum", ["x", "ax"], ["s"], {"keepdims": 0})]
    got, want = _run_both(gpu_runtime, nodes, env)
    for k in ("m", "s"):
        assert_same(got[k], want[k], f"{k} n={n}")
    buf = torch.empty(x.size + 1, device="cuda")
    xo = buf[1:].view(x.shape)
    xo.copy_(torch.from_numpy(x))
    got2 = {"x": xo, "ax": env["ax"]}
    gpu_runtime.run_nodes(nodes, got2)
    for k in ("m", "s"):
        assert_same(got2[k], want[k], f"{k} n={n} offset")

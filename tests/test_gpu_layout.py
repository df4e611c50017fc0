"""Chains through views on the GPU against the oracle: the reference keeps
Transpose outputs as numpy views and numpy's sums follow the memory layout,
so Transpose -> LayerNormalization (the Kokoro text encoder's cnn blocks),
Transpose -> ReduceMean and element-wise ops between them must reproduce
numpy's order bit for bit."""
import warnings

import numpy as np
import pytest
import torch

from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu
F16, F32, I64 = np.float16, np.float32, np.int64


def _run(rt, nodes, env, outs):
    want = {k: np.array(v, copy=True) for k, v in env.items()}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, want)
    got = dict(env)
    rt.run_nodes(nodes, got)
    torch.cuda.synchronize()
    for o in outs:
        g = got[o].cpu().numpy() if isinstance(got[o], torch.Tensor) else np.asarray(got[o])
        assert_same(g, np.asarray(want[o]), o)


def _ln_env(rng, B=1, C=512, T=9):
    return {"x": (rng.standard_normal((B, C, T)) * 1.5 + 0.2).astype(F32),
            "g": rng.uniform(0.5, 1.5, C).astype(F16), "b": (rng.standard_normal(C) * 0.1).astype(F16),
            "bias": rng.standard_normal(C).astype(F32), "skip": rng.standard_normal((B, T, C)).astype(F32),
            "ax": np.array([2], I64), "ax1": np.array([1], I64), "ax12": np.array([1, 2], I64)}


@pytest.mark.parametrize("C,T", [(512, 9), (128, 37), (768, 5), (96, 1000)])
def test_transpose_then_layernorm(gpu_runtime, C, T):
    env = _ln_env(np.random.default_rng(C + T), 2, C, T)
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 2, 1]}),
             ("LayerNormalization", ["xt", "g", "b"], ["y"], {"axis": -1, "epsilon": 1e-5}),
             ("LeakyRelu", ["y"], ["z"], {"alpha": 0.2}),
             ("Transpose", ["z"], ["zt"], {"perm": [0, 2, 1]}),
             ("ReduceMean", ["zt", "ax"], ["m"], {"keepdims": 1})]
    _run(gpu_runtime, nodes, env, ["y", "z", "zt", "m"])


def test_elementwise_between_transpose_and_norm(gpu_runtime):
    env = _ln_env(np.random.default_rng(1))
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 2, 1]}),
             ("Add", ["xt", "bias"], ["xb"], {}),
             ("Cast", ["xb"], ["xh"], {"to": 10}),
             ("LayerNormalization", ["xh", "g", "b"], ["y"], {"axis": -1, "epsilon": 1e-5}),
             ("SkipLayerNormalization", ["xt", "skip", "g", "b"], ["s"], {"epsilon": 1e-12}),
             ("SkipLayerNormalization", ["xt", "xb", "g", "b", "bias"], ["s2"], {"epsilon": 1e-12})]
    _run(gpu_runtime, nodes, env, ["xb", "xh", "y", "s", "s2"])


def test_transpose_keeping_the_last_axis_innermost(gpu_runtime):
    rng = np.random.default_rng(2)
    env = {"x": rng.standard_normal((9, 1, 512)).astype(F32), "g": rng.uniform(0.5, 1.5, 512).astype(F16),
           "b": rng.standard_normal(512).astype(F16)}
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [1, 0, 2]}),
             ("LayerNormalization", ["xt", "g", "b"], ["y"], {"axis": -1, "epsilon": 1e-5}),
             ("Softmax", ["xt"], ["p"], {"axis": -1})]
    _run(gpu_runtime, nodes, env, ["y", "p"])


@pytest.mark.parametrize("axes,keep", [("ax", 1), ("ax", 0), ("ax1", 1), ("ax12", 0)])
def test_transpose_then_reduce(gpu_runtime, axes, keep):
    env = _ln_env(np.random.default_rng(3), 3, 260, 33)
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 2, 1]}),
             ("ReduceMean", ["xt", axes], ["m"], {"keepdims": keep}),
             ("ReduceSum", ["xt", axes], ["s"], {"keepdims": keep})]
    _run(gpu_runtime, nodes, env, ["m", "s"])


def test_reshape_and_slice_of_views(gpu_runtime):
    rng = np.random.default_rng(4)
    env = {"x": rng.standard_normal((2, 12, 64, 9)).astype(F32), "shape": np.array([2, 9, 768], I64),
           "st": np.array([1], I64), "en": np.array([7], I64), "axs": np.array([1], I64),
           "ax": np.array([2], I64)}
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 3, 1, 2]}),
             ("Reshape", ["xt", "shape"], ["r"], {}),
             ("ReduceMean", ["r", "ax"], ["m"], {"keepdims": 1}),
             ("Transpose", ["r"], ["rt"], {"perm": [0, 2, 1]}),
             ("Slice", ["rt", "st", "en", "axs"], ["sl"], {}),
             ("ReduceSum", ["sl", "ax"], ["s"], {"keepdims": 0})]
    _run(gpu_runtime, nodes, env, ["r", "m", "sl", "s"])


def test_fortran_ordered_upload(gpu_runtime):
    """A numpy input already laid out with the last axis outermost (what a
    CPU op hands over) keeps that layout on the device."""
    rng = np.random.default_rng(5)
    env = {"x": np.asfortranarray(rng.standard_normal((1, 9, 512)).astype(F32)),
           "g": rng.uniform(0.5, 1.5, 512).astype(F16), "b": rng.standard_normal(512).astype(F16),
           "ax": np.array([2], I64)}
    nodes = [("LayerNormalization", ["x", "g", "b"], ["y"], {"axis": -1, "epsilon": 1e-5}),
             ("ReduceMean", ["x", "ax"], ["m"], {"keepdims": 1})]
    _run(gpu_runtime, nodes, env, ["y", "m"])


def test_same_dtype_cast_launches_nothing(gpu_runtime):
    """Cast to the dtype the tensor has (float32 -> float32, and the fp16
    target the reference computes in float32) hands back the tensor itself;
    a view with gaps is copied densely, as numpy's astype does."""
    rng = np.random.default_rng(6)
    env = {"x": rng.standard_normal((4, 96, 33)).astype(F32), "st": np.array([0], I64),
           "en": np.array([20], I64), "axs": np.array([2], I64)}
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 2, 1]}),
             ("Cast", ["xt"], ["c1"], {"to": 1}),
             ("Cast", ["c1"], ["c2"], {"to": 10}),
             ("DynamicQuantizeLinear", ["c2"], ["q", "qs", "qz"], {}),
             ("Slice", ["xt", "st", "en", "axs"], ["sl"], {}),
             ("Cast", ["sl"], ["c3"], {"to": 1})]
    _run(gpu_runtime, nodes, env, ["c1", "c2", "q", "qs", "qz", "sl", "c3"])
    got = dict(env)
    gpu_runtime.run_nodes(nodes[:1], got)
    before = gpu_runtime.launches
    gpu_runtime.run_nodes(nodes[1:3], got)
    assert gpu_runtime.launches == before and got["c2"] is got["xt"]


def test_upload_cache_follows_the_host_array(gpu_runtime):
    """An uploaded numpy array is reused while it lives and forgotten (its
    device copy released) when it dies."""
    import gc
    a = np.arange(1024, dtype=F32)
    t1 = gpu_runtime.to_device(a)
    assert gpu_runtime.to_device(a) is t1
    n = len(gpu_runtime._consts)
    del a, t1
    gc.collect()
    assert len(gpu_runtime._consts) == n - 1

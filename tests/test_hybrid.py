"""The whole-graph driver's host logic (bt_b200.hybrid) on the CPU: routing
by op, one host copy per device tensor, numpy's axis order kept across the
boundary, results equal to one op table running everything.  The GPU table
is stood in for by the oracle producing torch CPU tensors."""
import warnings

import numpy as np
import pytest
import torch

from bt_b200.hybrid import HybridRuntime, host_array
from oracle import OracleRuntime


class TensorTable:
    """The oracle, returning torch tensors like the GPU table does."""
    def __init__(self):
        self.ops = []

    def dispatch(self, op, ins, outs, at, env):
        self.ops.append(op)
        sub = {n: (env[n].numpy() if isinstance(env[n], torch.Tensor) else env[n]) for n in ins if n}
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            OracleRuntime().dispatch(op, ins, outs, at, sub)
        for o in outs:
            if o:
                env[o] = torch.from_numpy(np.array(sub[o], copy=True))


class CountingCpu:
    def __init__(self):
        self.ops, self.seen = [], []

    def dispatch(self, op, ins, outs, at, env):
        self.ops.append(op)
        self.seen += [type(env[n]) for n in ins if n]
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            OracleRuntime().dispatch(op, ins, outs, at, env)


def _graph():
    rng = np.random.default_rng(0)
    env = {"x": rng.standard_normal((2, 64, 9)).astype(np.float32), "b": rng.standard_normal(64).astype(np.float32),
           "g": rng.uniform(0.5, 1.5, 64).astype(np.float16), "ax": np.array([2], np.int64)}
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 2, 1]}),
             ("Add", ["xt", "b"], ["h"], {}),
             ("LayerNormalization", ["h", "g", ""], ["n"], {"axis": -1, "epsilon": 1e-5}),
             ("Mul", ["n", "h"], ["m"], {}),
             ("Sigmoid", ["h"], ["s"], {}),
             ("ReduceMean", ["m", "ax"], ["r"], {"keepdims": 1})]
    return nodes, env


@pytest.mark.parametrize("cpu_ops", [set(), {"LayerNormalization"}, {"Add", "ReduceMean"}, {"Sigmoid", "Mul"}])
def test_hybrid_equals_one_table(cpu_ops):
    nodes, env = _graph()
    want = dict(env)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, want)
    from bt_b200.runtime import BtRuntime
    gpu, cpu = TensorTable(), CountingCpu()
    hy = HybridRuntime(cpu, gpu_ops=set(BtRuntime.HOT_OPS) - cpu_ops, gpu_runtime=gpu)
    got = dict(env)
    hy.run_nodes(nodes, got)
    for o in ("xt", "h", "n", "m", "s", "r"):
        g = hy.result(got[o])
        assert g.dtype == want[o].dtype and np.array_equal(g, want[o]), o
    assert sorted(cpu.ops) == sorted(op for op, *_ in nodes if op in cpu_ops)
    assert hy.stats["cpu_nodes"] == len(cpu.ops) and hy.stats["gpu_nodes"] == len(gpu.ops)
    assert all(t is np.ndarray or issubclass(t, np.ndarray) for t in cpu.seen)   # the CPU table sees numpy only


def test_one_host_copy_per_tensor():
    nodes, env = _graph()
    nodes = nodes[:2] + [("Sigmoid", ["h"], ["s1"], {}), ("Sigmoid", ["h"], ["s2"], {})]
    hy = HybridRuntime(CountingCpu(), gpu_ops={"Transpose", "Add"}, gpu_runtime=TensorTable())
    hy.run_nodes(nodes, dict(env))
    assert hy.stats["d2h_bytes"] == 2 * 9 * 64 * 4    # h crosses once for its two CPU consumers


def test_gpu_ops_outside_the_path_are_rejected():
    with pytest.raises(ValueError):
        HybridRuntime(CountingCpu(), gpu_ops={"Conv"}, gpu_runtime=TensorTable())


def test_host_array_keeps_axis_order():
    base = torch.arange(2 * 512 * 9, dtype=torch.float32).reshape(2, 512, 9)
    v = base.permute(0, 2, 1)
    a = host_array(v)
    assert np.array_equal(a, v.numpy()) and not a.flags.c_contiguous
    assert sorted(range(3), key=lambda i: -a.strides[i]) == [0, 2, 1]
    s = base[:, ::2, :].permute(0, 2, 1)           # a view with gaps: made dense first
    assert np.array_equal(host_array(s), s.numpy())


def test_host_copies_do_not_keep_device_tensors_alive():
    import gc
    import weakref
    hy = HybridRuntime(CountingCpu(), gpu_ops={"Add"}, gpu_runtime=TensorTable())
    env = {"a": np.ones(8, np.float32), "b": np.ones(8, np.float32)}
    hy.run_nodes([("Add", ["a", "b"], ["c"], {}), ("Sigmoid", ["c"], ["d"], {})], env)
    ref = weakref.ref(env["c"])
    del env["c"]
    gc.collect()
    assert ref() is None

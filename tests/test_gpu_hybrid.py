"""The whole-graph driver on the GPU: BtRuntime for the GPU side, the oracle
standing in for the reference's RefRuntime on the CPU side, ops split both
ways across a graph with views (Transpose -> LayerNormalization, the text
encoder's pattern); every result equals one numpy table running the whole
graph, bit for bit."""
import warnings

import numpy as np
import pytest

from bt_b200.hybrid import HybridRuntime
from bt_b200.runtime import BtRuntime
from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu


def _graph():
    rng = np.random.default_rng(1)
    env = {"x": rng.standard_normal((2, 512, 9)).astype(np.float32), "b": rng.standard_normal(512).astype(np.float32),
           "g": rng.uniform(0.5, 1.5, 512).astype(np.float16), "beta": rng.standard_normal(512).astype(np.float16),
           "ax": np.array([2], np.int64), "sc": np.array(0.5, np.float16)}
    nodes = [("Transpose", ["x"], ["xt"], {"perm": [0, 2, 1]}),
             ("LayerNormalization", ["xt", "g", "beta"], ["n"], {"axis": -1, "epsilon": 1e-5}),
             ("LeakyRelu", ["n"], ["l"], {"alpha": 0.2}),
             ("Add", ["l", "b"], ["h"], {}),
             ("Transpose", ["h"], ["ht"], {"perm": [0, 2, 1]}),
             ("ReduceMean", ["ht", "ax"], ["m"], {"keepdims": 1}),
             ("Mul", ["ht", "sc"], ["y"], {}),
             ("DynamicQuantizeLinear", ["y"], ["q", "qs", "qz"], {})]
    return nodes, env


@pytest.mark.parametrize("cpu_ops", [set(), {"LayerNormalization"}, {"Transpose", "ReduceMean"},
                                     {"LeakyRelu", "Mul", "DynamicQuantizeLinear"}])
def test_hybrid_graph_equals_numpy(gpu_runtime, cpu_ops):
    nodes, env = _graph()
    want = dict(env)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, want)
    hy = HybridRuntime(OracleRuntime(), gpu_ops=set(BtRuntime.HOT_OPS) - cpu_ops, gpu_runtime=gpu_runtime)
    got = dict(env)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        hy.run_nodes(nodes, got)
    for o in ("xt", "n", "l", "h", "ht", "m", "y", "q", "qs", "qz"):
        assert_same(hy.result(got[o]), np.asarray(want[o]), o)
    assert hy.stats["cpu_nodes"] == sum(op in cpu_ops for op, *_ in nodes)

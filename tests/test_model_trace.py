"""The oracle on the real model's hot-path nodes (tests/golden/model_trace.*,
recorded from the reference's packed-model driver by make_model_trace.py).

Every sampled node -- at least one of each op type the model runs on the GPU
path, with the reference's own input arrays -- must give the reference's
outputs bit for bit, and every distinct node signature of the run (op,
attributes, dtypes, shapes) must run through the oracle on seeded inputs.
"""
import warnings

import numpy as np
import pytest

import modeltrace as T
from oracle import OracleRuntime
from parity import assert_same

META = T.load_meta()


@pytest.fixture(scope="module")
def arrays():
    return T.load_arrays()


def test_trace_covers_every_hot_op_type():
    from bt_b200.runtime import BtRuntime
    ops = set(META["op_counts"])
    assert ops <= set(BtRuntime.HOT_OPS)
    assert {n["op"] for n in META["sampled"]} == ops
    assert sum(META["op_counts"].values()) == META["hot_nodes"]
    assert sum(s["count"] for s in META["signatures"]) == META["hot_nodes"]


@pytest.mark.parametrize("node", META["sampled"], ids=[f'{n["op"]}@{n["pos"]}' for n in META["sampled"]])
def test_oracle_matches_reference_on_model_nodes(node, arrays):
    env = T.sampled_env(node, arrays)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().dispatch(node["op"], list(node["inputs"]), list(node["outputs"]), T.attrs(node["attrs"]), env)
    for name, want in T.sampled_outputs(node, arrays).items():
        assert_same(np.asarray(env[name]), want, f'{node["op"]}@{node["pos"]} -> {name}')


def test_oracle_runs_every_model_signature():
    for i, sig in enumerate(META["signatures"]):
        (op, ins, outs, at), env = T.synthetic_node(sig, seed=i)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            OracleRuntime().dispatch(op, ins, outs, at, env)
        assert all(o in env for o in outs), (op, sig["first"])

"""The oracle against fixtures produced by the reference interpreter itself.

tests/golden/make_golden.py ran every case of tests/golden/cases.py through
the reference's RefRuntime.dispatch (tools/ref_runtime.py:428-668); here the
oracle (oracle/ops.py) must reproduce those outputs bit for bit, including
the literal vectors of the reference's own GPU kernel test
(tests/test_gpu_elementwise.gd:165-181).
"""
import hashlib
import json
import os
import warnings

import numpy as np
import pytest

import cases as C
from oracle import OracleRuntime
from parity import assert_same

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def sha(a):
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def golden():
    with np.load(os.path.join(GOLD, "golden_ops.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    with open(os.path.join(GOLD, "golden_meta.json")) as f:
        meta = json.load(f)
    return arrays, meta


ALL = C.cases()


@pytest.mark.parametrize("case", ALL, ids=[c.name for c in ALL])
def test_oracle_matches_reference(case, golden):
    arrays, meta = golden
    assert {k: sha(v) for k, v in case.env.items()} == meta["inputs"][case.name], "case inputs changed"
    env = {k: np.array(v, copy=True) for k, v in case.env.items()}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(case.nodes, env)
    for o in case.outputs:
        assert_same(env[o], arrays[f"{case.name}/{o}"], f"{case.name}/{o}")
    for o, want in case.expect.items():
        assert_same(env[o], want, f"{case.name}/{o} (literal)")


def test_oracle_c5_stream_matches_reference(golden):
    from bt_b200.decoder import build_stream
    arrays, meta = golden
    S = build_stream(1, t0=8)
    env = C.c5_small_inputs(S)
    assert {k: sha(v) for k, v in env.items()} == meta["c5"]["inputs"]
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(S.nodes, env)
    for name in S.stage_outputs():
        assert_same(env[name], arrays[f"c5/{name}"], name)
    assert {n: sha(env[n]) for n in S.snake_names()} == meta["c5"]["snakes"]
    assert {n: sha(env[n]) for n in S.residual_names()} == meta["c5"]["residuals"]


def test_oracle_rejects_unknown_op():
    with pytest.raises(NotImplementedError):
        OracleRuntime().dispatch("Conv", ["x"], ["y"], {}, {"x": np.zeros(3, np.float32)})

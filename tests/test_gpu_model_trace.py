"""The real model's hot-path nodes through the drop-in op table on the GPU
(tests/golden/model_trace.*, recorded from the reference's packed-model
driver by make_model_trace.py).

* Every sampled node, with the reference's own input arrays, through
  ``BtRuntime.dispatch`` against the reference's own outputs.
* Every distinct node signature of the run (845: op, attributes, dtypes,
  shapes; the values of inputs of at most 64 elements) on seeded inputs,
  against the oracle.

Tolerances per op (modeltrace.tolerance): bit-exact except Tanh / Atan /
Erf and Pow with an exponent other than 2 (<= 2 ulp), float64 results of
integer inputs (<= 2 ulp), Sin / Cos beyond numpy's SIMD range (<= 1 ulp)
and FastGelu (|d| <= 1e-6 + 1e-5 |want|).
"""
import collections
import warnings

import numpy as np
import pytest
import torch

import modeltrace as T
from oracle import OracleRuntime

pytestmark = pytest.mark.gpu
META = T.load_meta()
BY_OP = collections.defaultdict(list)
for _i, _s in enumerate(META["signatures"]):
    BY_OP[_s["op"]].append((_i, _s))


@pytest.fixture(scope="module")
def arrays():
    return T.load_arrays()


def _host(v):
    return v.cpu().numpy() if isinstance(v, torch.Tensor) else np.asarray(v)


@pytest.mark.parametrize("node", META["sampled"], ids=[f'{n["op"]}@{n["pos"]}' for n in META["sampled"]])
def test_model_node_matches_reference(node, gpu_runtime, arrays):
    env = T.sampled_env(node, arrays)
    ins = [env[n] if n else None for n in node["inputs"]]
    gpu_runtime.dispatch(node["op"], list(node["inputs"]), list(node["outputs"]), T.attrs(node["attrs"]), env)
    torch.cuda.synchronize()
    for name, want in T.sampled_outputs(node, arrays).items():
        got = _host(env[name])
        T.compare(got, want, T.tolerance(node["op"], [a for a in ins if a is not None], want),
                  f'{node["op"]}@{node["pos"]} -> {name}')


@pytest.mark.parametrize("op", sorted(BY_OP))
def test_model_signatures_match_oracle(op, gpu_runtime):
    for i, sig in BY_OP[op]:
        (op_, ins, outs, at), env = T.synthetic_node(sig, seed=i)
        genv = {k: np.array(v, copy=True) for k, v in env.items()}
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            OracleRuntime().dispatch(op_, ins, outs, at, env)
        gpu_runtime.dispatch(op_, ins, outs, at, genv)
        torch.cuda.synchronize()
        args = [np.asarray(env[n]) for n in ins if n]
        for o in outs:
            want = np.asarray(env[o])
            T.compare(_host(genv[o]), want, T.tolerance(op_, args, want), f"{op} signature {i} (node {sig['first']}) -> {o}")

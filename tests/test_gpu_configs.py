"""GPU parity at the BASELINE configurations' full sizes (c1-c4), against the
oracle evaluated on the same seeded inputs in the same run.  Tolerances as in
test_gpu_ops.py: bit-exact except Tanh (<= 2 ulp)."""
import warnings

import numpy as np
import pytest
import torch

from bt_b200 import configs
from oracle import OracleRuntime
from parity import assert_same, assert_ulp

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def oracle(nodes, env):
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return OracleRuntime().run_nodes(nodes, dict(env))


def test_c1_broadcast_and_unary(gpu_runtime):
    c = configs.c1()
    nodes = [("Add", ["X", "B"], ["y"], {}), ("Mul", ["X", "B"], ["m"], {}), ("Sigmoid", ["y"], ["sg"], {}),
             ("Tanh", ["y"], ["th"], {}), ("LeakyRelu", ["y"], ["lr"], {"alpha": 0.2})]
    want = oracle(nodes, c)
    env = dict(c)
    gpu_runtime.run_nodes(nodes, env)
    for k in ("y", "m", "sg", "lr"):
        assert_same(env[k], want[k], k)
    assert_ulp(env["th"].cpu().numpy(), want["th"], 2, "th")


def test_c2_layernorm(gpu_runtime):
    c = configs.c2_layernorm()
    env = {"X": c["X"], "g": c["gamma"], "b": c["beta"]}
    nodes = [("LayerNormalization", ["X", "g", "b"], ["y"], {"axis": -1, "epsilon": c["eps"]})]
    want = oracle(nodes, env)
    gpu_runtime.run_nodes(nodes, env)
    assert_same(env["y"], want["y"], "layernorm")


def test_c2_adain(gpu_runtime):
    from test_gpu_decoder import oracle_adain_snake
    c = configs.c2_adain()
    Cc = c["X"].shape[1]
    _, want = oracle_adain_snake([c["X"]], c["h"], None, None, c["eps"], snake=False)
    h = dev(c["h"][:, :, 0])
    gain = gpu_runtime.elementwise("ADD", [h[:, :Cc], dev(np.array(1.0, np.float16))], (1, Cc), np.float32,
                                   np.float32)
    out = gpu_runtime.adain_snake([dev(c["X"])], gain, h[:, Cc:], np.float32(c["eps"]))
    assert_same(out[0], want, "adain")


def test_c2_reducemean(gpu_runtime):
    c = configs.c2_reducemean()
    env = {"X": c["X"], "ax": np.array([-1], np.int64)}
    nodes = [("ReduceMean", ["X", "ax"], ["y"], {"keepdims": 1})]
    want = oracle(nodes, env)
    gpu_runtime.run_nodes(nodes, env)
    assert_same(env["y"], want["y"], "reducemean")


@pytest.mark.parametrize("batch", [1, 16])
def test_c3_masked_softmax(gpu_runtime, batch):
    c = configs.c3(batch=batch)
    nodes = [("Add", ["X", "mask"], ["s"], {}), ("Softmax", ["s"], ["y"], {"axis": -1})]
    want = oracle(nodes, c)
    got = gpu_runtime.softmax(dev(c["X"]), dev(c["mask"]), -1)   # mask Add fused into the row kernel
    assert_same(got, want["y"], "masked softmax")


@pytest.mark.parametrize("shape", [(512, 512, 3), (256, 256, 7)])
def test_c4_dequant_gain(gpu_runtime, shape):
    c = configs.c4_dequant(shape=shape)
    nodes = [("DequantizeLinear", ["W", "scale", "zp"], ["d"], {"axis": 0}), ("Mul", ["d", "gain"], ["y"], {})]
    want = oracle(nodes, c)
    got = gpu_runtime.dequant_mul(dev(c["W"]), dev(c["scale"]), dev(c["zp"]), dev(c["gain"]))
    assert_same(got, want["y"], "dequant * gain")
    env = dict(c)
    gpu_runtime.run_nodes(nodes, env)
    assert_same(env["y"], want["y"], "dequant, mul (op by op)")


def test_c4_cast(gpu_runtime):
    c = configs.c4_cast()
    nodes = [("Cast", ["X"], ["y"], {"to": 1})]
    want = oracle(nodes, c)
    env = dict(c)
    gpu_runtime.run_nodes(nodes, env)
    assert_same(env["y"], want["y"], "cast fp16 -> fp32")

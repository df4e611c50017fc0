"""DynamicQuantizeLinear on the GPU (bt_dynamic_quantize) against the oracle,
bit for bit: the uint8 values, the float32 scale and the uint8 zero point.
Sizes on both sides of 2^17 values, where the one-cluster path for small
aligned float32 inputs hands over to the two-kernel path.

Sizes past one CTA's share and past the 16-value vector groups, inputs at
every 4-byte phase (the element-wise paths), float16 input, one-signed and
constant inputs, and the non-finite cases: a NaN gives scale 1, zero point 0
and 0 at the NaN elements; an infinity makes the scale infinite and every
value 0 (numpy turns its NaN zero point into 0 when it casts)."""
import warnings

import numpy as np
import pytest
import torch

from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu


def _oracle(x):
    env = {"x": x}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().dispatch("DynamicQuantizeLinear", ["x"], ["y", "sc", "zp"], {}, env)
    return env["y"], env["sc"], env["zp"]


def _gpu(rt, x, phase=0):
    flat = np.ascontiguousarray(x).reshape(-1)
    buf = torch.empty(flat.size + 4, dtype=torch.from_numpy(flat[:1]).dtype, device="cuda")
    xd = buf[phase:phase + flat.size].view(x.shape)
    xd.copy_(torch.from_numpy(np.ascontiguousarray(x)))
    y, sc, zp = rt.dynamic_quantize(xd)
    torch.cuda.synchronize()
    return y.cpu().numpy(), sc.cpu().numpy(), zp.cpu().numpy()


def _check(rt, x, phase=0, what=""):
    y, sc, zp = _gpu(rt, x, phase)
    wy, wsc, wzp = _oracle(x)
    assert_same(sc, np.asarray(wsc), f"scale {what}")
    assert_same(zp, np.asarray(wzp), f"zero point {what}")
    assert_same(y, wy, f"values {what}")


@pytest.mark.parametrize("n", [1, 3, 15, 16, 17, 4097, 32_768, 100_003, (1 << 17) - 1, 1 << 17, (1 << 17) + 1,
                               1 << 20, 3_000_001])
def test_sizes(gpu_runtime, n):
    rng = np.random.default_rng(n)
    _check(gpu_runtime, (rng.standard_normal(n) * 2.5).astype(np.float32), what=f"n={n}")


@pytest.mark.parametrize("phase", [1, 2, 3])
def test_unaligned(gpu_runtime, phase):
    rng = np.random.default_rng(10 + phase)
    _check(gpu_runtime, (rng.standard_normal(100_003) - 0.7).astype(np.float32), phase, f"phase {phase}")


def test_float16_and_shapes(gpu_runtime):
    rng = np.random.default_rng(3)
    _check(gpu_runtime, (rng.standard_normal((4, 512, 333)) * 4).astype(np.float16), what="fp16")
    _check(gpu_runtime, (rng.standard_normal((1, 512, 33)) * 4).astype(np.float16), what="fp16 small")
    _check(gpu_runtime, rng.uniform(0.1, 9.0, (2, 256, 4000)).astype(np.float32), what="positive")
    _check(gpu_runtime, -rng.uniform(0.1, 9.0, (2, 256, 4000)).astype(np.float32), what="negative")
    _check(gpu_runtime, np.full((7, 9), 2.5, np.float32), what="constant")
    _check(gpu_runtime, np.zeros((3, 1000), np.float32), what="zeros")


def test_halfway_quotients(gpu_runtime):
    """A range of exactly 255 makes the scale 1: x / scale = x, so values
    at .5 exercise rint's ties-to-even."""
    v = np.concatenate([[0.0, 255.0], np.arange(0.5, 255.0, 1.0), np.arange(0.25, 255.0, 0.5)]).astype(np.float32)
    _check(gpu_runtime, np.tile(v, 40), what="ties")


@pytest.mark.parametrize("seed", range(6))
def test_near_half_quotients(gpu_runtime, seed):
    """Values whose quotient x / scale lies within a few float ulps of a
    half-integer, at random scales: where the kernel's float32 shortcut
    hands over to the exact quotient."""
    rng = np.random.default_rng(100 + seed)
    lo = float(np.float32(-rng.uniform(0.01, 50.0)))
    hi = float(np.float32(rng.uniform(0.01, 50.0)))
    s32 = np.float32((hi - lo) / 255.0)     # the oracle's scale (double, then float32)
    k = rng.integers(-120, 120, 20_000).astype(np.float64)
    base = ((k + 0.5) * np.float64(s32)).astype(np.float32)
    steps = rng.integers(-4, 5, base.size)
    x = base.copy()
    for st in range(1, 5):
        x = np.where(steps >= st, np.nextafter(x, np.float32(np.inf)), x)
        x = np.where(steps <= -st, np.nextafter(x, np.float32(-np.inf)), x)
    x = np.clip(x, np.float32(lo), np.float32(hi))
    x = np.concatenate([[np.float32(lo), np.float32(hi)], x]).astype(np.float32)
    _check(gpu_runtime, x, what=f"near-half seed {seed}")


def test_non_finite(gpu_runtime):
    rng = np.random.default_rng(9)
    x = rng.standard_normal(50_000).astype(np.float32)
    xn = x.copy()
    xn[123] = np.nan
    y, sc, zp = _gpu(gpu_runtime, xn)
    assert float(sc) == 1.0 and int(zp) == 0 and y[123] == 0
    keep = np.ones(xn.size, bool)
    keep[123] = False
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        want = np.clip(np.rint(xn[keep] / np.float32(1.0)) + 0.0, 0, 255).astype(np.uint8)
    assert_same(y[keep], want, "NaN input: other values")
    xi = x.copy()
    xi[7] = np.inf
    y, sc, zp = _gpu(gpu_runtime, xi)
    assert np.isinf(sc) and int(zp) == 0 and not y.any()


def test_empty_is_an_error(gpu_runtime):
    with pytest.raises(RuntimeError):
        gpu_runtime.dynamic_quantize(torch.empty((0, 4), device="cuda"))

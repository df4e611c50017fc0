"""Rows held in registers: softmax over rows of 510 and 512 values (ALBERT's
attention rows) and layer norm over 768 channels (its hidden size), which
the register-resident kernel serves: numpy's pairwise sum unrolled at compile
time, bit-exact against the oracle's Add + Softmax for every mask layout the
kernel reads (one mask row for all rows, one per batch, a scalar, a strided
view, none), special values, and a misaligned input that takes the staged
kernel instead; rows of 300 values check the staged warp kernel on the same
mask layouts."""
import warnings

import numpy as np
import pytest
import torch

from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu


def _oracle(x, mask):
    env = {"x": x}
    nodes = [("Softmax", ["x"], ["y"], {"axis": -1})]
    if mask is not None:
        env["m"] = mask
        nodes = [("Add", ["x", "m"], ["s"], {}), ("Softmax", ["s"], ["y"], {"axis": -1})]
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, env)
    return env["y"]


@pytest.mark.parametrize("n", [300, 510, 512])
@pytest.mark.parametrize("mask_kind", ["row_const", "per_batch", "per_query", "per_head_query", "offset_view",
                                       "scalar", "strided", "none"])
def test_register_softmax_rows(gpu_runtime, n, mask_kind):
    rng = np.random.default_rng(n + len(mask_kind))
    B, H, Q = 3, 4, 37
    x = (rng.standard_normal((B, H, Q, n)) * 2).astype(np.float32)
    x[0, 0, 0, 5] = np.inf            # one +inf: that row is NaN / 0 as in numpy
    x[0, 1, 2, :] = -np.inf           # a row of -inf: all NaN
    x[1, 2, 3, 7] = np.nan
    x[2, 3, 4, :] = 80.0              # a constant row
    mask_dev = None
    if mask_kind == "row_const":
        mask = np.zeros((1, 1, 1, n), np.float32)
        mask[..., -37:] = -1e4
    elif mask_kind == "per_batch":
        mask = np.zeros((B, 1, 1, n), np.float32)
        for b in range(B):
            mask[b, ..., n - 10 * (b + 1):] = -1e4
    elif mask_kind == "per_query":          # [B, 1, Q, n]: three collapsed axes
        mask = (rng.standard_normal((B, 1, Q, n)) * 3).astype(np.float32)
    elif mask_kind == "per_head_query":     # [1, H, Q, n]: H and Q merge into one axis
        mask = (rng.standard_normal((1, H, Q, n)) * 3).astype(np.float32)
    elif mask_kind == "offset_view":        # per batch, rows 4 bytes off an 8-byte boundary
        wide = (rng.standard_normal(B * n + 1) * 3).astype(np.float32)
        mask = wide[1:].reshape(B, 1, 1, n)
        mask_dev = torch.from_numpy(wide).cuda()[1:].view(B, 1, 1, n)
    elif mask_kind == "scalar":
        mask = np.array([-3.0], np.float32)
    elif mask_kind == "strided":
        wide = (rng.standard_normal((1, 1, 1, 2 * n)) * 0.5).astype(np.float32)
        mask = wide[..., ::2]
        mask_dev = torch.from_numpy(wide).cuda()[..., ::2]
    else:
        mask = None
    want = _oracle(x, mask)
    if mask is not None and mask_dev is None:
        mask_dev = torch.from_numpy(np.ascontiguousarray(mask)).cuda()
    got = gpu_runtime.softmax(torch.from_numpy(x).cuda(), mask_dev, -1)
    assert_same(got.cpu().numpy(), want, f"softmax n={n} mask={mask_kind}")


@pytest.mark.parametrize("n", [510, 512])
def test_register_softmax_quotients_across_the_float_range(gpu_runtime, n):
    """Rows whose exponentials span every regime of the float32 quotient:
    values near the row maximum, tiny ones below 2^-60 (which the kernel
    divides in double), subnormal ones, exact zeros, and rows of equal
    values (a denominator of n)."""
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((6, 40, n)) * 2).astype(np.float32)
    x[0] = rng.uniform(-110.0, 0.0, (40, n)).astype(np.float32)      # exps from 1 down to subnormal and 0
    x[1] = rng.uniform(-45.0, 0.0, (40, n)).astype(np.float32)       # around 2^-60
    x[2, :, :] = 3.0                                                  # denominator n, every quotient 1 / n
    x[3, ::2, ::7] = -95.0                                            # a few subnormal exps per row
    x[4] = (rng.standard_normal((40, n)) * 20).astype(np.float32)    # wide logits
    x[5, :, n // 2:] = -1e30                                          # half the row exactly zero
    got = gpu_runtime.softmax(torch.from_numpy(x).cuda(), None, -1)
    assert_same(got.cpu().numpy(), _oracle(x, None), f"softmax n={n} across the float range")


def test_misaligned_rows_take_the_staged_kernel(gpu_runtime):
    rng = np.random.default_rng(9)
    n = 510
    x = (rng.standard_normal((2, 12, n)) * 2).astype(np.float32)
    base = torch.from_numpy(np.concatenate([np.zeros(1, np.float32), x.reshape(-1)])).cuda()
    xv = base[1:].view(2, 12, n)
    assert xv.data_ptr() % 8 == 4
    got = gpu_runtime.softmax(xv, None, -1)
    assert_same(got.cpu().numpy(), _oracle(x, None), "softmax of a 4-byte-offset input")


def _oracle_ln(x, skip, bias, gamma, beta, eps):
    env = {"x": x, "g": gamma}
    if skip is not None:
        env.update({"s": skip})
        ins = ["x", "s", "g", "b" if beta is not None else "", "bi" if bias is not None else ""]
        op, at = "SkipLayerNormalization", {"epsilon": eps}
    else:
        ins = ["x", "g"] + (["b"] if beta is not None else [])
        op, at = "LayerNormalization", {"epsilon": eps, "axis": -1}
    if beta is not None:
        env["b"] = beta
    if bias is not None:
        env["bi"] = bias
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes([(op, ins, ["y"], at)], env)
    return env["y"]


@pytest.mark.parametrize("variant", ["plain", "beta", "skip_bias", "skip_nobias", "f16_params", "specials", "scales"])
def test_register_layernorm_768(gpu_runtime, variant):
    """Rows of 768 values, enough of them (2400) for the warp-per-row path,
    which holds them in registers."""
    rng = np.random.default_rng(len(variant))
    x = (rng.standard_normal((4, 600, 768)) * 2 + 0.5).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 768).astype(np.float32)
    beta = (rng.standard_normal(768) * 0.1).astype(np.float32) if variant != "plain" else None
    skip = bias = None
    eps = 1e-12 if variant.startswith("skip") else 1e-5
    if variant.startswith("skip"):
        skip = rng.standard_normal(x.shape).astype(np.float32)
        bias = (rng.standard_normal(768) * 0.1).astype(np.float32) if variant == "skip_bias" else None
    if variant == "f16_params":
        gamma, beta = gamma.astype(np.float16), beta.astype(np.float16)
    if variant == "specials":
        x[0, 0, 3] = np.nan
        x[0, 1, :] = 7.0                 # zero variance: (x - mu) / sqrt(eps)
        x[1, 2, 5] = np.inf
        x[2, 3, 100] = 1e30
    if variant == "scales":
        # deviations and deviations over sd outside the float32 quotient's
        # window [2^-60, 2^60) (divided in double), inside it, and exactly zero
        x[0, :50] *= np.float32(1e-25)
        x[0, 50:100] *= np.float32(1e25)
        x[0, 100:150] *= np.float32(1e-12)
        x[1, :50, ::3] = 0.5
        x[1, 50:100] = np.float32(2.0) ** rng.integers(-70, 70, (50, 768)).astype(np.float32)
        x[2, :20] = np.float32(3.0)
    want = _oracle_ln(x, skip, bias, gamma, beta, eps)
    d = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()   # noqa: E731
    got = gpu_runtime.layernorm(d(x), d(skip), d(bias), d(gamma), d(beta), -1, eps)
    assert_same(got.cpu().numpy(), want, f"layernorm 768 {variant}")

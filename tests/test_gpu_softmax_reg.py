"""Softmax over rows of 510 and 512 values (ALBERT's attention rows), which
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
@pytest.mark.parametrize("mask_kind", ["row_const", "per_batch", "scalar", "strided", "none"])
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


def test_misaligned_rows_take_the_staged_kernel(gpu_runtime):
    rng = np.random.default_rng(9)
    n = 510
    x = (rng.standard_normal((2, 12, n)) * 2).astype(np.float32)
    base = torch.from_numpy(np.concatenate([np.zeros(1, np.float32), x.reshape(-1)])).cuda()
    xv = base[1:].view(2, 12, n)
    assert xv.data_ptr() % 8 == 4
    got = gpu_runtime.softmax(xv, None, -1)
    assert_same(got.cpu().numpy(), _oracle(x, None), "softmax of a 4-byte-offset input")

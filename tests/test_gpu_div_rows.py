"""Div by a divisor that is constant along each row (AdaIN's d / sd, a
[B, C, T] / [B, C, 1] broadcast): the row kernel divides through the
divisor's double reciprocal, RN32(RN64(x * r)), which must equal numpy's
float32 quotient for every x and b, special values included."""
import warnings

import numpy as np
import pytest
import torch

from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout", ["rows", "scalar"])
def test_div_by_row_constant_is_numpy_exact(gpu_runtime, layout):
    rng = np.random.default_rng(31)
    R, T = 700, 1024
    x = (rng.standard_normal((R, T)) * 10.0 ** rng.integers(-30, 30, (R, 1))).astype(np.float32)
    x[0, :8] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -3e-39, 3.4e38]
    if layout == "rows":
        b = (rng.standard_normal((R, 1)) * 10.0 ** rng.integers(-38, 38, (R, 1))).astype(np.float32)
        b[:12, 0] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -2e-40, 3.4e38, 1.0, -1.0, 3.0, 1e-38]
    else:
        b = np.array([[3.0]], np.float32)
    env = {"x": x, "b": b}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().dispatch("Div", ["x", "b"], ["y"], {}, env)
        genv = {"x": torch.from_numpy(x).cuda(), "b": torch.from_numpy(b).cuda()}
        gpu_runtime.dispatch("Div", ["x", "b"], ["y"], {}, genv)
    assert_same(genv["y"].cpu().numpy(), env["y"], f"Div {layout}")

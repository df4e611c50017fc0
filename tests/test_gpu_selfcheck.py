"""The fast division inside the device exp and sigmoid, checked on every
float32 input.

numpy's float32 exp ends with the IEEE quotient P5(r) / Q2(r) and the
Sigmoid op with 1 / (1 + exp(-x)).  The device routines compute both
quotients with Markstein's division (a reciprocal approximation refined by
Newton-Raphson, then one FMA residual correction).  bt_selfcheck runs each
routine over all 2^32 bit patterns beside the same routine with IEEE
division and counts the inputs whose results differ in any bit; the op tests
pin the IEEE forms to numpy, so zero mismatches make the fast routines
numpy-exact on every input.  Division by a per-row constant (softmax, layer
and instance norms) multiplies in double by a reciprocal formed by Newton-
Raphson steps; the check holds it within one double ulp of IEEE's 1/x on
every float, the bound under which RN32(RN64(a * (1/b))) is RN32(a/b).
Tanh is the library's own double evaluation; the check holds it within one
float ulp of the correctly rounded tanh on every input (numpy's float32 tanh
is within one ulp of that too, so the two stay within the 2-ulp bound of the
op tests).  DynamicQuantizeLinear's float32 shortcut (a reciprocal product,
with the exact double quotient near half-integers) must equal the exact path
on every input at each of eight scales.  Division by a per-row constant in
float32 alone (the correctly rounded reciprocal's product, corrected by one
FMA residual step) must give the correctly rounded quotient on all 2^46
pairs of significands, which covers every dividend and divisor inside the
window where the kernels use it."""
import ctypes

import pytest
import torch

from bt_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,name", [(0, "exp"), (1, "exp, two lanes"), (2, "sigmoid"),
                                       (3, "double reciprocal of a row constant"), (4, "sigmoid, two lanes"),
                                       (5, "tanh within one ulp of the correctly rounded value"),
                                       (6, "quantize shortcut against the exact quotient")])
def test_fast_division_equals_ieee_on_every_input(lib, kind, name):
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    _lib.check(lib.bt_selfcheck(kind, 0, 1 << 32, ctypes.c_void_p(count.data_ptr())), "bt_selfcheck")
    torch.cuda.synchronize()
    assert int(count.item()) == 0, f"{name}: {int(count.item())} inputs differ from IEEE division"


def test_row_division_in_float32_is_correctly_rounded_on_every_significand_pair(lib):
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    chunk = 1 << 20
    for first in range(0, 1 << 23, chunk):
        _lib.check(lib.bt_selfcheck(7, first, chunk, ctypes.c_void_p(count.data_ptr())), "bt_selfcheck")
    torch.cuda.synchronize()
    assert int(count.item()) == 0, f"{int(count.item())} (dividend, divisor) pairs differ from RN(a / b)"

"""CPU checks of the arithmetic identities the kernels rely on."""
import numpy as np


def test_division_by_shared_divisor_via_double_reciprocal_is_exact():
    """RN32(RN64(a * RN64(1/b))) == RN32(a / b): the row kernels divide by a
    per-row constant (sd, the softmax denominator, 3) this way.  Random bit
    patterns (all exponents, subnormals, specials) plus all-ones and
    near-power-of-two divisors."""
    rng = np.random.default_rng(2024)
    n = 4_000_000
    a = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    b = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    b[: n // 4] = (rng.integers(1, 254, n // 4).astype(np.uint32) << 23 | 0x7FFFFF).view(np.float32)
    b[n // 4: n // 2] = (rng.integers(1, 254, n // 4).astype(np.uint32) << 23
                         | rng.integers(0, 16, n // 4).astype(np.uint32)).view(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, 3.4e38, 1.0, 3.0], np.float32)
    a[:81] = np.repeat(special, 9)
    b[:81] = np.tile(special, 9)
    with np.errstate(all="ignore"):
        want = a / b
        got = (a.astype(np.float64) * (1.0 / b.astype(np.float64))).astype(np.float32)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), list(zip(a[~same][:5], b[~same][:5]))

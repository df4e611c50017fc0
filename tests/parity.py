"""Comparison helpers for parity tests (bit-exact and ulp-bounded)."""
import numpy as np


def _as_np(x):
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().cpu().numpy()
    except ImportError:
        pass
    return np.asarray(x)


def assert_same(got, want, what=""):
    """Same dtype, shape and bits (all NaNs count as equal)."""
    got, want = _as_np(got), _as_np(want)
    assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} != {want.dtype}"
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    if got.dtype.kind == "f":
        g = got.view(f"u{got.dtype.itemsize}")
        w = want.view(f"u{want.dtype.itemsize}")
        bad = (g != w) & ~(np.isnan(got) & np.isnan(want))
    else:
        bad = got != want
    if bad.any():
        idx = np.argwhere(bad)[:5]
        ex = [(tuple(i), got[tuple(i)].item(), want[tuple(i)].item()) for i in idx]
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.size} elements differ, e.g. {ex}")


def ulp_distance(a, b):
    """Distance in units in the last place between float arrays of one dtype
    (NaN vs NaN = 0, NaN vs number = huge)."""
    a, b = _as_np(a), _as_np(b)
    assert a.dtype == b.dtype and a.dtype.kind == "f"
    it = {2: np.int16, 4: np.int32, 8: np.int64}[a.dtype.itemsize]
    wide = np.int64
    ia = a.view(it).astype(wide)
    ib = b.view(it).astype(wide)
    top = np.iinfo(it).min
    ia = np.where(ia < 0, top - ia, ia)
    ib = np.where(ib < 0, top - ib, ib)
    d = np.abs(ia - ib)
    both_nan = np.isnan(a) & np.isnan(b)
    one_nan = np.isnan(a) ^ np.isnan(b)
    d = np.where(both_nan, 0, d)
    return np.where(one_nan, np.iinfo(wide).max, d)


def assert_ulp(got, want, max_ulp, what=""):
    got, want = _as_np(got), _as_np(want)
    assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} != {want.dtype}"
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    d = ulp_distance(got, want)
    if d.size and d.max() > max_ulp:
        i = np.unravel_index(int(np.argmax(d)), d.shape)
        raise AssertionError(f"{what}: max {int(d.max())} ulp > {max_ulp} at {i}: {got[i]} vs {want[i]}")

"""numpy's memory-layout rules as the GPU runtime models them, checked
against numpy itself on the CPU.

The reference keeps Transpose outputs as views and numpy allocates element-
wise results in order 'K', and numpy's float32 sums depend on that layout
(pairwise along the innermost axis in memory, slice after slice along outer
ones).  The runtime predicts the layout with ``_k_order`` and reduces a view
as its physical tensor over the mapped axes; both are pinned here."""
import itertools

import numpy as np
import pytest

from bt_b200.runtime import _inverse, _k_order


def _layouts(rng, shape):
    """Dense arrays of `shape` in every axis order (views of permuted buffers)."""
    nd = len(shape)
    for order in itertools.permutations(range(nd)):
        phys = rng.standard_normal([shape[a] for a in order]).astype(np.float32)
        yield order, phys.transpose(_inverse(list(order)))


def _mem_order(a):
    """Axes of size > 1, outermost in memory first."""
    return [i for i in sorted(range(a.ndim), key=lambda i: -a.strides[i]) if a.shape[i] > 1]


@pytest.mark.parametrize("shape", [(2, 3, 4), (1, 9, 5), (3, 1, 4, 2), (6, 7)])
def test_k_order_predicts_numpy_ufunc_layout(shape):
    rng = np.random.default_rng(len(shape))
    views = list(_layouts(rng, shape))
    for (_, a), (_, b) in itertools.product(views, views[:3]):
        for other in (b, b[..., :1], np.float32(2.0) * np.ones(shape[-1:], np.float32)):
            out = a + other
            order = _k_order([a, other], out.shape)
            want = _mem_order(out)
            assert [i for i in order if out.shape[i] > 1] == want, (a.strides, np.shape(other))


def test_k_order_of_a_transposed_view():
    x = np.zeros((1, 512, 9), np.float32).transpose(0, 2, 1)
    assert _k_order([x], x.shape)[1:] == [2, 1]
    assert _k_order([np.zeros((2, 3), np.float32)], (2, 3)) == [0, 1]


@pytest.mark.parametrize("shape,axes", [((1, 9, 512), (2,)), ((4, 6, 130), (2,)), ((4, 6, 130), (1,)),
                                        ((3, 5, 7, 11), (2, 3)), ((3, 5, 7, 11), (1,)), ((8, 300), (1,))])
def test_view_sums_equal_physical_sums(shape, axes):
    """numpy's sum over a view = its sum over the physical array with the
    axes mapped (the identity the GPU runtime's reductions rely on)."""
    rng = np.random.default_rng(7)
    for order, view in _layouts(rng, shape):
        phys = np.ascontiguousarray(view.transpose(order))
        paxes = tuple(sorted(list(order).index(a) for a in axes))
        want = view.sum(axis=axes, keepdims=True)
        got = phys.sum(axis=paxes, keepdims=True).transpose(_inverse(list(order)))
        assert got.tobytes() == np.ascontiguousarray(want).tobytes(), order
        assert want.mean() == want.mean()   # finite
    # and the layout does change the sum: the transposed LayerNorm input
    v = (rng.standard_normal((1, 512, 9)) * 3).astype(np.float32).transpose(0, 2, 1)
    c = np.ascontiguousarray(v)
    assert (v.sum(axis=2) != c.sum(axis=2)).any()

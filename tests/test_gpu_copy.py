"""Transpose, Concat, Slice and Expand through the op table (BtRuntime):
strided views copied by the library's IDENTITY kernel, bit for bit against
the oracle at sizes past the small golden cases -- the generator's [B, C, T]
layouts, every permutation of a rank-4 tensor, negative steps (negative
strides), the reference's empty full reversal, fp16 widening in Concat and
integer promotion."""
import itertools
import warnings

import numpy as np
import pytest
import torch

from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu


def _both(rt, nodes, env):
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        want = OracleRuntime().run_nodes(nodes, dict(env))
    got = dict(env)
    rt.run_nodes(nodes, got)
    torch.cuda.synchronize()
    return got, want


def test_all_rank4_permutations(gpu_runtime):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 4, 5, 6)).astype(np.float32)
    for perm in itertools.permutations(range(4)):
        got, want = _both(gpu_runtime, [("Transpose", ["x"], ["y"], {"perm": list(perm)})], {"x": x})
        assert_same(got["y"], want["y"], f"perm {perm}")


@pytest.mark.parametrize("shape,perm", [((2, 256, 4000), [0, 2, 1]), ((1, 510, 768), [0, 2, 1]),
                                        ((12, 510, 64), [1, 0, 2]), ((4, 37, 3, 5), [3, 1, 0, 2])])
def test_large_transposes(gpu_runtime, shape, perm):
    rng = np.random.default_rng(len(shape) + shape[-1])
    for dt in (np.float32, np.float16, np.int64):
        x = (rng.standard_normal(shape) * 5).astype(dt)
        got, want = _both(gpu_runtime, [("Transpose", ["x"], ["y"], {"perm": perm})], {"x": x})
        assert_same(got["y"], want["y"], f"{shape} {perm} {dt}")


def test_concat(gpu_runtime):
    rng = np.random.default_rng(2)
    env = {"a": rng.standard_normal((2, 128, 1000)).astype(np.float32),
           "b": rng.standard_normal((2, 64, 1000)).astype(np.float16),
           "c": rng.standard_normal((2, 3, 1000)).astype(np.float32),
           "i": rng.integers(-9, 9, (5, 7)).astype(np.int32), "j": rng.integers(-9, 9, (5, 2)).astype(np.int64)}
    nodes = [("Concat", ["a", "b", "c"], ["y"], {"axis": 1}), ("Concat", ["a", "c"], ["z"], {"axis": -2}),
             ("Concat", ["i", "j"], ["w"], {"axis": 1}), ("Concat", ["a", "a"], ["v"], {"axis": 2})]
    got, want = _both(gpu_runtime, nodes, env)
    for k in ("y", "z", "w", "v"):
        assert_same(got[k], want[k], f"concat {k}")


@pytest.mark.parametrize("starts,ends,axes,steps", [
    ([5], [-5], [2], None), ([0, 3], [2, 100], [0, 1], [1, 7]), ([-1], [-(1 << 62)], [2], [-1]),
    ([3999], [0], [2], [-3]), ([100], [10], [1], [-1]), ([-2, 1], [0, 5], [-1, -3], [-1, 2])])
def test_slices(gpu_runtime, starts, ends, axes, steps):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 256, 4000)).astype(np.float32)
    i64 = lambda v: np.array(v, np.int64)   # noqa: E731
    env = {"x": x, "s": i64(starts), "e": i64(ends), "a": i64(axes)}
    ins = ["x", "s", "e", "a"]
    if steps is not None:
        env["p"] = i64(steps)
        ins.append("p")
    got, want = _both(gpu_runtime, [("Slice", ins, ["y"], {})], env)
    assert_same(got["y"], want["y"], f"slice {starts} {ends} {axes} {steps}")


def test_expand(gpu_runtime):
    rng = np.random.default_rng(4)
    env = {"x": rng.standard_normal((256, 1)).astype(np.float32), "h": rng.standard_normal((1, 4000)).astype(np.float16),
           "s1": np.array([2, 256, 4000], np.int64), "s2": np.array([3, 1, 1], np.int64)}
    nodes = [("Expand", ["x", "s1"], ["y"], {}), ("Expand", ["h", "s2"], ["z"], {})]
    got, want = _both(gpu_runtime, nodes, env)
    assert_same(got["y"], want["y"], "expand fp32")
    assert_same(got["z"], want["z"], "expand fp16")


@pytest.mark.parametrize("shape,perm", [((2, 256, 4000), [0, 2, 1]), ((1, 510, 768), [0, 2, 1]), ((3, 33, 70), [0, 2, 1]),
                                        ((64, 40), [1, 0]), ((5, 96, 128), [0, 2, 1]), ((12, 510, 64), [1, 0, 2]),
                                        ((4, 37, 3, 5), [3, 1, 0, 2]), ((2, 8, 9), [0, 2, 1])])
def test_transpose_kernel(gpu_runtime, shape, perm):
    """The materialising transpose (BtRuntime.transpose: the tiled copy
    kernel), every element width, full and edge tiles, the 128-bit path
    (4-byte elements, aligned) and its scalar fallback (a start or a stride
    off the 16-byte grid)."""
    rng = np.random.default_rng(sum(shape))
    for dt in (np.float32, np.int32, np.float16, np.int64, np.uint8):
        x = (rng.standard_normal(shape) * 50).astype(dt)
        xd = torch.from_numpy(x).cuda()
        got = gpu_runtime.transpose(xd, perm)
        assert got.is_contiguous()
        assert_same(got.cpu().numpy(), np.ascontiguousarray(np.transpose(x, perm)), f"{shape} {perm} {dt}")
    # start one element off a 16-byte boundary, and an odd row stride
    x = rng.standard_normal(shape).astype(np.float32)
    buf = torch.empty(x.size + 1, device="cuda")
    off = buf[1:].view(shape)
    off.copy_(torch.from_numpy(x))
    assert_same(gpu_runtime.transpose(off, perm).cpu().numpy(), np.ascontiguousarray(np.transpose(x, perm)), "offset")
    wide = torch.from_numpy(np.concatenate([x, x[..., :1]], axis=-1)).cuda()[..., : shape[-1]]
    assert_same(gpu_runtime.transpose(wide, perm).cpu().numpy(), np.ascontiguousarray(np.transpose(x, perm)), "stride")

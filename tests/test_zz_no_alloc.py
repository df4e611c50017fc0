"""bt_dynamic_quantize_noalloc: DynamicQuantizeLinear for callers that cannot
allocate device memory while they run (an engine that hands a plugin only
buffers from its own pool, a serving process whose memory budget is fixed
before the first request, a real-time loop where an allocation could stall
or fail mid-frame).  The variant keeps its scratch in a static device array
instead of memory it allocates; its results must equal bt_dynamic_quantize's
and the numpy oracle's bit for bit.  Two calls in a row with different ranges
show the shared scratch record is cleared between calls.

The inputs cover every route through the shared record: float32 above 2^17
values (the two-pass path with 128-bit loads), float16 (scalar loads at any
size) and a float32 view 4 bytes past an aligned address (scalar loads
again).  Smaller aligned float32 inputs take the one-cluster path, which
needs no scratch record at all.

This file is collected last (its name), so a run that stops at the first
failure has already run every other test; it also passes alone in a fresh
process."""
import ctypes

import numpy as np
import pytest
import torch

from parity import assert_same

pytestmark = pytest.mark.gpu


def _desc(t):
    from bt_b200._lib import make_tensor
    from bt_b200.runtime import np_dtype
    return make_tensor(t.data_ptr(), np_dtype(t), tuple(t.shape), tuple(t.stride()))


def _quantize(lib, fn, x):
    from bt_b200._lib import check
    y = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    sc = torch.empty((), dtype=torch.float32, device=x.device)
    zp = torch.empty((), dtype=torch.uint8, device=x.device)
    check(getattr(lib, fn)(ctypes.byref(_desc(x)), ctypes.byref(_desc(y)), ctypes.c_void_p(sc.data_ptr()),
                           ctypes.c_void_p(zp.data_ptr())), fn)
    return y, sc, zp


def _oracle(xh):
    from oracle import OracleRuntime
    env = {"x": xh}
    OracleRuntime().dispatch("DynamicQuantizeLinear", ["x"], ["y", "s", "z"], {}, env)
    return env["y"], env["s"], env["z"]


def _inputs():
    rng = np.random.default_rng(2024)
    return [
        ("f32 mixed signs", (rng.standard_normal((3, 512, 1001)) * 3.0 + 1.0).astype(np.float32), 0),
        ("f32 positive, narrower range", rng.uniform(0.25, 0.75, (2, 300_001)).astype(np.float32), 0),
        ("f16", (rng.standard_normal((4, 2500)) * 5.0 - 2.0).astype(np.float16), 0),
        ("f32 view at a 4-byte offset", (rng.standard_normal(70_001) * 0.5 - 4.0).astype(np.float32), 1),
    ]


def test_noalloc_equals_allocating_entry_point_and_oracle_on_consecutive_calls(lib):
    from bt_b200._lib import check
    torch.cuda.set_device(0)
    check(lib.bt_init(0), "bt_init")
    check(lib.bt_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "bt_set_stream")
    for what, xh, offset in _inputs():
        if offset:
            base = torch.from_numpy(np.concatenate([np.zeros(offset, xh.dtype), xh])).cuda()
            x = base[offset:]
            assert x.data_ptr() % 16 != 0
        else:
            x = torch.from_numpy(xh).cuda()
        got = _quantize(lib, "bt_dynamic_quantize_noalloc", x)
        want = _quantize(lib, "bt_dynamic_quantize", x)
        torch.cuda.synchronize()
        assert torch.equal(got[1].view(torch.int32), want[1].view(torch.int32)), f"{what}: scale"
        assert torch.equal(got[2], want[2]), f"{what}: zero point"
        assert torch.equal(got[0], want[0]), f"{what}: values"
        y, s, z = _oracle(xh)
        assert_same(got[0].cpu().numpy(), y, f"{what}: values vs oracle")
        assert_same(got[1].cpu().numpy(), np.asarray(s), f"{what}: scale vs oracle")
        assert_same(got[2].cpu().numpy(), np.asarray(z), f"{what}: zero point vs oracle")

"""bt_dynamic_quantize_noalloc: DynamicQuantizeLinear for callers that cannot
allocate device memory while they run (an engine that hands a plugin only
buffers from its own pool, a serving process whose memory budget is fixed
before the first request, a real-time loop where an allocation could stall
or fail mid-frame).  The variant keeps its scratch in a static device array
instead of memory it allocates; its results must equal bt_dynamic_quantize's
bit for bit.  Two calls in a row with different ranges show the shared
scratch record is cleared between calls.

This file is collected last (its name), so a run that stops at the first
failure has already run every other test; it also passes alone in a fresh
process."""
import ctypes

import numpy as np
import pytest
import torch

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


def test_noalloc_equals_allocating_entry_point_on_two_calls(lib):
    from bt_b200._lib import check
    torch.cuda.set_device(0)
    check(lib.bt_init(0), "bt_init")
    check(lib.bt_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "bt_set_stream")
    rng = np.random.default_rng(2024)
    inputs = [(rng.standard_normal((3, 512, 1001)) * 3.0 + 1.0).astype(np.float32),   # mixed signs
              rng.uniform(0.25, 0.75, (2, 300_001)).astype(np.float32)]               # positive, a narrower range
    # (both above 2^17 values: smaller inputs take the one-cluster path, which
    # needs no scratch record at all)
    for k, xh in enumerate(inputs):
        x = torch.from_numpy(xh).cuda()
        got = _quantize(lib, "bt_dynamic_quantize_noalloc", x)
        want = _quantize(lib, "bt_dynamic_quantize", x)
        torch.cuda.synchronize()
        assert torch.equal(got[1].view(torch.int32), want[1].view(torch.int32)), f"call {k}: scale"
        assert torch.equal(got[2], want[2]), f"call {k}: zero point"
        assert torch.equal(got[0], want[0]), f"call {k}: values"

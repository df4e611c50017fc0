"""Whole-graph waveform parity: the reference's packed-model driver
(tools/kpk_runtime.py PackedModel.run, :52-81) on its own sample utterance
(voice_util.sample_tokens(9), voice af_heart), once with the reference's
numpy op table for every node and once with HybridRuntime in its place
(hot-path ops on the B200, every other op on the same numpy table).

Two runs through the GPU table:
  - every hot-path op whose kernels are bit-exact against numpy on the GPU,
    the four ops whose numpy results come from libm / vendor routines
    (Tanh, Atan, Erf inside FastGelu's tanh, FastGelu) on the CPU table: the
    waveform must be identical bit for bit;
  - every hot-path op on the GPU: those four ops are within 2 ulp of numpy,
    so the waveform may differ in its last bits; it must stay within
    1e-4 of the reference's peak amplitude.

This needs the reference's model and CPU ops, which are not part of this
repository: set BT_REFERENCE_CHECKOUT to a best-tts-godot checkout (it reads
tools/ref_runtime.py, kpk_runtime.py, voice_util.py, the packed model and the
af_heart voice).  Without it the test is skipped."""
import os
import sys
import warnings

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF = os.environ.get("BT_REFERENCE_CHECKOUT")
NOT_BIT_EXACT = {"Tanh", "Atan", "Erf", "FastGelu"}


@pytest.fixture(scope="module")
def reference():
    if not REF or not os.path.isdir(os.path.join(REF, "tools")):
        pytest.skip("BT_REFERENCE_CHECKOUT does not point at a best-tts-godot checkout")
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    from make_golden import import_reference
    ref_runtime, kpk_runtime = import_reference(REF)
    import voice_util
    pm = kpk_runtime.PackedModel()
    ids = voice_util.sample_tokens(9)
    style = voice_util.load_voice("af_heart", len(ids))
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        want = np.asarray(pm.run(ids, style))
    return ref_runtime, pm, ids, style, want


def _hybrid_run(reference, gpu_ops):
    """PackedModel.run with HybridRuntime taking every node: the run's own
    RefRuntime instance becomes its CPU table."""
    from bt_b200.hybrid import HybridRuntime
    from bt_b200.runtime import BtRuntime
    ref_runtime, pm, ids, style, _ = reference
    orig = ref_runtime.RefRuntime.dispatch
    gpu = BtRuntime(0)
    state = {}

    class Cpu:
        def __init__(self, rt):
            self.rt = rt

        def dispatch(self, op, ins, outs, at, env):
            return orig(self.rt, op, ins, outs, at, env)

    def routed(self, op, ins, outs, at, env):
        h = state.get(id(self))
        if h is None:
            h = state[id(self)] = HybridRuntime(Cpu(self), gpu_ops=gpu_ops, gpu_runtime=gpu)
            state["h"] = h
        return h.dispatch(op, ins, outs, at, env)

    ref_runtime.RefRuntime.dispatch = routed
    try:
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            out = pm.run(ids, style)
    finally:
        ref_runtime.RefRuntime.dispatch = orig
    h = state["h"]
    return h.result(out), h.stats


def test_waveform_bit_identical_with_exact_ops_on_the_gpu(reference):
    from bt_b200.runtime import BtRuntime
    want = reference[-1]
    ops = set(BtRuntime.HOT_OPS) - NOT_BIT_EXACT
    got, stats = _hybrid_run(reference, ops)
    assert stats["gpu_nodes"] > 3000
    assert got.dtype == want.dtype and got.shape == want.shape
    bad = got.view(np.uint32) != want.view(np.uint32)
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} samples differ, max |err| {np.abs(got - want).max()}"


def test_waveform_close_with_every_hot_op_on_the_gpu(reference):
    from bt_b200.runtime import BtRuntime
    want = reference[-1]
    got, stats = _hybrid_run(reference, set(BtRuntime.HOT_OPS))
    assert stats["gpu_nodes"] == 3442
    err = float(np.abs(got.astype(np.float64) - want).max())
    peak = float(np.abs(want).max())
    print(f"waveform: {want.size} samples, max |err| {err:.3e}, peak {peak:.3e}")
    assert err <= 1e-4 * peak

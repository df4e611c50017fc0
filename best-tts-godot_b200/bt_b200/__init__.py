"""B200 (sm_100a) tensor-op hot path of best-tts (Kokoro-82M).

Host side of the library: ``BtRuntime`` is the drop-in for the reference's
numpy op table (``RefRuntime.dispatch``), ``FusedDecoder`` runs the batched
decoder-stage op stream with row-fused kernels.  All arithmetic runs in
``libbt_ops.so`` (hand-written CUDA kernels behind a C ABI, include/bt_ops.h).
"""
from ._lib import load, BtError  # noqa: F401


def __getattr__(name):
    # torch-dependent parts are imported lazily so the C ABI binding can be
    # used (and tested) without initialising CUDA.
    if name in ("BtRuntime",):
        from .runtime import BtRuntime
        return BtRuntime
    if name in ("FusedDecoder", "build_stream"):
        from . import decoder
        return getattr(decoder, name)
    raise AttributeError(name)

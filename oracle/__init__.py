"""CPU oracle for the best-tts tensor-op hot path -- TEST INFRASTRUCTURE ONLY.

What this is
    A plain-numpy restatement of the semantics that the reference's numpy
    interpreter (``tools/ref_runtime.py`` in studio-ransom/best-tts-godot,
    ``RefRuntime.dispatch``, lines 428-668) gives to the elementwise,
    broadcast, reduction and dequantize ops that its graph executor runs for
    Kokoro-82M.  Every handler cites the reference line it follows.

Who may use it
    Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
    ``bench.py`` (``cpu_baseline`` and ``--impl reference``).  It is the
    checker, never the thing measured on the GPU and never shipped: the product
    package (``best-tts-godot_b200/bt_b200``) does not import it and fails
    loudly when its CUDA library is missing.

How it is pinned
    ``tests/golden/make_golden.py`` imports the reference interpreter itself
    (with a stub ``onnx`` module, the only missing import) and records its
    outputs on seeded inputs, including the literal vectors of the
    reference's own GPU kernel test (``tests/test_gpu_elementwise.gd``).
    ``tests/test_oracle_golden.py`` checks this module against those fixtures
    bit for bit.

Third-party arithmetic
    The arithmetic of the path lives in numpy (ufuncs ``exp``, ``sin``,
    ``tanh``, ``power``, ``add.reduce`` ...).  The reference pins no numpy
    version; the fixtures were produced with numpy 2.3.5 and record
    ``np.show_runtime()``'s SIMD dispatch next to them.
"""
from .ops import OracleRuntime, upcast, ONNX_TO_NUMPY, run_nodes_streaming  # noqa: F401

"""Generates the golden fixtures from the reference implementation itself.

    python tests/golden/make_golden.py [--reference /path/to/best-tts-godot]

Runs in a container that has the reference checkout (it is not needed, and not
read, anywhere else).  The reference's numpy interpreter
(tools/ref_runtime.py) imports ``onnx`` at module level (ref_runtime.py:15-16)
although the op table does not use it; a stub module is installed for the
import, which leaves ``RefRuntime.dispatch`` untouched.  The interpreter
instance is made the way the reference's own packed-model driver makes it
(kpk_runtime.py:53-56).

Writes, next to this script:
  golden_ops.npz   -- every case's reference outputs (cases.py) and the small
                      c5 decoder-stage stream's two stage outputs;
  golden_meta.json -- SHA-256 of every case input and of every large c5
                      intermediate (snake outputs, residuals), plus numpy's
                      version and SIMD dispatch on the generating host;
  generator_topology.json -- op-type sequences of the generator blocks in the
                      reference's packed model (assets/model.kpk), the source
                      of the c5 stream's topology.
"""
import argparse
import hashlib
import io
import json
import os
import sys
import types
import warnings
from contextlib import redirect_stdout

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(REPO, "best-tts-godot_b200"))

import cases as C  # noqa: E402


def sha(a):
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def import_reference(root):
    onnx = types.ModuleType("onnx")
    helper = types.ModuleType("onnx.numpy_helper")
    onnx.numpy_helper = helper
    onnx.AttributeProto = types.SimpleNamespace(INT=2, FLOAT=1, STRING=3, INTS=7, FLOATS=6, TENSOR=4)
    sys.modules.setdefault("onnx", onnx)
    sys.modules.setdefault("onnx.numpy_helper", helper)
    sys.path.insert(0, os.path.join(root, "tools"))
    import ref_runtime
    import kpk_runtime
    return ref_runtime, kpk_runtime


def reference_runtime(ref_runtime):
    rt = ref_runtime.RefRuntime.__new__(ref_runtime.RefRuntime)
    rt.quantized_lstm = False
    rt.fp16_boundaries = False
    rt.fp16_outputs = set()
    return rt


def run_nodes(rt, nodes, env):
    for op, ins, outs, at in nodes:
        rt.dispatch(op, list(ins), list(outs), dict(at), env)
    return env


def topology(kpk_runtime):
    """Op types, in packed-model order, of each generator block's hot-path
    nodes (the fc Linear, quantisation and conv epilogue nodes excluded)."""
    pm = kpk_runtime.PackedModel()
    names = pm.names
    blocks = [f"noise_res.{i}" for i in range(2)] + [f"resblocks.{i}" for i in range(6)]
    skip_ops = {"Cast", "DynamicQuantizeLinear", "ConvInteger", "MatMulInteger", "Reshape", "Unsqueeze",
                "Split", "Conv", "ConvTranspose"}
    seqs = {b: [] for b in blocks}
    stage_ops = {0: {}, 1: {}}
    for op_id, ins, outs, at, place in pm.nodes:
        op = pm.ops[op_id]
        out_names = [names[o] for o in outs if o >= 0]
        if not out_names:
            continue
        n0 = out_names[0]
        if op in skip_ops or "/fc/" in n0 or "/convs" in n0 or "quantized" in n0:
            continue
        for b in blocks:
            if f"/generator/{b}/" in n0:
                seqs[b].append(op)
    for b in blocks:
        idx = int(b.split(".")[1])
        stage = idx if b.startswith("noise_res") else idx // 3
        for op in seqs[b]:
            stage_ops[stage][op] = stage_ops[stage].get(op, 0) + 1
    return {"blocks": seqs, "stage_op_counts": {str(k): v for k, v in stage_ops.items()},
            "source": "assets/model.kpk nodes under /decoder/decoder/generator/"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BT_REFERENCE_CHECKOUT"),
                    required="BT_REFERENCE_CHECKOUT" not in os.environ,
                    help="path of a best-tts-godot checkout (or set BT_REFERENCE_CHECKOUT)")
    args = ap.parse_args()
    ref_runtime, kpk_runtime = import_reference(args.reference)
    rt = reference_runtime(ref_runtime)

    arrays, meta = {}, {"inputs": {}, "c5": {}, "numpy": np.__version__}
    buf = io.StringIO()
    with redirect_stdout(buf):
        np.show_runtime()
    meta["numpy_runtime"] = buf.getvalue()

    for case in C.cases():
        env = {k: np.array(v, copy=True) for k, v in case.env.items()}
        meta["inputs"][case.name] = {k: sha(v) for k, v in case.env.items()}
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            run_nodes(rt, case.nodes, env)
        for o in case.outputs:
            arrays[f"{case.name}/{o}"] = np.asarray(env[o])

    from bt_b200.decoder import build_stream
    S = build_stream(1, t0=8)
    env = C.c5_small_inputs(S)
    meta["c5"]["inputs"] = {k: sha(v) for k, v in env.items()}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        run_nodes(rt, S.nodes, env)
    for name in S.stage_outputs():
        arrays[f"c5/{name}"] = env[name]
    meta["c5"]["snakes"] = {n: sha(env[n]) for n in S.snake_names()}
    meta["c5"]["residuals"] = {n: sha(env[n]) for n in S.residual_names()}

    np.savez_compressed(os.path.join(HERE, "golden_ops.npz"), **arrays)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    with open(os.path.join(HERE, "generator_topology.json"), "w") as f:
        json.dump(topology(kpk_runtime), f, indent=1)
    print(f"{len(arrays)} arrays, {len(meta['inputs'])} cases")


if __name__ == "__main__":
    main()

"""The c5 stream builder against the reference's packed model.

generator_topology.json holds, per generator block of assets/model.kpk, the
op types of its elementwise / reduction nodes in graph order (extracted by
tests/golden/make_golden.py).  The stream the B200 path runs must have the
same op sequence per block and the same per-stage op counts.
"""
import json
import os

from bt_b200.decoder import build_stream, stream_launches

HERE = os.path.dirname(os.path.abspath(__file__))


def _topo():
    with open(os.path.join(HERE, "golden", "generator_topology.json")) as f:
        return json.load(f)


def _block_ops(S, block):
    ops = []
    for op, ins, outs, at in S.nodes:
        if op == "Split":
            continue
        if outs[0].startswith(f"G/{block}/"):
            ops.append(op)
    return ops


def test_block_sequences_match_packed_model():
    topo = _topo()
    S = build_stream(2, t0=16)
    for block, want in topo["blocks"].items():
        assert _block_ops(S, block) == want, block


def test_stage_op_counts_match_packed_model():
    topo = _topo()
    S = build_stream(1, t0=16)
    for stage in (0, 1):
        blocks = [f"noise_res.{stage}"] + [f"resblocks.{3 * stage + j}" for j in range(3)]
        counts = {}
        for b in blocks:
            for op in _block_ops(S, b):
                counts[op] = counts.get(op, 0) + 1
        assert counts == topo["stage_op_counts"][str(stage)]


def test_stream_shapes():
    S = build_stream(4, t0=400)
    assert [(st.C, st.T) for st in S.stages] == [(256, 4000), (128, 24001)]
    assert S.inputs["G/features"][0] == (4, 512, 400)
    assert stream_launches(S) == 49

"""The node-list fusion planner (bt_b200.chains.plan) on the CPU: which runs
of nodes it fuses in the c5 decoder stream, and that it never fuses away a
value that another node reads or that the caller keeps."""
from bt_b200 import chains
from bt_b200.decoder import build_stream


def test_c5_stream_snakes_and_affines_fuse():
    S = build_stream(2, t0=8)
    keep = set(S.stage_outputs())
    groups = chains.plan(S.nodes, keep)
    kinds = [g.kind for g in groups]
    # every AdaIN1d of both stages: its affine (Mul, Add) and its Snake
    assert kinds.count("snake") == 48
    assert kinds.count("mul_add") == 48
    for g in groups:
        ops = [S.nodes[i][0] for i in g.nodes]
        if g.kind == "snake":
            assert ops == ["Mul", "Sin", "Pow", "Mul", "Add"]
            x, alpha, p, inv = g.inputs
            assert alpha.endswith("alpha") and inv.endswith("inv_alpha") and p == "G/const/two"
        else:
            assert ops == ["Mul", "Add"]
        assert g.output == S.nodes[g.last][2][0]
    assert len({i for g in groups for i in g.nodes}) == sum(len(g.nodes) for g in groups)


def test_multiply_read_and_kept_values_are_not_fused():
    nodes = [("Add", ["x", "y"], ["s"], {}), ("Sigmoid", ["s"], ["z"], {})]
    assert [g.kind for g in chains.plan(nodes)] == ["add_sigmoid"]
    assert chains.plan(nodes, keep={"s"}) == []
    assert chains.plan(nodes + [("Mul", ["s", "s"], ["w"], {})]) == []
    dq = [("DequantizeLinear", ["q", "sc", "zp"], ["d"], {}), ("Mul", ["g", "d"], ["y"], {})]
    (g,) = chains.plan(dq)
    assert g.kind == "dequant_mul" and g.inputs == ["q", "sc", "g", "zp"] and g.output == "y"
    assert g.inputs_ok(["int8", "float32", "float16", "int8"])
    assert not g.inputs_ok(["int32", "float32", "float32", "int8"])
    assert not g.inputs_ok(["int8", "float32", "float64", "int8"])
    leaky = [("Add", ["x", "y"], ["s"], {}), ("LeakyRelu", ["s"], ["z"], {"alpha": 0.2})]
    (g,) = chains.plan(leaky)
    assert g.kind == "add_leaky" and abs(g.alpha - 0.2) < 1e-7

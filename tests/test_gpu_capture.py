"""A node list recorded as one CUDA graph (BtRuntime.capture_nodes) and
replayed: the outputs equal an eager run bit for bit, and a replay after new
input values are written in place recomputes them (the c5 stream's node
list at T0 = 8, every kernel kind of the element-wise and row paths)."""
import numpy as np
import pytest
import torch

from parity import assert_same

pytestmark = pytest.mark.gpu


def test_captured_node_list_replays_exactly(gpu_runtime):
    import cases as C
    from bt_b200.decoder import build_stream
    rt = gpu_runtime
    S = build_stream(2, t0=8)
    host = C.c5_small_inputs(S, seed=5)
    # activations on the device; the graph's constants (split sizes, axes,
    # alpha) stay numpy arrays, as a model's initializers do
    on_dev = lambda env: {k: (torch.from_numpy(np.ascontiguousarray(v)).cuda() if k in S.inputs else v)   # noqa: E731
                          for k, v in env.items()}
    dev = on_dev(host)
    cap = rt.capture_nodes(S.nodes, dev)
    out = cap.replay()
    torch.cuda.synchronize()
    eager = rt.run_nodes(S.nodes, dict(dev))
    for name in S.stage_outputs():
        assert_same(out[name].cpu().numpy(), eager[name].cpu().numpy(), f"replay {name}")
    # new input values, written in place, then replayed
    host2 = C.c5_small_inputs(S, seed=6)
    for k, v in host2.items():
        if isinstance(cap.env.get(k), torch.Tensor) and k in S.inputs:
            cap.env[k].copy_(torch.from_numpy(np.ascontiguousarray(v)).reshape(cap.env[k].shape))
    out = cap.replay()
    torch.cuda.synchronize()
    eager2 = rt.run_nodes(S.nodes, on_dev(host2))
    for name in S.stage_outputs():
        assert_same(out[name].cpu().numpy(), eager2[name].cpu().numpy(), f"replay 2 {name}")

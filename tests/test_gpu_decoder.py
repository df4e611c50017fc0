"""GPU parity of the fused kernels and of the batched decoder-stage stream.

Bit-exact against the oracle running the op-by-op chains of the packed graph
(every op of AdaIN1d + Snake, the residual Adds, the resblock mean and the
LeakyRelu are exact on both sides: numpy's pairwise means, numpy's float32
sin, IEEE division and square root), and against the reference's own
outputs for the small stream (tests/golden).
"""
import hashlib
import json
import os
import warnings

import numpy as np
import pytest
import torch

import cases as C
from oracle import OracleRuntime
from parity import assert_same

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a):
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def oracle_adain_snake(srcs, fc, alpha, inv, eps, snake=True):
    """The graph's op chain for one AdaIN1d (+ Snake), run by the oracle."""
    C_ = srcs[0].shape[1]
    env = {f"s{i}": s for i, s in enumerate(srcs)}
    env.update({"fc": fc, "ax": np.array([2], np.int64), "eps": eps, "one": np.array(1.0, np.float16),
                "two": np.array(2.0, np.float16), "alpha": alpha, "inv": inv,
                "split": np.array([C_, C_], np.int64)})
    nodes = [("Split", ["fc", "split"], ["gamma", "beta"], {"axis": 1}), ("Add", ["gamma", "one"], ["gain"], {})]
    h = "s0"
    for i in range(1, len(srcs)):
        nodes.append(("Add", [h, f"s{i}"], [f"h{i}"], {}))
        h = f"h{i}"
    nodes += [("ReduceMean", [h, "ax"], ["mu"], {"keepdims": 1}), ("Sub", [h, "mu"], ["d"], {}),
              ("Mul", ["d", "d"], ["d2"], {}), ("ReduceMean", ["d2", "ax"], ["var"], {"keepdims": 1}),
              ("Add", ["var", "eps"], ["ve"], {}), ("Sqrt", ["ve"], ["sd"], {}), ("Div", ["d", "sd"], ["n"], {}),
              ("Mul", ["gain", "n"], ["m"], {}), ("Add", ["m", "beta"], ["a"], {})]
    if snake:
        nodes += [("Mul", ["alpha", "a"], ["t"], {}), ("Sin", ["t"], ["s"], {}), ("Pow", ["s", "two"], ["p"], {}),
                  ("Mul", ["inv", "p"], ["q"], {}), ("Add", ["a", "q"], ["z"], {})]
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(nodes, env)
    return env[h], env["z" if snake else "a"]


@pytest.mark.parametrize("path", ["cluster", "one_cta"])
@pytest.mark.parametrize("B,Cc,T,n_src,snake", [
    (1, 8, 100, 1, True), (2, 16, 4000, 2, True), (1, 4, 24001, 3, True), (3, 5, 1023, 2, False),
    (1, 2, 7, 1, True), (2, 3, 129, 3, True), (1, 2, 2048, 1, False), (1, 3, 49152, 2, True),
    (2, 4, 24001, 1, True), (2, 4, 24001, 2, True), (1, 4, 7681, 3, False)])
def test_adain_snake_rows(gpu_runtime, monkeypatch, path, B, Cc, T, n_src, snake):
    """Both bt_adain_snake kernels: the cluster-split rows (default) and the
    one-CTA-per-row kernel (BT_ADAIN_ONE_CTA=1, the fallback for requests the
    cluster kernel does not cover)."""
    if path == "one_cta":
        monkeypatch.setenv("BT_ADAIN_ONE_CTA", "1")
    rt = gpu_runtime
    rng = np.random.default_rng(T + n_src)
    srcs = [(rng.standard_normal((B, Cc, T)) * 2).astype(np.float32) for _ in range(n_src)]
    fc = rng.standard_normal((B, 2 * Cc, 1)).astype(np.float32)
    alpha = rng.uniform(0.5, 1.5, (1, Cc, 1)).astype(np.float16)
    inv = (1.0 / alpha.astype(np.float64)).astype(np.float16)
    eps = np.array(1e-5, np.float16)
    h_want, z_want = oracle_adain_snake(srcs, fc, alpha, inv, eps, snake)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    fcd = d(fc[:, :, 0])
    gain = rt.elementwise("ADD", [fcd[:, :Cc], d(np.array(1.0, np.float16))], (B, Cc), np.float32, np.float32)
    res = torch.empty((B, Cc, T), dtype=torch.float32, device="cuda") if n_src > 1 else None
    out = rt.adain_snake([d(s) for s in srcs], gain, fcd[:, Cc:], np.float32(eps),
                         d(alpha.reshape(-1)) if snake else None, d(inv.reshape(-1)) if snake else None, res=res)
    torch.cuda.synchronize()
    assert_same(out[0], z_want, "adain/snake output")
    if res is not None:
        assert_same(res, h_want, "residual")


@pytest.mark.parametrize("path", ["cluster", "one_cta"])
@pytest.mark.parametrize("n_src", [1, 2])
def test_adain_snake_large_and_nonfinite_rows(gpu_runtime, monkeypatch, path, n_src):
    """Rows whose snake arguments leave numpy's sin reduction range (gain up
    to ~1e5, so alpha * y passes 117435.992 and takes the library fallback),
    plus rows holding a NaN or an Inf: the kernels' per-row range bound must
    fail for these and keep the checked sin, which still matches numpy."""
    if path == "one_cta":
        monkeypatch.setenv("BT_ADAIN_ONE_CTA", "1")
    rt = gpu_runtime
    rng = np.random.default_rng(77 + n_src)
    B, Cc, T = 2, 6, 3001
    srcs = [(rng.standard_normal((B, Cc, T)) * 2).astype(np.float32) for _ in range(n_src)]
    srcs[0][0, 1, 17] = np.nan
    srcs[0][1, 2, 2900] = np.inf
    fc = rng.standard_normal((B, 2 * Cc, 1)).astype(np.float32)
    fc[:, :Cc] *= np.float32(6.0e4)     # gamma, hence the gain, up to ~2e5
    alpha = rng.uniform(0.5, 1.5, (1, Cc, 1)).astype(np.float16)
    inv = (1.0 / alpha.astype(np.float64)).astype(np.float16)
    eps = np.array(1e-5, np.float16)
    h_want, z_want = oracle_adain_snake(srcs, fc, alpha, inv, eps, True)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    fcd = d(fc[:, :, 0])
    gain = rt.elementwise("ADD", [fcd[:, :Cc], d(np.array(1.0, np.float16))], (B, Cc), np.float32, np.float32)
    res = torch.empty((B, Cc, T), dtype=torch.float32, device="cuda") if n_src > 1 else None
    out = rt.adain_snake([d(s) for s in srcs], gain, fcd[:, Cc:], np.float32(eps), d(alpha.reshape(-1)),
                         d(inv.reshape(-1)), res=res)
    torch.cuda.synchronize()
    assert_same(out[0], z_want, "adain/snake output")
    if res is not None:
        assert_same(res, h_want, "residual")


@pytest.mark.parametrize("path", ["cluster", "one_cta"])
@pytest.mark.parametrize("n_src", [1, 2])
def test_adain_snake_rows_across_the_division_window(gpu_runtime, monkeypatch, path, n_src):
    """Rows whose deviations (h - mu) and standard deviations fall inside and
    outside the float32 division's window [2^-60, 2^60): tiny rows (1e-25,
    where sd is sqrt(eps)), huge rows (1e25: sd beyond the window), constant
    rows (every deviation exactly zero), rows with values exactly at the mean
    and rows spanning many binades."""
    if path == "one_cta":
        monkeypatch.setenv("BT_ADAIN_ONE_CTA", "1")
    rt = gpu_runtime
    rng = np.random.default_rng(91 + n_src)
    B, Cc, T = 2, 6, 3001
    srcs = [(rng.standard_normal((B, Cc, T)) * 2).astype(np.float32) for _ in range(n_src)]
    srcs[0][0, 0] *= np.float32(1e-25)
    srcs[0][0, 1] *= np.float32(1e25)
    srcs[0][0, 2] = np.float32(0.75)
    srcs[0][1, 0] = np.float32(2.0) ** rng.integers(-70, 70, T).astype(np.float32)
    srcs[0][1, 1, ::2] = np.float32(1.0)
    srcs[0][1, 1, 1::2] = np.float32(-1.0)
    for s_ in srcs[1:]:
        s_[0, :3] = 0.0                  # keep the planted rows as planted
        s_[1, :2] = 0.0
    fc = rng.standard_normal((B, 2 * Cc, 1)).astype(np.float32)
    alpha = rng.uniform(0.5, 1.5, (1, Cc, 1)).astype(np.float16)
    inv = (1.0 / alpha.astype(np.float64)).astype(np.float16)
    eps = np.array(1e-5, np.float16)
    h_want, z_want = oracle_adain_snake(srcs, fc, alpha, inv, eps, True)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    fcd = d(fc[:, :, 0])
    gain = rt.elementwise("ADD", [fcd[:, :Cc], d(np.array(1.0, np.float16))], (B, Cc), np.float32, np.float32)
    res = torch.empty((B, Cc, T), dtype=torch.float32, device="cuda") if n_src > 1 else None
    out = rt.adain_snake([d(s) for s in srcs], gain, fcd[:, Cc:], np.float32(eps), d(alpha.reshape(-1)),
                         d(inv.reshape(-1)), res=res)
    torch.cuda.synchronize()
    assert_same(out[0], z_want, "adain/snake output")
    if res is not None:
        assert_same(res, h_want, "residual")


def test_adain_three_outputs_share_norm(gpu_runtime):
    rt = gpu_runtime
    rng = np.random.default_rng(5)
    B, Cc, T = 2, 6, 777
    srcs = [rng.standard_normal((B, Cc, T)).astype(np.float32) for _ in range(3)]
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    fcs = [rng.standard_normal((B, 2 * Cc, 1)).astype(np.float32) for _ in range(3)]
    alphas = [rng.uniform(0.5, 1.5, (1, Cc, 1)).astype(np.float16) for _ in range(3)]
    invs = [(1.0 / a.astype(np.float64)).astype(np.float16) for a in alphas]
    gains, shifts = [], []
    for fc in fcs:
        f = d(fc[:, :, 0])
        gains.append(rt.elementwise("ADD", [f[:, :Cc], d(np.array(1.0, np.float16))], (B, Cc), np.float32, np.float32))
        shifts.append(f[:, Cc:])
    res = torch.empty((B, Cc, T), dtype=torch.float32, device="cuda")
    outs = rt.adain_snake([d(s) for s in srcs], gains, shifts, np.float32(np.float16(1e-5)),
                          [d(a.reshape(-1)) for a in alphas], [d(v.reshape(-1)) for v in invs], res=res)
    for k in range(3):
        h, z = oracle_adain_snake(srcs, fcs[k], alphas[k], invs[k], np.array(1e-5, np.float16))
        assert_same(outs[k], z, f"output {k}")
    assert_same(res, h, "residual")


def test_resblock_mean_leaky(gpu_runtime):
    from bt_b200 import _lib
    import ctypes
    rng = np.random.default_rng(9)
    n = 3 * 1000 + 3
    a = [rng.standard_normal(n).astype(np.float32) for _ in range(3)]
    b = [rng.standard_normal(n).astype(np.float32) for _ in range(3)]
    env = {f"a{i}": a[i] for i in range(3)}
    env.update({f"b{i}": b[i] for i in range(3)})
    env["three"] = np.array(3.0, np.float16)
    nodes = [("Add", ["a0", "b0"], ["o0"], {}), ("Add", ["a1", "b1"], ["o1"], {}), ("Add", ["a2", "b2"], ["o2"], {}),
             ("Add", ["o0", "o1"], ["m"], {}), ("Add", ["m", "o2"], ["m2"], {}), ("Div", ["m2", "three"], ["q"], {}),
             ("LeakyRelu", ["q"], ["y"], {"alpha": 0.009999999776482582})]
    OracleRuntime().run_nodes(nodes, env)
    for off in (0, 1):   # aligned and misaligned starts
        da = [torch.from_numpy(x).cuda() for x in a]
        db = [torch.from_numpy(x).cuda() for x in b]
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        lib = _lib.load()
        pa = (ctypes.c_void_p * 3)(*[t[off:].data_ptr() for t in da])
        pb = (ctypes.c_void_p * 3)(*[t[off:].data_ptr() for t in db])
        _lib.check(lib.bt_set_stream(torch.cuda.current_stream().cuda_stream), "stream")
        _lib.check(lib.bt_resblock_mean_leaky(pa, pb, n - off, 3.0, float(np.float32(0.01)), out[off:].data_ptr()),
                   "mean_leaky")
        torch.cuda.synchronize()
        assert_same(out[off:], env["y"][off:], f"offset {off}")


def _run_fused(S, host):
    from bt_b200.decoder import FusedDecoder
    dec = FusedDecoder(S)
    for name, t in dec.inputs.items():
        t.copy_(torch.from_numpy(np.ascontiguousarray(host[name])).reshape(t.shape))
    dec.launch()
    torch.cuda.synchronize()
    return dec


def test_fused_stream_matches_reference_golden(lib):
    """The small stream (B=1, T0=8) against the reference's own outputs."""
    from bt_b200.decoder import build_stream
    with np.load(os.path.join(HERE, "golden", "golden_ops.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    meta = json.load(open(os.path.join(HERE, "golden", "golden_meta.json")))
    S = build_stream(1, t0=8)
    host = C.c5_small_inputs(S)
    dec = _run_fused(S, host)
    for name in S.stage_outputs():
        assert_same(dec.out[name], arrays[f"c5/{name}"], name)
    assert {n: sha(dec.out[n].cpu().numpy()) for n in S.snake_names()} == meta["c5"]["snakes"]
    assert {n: sha(dec.out[n].cpu().numpy()) for n in S.residual_names()} == meta["c5"]["residuals"]


def test_fused_stream_full_length_matches_oracle(lib):
    """One utterance at the full c5 lengths (T = 4000 and 24001)."""
    from bt_b200.decoder import build_stream
    S = build_stream(1, t0=400)
    host = C.c5_small_inputs(S, seed=21)
    dec = _run_fused(S, host)
    env = dict(host)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(S.nodes, env)
    for name in S.stage_outputs() + S.residual_names() + S.snake_names()[::7]:
        assert_same(dec.out[name], env[name], name)


def test_op_by_op_dispatch_matches_fused(gpu_runtime):
    """The drop-in op table walking the node list equals the fused plan."""
    from bt_b200.decoder import build_stream
    S = build_stream(2, t0=40)
    host = C.c5_small_inputs(S, seed=3)
    dec = _run_fused(S, host)
    env = dict(host)
    gpu_runtime.run_nodes(S.nodes, env)
    torch.cuda.synchronize()
    for name in S.stage_outputs() + S.snake_names() + S.residual_names():
        assert_same(env[name], dec.out[name], name)


def test_full_batch_utterances_are_independent_and_exact(lib):
    """B = 64 at full length with GPU-drawn conv stand-ins; utterance 37 is
    recomputed alone by the oracle and must match its slice bit for bit."""
    from bt_b200.decoder import build_stream, FusedDecoder, fill_conv_standins, host_inputs, load_host_inputs
    S = build_stream(64, t0=400)
    dec = FusedDecoder(S)
    fill_conv_standins(dec, seed=2)
    load_host_inputs(dec, host_inputs(S, seed=4))
    dec.launch()
    torch.cuda.synchronize()
    u = 37
    S1 = build_stream(1, t0=400)
    env = {name: dec.inputs[name][u:u + 1].cpu().numpy() for name in S.inputs}
    env.update(S1.consts)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(S1.nodes, env)
    for name in S.stage_outputs():
        assert_same(dec.out[name][u:u + 1], env[name], name)
    for name in S.snake_names()[::11]:
        assert_same(dec.out[name][u:u + 1], env[name], name)


def test_cuda_graph_replay_matches_eager(lib):
    from bt_b200.decoder import build_stream, FusedDecoder
    S = build_stream(2, t0=40)
    host = C.c5_small_inputs(S, seed=8)
    dec = _run_fused(S, host)
    want = {n: dec.out[n].clone() for n in S.stage_outputs()}
    for n in S.stage_outputs():
        dec.out[n].zero_()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dec.launch()                       # warm-up on the side stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dec.launch()
    for n in S.stage_outputs():
        dec.out[n].zero_()
    g.replay()
    torch.cuda.synchronize()
    for n in S.stage_outputs():
        assert_same(dec.out[n], want[n], n)


def test_host_pipeline_matches_run_host(lib):
    """The overlapped host-buffer loop (HostPipeline: copies on side streams,
    ordered by events against the compute stream) returns, after several
    steps, exactly what the serial FusedDecoder.run_host returns."""
    from bt_b200.decoder import build_stream, FusedDecoder, fill_conv_standins, host_inputs, load_host_inputs
    S = build_stream(3, t0=40)
    dec = FusedDecoder(S)
    fill_conv_standins(dec, seed=11)
    load_host_inputs(dec, host_inputs(S, seed=12))
    hin, hout = dec.host_buffers()
    feat = S.stages[0].x_in
    hin[feat].copy_(dec.inputs[feat].cpu())
    for i, fc in enumerate(dec.fc_bufs):
        hin[f"fc{i}"].copy_(fc.cpu())
    dec.run_host(hin, hout)
    torch.cuda.synchronize()
    want = hout.clone()
    hout.zero_()
    pipe = dec.host_pipeline(hin, hout)
    for _ in range(4):
        pipe.step()
    pipe.finish()
    torch.cuda.synchronize()
    assert torch.equal(hout.view(torch.int32), want.view(torch.int32))


def test_zz_every_bulk_copy_completed(lib):
    """The AdaIN kernels stage rows with bulk copies behind bounded waits; a
    wait that gave up would have counted itself (none may have, after the
    fused-stream tests above)."""
    import ctypes
    from bt_b200 import _lib
    n = ctypes.c_uint32(99)
    _lib.check(lib.bt_wait_timeouts(ctypes.byref(n)), "bt_wait_timeouts")
    assert n.value == 0

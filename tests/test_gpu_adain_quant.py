"""AdaIN1d + Snake feeding DynamicQuantizeLinear with the range pass fused
into the producer (bt_adain_snake_range, then bt_dynamic_quantize_ranged),
bit for bit against the oracle's op-by-op chain followed by its
DynamicQuantizeLinear: the Snake outputs, the uint8 values, the scale and the
zero point.  Both AdaIN kernels (the cluster kernel folds the range into its
output pass; the one-CTA fallback runs a separate range pass), one to three
outputs, rows at every 4-byte phase (odd T), and rows holding a NaN (the
whole row's outputs turn NaN, so the record's NaN flag decides the scale)."""
import numpy as np
import pytest
import torch

from parity import assert_same
from test_gpu_decoder import oracle_adain_snake
from test_gpu_quant import _oracle as oracle_quantize

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(rt, B, Cc, T, n_src, n_out, snake, seed, nan=False):
    rng = np.random.default_rng(seed)
    srcs = [(rng.standard_normal((B, Cc, T)) * 2).astype(np.float32) for _ in range(n_src)]
    if nan:
        srcs[0][B - 1, Cc // 2, T // 3] = np.nan
    fcs = [rng.standard_normal((B, 2 * Cc, 1)).astype(np.float32) for _ in range(n_out)]
    alphas = [rng.uniform(0.5, 1.5, (1, Cc, 1)).astype(np.float16) for _ in range(n_out)]
    invs = [(1.0 / a.astype(np.float64)).astype(np.float16) for a in alphas]
    eps = np.array(1e-5, np.float16)
    gains, shifts = [], []
    for fc in fcs:
        f = _dev(fc[:, :, 0])
        gains.append(rt.elementwise("ADD", [f[:, :Cc], _dev(np.array(1.0, np.float16))], (B, Cc), np.float32,
                                    np.float32))
        shifts.append(f[:, Cc:])
    al = [_dev(a.reshape(-1)) for a in alphas] if snake else None
    iv = [_dev(v.reshape(-1)) for v in invs] if snake else None
    res = torch.empty((B, Cc, T), dtype=torch.float32, device="cuda") if n_src > 1 else None
    srcs_d = [_dev(s) for s in srcs]
    ranges = rt.range_records(n_out)
    ranges.fill_(0x5a5a5a5a)    # the call zeroes the records itself
    outs = rt.adain_snake(srcs_d, gains, shifts, np.float32(eps), al, iv, res=res, ranges=ranges)
    plain = rt.adain_snake(srcs_d, gains, shifts, np.float32(eps), al, iv)
    quant = [rt.dynamic_quantize(outs[k], range=ranges[k]) for k in range(n_out)]
    unfused = [rt.dynamic_quantize(outs[k]) for k in range(n_out)]
    torch.cuda.synchronize()
    for k in range(n_out):
        _, z = oracle_adain_snake(srcs, fcs[k], alphas[k], invs[k], eps, snake)
        assert_same(outs[k], z, f"output {k}")
        assert_same(plain[k], z, f"output {k} without the range")
        wy, wsc, wzp = oracle_quantize(z)
        y, sc, zp = (t.cpu().numpy() for t in quant[k])
        assert_same(sc, np.asarray(wsc), f"scale {k}")
        assert_same(zp, np.asarray(wzp), f"zero point {k}")
        assert_same(y, wy, f"values {k}")
        for a, b in zip(quant[k], unfused[k]):
            assert torch.equal(a, b)
        if nan:
            assert float(sc) == 1.0 and int(zp) == 0
    return ranges


@pytest.mark.parametrize("path", ["cluster", "one_cta"])
@pytest.mark.parametrize("B,Cc,T,n_src,n_out,snake", [
    (1, 8, 100, 1, 1, True), (2, 16, 4000, 2, 3, True), (1, 4, 24001, 3, 2, True), (3, 5, 1023, 2, 1, False),
    (1, 2, 7, 1, 1, True), (2, 3, 129, 3, 3, True), (1, 3, 49152, 2, 1, True), (4, 64, 1537, 1, 2, True)])
def test_fused_range_matches_unfused(gpu_runtime, monkeypatch, path, B, Cc, T, n_src, n_out, snake):
    if path == "one_cta":
        monkeypatch.setenv("BT_ADAIN_ONE_CTA", "1")
    _run(gpu_runtime, B, Cc, T, n_src, n_out, snake, seed=T * 7 + n_out)


@pytest.mark.parametrize("path", ["cluster", "one_cta"])
def test_fused_range_nan_row(gpu_runtime, monkeypatch, path):
    if path == "one_cta":
        monkeypatch.setenv("BT_ADAIN_ONE_CTA", "1")
    rec = _run(gpu_runtime, 2, 6, 3001, 2, 2, True, seed=11, nan=True)
    assert (rec[:, 2].cpu().numpy() != 0).all()


def test_fused_range_argument_errors(gpu_runtime):
    rt = gpu_runtime
    x = torch.zeros((1, 2, 8), device="cuda")
    g = torch.ones((1, 2), device="cuda")
    rec = rt.range_records(1)
    with pytest.raises(RuntimeError):
        rt.dynamic_quantize(torch.empty((0,), device="cuda"), range=rec[0])
    # a record not on a 16-byte boundary
    flat = torch.zeros(12, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError):
        rt.adain_snake([x], g, g, np.float32(1e-5), ranges=flat[1:9])

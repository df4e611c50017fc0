"""Benchmark: the batched Kokoro-82M decoder-stage op stream on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload: the ISTFTNet generator's elementwise /
broadcast / reduction op stream for ONE fixed batch of 64 utterances,
features [512, 400] -> stages [256, 4000] and [128, 24001], conv and fc
outputs as seeded stand-ins resident in HBM.  One step = the whole stream for
the batch (49 kernel launches per decoder).  With torchrun (N > 1) the batch
is split by utterance (64 / N per rank, shard.split_utterances; "scaling":
"strong"), every rank runs its share with no collective on the data path,
and the job's time is the max over ranks.  A rank with 2-32 utterances
splits them again over two FusedDecoders on two concurrent CUDA streams
(--streams), which keeps the GPU busy where one decoder's launches are too
small to.  At N > 1 the weak-scaling figure (64 utterances on every rank)
is reported beside it under "weak".

Printed (rank 0, one JSON line): utt/s of the whole batch from CUDA events
with inputs resident; ``e2e`` through FusedDecoder.host_pipeline with pinned
host buffers (features + fc outputs in, final stage output out, every step)
and ``e2e_limit``, which names what bounds it (the device step or the
device-to-host copy of the result); ``roofline`` for the dominant kernel
(bt_adain_snake) from per-launch CUDA events, taken in a second pass of the
same steps (events between launches would slow the timed one); ``cpu_baseline`` = the numpy
oracle on the host cores; ``per_op`` = each BASELINE op config c1-c4 (GB/s,
fraction of the measured HBM peak and of the nominal 8 TB/s) plus a >= 256 MB
sweep, each next to the oracle's single-core numpy time; ``clocks`` sampled
with nvidia-smi during the timed region.  ``--impl reference`` times the
oracle port (the reference's numpy op table, restated in oracle/) on the
host cores instead.
"""
import argparse
import json
import os
import subprocess
import sys
import time
import warnings

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [REPO, os.path.join(REPO, "best-tts-godot_b200")]

METRIC = "Kokoro decoder op-stream utt/s"
UNIT = "utt/s"
NOMINAL_HBM = 8000.0
DATA = ("synthetic: seeded N(0,1) features, fc outputs (from N(0,1) style vectors through seeded "
        "Linear(128->2C)) and conv-output stand-ins; seeded alpha ~ U(0.5,1.5)")


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def rank_batches(total, n):
    """Utterances of each rank when one batch of `total` is split over n GPUs."""
    from bt_b200 import shard
    return [shard.split_utterances(total, n, r)[1] for r in range(n)]


def config(args, n, groups=None):
    from bt_b200.decoder import stage_shapes
    per = rank_batches(args.batch, n)
    if groups is None:
        groups = stream_groups(max(per), getattr(args, "streams", 0))
    gpu_bytes = max(per) * 128 * (args.t0 * 60 + 1) * 4
    return {"workload": "c5: batched Kokoro-82M ISTFTNet decoder-stage op stream (BASELINE configs[4])",
            "global_batch": args.batch, "batch_per_gpu": max(per), "batch_split": per, "t0": args.t0,
            "stage_shapes": [[c, t] for (_, _, c, t) in stage_shapes(args.t0)],
            "parallelism": f"dp{n}: one batch of {args.batch} utterances split by utterance over {n} GPU(s) "
                           f"(strong scaling), no collective on the data path; {groups} concurrent stream(s) "
                           "per GPU, each over its share of the GPU's utterances",
            "streams_per_gpu": groups,
            "l2": "no flush needed: every step moves "
                  f"{75.6 * max(per) / 64:.1f} GB per GPU through HBM, far more than L2, so no step starts "
                  f"with the previous step's data cached (a stage-2 tensor is {gpu_bytes / 1e6:.0f} MB per GPU)",
            "launches_per_step": 49 * groups}


# ---------------------------------------------------------------------------
# CPU side: the oracle (numpy op table) on the host cores
# ---------------------------------------------------------------------------
def _oracle_utterance(args):
    t0, seed = args
    sys.path[:0] = [REPO, os.path.join(REPO, "best-tts-godot_b200")]
    import numpy as np  # noqa
    from bt_b200.decoder import build_stream
    from oracle import OracleRuntime, run_nodes_streaming
    S = build_stream(1, t0=t0)
    rng = np.random.default_rng(seed)
    env = {name: rng.standard_normal(shape, dtype=np.float32) for name, (shape, dt, kind) in sorted(S.inputs.items())}
    env.update(S.consts)
    t = time.perf_counter()
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        run_nodes_streaming(OracleRuntime(), S.nodes, env, keep=[S.final])
    return time.perf_counter() - t


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_pool(procs):
    import multiprocessing as mp
    return mp.get_context("spawn").Pool(procs)


def oracle_step(pool, procs, t0, step):
    """procs utterances, one per worker; returns (wall seconds, utterances)."""
    t = time.perf_counter()
    pool.map(_oracle_utterance, [(t0, 1000 * step + i) for i in range(procs)])
    return time.perf_counter() - t, procs


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    n = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    procs = max(1, min(cpu_cores(), args.cpu_procs))
    pool = cpu_pool(procs)
    for w in range(args.warmup):
        oracle_step(pool, procs, args.t0, w)
    tot, utts = 0.0, 0
    for k in range(args.steps):
        dt, u = oracle_step(pool, procs, args.t0, args.warmup + k)
        tot += dt
        utts += u
    pool.close()
    value = utts / tot
    sample = (f"{procs} full-length utterances per step, one per worker process (numpy oracle, "
              f"oracle/ops.py, the reference's op table restated), {args.steps} steps")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": DATA,
            "config": config(args, n),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": procs, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def read_profile_traffic():
    """Per-launch DRAM traffic of the dominant kernel from the committed ncu
    summary (profiles/adain_snake_c5.md, line 'traffic_bytes_per_launch: N'),
    or None when no capture has been summarised."""
    p = os.path.join(REPO, "profiles", "adain_snake_c5.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def adain_bytes(rows, cols, n_src, n_out, has_res):
    """Algorithmic bytes of one bt_adain_snake launch: each source row read
    once, the residual and every output written once (fp32); the per-row
    parameters are included."""
    n = rows * cols * 4
    return n * (n_src + n_out + (1 if has_res else 0)) + rows * n_out * 8


def measure_op(fn, bytes_, flush, reps, torch):
    """Median CUDA-event time of fn() over reps, L2 flushed before each: the
    flush buffer (larger than L2) is written, then read, so that L2 holds only
    clean lines of it when fn() starts (dirty flush lines would otherwise be
    written back during fn and charge it DRAM traffic it never asked for).  A
    short device-side sleep queued after the flush keeps the GPU busy while
    the host enqueues fn(), so the interval between the events holds fn's
    kernels only, not the host's dispatch time."""
    import statistics
    for _ in range(3):
        fn()
    times = []
    for _ in range(reps):
        flush.fill_(1.0)
        flush.sum()
        torch.cuda._sleep(400_000)   # ~0.2 ms at 1.965 GHz
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    return ms, bytes_ / (ms * 1e-3) / 1e9


def per_op(rt, torch, peak):
    """BASELINE configs c1-c4 and a >= 256 MB sweep (rank 0, N = 1)."""
    from bt_b200 import configs
    from oracle import OracleRuntime
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()   # noqa: E731
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")   # 256 MB > L2
    res = {}

    def entry(name, fn, nbytes, cpu_fn=None, reps=10):
        ms, gbs = measure_op(fn, nbytes, flush, reps, torch)
        e = {"ms": round(ms, 5), "bytes": int(nbytes), "GBps": round(gbs, 1),
             "frac_of_measured": round(gbs / peak, 4), "frac_of_8TBps": round(gbs / NOMINAL_HBM, 4)}
        if cpu_fn is not None:
            with warnings.catch_warnings():
                warnings.simplefilter("ignore")
                t = time.perf_counter()
                cpu_fn()
                e["cpu_ms_1core"] = round(1e3 * (time.perf_counter() - t), 2)
        res[name] = e

    orc = OracleRuntime()

    def onode(op, env, ins, at=None):
        return lambda: orc.dispatch(op, ins, ["_o"], at or {}, dict(env))

    c = configs.c1()
    X, B = dev(c["X"]), dev(c["B"])
    entry("c1_add", lambda: rt.elementwise("ADD", [X, B], X.shape, np.float32, np.float32), 4196352,
          onode("Add", c, ["X", "B"]))
    entry("c1_mul", lambda: rt.elementwise("MUL", [X, B], X.shape, np.float32, np.float32), 4196352,
          onode("Mul", c, ["X", "B"]))
    y = rt.elementwise("ADD", [X, B], X.shape, np.float32, np.float32)
    yh = {"y": (c["X"] + c["B"]).astype(np.float32)}
    for nm, op, onnx, at in [("c1_sigmoid", "SIGMOID", "Sigmoid", {}), ("c1_tanh", "TANH", "Tanh", {}),
                             ("c1_leakyrelu", "LEAKYRELU", "LeakyRelu", {"alpha": 0.2})]:
        entry(nm, lambda op=op: rt.elementwise(op, [y], y.shape, np.float32, np.float32, alpha=0.2), 4194304,
              onode(onnx, yh, ["y"], at))
    c = configs.c2_layernorm()
    Xl, g, b = dev(c["X"]), dev(c["gamma"]), dev(c["beta"])
    entry("c2_layernorm", lambda: rt.layernorm(Xl, None, None, g, b, -1, 1e-12), 3139584,
          onode("LayerNormalization", {"X": c["X"], "g": c["gamma"], "b": c["beta"]}, ["X", "g", "b"],
                {"epsilon": 1e-12}))
    c = configs.c2_adain()
    Xa, h = dev(c["X"]), dev(c["h"][:, :, 0])
    Cc = c["X"].shape[1]
    gain = rt.elementwise("ADD", [h[:, :Cc], dev(np.array(1.0, np.float16))], (1, Cc), np.float32, np.float32)
    outa = [torch.empty_like(Xa)]
    entry("c2_adain", lambda: rt.adain_snake([Xa], gain, h[:, Cc:], np.float32(c["eps"]), outs=outa), 8392704)
    c = configs.c2_reducemean()
    Xr = dev(c["X"])
    entry("c2_reducemean", lambda: rt._reduce_block(Xr, [2], 1), 268566528,
          onode("ReduceMean", {"X": c["X"], "ax": np.array([-1], np.int64)}, ["X", "ax"]))
    del Xr
    for bsz, nbytes in ((1, 24971640), (16, 399515640)):
        c = configs.c3(batch=bsz)
        Xs, M = dev(c["X"]), dev(c["mask"])
        entry(f"c3_softmax_b{bsz}", lambda: rt.softmax(Xs, M, -1), nbytes,
              lambda c=c: OracleRuntime().run_nodes([("Add", ["X", "mask"], ["s"], {}),
                                                     ("Softmax", ["s"], ["y"], {})], dict(c)))
        del Xs
    for shape, nbytes in (((512, 512, 3), 3936256), ((256, 256, 7), 2295808)):
        c = configs.c4_dequant(shape=shape)
        W, s, z, gn = dev(c["W"]), dev(c["scale"]), dev(c["zp"]), dev(c["gain"])
        entry(f"c4_dequant_{shape[0]}", lambda: rt.dequant_mul(W, s, z, gn), nbytes,
              lambda c=c: OracleRuntime().run_nodes([("DequantizeLinear", ["W", "scale", "zp"], ["d"], {}),
                                                     ("Mul", ["d", "gain"], ["y"], {})], dict(c)))
    c = configs.c4_cast()
    Xc = dev(c["X"])
    entry("c4_cast", lambda: rt.elementwise("IDENTITY", [Xc], Xc.shape, np.float32,
                                            rt._cast_compute(np.float16, np.float32)), 492000000,
          onode("Cast", c, ["X"], {"to": 1}))
    del Xc
    # DynamicQuantizeLinear of a stage-1-sized activation [1, 512, 4000]
    # (algorithmic bytes: x read once, y written once, 5 bytes per value)
    xq = (np.random.default_rng(0).standard_normal((1, 512, 4000)) * 2).astype(np.float32)
    Xq = dev(xq)
    entry("dynquant_8MB", lambda: rt.dynamic_quantize(Xq), xq.size * 5 + 5,
          onode("DynamicQuantizeLinear", {"x": xq}, ["x"]))
    del Xq
    # the model's typical quantised activations (one-cluster path)
    for nm, shape in (("dynquant_128KB", (1, 128, 256)), ("dynquant_512KB", (1, 256, 512))):
        xs = (np.random.default_rng(1).standard_normal(shape) * 2).astype(np.float32)
        Xs_ = dev(xs)
        entry(nm, lambda Xs_=Xs_: rt.dynamic_quantize(Xs_), xs.size * 5 + 5,
              onode("DynamicQuantizeLinear", {"x": xs}, ["x"]))
    # the integer convolution epilogue of a stage-0 conv output [1, 256, 4000]
    # (algorithmic bytes: int32 accumulators read, float32 written)
    gq = torch.Generator(device="cuda").manual_seed(0)
    accq = torch.randint(-(1 << 24), 1 << 24, (1, 256, 4000), dtype=torch.int32, device="cuda", generator=gq)
    biasq = torch.randn(256, device="cuda", generator=gq).half()
    xsq, wsq = torch.tensor(0.0173, device="cuda"), torch.tensor(0.0021, device="cuda").half()
    entry("conv_epilogue_8MB", lambda: rt.conv_int_epilogue(accq, biasq, xsq, wsq), accq.numel() * 8 + 256 * 2 + 6)
    # Transpose of a stage-0 activation [2, 256, 4000] -> [2, 4000, 256]
    Xt = torch.randn((2, 256, 4000), device="cuda", generator=gq)
    entry("transpose_8MB", lambda: rt.transpose(Xt, [0, 2, 1]), Xt.numel() * 8)
    # >= 256 MB sweep
    n = 64 * 1024 * 1024
    A = torch.randn((8192, 8192), device="cuda")
    A2 = torch.randn((8192, 8192), device="cuda")
    Bv = torch.randn((8192, 1), device="cuda")
    sweep = {}
    for nm, op, ins, nb in [("add_rowbcast", "ADD", [A, Bv], 2 * n * 4 + 8192 * 4), ("mul_same_shape", "MUL", [A, A2], 3 * n * 4),
                            ("sigmoid", "SIGMOID", [A], 2 * n * 4), ("tanh", "TANH", [A], 2 * n * 4),
                            ("leakyrelu", "LEAKYRELU", [A], 2 * n * 4), ("sin", "SIN", [A], 2 * n * 4),
                            ("exp", "EXP", [A], 2 * n * 4)]:
        ms, gbs = measure_op(lambda op=op, ins=ins: rt.elementwise(op, ins, A.shape, np.float32, np.float32,
                                                                     alpha=0.2), nb, flush, 5, torch)
        sweep[nm] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    # the rest of the listed element-wise ops
    Aabs = A.abs()
    two = torch.tensor(2.0, device="cuda")
    p17 = torch.tensor(1.7, device="cuda")
    for nm, op, ins, nb in [("sub_same_shape", "SUB", [A, A2], 3 * n * 4), ("div_rowbcast", "DIV", [A, Bv],
                                                                              2 * n * 4 + 8192 * 4),
                            ("pow2", "POW", [A, two], 2 * n * 4 + 4), ("pow_general", "POW", [Aabs, p17], 2 * n * 4 + 4),
                            ("sqrt", "SQRT", [Aabs], 2 * n * 4)]:
        ms, gbs = measure_op(lambda op=op, ins=ins: rt.elementwise(op, ins, A.shape, np.float32, np.float32),
                             nb, flush, 5, torch)
        sweep[nm] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    del Aabs
    # int8 weights: DequantizeLinear alone (per-row scale) and fused with the
    # gain Mul (one pass, bt_fused_chain); Snake as one chain
    gq8 = torch.Generator(device="cuda").manual_seed(1)
    W8 = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda", generator=gq8)
    sc8 = torch.rand((8192, 1), device="cuda", generator=gq8) * 0.02 + 1e-3
    gn8 = torch.rand((8192, 1), device="cuda", generator=gq8) + 0.5
    ms, gbs = measure_op(lambda: rt.dequantize(W8, sc8), n * 5 + 8192 * 4, flush, 5, torch)
    sweep["dequant_int8"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    ms, gbs = measure_op(lambda: rt.dequant_mul(W8, sc8, None, gn8), n * 5 + 8192 * 8, flush, 5, torch)
    sweep["dequant_int8_x_gain_chain"] = {"ms": round(ms, 4), "GBps": round(gbs, 1),
                                          "frac_of_measured": round(gbs / peak, 4), "launches": 1}
    del W8
    A3s = A.reshape(64, 128, 8192)
    al8 = (torch.rand((1, 128, 1), device="cuda", generator=gq8) + 0.5).half()
    ial8 = (1.0 / al8.float()).half()
    two16 = torch.tensor(2.0, device="cuda").half()
    ms, gbs = measure_op(lambda: rt.snake(A3s, al8, ial8, two16), 2 * n * 4 + 128 * 4, flush, 5, torch)
    sweep["snake_chain"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4),
                            "launches": 1}
    from bt_b200 import chains
    ms, gbs = measure_op(lambda: rt.chain(chains.add_unary_program("SIGMOID"), [A, A2]), 3 * n * 4, flush, 5, torch)
    sweep["add_sigmoid_chain"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4),
                                  "launches": 1}
    gl = torch.rand(768, device="cuda")
    Al = A.reshape(-1)[: (n // 768) * 768].reshape(-1, 768)
    Al2 = A2.reshape(-1)[: (n // 768) * 768].reshape(-1, 768)
    ms, gbs = measure_op(lambda: rt.layernorm(Al, Al2, None, gl, gl, -1, 1e-12), 3 * Al.numel() * 4 + 6144,
                         flush, 5, torch)
    sweep["skip_layernorm_768"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    ms, gbs = measure_op(lambda: rt.layernorm(Al, None, None, gl, None, -1, 1e-5), 2 * Al.numel() * 4 + 3072,
                         flush, 5, torch)
    sweep["layernorm_768"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    A3 = A.reshape(64, 128, 8192)
    gsw = torch.rand((64, 128), device="cuda")
    osw = [torch.empty_like(A3)]
    ms, gbs = measure_op(lambda: rt.adain_snake([A3], gsw, gsw, 1e-5, outs=osw), 2 * n * 4, flush, 5, torch)
    sweep["adain_8192"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    # AdaIN + Snake whose output feeds DynamicQuantizeLinear, the range pass
    # separate (adain, range, quantize) and folded into the AdaIN kernel
    # (adain + range, quantize); algorithmic bytes of the pair: x read,
    # the Snake output written and read back once, y written
    al3 = (torch.rand(128, device="cuda") + 0.5).half()
    ial3 = (1.0 / al3.float()).half()
    rec3 = rt.range_records(1)
    for nm, fused in (("adain_snake_dynquant_separate", False), ("adain_snake_dynquant_fused", True)):
        def pair(fused=fused):
            rt.adain_snake([A3], gsw, gsw, 1e-5, al3, ial3, outs=osw, ranges=rec3 if fused else None)
            rt.dynamic_quantize(osw[0], range=rec3[0] if fused else None)
        ms, gbs = measure_op(pair, 13 * n, flush, 5, torch)
        sweep[nm] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    ms, gbs = measure_op(lambda: rt._reduce_block(A3, [2], 1), n * 4, flush, 5, torch)
    sweep["reducemean_8192"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    ms, gbs = measure_op(lambda: rt.dynamic_quantize(A), 5 * n + 5, flush, 5, torch)
    sweep["dynquant"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    acc3 = A.view(torch.int32).reshape(64, 128, 8192)
    bias3 = torch.rand(128, device="cuda").half()
    ms, gbs = measure_op(lambda: rt.conv_int_epilogue(acc3, bias3, xsq, wsq), 8 * n + 128 * 2 + 6, flush, 5, torch)
    sweep["conv_epilogue"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    ms, gbs = measure_op(lambda: rt.transpose(A3, [0, 2, 1]), 8 * n, flush, 5, torch)
    sweep["transpose_last2"] = {"ms": round(ms, 4), "GBps": round(gbs, 1), "frac_of_measured": round(gbs / peak, 4)}
    res["sweep_256MB"] = sweep
    del A, A2, A3, acc3, osw, flush
    res["model_hot_nodes"] = model_hot_nodes(rt, torch)
    return res


KPK_DTYPES = {0: np.float32, 1: np.int8, 2: np.uint8, 3: np.int32, 4: np.int64, 5: np.bool_, 6: np.float16}


def _trace_node(sig, seed):
    """A node of the recorded signature (tests/golden/model_trace.json): the
    recorded values for inputs of at most 64 elements, seeded data else."""
    rng = np.random.default_rng(seed)
    names, env = [], {}
    for j, sp in enumerate(sig["inputs"]):
        if sp is None:
            names.append("")
            continue
        name = f"x{j}"
        names.append(name)
        dt, shape = np.dtype(sp["dtype"]), tuple(sp["shape"])
        if "values" in sp:
            a = np.array(sp["values"], dtype=dt).reshape(shape)
        elif dt.kind == "f":
            a = (rng.standard_normal(shape) * 2).astype(dt)
        elif dt.kind == "b":
            a = rng.random(shape) < 0.5
        else:
            a = rng.integers(-1000, 1001, shape).astype(dt)
        env[name] = a
    at = {}
    for k, v in (sig["attrs"] or {}).items():
        if isinstance(v, dict) and "__t" in v:
            v = np.array(v["v"], dtype=KPK_DTYPES[v["__t"]]).reshape(v["s"])
        at[k] = v
    return (sig["op"], names, [f"y{i}" for i in range(sig["n_out"])], at), env


def model_hot_nodes(rt, torch):
    """Every hot-path node execution of one real model run (3442 nodes of a
    9-token utterance, recorded from the reference's packed-model driver:
    845 distinct signatures with their counts) replayed on seeded inputs of
    the recorded shapes: through BtRuntime.dispatch (device-resident inputs,
    timed end to end on the host clock with a synchronize, so Python
    dispatch counts; constants of at most 64 elements stay numpy arrays, as
    the model's initializers do) and through the numpy oracle on one core."""
    from oracle import OracleRuntime
    path = os.path.join(REPO, "tests", "golden", "model_trace.json")
    with open(path) as f:
        sigs = json.load(f)["signatures"]
    nodes = []
    for i, sig in enumerate(sigs):
        node, env = _trace_node(sig, i)
        # inputs recorded with their values (axes, shapes, split sizes,
        # scalar constants: the model's initializers) stay numpy, as in the
        # model's env; activations are resident on the device
        small = {f"x{j}" for j, sp in enumerate(sig["inputs"]) if sp is not None and "values" in sp}
        denv = {k: (v if k in small else torch.from_numpy(np.ascontiguousarray(v)).cuda()) for k, v in env.items()}
        nodes.append((node, env, denv, sig["count"]))

    def gpu_pass():
        for (op, ins, outs, at), _, denv, count in nodes:
            for _ in range(count):
                e = dict(denv)
                rt.dispatch(op, ins, outs, at, e)

    gpu_pass()
    torch.cuda.synchronize()
    l0 = rt.launches
    t = time.perf_counter()
    gpu_pass()
    torch.cuda.synchronize()
    gpu_ms = 1e3 * (time.perf_counter() - t)
    launches = rt.launches - l0
    # the same node executions recorded once as a CUDA graph and replayed
    # (the serving form: per-node host work paid at capture)
    captured_ms = None
    try:
        cap_stream = torch.cuda.Stream()
        cap_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap_stream):
            gpu_pass()
        cap_stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap_stream):
            gpu_pass()
        graph.replay()
        torch.cuda.synchronize()
        reps = 5
        t = time.perf_counter()
        for _ in range(reps):
            graph.replay()
        torch.cuda.synchronize()
        captured_ms = round(1e3 * (time.perf_counter() - t) / reps, 2)
        del graph
    except RuntimeError as exc:   # a node that needs a host value cannot be captured
        captured_ms = f"not captured: {str(exc).splitlines()[0][:120]}"
        torch.cuda.synchronize()
    orc = OracleRuntime()
    cpu_ms = 0.0
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        for (op, ins, outs, at), env, _, count in nodes:
            t = time.perf_counter()
            orc.dispatch(op, ins, outs, at, dict(env))
            cpu_ms += 1e3 * (time.perf_counter() - t) * count
    n = sum(c for *_, c in nodes)
    return {"nodes": n, "signatures": len(nodes), "gpu_ms_per_utterance": round(gpu_ms, 2),
            "captured_ms_per_utterance": captured_ms,
            "gpu_launches": launches, "numpy_ms_per_utterance_1core": round(cpu_ms, 1),
            "speedup": round(cpu_ms / gpu_ms, 1),
            "note": "host clock around BtRuntime.dispatch of every node (Python dispatch included), inputs "
                    "resident; captured: the same node executions replayed as one CUDA graph"}


def stream_groups(batch, streams):
    """Concurrent groups a rank splits its utterances into: `streams`, or by
    default 2 for 2-32 utterances (measured on one B200: at 8 and 16
    utterances two concurrent streams run 21 % and 9 % faster, because one
    group's row staging overlaps the other's statistics and output passes
    and a launch's partial last wave no longer idles the GPU), else 1."""
    if streams:
        return max(1, min(int(streams), batch))
    return 2 if 2 <= batch <= 32 else 1


class RankStream:
    """One rank's share of the job: its utterances in `groups` FusedDecoders
    (each on its own CUDA stream when there are several), conv stand-ins
    drawn on the device, pinned host buffers holding the per-step inputs
    (features, fc outputs), all seeded per rank and group."""

    def __init__(self, batch, t0, rank, dev, groups=1):
        from bt_b200.decoder import FusedDecoder, build_stream, fill_conv_standins, host_inputs
        from bt_b200 import shard
        import torch
        self.batch = batch
        self.parts = []
        sizes = [batch // groups + (1 if g < batch % groups else 0) for g in range(groups)]
        for g, b in enumerate(sizes):
            S = build_stream(b, t0=t0)
            dec = FusedDecoder(S, dev)
            fill_conv_standins(dec, seed=shard.rank_seed(17, rank) + 7919 * g)
            host = host_inputs(S, seed=shard.rank_seed(100, rank) + 7919 * g)
            hin, hout = dec.host_buffers()
            dec.fill_host(hin, host)
            dec.run_host(hin, hout)                        # inputs resident from here on
            self.parts.append((S, dec, hin, hout))
        self.streams = [torch.cuda.Stream(dev) for _ in self.parts] if len(self.parts) > 1 else []
        torch.cuda.synchronize()

    @property
    def stages(self):
        return [S for S, *_ in self.parts]

    def _fan(self, fn):
        """fn(g, part) for every group: on its own stream when there are
        several (forked from and joined back into the current stream)."""
        import torch
        if not self.streams:
            return [fn(0, self.parts[0])]
        main = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        res = []
        for g, (part, st) in enumerate(zip(self.parts, self.streams)):
            st.wait_event(fork)
            with torch.cuda.stream(st):
                res.append(fn(g, part))
            join = torch.cuda.Event()
            join.record(st)
            main.wait_event(join)
        return res

    def launch(self, record=None, serial=False):
        """One step of every group (concurrently unless `serial`); returns
        the kernel launches."""
        if serial or not self.streams:
            return sum(dec.launch(record=record) for _, dec, _, _ in self.parts)
        return sum(self._fan(lambda g, part: part[1].launch(record=record)))

    def device_steps(self, steps, warmup, barrier, record=None, serial=False):
        """Seconds for `steps` steps of the stream (CUDA events on the
        launch stream, barrier + synchronize on both sides); returns
        (seconds, kernel launches).  With `record`, every launch is also
        bracketed by CUDA events (run with `serial`: the groups one after
        the other, so that no two launches overlap)."""
        import torch
        for _ in range(warmup):
            self.launch(serial=serial)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        launches = 0
        for _ in range(steps):
            launches += self.launch(record=record, serial=serial)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / 1e3, launches

    def e2e_steps(self, steps, warmup, barrier):
        """Seconds for `steps` end-to-end steps through the host-buffer API
        (FusedDecoder.host_pipeline: each step copies its inputs in from
        pinned host memory and its result out, overlapped with the
        neighbouring steps' compute); returns (seconds, h2d, d2h bytes per
        step)."""
        import torch
        pipes = [dec.host_pipeline(hin, hout) for _, dec, hin, hout in self.parts]

        def step():
            moved = self._fan(lambda g, part: pipes[g].step())
            return sum(m[0] for m in moved), sum(m[1] for m in moved)

        def finish():
            self._fan(lambda g, part: pipes[g].finish())

        for _ in range(warmup):
            step()
        finish()
        torch.cuda.synchronize()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        h2d = d2h = 0
        for _ in range(steps):
            h2d, d2h = step()
        finish()
        f1.record()
        torch.cuda.synchronize()
        barrier()
        return f0.elapsed_time(f1) / 1e3, h2d, d2h

    def release(self):
        import torch
        del self.parts
        torch.cuda.empty_cache()


def run_b200(args):
    import torch
    import torch.distributed as dist
    from bt_b200.decoder import stream_algorithmic_bytes
    from bt_b200.runtime import BtRuntime
    from bt_b200 import shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = world
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    peak, peak_kind = peaks()

    # CPU baseline pool first (spawned workers; rank 0 at N = 1 only)
    do_cpu = rank == 0 and n == 1 and not args.no_cpu_baseline
    pool = None
    if do_cpu:
        procs = max(1, min(cpu_cores(), args.cpu_procs))
        pool = cpu_pool(procs)

    # this rank's share of the one batch (strong scaling): utterances
    # shard.split_utterances(batch, n, rank), inputs seeded per rank
    _, mine = shard.split_utterances(args.batch, n, rank)
    groups = stream_groups(mine, args.streams)
    rs = RankStream(mine, args.t0, rank, dev, groups)

    def barrier():
        shard.barrier(dev)

    def max_over_ranks(v):
        return shard.max_over_ranks(v, device=dev)

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    # the timed steps: no event between launches (a pair of CUDA events
    # around every launch adds a gap after each kernel: 11 % of the step at
    # 8 utterances per GPU, 2-3 % at 64)
    dt, launches = rs.device_steps(args.steps, args.warmup, barrier)
    clk = clocks.stop()
    elapsed = max_over_ranks(dt)
    value = args.batch * args.steps / elapsed
    ms_step = 1e3 * elapsed / args.steps
    # the roofline pass: the same steps again, every launch bracketed by CUDA
    # events on its stream and the groups run one after the other, so that
    # each launch's duration is its own
    record = []
    rdt, _ = rs.device_steps(args.steps, 1, barrier, record=record, serial=True)
    roofline_ms_step = 1e3 * max_over_ranks(rdt) / args.steps

    # dominant kernel: bt_adain_snake launches of the timed region
    ad_bytes = ad_time = 0.0
    ad_n = 0
    kind_time = {}
    for kind, rows, cols, n_src, n_out, has_res, a, b in record:
        t = a.elapsed_time(b) / 1e3
        kind_time[kind] = kind_time.get(kind, 0.0) + t
        if kind == "adain":
            ad_bytes += adain_bytes(rows, cols, n_src, n_out, has_res)
            ad_time += t
            ad_n += 1
    achieved = ad_bytes / ad_time / 1e9
    traffic = read_profile_traffic()
    roofline = {"bound": "hbm", "kernel": "bt_adain_snake (adain_cluster_kernel)", "achieved": round(achieved, 1),
                "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "frac_of_8TBps": round(achieved / NOMINAL_HBM, 4), "peak_kind": peak_kind,
                "traffic": traffic, "launches_timed": ad_n,
                "algorithmic_bytes_per_launch": round(ad_bytes / max(ad_n, 1)),
                "avg_launch_ms": round(1e3 * ad_time / max(ad_n, 1), 4),
                "share_of_step_time": round(ad_time / max(sum(kind_time.values()), 1e-12), 4),
                "measured": "CUDA events around every launch, in a second pass of the same steps (groups run "
                            "one after the other) right after the timed one",
                "pass_ms_per_step": round(roofline_ms_step, 3)}
    stream_bytes = sum(stream_algorithmic_bytes(S) for S in rs.stages)
    stream_bytes_all = int(shard.sum_over_ranks(stream_bytes, device=dev))

    # end to end through the host-buffer API
    e2e_dt, h2d, d2h = rs.e2e_steps(args.steps, args.warmup, barrier)
    e2e_s = max_over_ranks(e2e_dt)
    h2d_all = int(shard.sum_over_ranks(h2d, device=dev))
    d2h_all = int(shard.sum_over_ranks(d2h, device=dev))
    e2e = {"value": args.batch * args.steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d_all,
           "d2h_bytes_per_step": d2h_all, "ms_per_step": round(1e3 * e2e_s / args.steps, 3),
           "api": "FusedDecoder.host_pipeline(...).step() on every rank (pinned host buffers; each step's copies "
                  "overlap the neighbouring steps' compute)"}
    # what bounds the end-to-end step: the device's own step, or the copy
    # of the result to the host (all ranks share the host link)
    e2e_ms = 1e3 * e2e_s / args.steps
    d2h_gbs = d2h_all / (e2e_s / args.steps) / 1e9
    e2e_limit = {"device_ms_per_step": round(ms_step, 3), "e2e_ms_per_step": round(e2e_ms, 3),
                 "d2h_bytes_per_step_all_ranks": d2h_all, "h2d_bytes_per_step_all_ranks": h2d_all,
                 "d2h_GBps_all_ranks": round(d2h_gbs, 1),
                 "limited_by": ("device step" if e2e_ms < 1.1 * ms_step else
                                "device-to-host copy of the result (the host link)")}

    # weak scaling beside it (N > 1): 64 utterances on every rank
    weak = None
    if n > 1 and not args.no_weak:
        rs.release()
        rw = RankStream(args.weak_batch, args.t0, rank, dev, stream_groups(args.weak_batch, args.streams))
        wdt, _ = rw.device_steps(args.steps, args.warmup, barrier)
        wdt = max_over_ranks(wdt)
        we_dt, _, wd2h = rw.e2e_steps(args.steps, args.warmup, barrier)
        we_dt = max_over_ranks(we_dt)
        wd2h = int(shard.sum_over_ranks(wd2h, device=dev))
        weak = {"batch_per_gpu": args.weak_batch, "global_batch": args.weak_batch * n,
                "value": args.weak_batch * n * args.steps / wdt, "unit": UNIT,
                "ms_per_step": round(1e3 * wdt / args.steps, 3),
                "e2e": {"value": args.weak_batch * n * args.steps / we_dt, "unit": UNIT,
                        "ms_per_step": round(1e3 * we_dt / args.steps, 3), "d2h_bytes_per_step": wd2h}}
        rw.release()

    extra = {}
    if rank == 0 and n == 1 and not args.no_per_op:
        rs.release()
        rt = BtRuntime(dev)
        extra["per_op"] = per_op(rt, torch, peak)

    cpu = None
    if do_cpu:
        procs = pool._processes
        oracle_step(pool, procs, args.t0, 0)             # warm the workers (imports)
        dt_c, u = oracle_step(pool, procs, args.t0, 1)
        pool.close()
        cpu = {"value": u / dt_c, "unit": UNIT, "cores": procs, "kind": "port",
               "sample": f"{u} full-length utterances, one per worker process, through the numpy oracle "
                         "(oracle/ops.py, the reference's op table restated), after one warm-up round"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": DATA, "config": config(args, n, groups),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "e2e_limit": e2e_limit,
                "gpu_launches": launches * n, "gpu_launches_per_rank": launches,
                "clocks": clk, "stream_algorithmic_bytes_per_step": stream_bytes_all,
                "stream_GBps_per_gpu": round(stream_bytes_all / n * args.steps / elapsed / 1e9, 1),
                "stream_frac_of_measured": round(stream_bytes_all / n / (elapsed / args.steps) / 1e9 / peak, 4)}
        if weak is not None:
            line["weak"] = weak
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


PROFILE_KINDS = {
    # name: (sources, residual written, outputs)
    "2src": (2, True, 1),      # pairs 1-2 first AdaIN: conv output + residual
    "1src": (1, False, 1),     # second AdaIN of every pair
    "shared3": (2, True, 3),   # the shared instance norm of the three resblocks
}


def run_profile_adain(args):
    """One kind of stage-2 bt_adain_snake launch on its own, for ncu:
    batch x 128 rows of 24001 values (every array larger than L2 from batch
    16 up).  --profile-kind picks the launch: '2src' (two sources + residual
    + snake output, the most common launch of the stream), '1src' (one
    source, one snake output) or 'shared3' (two sources + residual, three
    snake outputs)."""
    import torch
    from bt_b200.runtime import BtRuntime
    torch.cuda.set_device(0)
    rt = BtRuntime(0)
    n_src, with_res, n_out = PROFILE_KINDS[args.profile_kind]
    B, C, T = args.batch, 128, args.t0 * 60 + 1
    g = torch.Generator(device="cuda").manual_seed(5)
    srcs = [torch.randn((B, C, T), device="cuda", generator=g) for _ in range(n_src)]
    res = torch.empty((B, C, T), device="cuda") if with_res else None
    out = [torch.empty((B, C, T), device="cuda") for _ in range(n_out)]
    fc = [torch.randn((B, 2 * C), device="cuda", generator=g) for _ in range(n_out)]
    alpha = [(torch.rand(C, device="cuda", generator=g) + 0.5).half() for _ in range(n_out)]
    inv = [(1.0 / a.float()).half() for a in alpha]
    gains = [f[:, :C] for f in fc]
    shifts = [f[:, C:] for f in fc]
    for _ in range(args.warmup + args.steps):
        if n_out == 1:
            rt.adain_snake(srcs, gains[0], shifts[0], 1e-5, alpha[0], inv[0], res=res, outs=out)
        else:
            rt.adain_snake(srcs, gains, shifts, 1e-5, alpha, inv, res=res, outs=out)
    torch.cuda.synchronize()
    print(json.dumps({"profile": f"adain_snake stage 2, kind {args.profile_kind}", "rows": B * C, "cols": T,
                      "sources": n_src, "residual": with_res, "outputs": n_out,
                      "launches": args.warmup + args.steps}))
    return 0


PROFILE_OPS = ("reducemean_c2", "softmax_c3_b16", "layernorm_768", "reducemean_8192", "dynquant_256MB",
               "conv_epilogue_256MB", "transpose_256MB", "tanh_256MB", "adain_dq_256MB", "dequant_gain_320MB",
               "snake_512MB")


def run_profile_op(args):
    """One per-op workload, launched warmup + steps times, for ncu:
    'reducemean_c2' (BASELINE c2 ReduceMean, [64,512,2048]), 'softmax_c3_b16'
    (c3 masked softmax at batch 16) or 'layernorm_768' (LayerNormalization
    over 768 channels of a 256 MB tensor); the 256 MB sweep's
    'reducemean_8192', 'dynquant_256MB', 'conv_epilogue_256MB',
    'transpose_256MB' ([64,128,8192] -> [64,8192,128]), 'tanh_256MB',
    'adain_dq_256MB' (AdaIN+Snake with the range folded in, then the
    quantize pass), 'dequant_gain_320MB' (int8 [8192, 8192] dequantised
    and scaled in one chain) and 'snake_512MB' (Snake as one chain over
    [64, 128, 8192])."""
    import torch
    from bt_b200 import configs
    from bt_b200.runtime import BtRuntime
    torch.cuda.set_device(0)
    rt = BtRuntime(0)
    name = args.profile_op
    if name == "reducemean_c2":
        X = torch.from_numpy(configs.c2_reducemean()["X"]).cuda()
        fn = lambda: rt._reduce_block(X, [2], 1)
    elif name == "softmax_c3_b16":
        c = configs.c3(batch=16)
        Xs, M = torch.from_numpy(c["X"]).cuda(), torch.from_numpy(c["mask"]).cuda()
        fn = lambda: rt.softmax(Xs, M, -1)
    elif name == "layernorm_768":
        A = torch.randn((64 * 1024 * 1024 // 768, 768), device="cuda")
        g = torch.rand(768, device="cuda")
        fn = lambda: rt.layernorm(A, None, None, g, None, -1, 1e-5)
    elif name == "dequant_gain_320MB":
        W8 = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        sc, gn = torch.rand((8192, 1), device="cuda") * 0.02, torch.rand((8192, 1), device="cuda") + 0.5
        fn = lambda: rt.dequant_mul(W8, sc, None, gn)
    elif name == "snake_512MB":
        X = torch.randn((64, 128, 8192), device="cuda")
        al = (torch.rand((1, 128, 1), device="cuda") + 0.5).half()
        ial, two = (1.0 / al.float()).half(), torch.tensor(2.0, device="cuda").half()
        fn = lambda: rt.snake(X, al, ial, two)
    else:
        A = torch.randn((64, 128, 8192), device="cuda")
        if name == "reducemean_8192":
            fn = lambda: rt._reduce_block(A, [2], 1)
        elif name == "dynquant_256MB":
            fn = lambda: rt.dynamic_quantize(A)
        elif name == "conv_epilogue_256MB":
            acc, b = A.view(torch.int32), torch.rand(128, device="cuda").half()
            xs, ws = torch.tensor(0.0173, device="cuda"), torch.tensor(0.0021, device="cuda").half()
            fn = lambda: rt.conv_int_epilogue(acc, b, xs, ws)
        elif name == "transpose_256MB":
            fn = lambda: rt.transpose(A, [0, 2, 1])
        elif name == "adain_dq_256MB":
            g = torch.rand((64, 128), device="cuda")
            al = (torch.rand(128, device="cuda") + 0.5).half()
            ial = (1.0 / al.float()).half()
            rec, out = rt.range_records(1), [torch.empty_like(A)]

            def fn():
                rt.adain_snake([A], g, g, 1e-5, al, ial, outs=out, ranges=rec)
                rt.dynamic_quantize(out[0], range=rec[0])
        else:
            fn = lambda: rt.elementwise("TANH", [A], A.shape, np.float32, np.float32)
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"profile_op": name, "launches": args.warmup + args.steps}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=64,
                    help="utterances in the batch, split over the GPUs (strong scaling)")
    ap.add_argument("--streams", type=int, default=0,
                    help="concurrent decoder streams per GPU (0: 2 for 2-32 utterances per GPU, else 1)")
    ap.add_argument("--weak-batch", type=int, default=64,
                    help="utterances per GPU of the weak-scaling figure reported beside it at N > 1")
    ap.add_argument("--no-weak", action="store_true", help="skip the weak-scaling figure at N > 1")
    ap.add_argument("--t0", type=int, default=400)
    ap.add_argument("--cpu-procs", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-op", action="store_true")
    ap.add_argument("--profile-adain", action="store_true",
                    help="run only stage-2 bt_adain_snake launches (for ncu)")
    ap.add_argument("--profile-kind", default="2src", choices=sorted(PROFILE_KINDS),
                    help="which bt_adain_snake launch --profile-adain runs")
    ap.add_argument("--profile-op", default=None, choices=PROFILE_OPS,
                    help="run only one per-op workload (for ncu)")
    args = ap.parse_args()
    if args.profile_adain:
        return run_profile_adain(args)
    if args.profile_op:
        return run_profile_op(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())

"""Kokoro-82M ISTFTNet generator: the decoder-stage op stream (config c5).

The stream is the part of the packed Kokoro graph (model.kpk, nodes under
``/decoder/decoder/generator/``) that runs on the elementwise / reduction hot
path between the generator's convolutions:

    stage s (s = 0: [256, 10*T], s = 1: [128, 60*T + 1]):
      x0   = LeakyRelu(x_in, 0.1)                     -> ups conv (stand-in u)
      xs   = noise conv output (stand-in)
      noise_res.s:   3 dilation pairs on xs            (AdaINResBlock1)
      x    = u + xs
      resblocks.3s+j, j = 0..2: 3 dilation pairs on x  (AdaINResBlock1)
      m    = ((r0 + r1) + r2) / 3                      -> next stage's LeakyRelu
    final = LeakyRelu(m_1, 0.01)                       -> conv_post

    dilation pair k of a block with residual h:
      a  = AdaIN1d(h)  = (1 + gamma) * InstanceNorm(h) + beta
           InstanceNorm = ReduceMean, Sub, Mul, ReduceMean, Add eps, Sqrt, Div
      s1 = Snake(a)    = a + inv_alpha * sin(alpha * a) ** 2
           (Mul, Sin, Pow 2, Mul, Add; inv_alpha is a stored fp16 constant)
      c1 = conv1(s1)   (stand-in)
      s2 = Snake(AdaIN1d(c1));  c2 = conv2(s2)  (stand-in)
      h  = c2 + h

The graph computes the instance norm of x once for the three resblocks that
read it (their adain1.0 share ReduceMean..Div, then apply their own affine).
gamma / beta come from each AdaIN's fc Linear on the style half of the style
vector; the Linear is a contraction, so its outputs h = [gamma | beta] are
inputs here (``fc`` stand-ins), split with ``Split`` and offset with
``Add(gamma, 1)`` exactly as in the graph.  Convolution outputs are seeded
N(0,1) stand-ins of the matching shapes.

``build_stream`` returns one ``Stream`` description rendered two ways:
``Stream.nodes`` is the op-table node list (what the reference interpreter
or ``BtRuntime`` executes node by node) and ``FusedDecoder`` is the B200
plan: per dilation pair one row-fused AdaIN->Snake kernel per AdaIN (the
residual Add folded into the next AdaIN's row staging), the shared
normalisation producing three outputs, and one kernel for the resblock mean
plus the LeakyRelu that follows.  Both compute the same values bit for bit.
"""
import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import check, load, make_tensor
from .runtime import as_cuda_device, tensor_desc

EPS = np.float16(1e-5)           # the graph's AdaIN epsilon constant (fp16)
STYLE_DIM = 128


def stage_shapes(t0=400, channels=(512, 256, 128), rates=(10, 6)):
    """[(C_in, T_in, C, T)] of the two generator stages (stage 1 adds the
    one-sample reflection pad of the generator)."""
    t1 = t0 * rates[0]
    t2 = t1 * rates[1] + 1
    return [(channels[0], t0, channels[1], t1), (channels[1], t1, channels[2], t2)]


@dataclass
class AdaIN:
    fc: str            # [B, 2C, 1] fc output (gamma | beta)
    gamma: str
    beta: str
    gain: str          # 1 + gamma
    alpha: str         # [1, C, 1] fp16
    inv_alpha: str
    norm: str = ""     # Div output (instance norm) this AdaIN scales
    affine: str = ""   # Add(beta) output
    snake: str = ""    # snake Add output


@dataclass
class Pair:
    src: list          # names summed (left to right) to form this pair's input h
    h: str             # name of h (the residual entering the pair)
    a1: AdaIN = None
    c1: str = ""
    a2: AdaIN = None
    c2: str = ""
    out: str = ""      # c2 + h


@dataclass
class Block:
    name: str
    pairs: list = field(default_factory=list)


@dataclass
class Stage:
    index: int
    C: int
    T: int
    x_in: str
    leaky_in: str      # LeakyRelu(x_in) output (feeds the ups conv)
    ups: str
    noise_x: str
    noise: Block = None
    x: str = ""        # u + noise output
    shared_norm: str = ""
    res: list = field(default_factory=list)
    mean: str = ""     # Div output


@dataclass
class Stream:
    batch: int
    nodes: list = field(default_factory=list)
    inputs: dict = field(default_factory=dict)   # name -> (shape, dtype, kind)
    consts: dict = field(default_factory=dict)   # name -> np.ndarray
    stages: list = field(default_factory=list)
    final: str = ""

    def snake_names(self):
        out = []
        for st in self.stages:
            for blk in [st.noise] + st.res:
                for p in blk.pairs:
                    for a in (p.a1, p.a2):
                        out.append(a.snake)
        return out

    def residual_names(self):
        """Residuals the fused plan materialises: x of each stage and the
        pair inputs h of pairs 1 and 2 of every block."""
        out = []
        for st in self.stages:
            out.append(st.x)
            for blk in [st.noise] + st.res:
                out.extend(p.h for p in blk.pairs[1:])
        return out

    def stage_outputs(self):
        """LeakyRelu(stage-0 mean) (input of the second ups conv) and the
        final LeakyRelu (input of conv_post)."""
        return [self.stages[1].leaky_in, self.final]

    def adains(self, stage):
        return [a for blk in [stage.noise] + stage.res for p in blk.pairs for a in (p.a1, p.a2)]


def build_stream(batch, t0=400, seed=0):
    """The c5 op stream for ``batch`` utterances (see module docstring).

    Constants drawn from ``np.random.default_rng(seed)``: per snake, alpha ~
    U(0.5, 1.5) per channel stored as fp16, inv_alpha = fp16(1 / alpha)."""
    rng = np.random.default_rng(seed)
    S = Stream(batch=batch)
    nodes = S.nodes
    counter = [0]

    def nm(prefix):
        counter[0] += 1
        return f"{prefix}#{counter[0]}"

    def const(name, value):
        S.consts[name] = value
        return name

    def inp(name, shape, dtype, kind):
        S.inputs[name] = (tuple(shape), np.dtype(dtype), kind)
        return name

    one = const("G/const/one", np.array(1.0, dtype=np.float16))
    two = const("G/const/two", np.array(2.0, dtype=np.float16))
    eps = const("G/const/eps", np.array(EPS, dtype=np.float16))
    axes = const("G/const/axes", np.array([2], dtype=np.int64))
    three = [const("G/const/three0", np.array(3.0, dtype=np.float32)),
             const("G/const/three1", np.array(3.0, dtype=np.float16))]

    feat = inp("G/features", (batch, 512, t0), np.float32, "features")
    shapes = stage_shapes(t0)
    prelude, body = [], []

    def adain_params(prefix, C):
        fc = inp(f"{prefix}/fc", (batch, 2 * C, 1), np.float32, "fc")
        split = const(f"{prefix}/splits", np.array([C, C], dtype=np.int64))
        g, b = nm(f"{prefix}/gamma"), nm(f"{prefix}/beta")
        prelude.append(("Split", [fc, split], [g, b], {"axis": 1}))
        gain = nm(f"{prefix}/gain")
        prelude.append(("Add", [g, one], [gain], {}))
        return fc, g, b, gain

    def snake_consts(prefix, C):
        alpha = rng.uniform(0.5, 1.5, (1, C, 1)).astype(np.float16)
        inv = (1.0 / alpha.astype(np.float64)).astype(np.float16)
        return const(f"{prefix}/alpha", alpha), const(f"{prefix}/inv_alpha", inv)

    def instance_norm(prefix, h):
        mu, d, d2, var, ve, sd, n = (nm(f"{prefix}/{k}") for k in
                                      ("ReduceMean", "Sub", "Mul", "ReduceMean_2", "Add", "Sqrt", "Div"))
        body.extend([
            ("ReduceMean", [h, axes], [mu], {"keepdims": 1, "noop_with_empty_axes": 0}),
            ("Sub", [h, mu], [d], {}),
            ("Mul", [d, d], [d2], {}),
            ("ReduceMean", [d2, axes], [var], {"keepdims": 1, "noop_with_empty_axes": 0}),
            ("Add", [var, eps], [ve], {}),
            ("Sqrt", [ve], [sd], {}),
            ("Div", [d, sd], [n], {}),
        ])
        return n

    def affine_snake(a, prefix):
        m, y = nm(f"{prefix}/Mul_3"), nm(f"{prefix}/Add_3")
        body.extend([("Mul", [a.gain, a.norm], [m], {}), ("Add", [m, a.beta], [y], {})])
        a.affine = y
        t, s, p, q, z = (nm(f"{prefix}/snake/{k}") for k in ("Mul", "Sin", "Pow", "Mul_1", "Add"))
        body.extend([
            ("Mul", [a.alpha, y], [t], {}),
            ("Sin", [t], [s], {}),
            ("Pow", [s, two], [p], {}),
            ("Mul", [a.inv_alpha, p], [q], {}),
            ("Add", [y, q], [z], {}),
        ])
        a.snake = z

    def make_adain(prefix, C, alpha_prefix):
        fc, g, b, gain = adain_params(prefix, C)
        al, inv = snake_consts(alpha_prefix, C)
        return AdaIN(fc=fc, gamma=g, beta=b, gain=gain, alpha=al, inv_alpha=inv)

    def block(name, h0, C, T, shared_norm=None):
        blk = Block(name=name)
        h = h0
        for k in range(3):
            p = Pair(src=[], h=h)
            p.a1 = make_adain(f"{name}/adain1.{k}", C, f"{name}/alpha1.{k}")
            p.a2 = make_adain(f"{name}/adain2.{k}", C, f"{name}/alpha2.{k}")
            p.c1 = inp(f"{name}/convs1.{k}", (batch, C, T), np.float32, "conv")
            p.c2 = inp(f"{name}/convs2.{k}", (batch, C, T), np.float32, "conv")
            blk.pairs.append(p)
            if k == 0 and shared_norm is not None:
                p.a1.norm = shared_norm
            else:
                p.a1.norm = instance_norm(f"{name}/adain1.{k}", h)
            affine_snake(p.a1, f"{name}/adain1.{k}")
            p.a2.norm = instance_norm(f"{name}/adain2.{k}", p.c1)
            affine_snake(p.a2, f"{name}/adain2.{k}")
            p.out = nm(f"{name}/Add_res{k}")
            body.append(("Add", [p.c2, h], [p.out], {}))
            h = p.out
        return blk

    x_in = feat
    for s, (cin, tin, C, T) in enumerate(shapes):
        leaky = nm(f"G/LeakyRelu_{s}")
        body.append(("LeakyRelu", [x_in], [leaky], {"alpha": 0.10000000149011612}))
        st = Stage(index=s, C=C, T=T, x_in=x_in, leaky_in=leaky,
                   ups=inp(f"G/ups.{s}", (batch, C, T), np.float32, "conv"),
                   noise_x=inp(f"G/noise_convs.{s}", (batch, C, T), np.float32, "conv"))
        st.noise = block(f"G/noise_res.{s}", st.noise_x, C, T)
        st.x = nm(f"G/Add_x{s}")
        body.append(("Add", [st.ups, st.noise.pairs[-1].out], [st.x], {}))
        st.shared_norm = instance_norm(f"G/resblocks.{3 * s}/adain1.0", st.x)
        for j in range(3):
            st.res.append(block(f"G/resblocks.{3 * s + j}", st.x, C, T, shared_norm=st.shared_norm))
        m01, m012, st.mean = nm(f"G/Add_m{s}"), nm(f"G/Add_m{s}b"), nm(f"G/Div_m{s}")
        body.extend([
            ("Add", [st.res[0].pairs[-1].out, st.res[1].pairs[-1].out], [m01], {}),
            ("Add", [m01, st.res[2].pairs[-1].out], [m012], {}),
            ("Div", [m012, three[s]], [st.mean], {}),
        ])
        S.stages.append(st)
        x_in = st.mean
    S.final = nm("G/LeakyRelu_final")
    body.append(("LeakyRelu", [x_in], [S.final], {"alpha": 0.009999999776482582}))
    nodes.extend(prelude)
    nodes.extend(body)
    return S


LEAKY_STAGE = 0.10000000149011612   # LeakyRelu slope at each stage start (float32 0.1)
LEAKY_FINAL = 0.009999999776482582  # final LeakyRelu slope (float32 0.01)


def stream_algorithmic_bytes(S):
    """HBM bytes the fused plan must move per batch: each kernel reads every
    input element once and writes every output element once (fp32).  Per
    stage with n = B*C*T*4: noise_res 16n, shared-norm kernel 7n, resblocks
    3 * 14n, mean + LeakyRelu 7n = 72n; plus the features LeakyRelu and the
    per-stage gain Add."""
    B = S.batch
    st0 = S.stages[0]
    fb = 1
    for s in S.inputs[st0.x_in][0]:
        fb *= s
    total = 2 * fb * 4
    for st in S.stages:
        n = B * st.C * st.T * 4
        total += 72 * n
        total += 2 * len(S.adains(st)) * B * st.C * 4
    return total


def stream_launches(S):
    """Kernel launches of one FusedDecoder.launch()."""
    n = 1                                   # features LeakyRelu
    for st in S.stages:
        n += 1                              # gains
        n += 6 + 1 + 3 * 5                  # noise pairs, shared norm, resblock pairs
        n += 1                              # mean + LeakyRelu
    return n


class FusedDecoder:
    """B200 execution of a ``Stream`` (see module docstring).

    The decoder owns its device buffers.  ``inputs`` maps every input name of
    the stream (features, conv and fc stand-ins) to a CUDA tensor view the
    caller fills; the fc stand-ins of one stage live in one [n_adain, B, 2C]
    buffer so the 24 gain Adds of the stage are one launch.  ``launch()``
    issues the whole stream on the current CUDA stream with library kernels
    only (no torch compute), so it can be captured in a CUDA graph.
    ``out`` holds every tensor the plan materialises: all snake outputs, the
    residuals, and the two stage outputs."""

    def __init__(self, S, device=None):
        self.S = S
        self.device = as_cuda_device(device)
        self.lib = load()
        with torch.cuda.device(self.device):
            check(self.lib.bt_init(self.device.index), "bt_init")
        dev, B = self.device, S.batch
        f32 = dict(dtype=torch.float32, device=dev)
        self.inputs, self.out, self.t = {}, {}, {}
        for name, (shape, dt, kind) in S.inputs.items():
            if kind != "fc":
                self.inputs[name] = torch.empty(shape, **f32)
        self.fc_bufs, self.gain_bufs = [], []
        for st in S.stages:
            ads = S.adains(st)
            fc = torch.empty((len(ads), B, 2 * st.C), **f32)
            gains = torch.empty((len(ads), B, st.C), **f32)
            self.fc_bufs.append(fc)
            self.gain_bufs.append(gains)
            for i, a in enumerate(ads):
                self.inputs[a.fc] = fc[i].unsqueeze(-1)
                self.t[a.gain] = gains[i]
                self.t[a.beta] = fc[i, :, st.C:]
        for k, v in S.consts.items():
            self.t[k] = torch.from_numpy(np.ascontiguousarray(v)).to(dev)
        for st in S.stages:
            for blk in [st.noise] + st.res:
                for p in blk.pairs:
                    for a in (p.a1, p.a2):
                        self.out[a.snake] = torch.empty((B, st.C, st.T), **f32)
                for p in blk.pairs[1:]:
                    self.out[p.h] = torch.empty((B, st.C, st.T), **f32)
            self.out[st.x] = torch.empty((B, st.C, st.T), **f32)
        self.out[S.stages[0].leaky_in] = torch.empty(S.inputs[S.stages[0].x_in][0], **f32)
        self.out[S.stages[1].leaky_in] = torch.empty((B, S.stages[0].C, S.stages[0].T), **f32)
        self.out[S.final] = torch.empty((B, S.stages[1].C, S.stages[1].T), **f32)
        self._plan()

    def _ptr(self, name):
        for d in (self.inputs, self.out, self.t):
            if name in d:
                return d[name].data_ptr()
        raise KeyError(name)

    def _adain(self, st, srcs, res, adains):
        a = _lib.BtAdainArgs()
        a.rows, a.cols, a.channels = self.S.batch * st.C, st.T, st.C
        a.n_src, a.n_out = len(srcs), len(adains)
        for i, s in enumerate(srcs):
            a.src[i] = self._ptr(s)
        a.res = self._ptr(res) if res else None
        a.eps = float(np.float32(EPS))
        a.gain_stride, a.shift_stride = st.C, 2 * st.C
        a.alpha_dtype = _lib.BT_F16
        for i, ad in enumerate(adains):
            a.gain[i] = self._ptr(ad.gain)
            a.shift[i] = self._ptr(ad.beta)
            a.alpha[i] = self._ptr(ad.alpha)
            a.inv_alpha[i] = self._ptr(ad.inv_alpha)
            a.out[i] = self._ptr(ad.snake)
        return a

    def _plan(self):
        S, B = self.S, self.S.batch
        L = []
        st0 = S.stages[0]
        L.append(("ew", "LEAKYRELU", [self.inputs[st0.x_in]], self.out[st0.leaky_in], LEAKY_STAGE))
        # plan positions the host pipeline synchronises on: the first reader
        # of each stage's fc buffer and the last item of each stage (after it
        # the stage's fc buffer is free; the last one writes S.final)
        self.stage_first, self.stage_last = [], []
        for st in S.stages:
            fc, gains = self.fc_bufs[st.index], self.gain_bufs[st.index]
            self.stage_first.append(len(L))
            L.append(("ew", "ADD", [fc[:, :, :st.C], self.t["G/const/one"]], gains, 0.0))
            nb = st.noise
            for k, p in enumerate(nb.pairs):
                if k == 0:
                    L.append(("adain", self._adain(st, [st.noise_x], None, [p.a1])))
                else:
                    prev = nb.pairs[k - 1]
                    L.append(("adain", self._adain(st, [prev.c2, prev.h], p.h, [p.a1])))
                L.append(("adain", self._adain(st, [p.c1], None, [p.a2])))
            last = nb.pairs[-1]
            L.append(("adain", self._adain(st, [last.c2, last.h, st.ups], st.x,
                                           [blk.pairs[0].a1 for blk in st.res])))
            for blk in st.res:
                for k, p in enumerate(blk.pairs):
                    if k > 0:
                        prev = blk.pairs[k - 1]
                        L.append(("adain", self._adain(st, [prev.c2, prev.h], p.h, [p.a1])))
                    L.append(("adain", self._adain(st, [p.c1], None, [p.a2])))
            last_stage = st.index + 1 == len(S.stages)
            nxt = S.final if last_stage else S.stages[st.index + 1].leaky_in
            slope = LEAKY_FINAL if last_stage else LEAKY_STAGE
            a = (ctypes.c_void_p * 3)(*[self._ptr(blk.pairs[-1].c2) for blk in st.res])
            b = (ctypes.c_void_p * 3)(*[self._ptr(blk.pairs[-1].h) for blk in st.res])
            self.stage_last.append(len(L))
            L.append(("mean", a, b, B * st.C * st.T, float(np.float32(slope)), self._ptr(nxt)))
        # elementwise descriptors are built once, here
        plan = []
        for item in L:
            if item[0] == "ew":
                _, opname, ins, out, alpha = item
                descs = (_lib.BtTensor * len(ins))(*[tensor_desc(t) for t in ins])
                plan.append(("ew", _lib.OP[opname], len(ins), descs, tensor_desc(out),
                             _lib.BtEwAttrs(_lib.BT_F32, float(np.float32(alpha)))))
            else:
                plan.append(item)
        self.plan = plan
        assert len(plan) == stream_launches(S)

    def launch(self, record=None, wait=None, signal=None):
        """Issues the stream on the current CUDA stream; returns the number of
        kernel launches.  With ``record`` (a list), each launch is bracketed by
        CUDA events on that stream and ``(kind, rows, cols, n_src, n_out,
        has_res, start, end)`` is appended (timing of individual kernels).
        ``wait`` maps a plan position to CUDA events the stream waits for
        before that launch; ``signal`` maps a plan position to an event
        recorded right after it (both used by HostPipeline)."""
        lib = self.lib
        stream = torch.cuda.current_stream(self.device)
        check(lib.bt_set_stream(stream.cuda_stream), "bt_set_stream")
        for pos, item in enumerate(self.plan):
            for ev in (wait or {}).get(pos, ()):
                stream.wait_event(ev)
            kind = item[0]
            if record is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record(stream)
            if kind == "adain":
                check(lib.bt_adain_snake(ctypes.byref(item[1])), "bt_adain_snake")
            elif kind == "ew":
                _, op, n, descs, od, attrs = item
                check(lib.bt_elementwise(op, n, descs, ctypes.byref(od), ctypes.byref(attrs)), "bt_elementwise")
            else:
                _, a, b, nel, slope, out = item
                check(lib.bt_resblock_mean_leaky(a, b, nel, 3.0, slope, out), "bt_resblock_mean_leaky")
            if record is not None:
                ev1.record(stream)
                if kind == "adain":
                    A = item[1]
                    record.append((kind, A.rows, A.cols, A.n_src, A.n_out, bool(A.res), ev0, ev1))
                else:
                    record.append((kind, 0, 0, 0, 0, False, ev0, ev1))
            if signal and pos in signal:
                signal[pos].record(stream)
        return len(self.plan)

    # ---- end-to-end path (host buffers) ------------------------------------------
    def host_buffers(self, pin=True):
        """Pinned host buffers of the per-step inputs (features, the stacked
        fc outputs of each stage) and of the step's result (the final
        LeakyRelu output, the input of conv_post)."""
        S = self.S
        feat = S.stages[0].x_in
        hin = {feat: torch.empty(self.inputs[feat].shape, dtype=torch.float32, pin_memory=pin)}
        for i, fc in enumerate(self.fc_bufs):
            hin[f"fc{i}"] = torch.empty(fc.shape, dtype=torch.float32, pin_memory=pin)
        hout = torch.empty(self.out[S.final].shape, dtype=torch.float32, pin_memory=pin)
        return hin, hout

    def fill_host(self, hin, host):
        """Copies ``host_inputs()`` arrays into the pinned input buffers."""
        S = self.S
        feat = S.stages[0].x_in
        hin[feat].copy_(torch.from_numpy(host[feat]))
        for i, st in enumerate(S.stages):
            stacked = np.stack([host[a.fc].reshape(S.batch, 2 * st.C) for a in S.adains(st)])
            hin[f"fc{i}"].copy_(torch.from_numpy(stacked))

    def host_pipeline(self, hin, hout):
        """A HostPipeline over this decoder and the given host buffers."""
        return HostPipeline(self, hin, hout)

    def run_host(self, hin, hout):
        """One end-to-end step on the current stream: host-to-device copies
        of the step's inputs, the fused stream, device-to-host copy of the
        result.  Returns (h2d_bytes, d2h_bytes)."""
        S = self.S
        feat = S.stages[0].x_in
        self.inputs[feat].copy_(hin[feat], non_blocking=True)
        h2d = hin[feat].numel() * 4
        for i, fc in enumerate(self.fc_bufs):
            fc.copy_(hin[f"fc{i}"], non_blocking=True)
            h2d += fc.numel() * 4
        self.launch()
        hout.copy_(self.out[S.final], non_blocking=True)
        return h2d, hout.numel() * 4


def fc_weights(S, seed=1):
    """Random Linear(128 -> 2C) weights of every AdaIN fc, in stream order."""
    rng = np.random.default_rng(seed)
    ws = []
    for st in S.stages:
        for _ in S.adains(st):
            w = (rng.standard_normal((2 * st.C, STYLE_DIM)) / np.sqrt(STYLE_DIM)).astype(np.float32)
            b = (rng.standard_normal(2 * st.C) * 0.1).astype(np.float32)
            ws.append((w, b))
    return ws


def host_inputs(S, seed=0):
    """Host-side per-step inputs of the stream: features [B,512,T0] ~ N(0,1),
    style [B,128] ~ N(0,1), and the fc outputs h = fc(style) of every AdaIN
    (float64 Linear rounded to float32, see configs.adain_affine), in
    stream order.  Drawn from np.random.default_rng(seed)."""
    from .configs import adain_affine
    rng = np.random.default_rng(seed)
    feat_name = S.stages[0].x_in
    feats = rng.standard_normal(S.inputs[feat_name][0], dtype=np.float32)
    style = rng.standard_normal((S.batch, STYLE_DIM), dtype=np.float32)
    out = {feat_name: feats, "style": style}
    i = 0
    ws = fc_weights(S)
    for st in S.stages:
        for a in S.adains(st):
            w, b = ws[i]
            out[a.fc] = adain_affine(style, w, b).reshape(S.batch, 2 * st.C, 1)
            i += 1
    return out


def fill_conv_standins(dec, seed=0):
    """Seeded N(0,1) conv-output stand-ins, drawn on the GPU (setup only)."""
    g = torch.Generator(device=dec.device)
    for i, (name, (shape, dt, kind)) in enumerate(sorted(dec.S.inputs.items())):
        if kind == "conv":
            g.manual_seed(seed * 1000003 + i)
            dec.inputs[name].normal_(0.0, 1.0, generator=g)


def load_host_inputs(dec, host):
    """Copies host inputs (features, fc outputs) into the decoder's buffers."""
    for name, arr in host.items():
        if name in dec.inputs:
            dec.inputs[name].copy_(torch.from_numpy(np.ascontiguousarray(arr)).reshape(dec.inputs[name].shape),
                                   non_blocking=False)


class HostPipeline:
    """End-to-end steps whose host transfers overlap the neighbouring steps'
    compute (the serving loop of the host-buffer API).

    Each ``step()`` copies the step's inputs from the pinned host buffers,
    runs the fused stream on the current stream and copies the final stage
    output back, like ``FusedDecoder.run_host``, but with the copies on two
    side streams (host-to-device and device-to-host run concurrently over the
    full-duplex link), ordered by events instead of by the compute stream:

    - the features of step i+1 are copied once step i's first kernel has
      read them, each stage's fc outputs once step i's last kernel of that
      stage has run;
    - step i's result is copied out while step i+1 computes; step i+1's last
      kernel, which rewrites that buffer, waits for the copy.

    ``finish()`` makes the current stream wait for the last copy-out; after
    it, ``hout`` holds the last step's result."""

    def __init__(self, dec, hin, hout):
        self.dec, self.hin, self.hout = dec, hin, hout
        self.h2d = torch.cuda.Stream(dec.device)
        self.d2h = torch.cuda.Stream(dec.device)
        self.prev = None

    def step(self):
        dec, S = self.dec, self.dec.S
        comp = torch.cuda.current_stream(dec.device)
        feat = S.stages[0].x_in
        prev = self.prev
        ev = lambda: torch.cuda.Event()   # noqa: E731
        cur = {"feat_free": ev(), "fc_free": [ev() for _ in S.stages], "d2h_done": ev()}
        feat_ready, fc_ready = ev(), [ev() for _ in S.stages]
        h2d = self.hin[feat].numel() * 4
        with torch.cuda.stream(self.h2d):
            if prev is None:
                self.h2d.wait_stream(comp)
            else:
                self.h2d.wait_event(prev["feat_free"])
            dec.inputs[feat].copy_(self.hin[feat], non_blocking=True)
            feat_ready.record(self.h2d)
            for i, fc in enumerate(dec.fc_bufs):
                if prev is not None:
                    self.h2d.wait_event(prev["fc_free"][i])
                fc.copy_(self.hin[f"fc{i}"], non_blocking=True)
                fc_ready[i].record(self.h2d)
                h2d += fc.numel() * 4
        wait = {0: [feat_ready]}
        for i, pos in enumerate(dec.stage_first):
            wait.setdefault(pos, []).append(fc_ready[i])
        last = dec.stage_last[-1]
        if prev is not None:
            wait.setdefault(last, []).append(prev["d2h_done"])
        signal = {0: cur["feat_free"]}
        for i, pos in enumerate(dec.stage_last):
            signal[pos] = cur["fc_free"][i]
        out_ready = cur["fc_free"][-1]   # the last stage's last kernel writes S.final
        dec.launch(wait=wait, signal=signal)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(out_ready)
            self.hout.copy_(dec.out[S.final], non_blocking=True)
            cur["d2h_done"].record(self.d2h)
        self.prev = cur
        return h2d, self.hout.numel() * 4

    def finish(self):
        if self.prev is not None:
            torch.cuda.current_stream(self.dec.device).wait_event(self.prev["d2h_done"])

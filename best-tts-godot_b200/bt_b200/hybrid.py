"""Whole-graph driver: a packed model's nodes through the GPU op table where
the op is on the B200 path and through a CPU op table everywhere else.

The reference runs a packed model by walking its nodes and calling
``RefRuntime.dispatch`` for each (tools/kpk_runtime.py:52-81).
``HybridRuntime`` has the same ``dispatch`` signature, so it drops into that
loop in place of the ``RefRuntime`` instance:

* ops in ``BtRuntime.HOT_OPS`` run on the GPU (``BtRuntime.dispatch``);
  numpy inputs (weights, outputs of CPU ops) are uploaded on first use and
  cached by the GPU table;
* every other op (convolutions, LSTM, STFT, Gather, ...) runs on the CPU
  table it wraps -- the reference's own ``RefRuntime`` -- with its CUDA
  inputs copied to the host once each (numpy's axis order kept) and its
  outputs left in ``env`` as numpy arrays.

A tensor therefore crosses between host and device only where its consumer
runs on the other side, once per direction.  ``stats`` counts the nodes on
each side and the bytes moved.
"""
import weakref

import numpy as np
import torch

from .runtime import BtRuntime


class HybridRuntime:
    def __init__(self, cpu_runtime, device=None, gpu_ops=None, gpu_runtime=None):
        """cpu_runtime: any object with ``dispatch(op, node_input,
        node_output, at, env)`` over numpy arrays (the reference's
        RefRuntime).  gpu_ops: the ops sent to the GPU (default: all of
        BtRuntime.HOT_OPS)."""
        self.cpu = cpu_runtime
        self.gpu = gpu_runtime if gpu_runtime is not None else BtRuntime(device)
        self.gpu_ops = frozenset(BtRuntime.HOT_OPS if gpu_ops is None else gpu_ops)
        unknown = self.gpu_ops - set(BtRuntime.HOT_OPS)
        if unknown:
            raise ValueError(f"not on the GPU path: {sorted(unknown)}")
        self._host = {}       # id(CUDA tensor) -> (weak reference to it, its host copy)
        self.stats = {"gpu_nodes": 0, "cpu_nodes": 0, "d2h_bytes": 0}

    def _to_host(self, t):
        hit = self._host.get(id(t))
        if hit is not None and hit[0]() is t:
            return hit[1]
        a = host_array(t, self._dense)
        self.stats["d2h_bytes"] += a.nbytes
        if len(self._host) >= 1024:
            # forget the copies of device tensors that no longer exist
            self._host = {k: v for k, v in self._host.items() if v[0]() is not None}
        self._host[id(t)] = (weakref.ref(t), a)
        return a

    def dispatch(self, op, node_input, node_output, at, env):
        if op in self.gpu_ops:
            self.gpu.dispatch(op, node_input, node_output, at, env)
            self.stats["gpu_nodes"] += 1
            return
        sub = {}
        for n in node_input:
            if n and n in env:
                v = env[n]
                sub[n] = self._to_host(v) if isinstance(v, torch.Tensor) else v
        self.cpu.dispatch(op, node_input, node_output, at, sub)
        for n in node_output:
            if n and n in sub:
                env[n] = sub[n]
        self.stats["cpu_nodes"] += 1

    def run_nodes(self, nodes, env):
        """Runs ``(op, inputs, outputs, attrs)`` nodes in order."""
        for op, ins, outs, at in nodes:
            try:
                self.dispatch(op, list(ins), list(outs), at, env)
            except Exception as exc:
                raise RuntimeError(f"{op} ({list(ins)} -> {list(outs)}): {exc}") from exc
        return env

    def result(self, value):
        """A graph output as numpy (the reference's drivers return arrays)."""
        return host_array(value, self._dense) if isinstance(value, torch.Tensor) else np.asarray(value)

    def _dense(self, t):
        return self.gpu._contig(t) if t.is_cuda else t.contiguous()


def host_array(t, dense=None):
    """numpy copy of a tensor in the tensor's own axis order: a permuted view
    comes back as a permuted view of a dense host array, as numpy would hold
    it.  A view with gaps is first made C-contiguous by ``dense``."""
    if t.is_contiguous():
        return t.cpu().numpy()
    order = sorted(range(t.dim()), key=lambda i: (-t.stride(i), i))
    phys = t.permute(order)
    if not phys.is_contiguous():
        return (dense(t) if dense is not None else t.contiguous()).cpu().numpy()
    inv = [0] * len(order)
    for i, p in enumerate(order):
        inv[p] = i
    return phys.cpu().numpy().transpose(inv)

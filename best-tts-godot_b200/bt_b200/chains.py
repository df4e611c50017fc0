"""Fused elementwise chains: the programs bt_fused_chain runs, and the pass
that finds them in a node list.

The reference runs every node as its own dispatch followed by a barrier
(executor.gd:678-699): Snake is five passes over its activation (Mul, Sin,
Pow 2, Mul, Add), DequantizeLinear followed by a gain Mul two
(executor.gd:822-827).  ``plan`` finds such runs of nodes whose intermediate
values nothing else reads, and ``BtRuntime.run_nodes`` executes each as one
``bt_fused_chain`` launch: every input read once, the result written once,
each op rounded as numpy rounds it (the kernels are bit-exact against the
op-by-op chain).

A chain is valid in float32 only where numpy computes each of its ops in
float32: every input is float32 or float16 (widened, ref_runtime.py:49-51),
except the quantised values and zero point of a DequantizeLinear (int8 /
uint8, which the reference casts to float32 itself, ref_runtime.py:631-636).
``FusedGroup.inputs_ok`` checks that on the actual tensors; a group whose
inputs fail it runs node by node.
"""
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import OP

FLOAT_DTYPES = (np.dtype(np.float32), np.dtype(np.float16))
QUANT_DTYPES = (np.dtype(np.int8), np.dtype(np.uint8))


def program(n_in, code, out_reg):
    """A bt_chain from [(opname, dst, a, b[, alpha])] register instructions."""
    prog = _lib.BtChain()
    prog.n_in = n_in
    prog.n_instr = len(code)
    prog.out_reg = out_reg
    for i, ins in enumerate(code):
        op, d, a, b = ins[:4]
        alpha = float(np.float32(ins[4])) if len(ins) > 4 else 0.0
        prog.instr[i] = _lib.BtChainInstr(OP[op], d, a, b, alpha)
    return prog


# The library's catalog (bt_chain_kind 0-7), inputs in the order listed.
def dequant_mul_program(with_zp):
    """Mul(DequantizeLinear(q, scale[, zp]), gain): inputs q, scale, gain[, zp]."""
    if with_zp:
        return program(4, [("SUB", 4, 0, 3), ("MUL", 4, 4, 1), ("MUL", 4, 4, 2)], 4)
    return program(3, [("MUL", 3, 0, 1), ("MUL", 3, 3, 2)], 3)


def dequant_program(with_zp):
    """DequantizeLinear(q, scale[, zp]) = (q [- zp]) * scale: inputs q, scale[, zp]."""
    if with_zp:
        return program(3, [("SUB", 3, 0, 2), ("MUL", 3, 3, 1)], 3)
    return program(2, [("MUL", 2, 0, 1)], 2)


def snake_program():
    """x + inv_alpha * sin(alpha * x) ** p in the graph's order (Mul, Sin,
    Pow, Mul, Add): inputs x, alpha, p, inv_alpha."""
    return program(4, [("MUL", 4, 1, 0), ("SIN", 4, 4, 4), ("POW", 4, 4, 2), ("MUL", 4, 3, 4),
                       ("ADD", 4, 0, 4)], 4)


def add_unary_program(unary, alpha=0.0):
    """unary(Add(x, y)) (unary SIGMOID or LEAKYRELU): inputs x, y."""
    return program(2, [("ADD", 2, 0, 1), (unary, 2, 2, 2, alpha)], 2)


def mul_add_program():
    """Add(Mul(x, g), b): inputs x, g, b."""
    return program(3, [("MUL", 3, 0, 1), ("ADD", 3, 3, 2)], 3)


@dataclass
class FusedGroup:
    """Nodes first..last of a node list replaced by one chain launch."""
    first: int
    last: int
    kind: str               # "dequant_mul", "snake", "add_sigmoid", "add_leaky", "mul_add"
    inputs: list            # env names, in the program's input order ("" = absent zero point)
    output: str
    alpha: float = 0.0      # LeakyRelu slope
    quant: tuple = ()       # positions of inputs that may be int8 / uint8
    nodes: tuple = ()       # positions of the fused nodes (first .. last)

    def prog(self):
        if self.kind == "dequant_mul":
            return dequant_mul_program(len(self.inputs) == 4)
        if self.kind == "snake":
            return snake_program()
        if self.kind == "add_sigmoid":
            return add_unary_program("SIGMOID")
        if self.kind == "add_leaky":
            return add_unary_program("LEAKYRELU", self.alpha)
        return mul_add_program()

    def inputs_ok(self, dtypes):
        """Whether numpy computes every op of the chain in float32 for inputs
        of these dtypes (then the float32 chain is bit-exact)."""
        for i, dt in enumerate(dtypes):
            ok = QUANT_DTYPES if i in self.quant else FLOAT_DTYPES
            if np.dtype(dt) not in ok:
                return False
        return True


def _uses(nodes):
    n = {}
    for _, ins, _, _ in nodes:
        for name in ins:
            if name:
                n[name] = n.get(name, 0) + 1
    return n


def plan(nodes, keep=()):
    """Non-overlapping FusedGroups of a node list, in order.  A run of nodes
    fuses only where each intermediate value is read by the next node of the
    run alone and is not in ``keep`` (values the caller needs afterwards)."""
    uses = _uses(nodes)
    keep = set(keep)
    consumer = {}
    for i, (_, ins, _, _) in enumerate(nodes):
        for name in ins:
            if name:
                consumer.setdefault(name, []).append(i)

    def single(name, j=None):
        """The one node reading `name` (after j), if the value may vanish."""
        if not name or name in keep or uses.get(name, 0) != 1:
            return None
        c = consumer[name][0]
        return c if j is None or c > j else None

    def node(i):
        op, ins, outs, at = nodes[i]
        return op, list(ins), list(outs), dict(at or {})

    groups = []
    taken = set()
    for i in range(len(nodes)):
        if i in taken:
            continue
        op, ins, outs, at = node(i)
        g = None
        if op == "DequantizeLinear" and len(outs) == 1:
            j = single(outs[0], i)
            if j is not None:
                op2, ins2, outs2, _ = node(j)
                if op2 == "Mul" and len(ins2) == 2 and outs[0] in ins2 and ins2[0] != ins2[1]:
                    gain = ins2[1] if ins2[0] == outs[0] else ins2[0]
                    zp = ins[2] if len(ins) > 2 and ins[2] else ""
                    names = [ins[0], ins[1], gain] + ([zp] if zp else [])
                    g = FusedGroup(i, j, "dequant_mul", names, outs2[0], quant=(0, 3), nodes=(i, j))
        elif op == "Mul" and len(ins) == 2:
            g = _match_snake(i, node, single) or _match_mul_add(i, node, single)
        elif op == "Add" and len(ins) == 2:
            j = single(outs[0], i)
            if j is not None:
                op2, ins2, outs2, at2 = node(j)
                if op2 == "Sigmoid":
                    g = FusedGroup(i, j, "add_sigmoid", [ins[0], ins[1]], outs2[0], nodes=(i, j))
                elif op2 == "LeakyRelu":
                    g = FusedGroup(i, j, "add_leaky", [ins[0], ins[1]], outs2[0],
                                   alpha=float(np.float32(at2.get("alpha", 0.01))), nodes=(i, j))
        if g is not None and not (set(g.nodes) & taken):
            groups.append(g)
            taken.update(g.nodes)
    return groups


def _match_snake(i, node, single):
    """Mul(alpha, x) -> Sin -> Pow(., p) -> Mul(inv, .) -> Add(x, .) (either
    operand order of the Muls and the Add: IEEE products and sums are
    commutative bit for bit)."""
    _, ins, outs, _ = node(i)
    chain = [i]
    j = single(outs[0], i)
    if j is None or node(j)[0] != "Sin":
        return None
    chain.append(j)
    k = single(node(j)[2][0], j)
    if k is None or node(k)[0] != "Pow" or node(k)[1][0] != node(j)[2][0]:
        return None
    p = node(k)[1][1]
    chain.append(k)
    m = single(node(k)[2][0], k)
    if m is None or node(m)[0] != "Mul":
        return None
    mins = node(m)[1]
    pw = node(k)[2][0]
    if mins.count(pw) != 1:
        return None
    inv = mins[1] if mins[0] == pw else mins[0]
    chain.append(m)
    n = single(node(m)[2][0], m)
    if n is None or node(n)[0] != "Add":
        return None
    ains = node(n)[1]
    q = node(m)[2][0]
    if ains.count(q) != 1:
        return None
    x = ains[1] if ains[0] == q else ains[0]
    if x not in ins or ins[0] == ins[1]:
        return None
    alpha = ins[1] if ins[0] == x else ins[0]
    chain.append(n)
    return FusedGroup(i, n, "snake", [x, alpha, p, inv], node(n)[2][0], nodes=tuple(chain))


def _match_mul_add(i, node, single):
    _, ins, outs, _ = node(i)
    j = single(outs[0], i)
    if j is None:
        return None
    op2, ins2, outs2, _ = node(j)
    if op2 != "Add" or ins2.count(outs[0]) != 1:
        return None
    b = ins2[1] if ins2[0] == outs[0] else ins2[0]
    return FusedGroup(i, j, "mul_add", [ins[0], ins[1], b], outs2[0], nodes=(i, j))

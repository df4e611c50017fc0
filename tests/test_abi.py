"""The C ABI without a GPU: exports, error paths, the broadcast planner and
the library's float32 math evaluated on the host."""
import ctypes
import os
import re

import numpy as np
import pytest

from bt_b200 import _lib

HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = os.path.join(os.path.dirname(HERE), "include", "bt_ops.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bt_[a-z0-9_]+)\s*\(", src)))


def test_header_and_binding_agree(lib):
    decl = declared_functions()
    assert decl, "no declarations parsed"
    assert sorted(_lib.SIGNATURES) == decl


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.bt_abi_version() == 1


def test_errors_set_message(lib):
    rc = lib.bt_elementwise(0, 0, None, None, None)
    assert rc == -1
    assert b"n_in" in lib.bt_last_error()
    x = _lib.make_tensor(0, np.float32, (4,))
    attrs = _lib.BtEwAttrs(_lib.BT_F32, 0.0)
    ins = (_lib.BtTensor * 1)(x)
    rc = lib.bt_elementwise(99, 1, ins, ctypes.byref(x), ctypes.byref(attrs))
    assert rc == -1 and b"unknown op" in lib.bt_last_error()
    rc = lib.bt_reduce(7, ctypes.byref(x), None, 0, 1, ctypes.byref(x))
    assert rc == -1
    args = _lib.BtAdainArgs()
    args.rows, args.cols, args.channels, args.n_src, args.n_out = 4, 8, 2, 0, 1
    assert lib.bt_adain_snake(ctypes.byref(args)) == -1
    args.n_src = 1
    assert lib.bt_adain_snake(ctypes.byref(args)) == -1     # src[0] null
    assert b"src[0]" in lib.bt_last_error()
    assert lib.bt_adain_snake_range(ctypes.byref(args), ctypes.c_void_p(16)) == -1     # validated first
    assert b"src[0]" in lib.bt_last_error()
    args.src[0] = args.out[0] = args.gain[0] = args.shift[0] = 16
    args.gain_stride = args.shift_stride = 2
    args.alpha_dtype = _lib.BT_F32
    assert lib.bt_adain_snake_range(ctypes.byref(args), None) == -1
    assert b"null range" in lib.bt_last_error()
    assert lib.bt_adain_snake_range(ctypes.byref(args), ctypes.c_void_p(20)) == -1
    assert b"16-byte" in lib.bt_last_error()
    y = _lib.make_tensor(0, np.uint8, (4,))
    assert lib.bt_dynamic_quantize_ranged(ctypes.byref(x), ctypes.byref(y), None, None, None) == -1
    assert lib.bt_selfcheck(8, 0, 16, None) == -1 and b"kind" in lib.bt_last_error()
    assert lib.bt_selfcheck(7, 1, 1 << 23, ctypes.c_void_p(16)) == -1 and b"2^23" in lib.bt_last_error()
    assert lib.bt_selfcheck(0, 0, 16, None) == -1 and b"null" in lib.bt_last_error()
    assert lib.bt_selfcheck(0, 1, 1 << 32, ctypes.c_void_p(16)) == -1


def _plan(shapes, out_shape):
    ops = [_lib.make_tensor(0, np.float32, s) for s in shapes]
    arr = (_lib.BtTensor * len(ops))(*ops)
    osh = (ctypes.c_int64 * max(1, len(out_shape)))(*out_shape)
    rank = ctypes.c_int(0)
    shp = (ctypes.c_int64 * 8)()
    st = (ctypes.c_int64 * (8 * len(ops)))()
    rc = _lib.load().bt_plan_broadcast(len(ops), arr, osh, len(out_shape), ctypes.byref(rank), shp, st)
    return rc, rank.value, list(shp[:rank.value]), [list(st[k * 8:k * 8 + rank.value]) for k in range(len(ops))]


def _walk(rank, shape, strides, n):
    """Element offsets the planned iteration visits, in order."""
    offs = []
    for i in range(n):
        rem, off = i, 0
        for d in range(rank - 1, -1, -1):
            c = rem % shape[d]
            rem //= shape[d]
            off += c * strides[d]
        offs.append(off)
    return offs


@pytest.mark.parametrize("shapes", [
    [(2, 3, 4), (3, 1)], [(5, 7), ()], [(4, 6), (4, 6)], [(2, 1, 5), (2, 4, 5)],
    [(1, 512, 1024), (1, 512, 1)], [(2, 1, 3, 1, 2), (1, 4, 1, 5, 1)], [(6,), (2, 1, 6)],
    [(512, 512, 3), (512, 1, 1), ()], [(8, 1, 1), (1, 9, 1), (1, 1, 10)]])
def test_planner_visits_numpy_broadcast_order(lib, shapes):
    out_shape = np.broadcast_shapes(*shapes)
    rc, rank, shape, strides = _plan(list(shapes) + [out_shape], out_shape)
    assert rc == 0
    n = int(np.prod(out_shape))
    assert int(np.prod(shape)) == n
    for k, s in enumerate(shapes):
        want = np.broadcast_to(np.arange(int(np.prod(s))).reshape(s), out_shape).reshape(-1)
        assert _walk(rank, shape, strides[k], n) == want.tolist()
    assert _walk(rank, shape, strides[-1], n) == list(range(n))


def test_planner_collapses_contiguous_axes(lib):
    rc, rank, shape, _ = _plan([(2, 3, 4, 5), (2, 3, 4, 5)], (2, 3, 4, 5))
    assert rc == 0 and rank == 1 and shape == [120]
    rc, rank, shape, st = _plan([(1, 512, 1024), (1, 512, 1), (1, 512, 1024)], (1, 512, 1024))
    assert rc == 0 and rank == 2 and shape == [512, 1024] and st[1] == [1, 0]


def test_planner_rejects_bad_broadcast(lib):
    rc, *_ = _plan([(3, 4), (5,)], (3, 4))
    assert rc == -2
    assert b"does not broadcast" in lib.bt_last_error()


def _host_math(kind, x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(1 if kind == 4 else x.size, np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    rc = _lib.load().bt_host_math(kind, x.ctypes.data_as(fp), out.ctypes.data_as(fp), x.size)
    assert rc == 0
    return out


def _inputs():
    rng = np.random.default_rng(11)
    return np.concatenate([rng.standard_normal(300_000).astype(np.float32) * 10,
                           rng.uniform(-2e5, 2e5, 300_000).astype(np.float32),
                           rng.integers(0, 2**32, 600_000, dtype=np.uint64).astype(np.uint32).view(np.float32)])


@pytest.mark.parametrize("kind,fn", [(0, np.exp), (1, np.sin), (2, np.cos),
                                     (3, lambda v: 1.0 / (1.0 + np.exp(-v)))])
def test_host_math_is_numpy_exact(lib, kind, fn):
    """The library's float32 exp / sin / cos / sigmoid (the code the kernels
    run) reproduce numpy bit for bit, except sin/cos beyond numpy's SIMD
    range, where numpy calls the C library (those may differ by 1 ulp)."""
    x = _inputs()
    with np.errstate(all="ignore"):
        want = fn(x).astype(np.float32)
    got = _host_math(kind, x)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    if kind in (1, 2):
        lim = 117435.992 if kind == 1 else 71476.0625
        big = ~(np.abs(x) <= lim)
        assert same[~big].all()
        from parity import ulp_distance
        assert ulp_distance(got[big], want[big]).max() <= 1
    else:
        assert same.all(), x[~same][:5]


@pytest.mark.parametrize("n", [0, 1, 5, 7, 8, 9, 100, 128, 129, 255, 510, 768, 2048, 4000, 24001, 100000])
def test_host_pairwise_sum_is_numpy_exact(lib, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    got = _host_math(4, x)[0]
    want = np.float32(x.sum())
    assert got.view(np.uint32) == want.view(np.uint32)


def test_fused_chain_validates_programs(lib):
    """bt_fused_chain rejects malformed programs before touching the GPU:
    bad header, unknown op, register out of range, a register read before
    anything wrote it, an output register never written."""
    from bt_b200 import chains
    x = _lib.make_tensor(0x1000, np.float32, (4,))
    one = (_lib.BtTensor * 1)(x)

    def status(prog):
        return lib.bt_fused_chain(ctypes.byref(prog), one, ctypes.byref(x)), lib.bt_chain_kind(ctypes.byref(prog))

    prog = _lib.BtChain()
    prog.n_in = 0
    assert status(prog) == (-1, -1)
    assert status(chains.program(1, [("ADD", 1, 0, 5)], 1)) == (-1, -1)         # r5 never written
    assert status(chains.program(1, [("ADD", 16, 0, 0)], 16)) == (-1, -1)       # register 16
    assert status(chains.program(1, [("WHERE", 1, 0, 0)], 1)) == (-1, -1)       # not a chain op
    assert status(chains.program(1, [("SIN", 1, 0, 0)], 2)) == (-1, -1)         # output never written
    assert b"never written" in lib.bt_last_error()
    bad = chains.program(1, [("ADD", 1, 0, 0)], 1)
    bad.instr[0].op = 99
    assert status(bad) == (-1, -1)


def test_chain_catalog_kinds(lib):
    """Programs are matched to the compiled catalog after renaming their
    registers to single-assignment form, so register reuse does not matter;
    any other valid program goes to the interpreter."""
    from bt_b200 import chains
    kind = lambda p: lib.bt_chain_kind(ctypes.byref(p))   # noqa: E731
    assert kind(chains.dequant_mul_program(False)) == 0
    assert kind(chains.dequant_mul_program(True)) == 1
    assert kind(chains.snake_program()) == 2
    assert kind(chains.add_unary_program("SIGMOID")) == 3
    assert kind(chains.mul_add_program()) == 4
    assert kind(chains.add_unary_program("LEAKYRELU", 0.1)) == 5
    assert kind(chains.dequant_program(False)) == 6
    assert kind(chains.dequant_program(True)) == 7
    # Snake written with fresh registers for every step: the same program
    fresh = chains.program(4, [("MUL", 4, 1, 0), ("SIN", 5, 4, 4), ("POW", 6, 5, 2), ("MUL", 7, 3, 6),
                               ("ADD", 8, 0, 7)], 8)
    assert kind(fresh) == 2
    # overwriting an input register is allowed (single-assignment renaming)
    assert kind(chains.program(2, [("ADD", 0, 0, 1), ("SIGMOID", 0, 0, 0)], 0)) == 3
    # other programs: the interpreter
    assert kind(chains.program(2, [("SUB", 2, 0, 1), ("EXP", 2, 2, 2)], 2)) == 64
    assert kind(chains.program(2, [("ADD", 2, 1, 0), ("SIGMOID", 2, 2, 2)], 2)) == 64   # operands swapped
    assert kind(chains.program(1, [], 0)) == 64


@pytest.mark.gpu
def test_ctypes_binding_without_torch_tensors():
    """A caller without torch: device memory from the CUDA runtime through
    ctypes, one broadcast Add through bt_elementwise, numpy's bits back."""
    import ctypes
    import os
    lib = ctypes.CDLL(_lib.LIB_PATH)
    cudart = None
    for name in ("/usr/local/cuda/lib64/libcudart.so", "libcudart.so", "libcudart.so.12"):
        try:
            cudart = ctypes.CDLL(name)
            break
        except OSError:
            continue
    if cudart is None:
        pytest.skip("no libcudart to load by name")

    class BtTensor(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                    ("shape", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8)]

    class BtEwAttrs(ctypes.Structure):
        _fields_ = [("compute_dtype", ctypes.c_int32), ("alpha", ctypes.c_float)]

    lib.bt_elementwise.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(BtTensor),
                                   ctypes.POINTER(BtTensor), ctypes.POINTER(BtEwAttrs)]
    lib.bt_last_error.restype = ctypes.c_char_p
    ptrs = []

    def device_copy(a):
        p = ctypes.c_void_p()
        assert cudart.cudaMalloc(ctypes.byref(p), ctypes.c_size_t(a.nbytes)) == 0
        ptrs.append(p)
        assert cudart.cudaMemcpy(p, a.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(a.nbytes), 1) == 0
        return p

    def view(p, shape, strides):
        t = BtTensor()
        t.data, t.dtype, t.rank = p, 10, len(shape)
        for i, (n, s) in enumerate(zip(shape, strides)):
            t.shape[i], t.strides[i] = n, s
        return t

    rng = np.random.default_rng(0)
    x = rng.standard_normal((512, 1024), dtype=np.float32)
    b = rng.standard_normal((512, 1), dtype=np.float32)
    try:
        dx, db, dy = device_copy(x), device_copy(b), device_copy(np.zeros_like(x))
        ins = (BtTensor * 2)(view(dx, (512, 1024), (1024, 1)), view(db, (512, 1024), (1, 0)))
        out = view(dy, (512, 1024), (1024, 1))
        assert lib.bt_init(0) == 0
        rc = lib.bt_elementwise(0, 2, ins, ctypes.byref(out), ctypes.byref(BtEwAttrs(10, 0.0)))
        assert rc == 0, lib.bt_last_error()
        assert lib.bt_sync() == 0
        y = np.empty_like(x)
        assert cudart.cudaMemcpy(y.ctypes.data_as(ctypes.c_void_p), dy, ctypes.c_size_t(y.nbytes), 2) == 0
        assert np.array_equal(y.view(np.uint32), (x + b).view(np.uint32))
    finally:
        for p in ptrs:
            cudart.cudaFree(p)

"""ctypes binding of libbt_ops.so (the C ABI declared in include/bt_ops.h).

The library is loaded from this package's directory.  There is no fallback:
if it is missing or fails to load, every entry point raises, so a GPU run can
never silently compute on the CPU.
"""
import ctypes
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbt_ops.so")
MAX_RANK = 8

# status codes (bt_ops.h)
BT_OK = 0
STATUS_NAMES = {-1: "BT_EINVAL", -2: "BT_ESHAPE", -3: "BT_EDTYPE", -4: "BT_ECUDA",
                -5: "BT_EUNSUPPORTED", -6: "BT_ETOOBIG"}

# element types (bt_dtype)
BT_BOOL, BT_I8, BT_U8, BT_I16, BT_U16, BT_I32, BT_U32, BT_I64, BT_U64, BT_F16, BT_F32, BT_F64 = range(12)
NP_TO_BT = {
    np.dtype(np.bool_): BT_BOOL, np.dtype(np.int8): BT_I8, np.dtype(np.uint8): BT_U8,
    np.dtype(np.int16): BT_I16, np.dtype(np.uint16): BT_U16, np.dtype(np.int32): BT_I32,
    np.dtype(np.uint32): BT_U32, np.dtype(np.int64): BT_I64, np.dtype(np.uint64): BT_U64,
    np.dtype(np.float16): BT_F16, np.dtype(np.float32): BT_F32, np.dtype(np.float64): BT_F64,
}

# elementwise op codes (bt_op; 0-31 follow runtime/ops.gd:12-19)
OP = {
    "ADD": 0, "SUB": 1, "MUL": 2, "DIV": 3, "POW": 4, "SQRT": 5, "EXP": 6, "SIN": 7,
    "COS": 8, "ATAN": 9, "TANH": 10, "SIGMOID": 11, "FLOOR": 12, "ROUND": 13,
    "LEAKYRELU": 14, "CLIP": 15, "EQUAL": 16, "GREATER": 17, "LESS": 18, "GEQ": 19,
    "AND": 20, "WHERE": 21, "CAST_INT": 22, "CAST_BOOL": 23, "IDENTITY": 24, "NEG": 25,
    "ABS": 26, "LOG": 27, "MIN": 28, "MAX": 29, "ERF": 30, "GELU": 31, "DEQUANT": 40,
}
CHAIN_MAX_INSTR = 16
CHAIN_MAX_IN = 6
ADAIN_MAX_SRC = 3
ADAIN_MAX_OUT = 3


class BtTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.c_int64 * MAX_RANK), ("strides", ctypes.c_int64 * MAX_RANK)]


class BtEwAttrs(ctypes.Structure):
    _fields_ = [("compute_dtype", ctypes.c_int32), ("alpha", ctypes.c_float)]


class BtChainInstr(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("dst", ctypes.c_int32), ("a", ctypes.c_int32),
                ("b", ctypes.c_int32), ("alpha", ctypes.c_float)]


class BtChain(ctypes.Structure):
    _fields_ = [("n_in", ctypes.c_int32), ("n_instr", ctypes.c_int32), ("out_reg", ctypes.c_int32),
                ("instr", BtChainInstr * CHAIN_MAX_INSTR)]


class BtAdainArgs(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("channels", ctypes.c_int64),
                ("n_src", ctypes.c_int32), ("n_out", ctypes.c_int32),
                ("src", ctypes.c_void_p * ADAIN_MAX_SRC), ("res", ctypes.c_void_p),
                ("eps", ctypes.c_float),
                ("gain_stride", ctypes.c_int64), ("shift_stride", ctypes.c_int64),
                ("gain", ctypes.c_void_p * ADAIN_MAX_OUT), ("shift", ctypes.c_void_p * ADAIN_MAX_OUT),
                ("alpha", ctypes.c_void_p * ADAIN_MAX_OUT), ("inv_alpha", ctypes.c_void_p * ADAIN_MAX_OUT),
                ("alpha_dtype", ctypes.c_int32),
                ("out", ctypes.c_void_p * ADAIN_MAX_OUT)]


# Every symbol include/bt_ops.h declares, with its ctypes signature.
_P = ctypes.POINTER
SIGNATURES = {
    "bt_abi_version": (ctypes.c_int, []),
    "bt_last_error": (ctypes.c_char_p, []),
    "bt_init": (ctypes.c_int, [ctypes.c_int]),
    "bt_set_stream": (ctypes.c_int, [ctypes.c_void_p]),
    "bt_sync": (ctypes.c_int, []),
    "bt_elementwise": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P(BtTensor), _P(BtTensor), _P(BtEwAttrs)]),
    "bt_fused_chain": (ctypes.c_int, [_P(BtChain), _P(BtTensor), _P(BtTensor)]),
    "bt_chain_kind": (ctypes.c_int, [_P(BtChain)]),
    "bt_reduce": (ctypes.c_int, [ctypes.c_int, _P(BtTensor), _P(ctypes.c_int64), ctypes.c_int, ctypes.c_int,
                                 _P(BtTensor)]),
    "bt_softmax": (ctypes.c_int, [_P(BtTensor), _P(BtTensor), ctypes.c_int, _P(BtTensor)]),
    "bt_layernorm": (ctypes.c_int, [_P(BtTensor), _P(BtTensor), _P(BtTensor), _P(BtTensor), _P(BtTensor),
                                    ctypes.c_int, ctypes.c_float, _P(BtTensor)]),
    "bt_adain_snake": (ctypes.c_int, [_P(BtAdainArgs)]),
    "bt_adain_snake_range": (ctypes.c_int, [_P(BtAdainArgs), ctypes.c_void_p]),
    "bt_resblock_mean_leaky": (ctypes.c_int, [_P(ctypes.c_void_p), _P(ctypes.c_void_p), ctypes.c_int64,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_void_p]),
    "bt_plan_broadcast": (ctypes.c_int, [ctypes.c_int, _P(BtTensor), _P(ctypes.c_int64), ctypes.c_int,
                                         _P(ctypes.c_int), _P(ctypes.c_int64), _P(ctypes.c_int64)]),
    "bt_host_math": (ctypes.c_int, [ctypes.c_int, _P(ctypes.c_float), _P(ctypes.c_float), ctypes.c_int64]),
    "bt_selfcheck": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p]),
    "bt_wait_timeouts": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "bt_dynamic_quantize": (ctypes.c_int, [_P(BtTensor), _P(BtTensor), ctypes.c_void_p, ctypes.c_void_p]),
    "bt_dynamic_quantize_noalloc": (ctypes.c_int, [_P(BtTensor), _P(BtTensor), ctypes.c_void_p, ctypes.c_void_p]),
    "bt_dynamic_quantize_ranged": (ctypes.c_int, [_P(BtTensor), _P(BtTensor), ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_void_p]),
    "bt_conv_int_epilogue": (ctypes.c_int, [_P(BtTensor)] * 5),
}

_lib = None
_lock = threading.Lock()


def load():
    """Loads libbt_ops.so once; raises RuntimeError if it is absent."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python best-tts-godot_b200/build.py` "
                    "(there is no CPU fallback for the B200 path)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class BtError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, what, code, msg):
        super().__init__(f"{what}: {msg} ({STATUS_NAMES.get(code, code)})")
        self.code = code


def check(rc, what):
    if rc != BT_OK:
        msg = load().bt_last_error()
        raise BtError(what, rc, msg.decode() if msg else "")
    return rc


def make_tensor(ptr, np_dtype, shape, strides=None):
    """Fills a BtTensor from a device pointer, numpy dtype, shape and element strides."""
    t = BtTensor()
    shape = tuple(int(s) for s in shape)
    if len(shape) > MAX_RANK:
        raise ValueError(f"rank {len(shape)} exceeds {MAX_RANK}")
    if strides is None:
        strides, acc = [], 1
        for s in reversed(shape):
            strides.append(acc)
            acc *= s
        strides = list(reversed(strides))
    t.data = ptr
    t.dtype = NP_TO_BT[np.dtype(np_dtype)]
    t.rank = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        t.shape[i] = s
        t.strides[i] = int(st)
    return t

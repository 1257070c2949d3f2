"""ctypes binding of libqb_gdn.so (include/qb_gdn.h).

The library is the product: every compute call below goes through its C ABI.  There is no
fallback: if the library is missing or a call fails, an exception says why.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqb_gdn.so")

QB_DTYPE_F32 = 0
QB_DTYPE_BF16 = 1
QB_OP_FWD = 0
QB_OP_BWD = 1
QB_OP_LAYER_FWD = 2
QB_OP_LAYER_BWD = 3
QB_OP_BWD_CKPT = 4
QB_ALGO_AUTO = 0
QB_ALGO_ROWS = 1
QB_ALGO_CHUNKED = 2

# Every extern "C" symbol include/qb_gdn.h declares.
SYMBOLS = (
    "qb_gdn_version", "qb_gdn_launches", "qb_gdn_workspace_bytes", "qb_gdn_saved_bytes", "qb_gdn_fwd", "qb_gdn_bwd",
    "qb_gdn_step", "qb_gdn_verify", "qb_gdn_keep_rows", "qb_gdn_gate_fwd", "qb_gdn_gate_bwd",
    "qb_gdn_gate_workspace_bytes", "qb_gdn_gate_bwd_noalloc", "qb_gdn_layer_saved_bytes", "qb_gdn_layer_fwd",
    "qb_gdn_layer_bwd", "qb_gdn_status", "qb_gdn_set_wait_limit", "qb_gdn_count_nonfinite",
    "qb_gdn_conv_workspace_bytes", "qb_gdn_conv_fwd", "qb_gdn_conv_bwd", "qb_gdn_conv_verify", "qb_gdn_keep_conv_rows",
    "qb_gdn_gated_norm_fwd", "qb_gdn_gated_norm_workspace_bytes", "qb_gdn_gated_norm_bwd", "qb_gdn_ckpt_bytes",
    "qb_gdn_bwd_from_ckpt",
)


class Desc(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("Hk", ctypes.c_int32), ("Hv", ctypes.c_int32),
        ("Dk", ctypes.c_int32), ("Dv", ctypes.c_int32), ("n_seqs", ctypes.c_int32),
        ("cu_seqlens", ctypes.c_void_p), ("cu_seqlens_host", ctypes.c_void_p),
        ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32), ("algo", ctypes.c_int32),
    ]


class ConvDesc(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("Hk", ctypes.c_int32), ("Hv", ctypes.c_int32),
        ("Dk", ctypes.c_int32), ("Dv", ctypes.c_int32), ("K", ctypes.c_int32), ("n_seqs", ctypes.c_int32),
        ("cu_seqlens", ctypes.c_void_p), ("cu_seqlens_host", ctypes.c_void_p), ("dtype", ctypes.c_int32),
    ]


class QbError(RuntimeError):
    pass


_lib = None


def load():
    """The loaded library (raises if it was never built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise QbError(f"{LIB_PATH} is missing: build it with `python -m quotebound_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64, cp = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_char_p
    dp = ctypes.POINTER(Desc)
    L.qb_gdn_version.restype = cp
    L.qb_gdn_version.argtypes = []
    L.qb_gdn_launches.restype = i64
    L.qb_gdn_launches.argtypes = []
    L.qb_gdn_workspace_bytes.restype = i64
    L.qb_gdn_workspace_bytes.argtypes = [dp, i32, cp, ctypes.c_int]
    L.qb_gdn_saved_bytes.restype = i64
    L.qb_gdn_saved_bytes.argtypes = [dp, cp, ctypes.c_int]
    L.qb_gdn_fwd.restype = ctypes.c_int
    L.qb_gdn_fwd.argtypes = [dp] + [vp] * 10 + [i64, vp, cp, ctypes.c_int]
    L.qb_gdn_bwd.restype = ctypes.c_int
    L.qb_gdn_bwd.argtypes = [dp] + [vp] * 16 + [i64, vp, cp, ctypes.c_int]
    L.qb_gdn_step.restype = ctypes.c_int
    L.qb_gdn_step.argtypes = [i32] * 7 + [vp] * 8 + [vp, cp, ctypes.c_int]
    L.qb_gdn_verify.restype = ctypes.c_int
    L.qb_gdn_verify.argtypes = [i32] * 8 + [vp] * 8 + [vp, cp, ctypes.c_int]
    L.qb_gdn_keep_rows.restype = ctypes.c_int
    L.qb_gdn_keep_rows.argtypes = [i32] * 5 + [vp] * 4 + [vp, cp, ctypes.c_int]
    L.qb_gdn_gate_fwd.restype = ctypes.c_int
    L.qb_gdn_gate_fwd.argtypes = [i64] + [i32] * 5 + [vp] * 10 + [vp, cp, ctypes.c_int]
    L.qb_gdn_gate_bwd.restype = ctypes.c_int
    L.qb_gdn_gate_bwd.argtypes = [i64] + [i32] * 5 + [vp] * 16 + [vp, i64, vp, cp, ctypes.c_int]
    L.qb_gdn_layer_saved_bytes.restype = i64
    L.qb_gdn_layer_saved_bytes.argtypes = [dp, cp, ctypes.c_int]
    L.qb_gdn_layer_fwd.restype = ctypes.c_int
    L.qb_gdn_layer_fwd.argtypes = [dp] + [vp] * 12 + [i64, vp, cp, ctypes.c_int]
    L.qb_gdn_layer_bwd.restype = ctypes.c_int
    L.qb_gdn_layer_bwd.argtypes = [dp] + [vp] * 20 + [i64, vp, cp, ctypes.c_int]
    L.qb_gdn_gate_bwd_noalloc.restype = ctypes.c_int
    L.qb_gdn_gate_bwd_noalloc.argtypes = [i64] + [i32] * 5 + [vp] * 16 + [vp, cp, ctypes.c_int]
    L.qb_gdn_gate_workspace_bytes.restype = i64
    L.qb_gdn_gate_workspace_bytes.argtypes = [i64, i32]
    L.qb_gdn_status.restype = ctypes.c_int
    L.qb_gdn_status.argtypes = [vp, ctypes.POINTER(i32), vp, cp, ctypes.c_int]
    L.qb_gdn_set_wait_limit.restype = ctypes.c_int
    L.qb_gdn_set_wait_limit.argtypes = [i32, i32, cp, ctypes.c_int]
    L.qb_gdn_count_nonfinite.restype = ctypes.c_int
    L.qb_gdn_count_nonfinite.argtypes = [vp, i64, i32, vp, vp, cp, ctypes.c_int]
    L.qb_gdn_ckpt_bytes.restype = i64
    L.qb_gdn_ckpt_bytes.argtypes = [dp, cp, ctypes.c_int]
    L.qb_gdn_bwd_from_ckpt.restype = ctypes.c_int
    L.qb_gdn_bwd_from_ckpt.argtypes = [dp] + [vp] * 16 + [i64, vp, cp, ctypes.c_int]
    cdp = ctypes.POINTER(ConvDesc)
    L.qb_gdn_conv_workspace_bytes.restype = i64
    L.qb_gdn_conv_workspace_bytes.argtypes = [cdp, cp, ctypes.c_int]
    L.qb_gdn_conv_fwd.restype = ctypes.c_int
    L.qb_gdn_conv_fwd.argtypes = [cdp] + [vp] * 8 + [i64, vp, cp, ctypes.c_int]
    L.qb_gdn_conv_bwd.restype = ctypes.c_int
    L.qb_gdn_conv_bwd.argtypes = [cdp] + [vp] * 11 + [i64, vp, cp, ctypes.c_int]
    L.qb_gdn_conv_verify.restype = ctypes.c_int
    L.qb_gdn_conv_verify.argtypes = [cdp] + [vp] * 7 + [vp, cp, ctypes.c_int]
    L.qb_gdn_keep_conv_rows.restype = ctypes.c_int
    L.qb_gdn_keep_conv_rows.argtypes = [i32] * 5 + [vp] * 4 + [vp, cp, ctypes.c_int]
    f32 = ctypes.c_float
    L.qb_gdn_gated_norm_fwd.restype = ctypes.c_int
    L.qb_gdn_gated_norm_fwd.argtypes = [i64, i32, i32, f32, i32] + [vp] * 4 + [vp, cp, ctypes.c_int]
    L.qb_gdn_gated_norm_workspace_bytes.restype = i64
    L.qb_gdn_gated_norm_workspace_bytes.argtypes = [i64, i32, i32]
    L.qb_gdn_gated_norm_bwd.restype = ctypes.c_int
    L.qb_gdn_gated_norm_bwd.argtypes = [i64, i32, i32, f32, i32] + [vp] * 7 + [vp, i64, vp, cp, ctypes.c_int]
    _lib = L
    return L


def err_buf():
    return ctypes.create_string_buffer(512)


def check(rc: int, err) -> None:
    if rc != 0:
        raise QbError(err.value.decode(errors="replace") or f"qb_gdn call failed ({rc})")


def version() -> str:
    return load().qb_gdn_version().decode()


def launches() -> int:
    """Kernels the library has launched in this process so far."""
    return int(load().qb_gdn_launches())


# Meaning of the device status codes (include/qb_gdn.h, qb_gdn_status).
STATUS_CODES = {
    1: "prep: the K / Q tiles", 2: "prep: K K^T, Q K^T",
    10: "forward walk: a chunk's tiles", 11: "forward walk: product round 1", 12: "forward walk: product round 2",
    13: "forward walk: product round 3", 14: "forward walk: the last chunk's output product",
    15: "forward walk: a chunk's P image",
    20: "reverse walk: a chunk's images and gates", 21: "reverse walk: product round 1",
    22: "reverse walk: product round 2", 23: "reverse walk: product round 3",
    26: "reverse walk: a chunk's P image and rows",
    30: "gradient: the [K; Q] image", 31: "gradient: a value head's P image and gates",
    34: "gradient: a slice's products", 35: "gradient: K K^T", 36: "gradient: the finalize's products",
    37: "gradient: a slice's tiles",
}


def status(ws, stream) -> int:
    """The device status code the last call that used workspace ``ws`` (a CUDA tensor) left; syncs ``stream``."""
    err, code = err_buf(), ctypes.c_int32(0)
    check(load().qb_gdn_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(code), stream, err, len(err)), err)
    return int(code.value)


def set_wait_limit(code: int, polls: int = 1) -> None:
    """Test hook: the bounded wait with this code gives up after ``polls`` polls (code 0 = off)."""
    err = err_buf()
    check(load().qb_gdn_set_wait_limit(int(code), int(polls), err, len(err)), err)

"""Host-side checks of a call's outcome: the device status its bounded waits left, and the finite
check of the reference's training step.

quotebound refuses a training step whose loss or gradient norm is not finite (src/train.cpp:266-271)
and throws on bad shapes (src/delta_grad.cpp:164-170).  Here the recurrence's calls are asynchronous,
so both checks read device-side results back: ``require_ok`` the status code that opens the call's
workspace (qb_gdn_status; nonzero when a bounded wait gave up and the outputs are not valid) and
``require_finite`` the count of NaN / infinite entries (qb_gdn_count_nonfinite).  Each synchronises
the current stream, so they are opt-in: ``check=True`` on a call, or ``QB_GDN_CHECK=1`` in the
environment for every call.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from ._lib import QbError, check, err_buf, load

DEFAULT = os.environ.get("QB_GDN_CHECK", "0") not in ("", "0")


def enabled(flag) -> bool:
    return DEFAULT if flag is None else bool(flag)


def nonfinite(t: torch.Tensor) -> int:
    """Number of NaN or infinite entries of a float32 / bfloat16 CUDA tensor (syncs its stream)."""
    if t.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"finite check: float32 or bfloat16 only (got {t.dtype})")
    t = t.contiguous()
    count = torch.empty(1, dtype=torch.int64, device=t.device)
    err = err_buf()
    dtype = _lib.QB_DTYPE_BF16 if t.dtype == torch.bfloat16 else _lib.QB_DTYPE_F32
    stream = ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
    check(load().qb_gdn_count_nonfinite(ctypes.c_void_p(t.data_ptr()), t.numel(), dtype,
                                        ctypes.c_void_p(count.data_ptr()), stream, err, len(err)), err)
    return int(count.item())


def require_finite(what: str, **tensors) -> None:
    """Raises QbError naming every tensor with a NaN or infinite entry (None entries are skipped)."""
    bad = []
    for name, t in tensors.items():
        if t is not None:
            n = nonfinite(t)
            if n:
                bad.append(f"{name} ({n} of {t.numel()})")
    if bad:
        raise QbError(f"{what}: not finite: {', '.join(bad)}")


def require_ok(what: str, ws: torch.Tensor) -> None:
    """Raises QbError if the call that used workspace ``ws`` left a nonzero device status."""
    code = _lib.status(ws, ctypes.c_void_p(torch.cuda.current_stream(ws.device).cuda_stream))
    if code:
        raise QbError(f"{what}: device wait {code} gave up ({_lib.STATUS_CODES.get(code, 'unknown')}); "
                      "the outputs of this call are not valid")

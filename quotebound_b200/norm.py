"""The gated RMSNorm after the recurrence, over the C ABI (qb_gdn_gated_norm_*).

quotebound's deltanet() ends with o = precise_swiglu(y, z, rms_norm(y, w.norm, eps))
(src/deltanet.cpp:35-45, :122): per (token, value head) row, n = y rsqrt(mean(y^2) + eps) w rounded to
y's dtype, o = silu(z) n in float32 rounded to y's dtype.

* ``gated_norm_fwd(y, z, w, eps) -> o``;  ``gated_norm_bwd(y, z, w, do, eps) -> (dy, dz, dw)``
* ``gated_norm(y, z, w, eps)``  the two as a torch.autograd.Function
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import err_buf, load

__all__ = ["gated_norm_fwd", "gated_norm_bwd", "gated_norm"]


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dtype(t):
    if t.dtype == torch.bfloat16:
        return _lib.QB_DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.QB_DTYPE_F32
    raise ValueError(f"gated norm: bfloat16 or float32 only (got {t.dtype})")


def _shape(y):
    if y.dim() < 2:
        raise ValueError(f"gated norm: y must be [..., Hv, Dv] (got {tuple(y.shape)})")
    Hv, Dv = y.shape[-2], y.shape[-1]
    return y.numel() // (Hv * Dv), Hv, Dv


def gated_norm_fwd(y, z, w, eps=1e-6):
    y, z = y.contiguous(), z.to(y.dtype).contiguous()
    w = w.to(torch.float32).contiguous()
    P, Hv, Dv = _shape(y)
    o = torch.empty_like(y)
    err = err_buf()
    _lib.check(load().qb_gdn_gated_norm_fwd(P, Hv, Dv, float(eps), _dtype(y), _ptr(y), _ptr(z), _ptr(w), _ptr(o),
                                            ctypes.c_void_p(torch.cuda.current_stream(y.device).cuda_stream), err,
                                            len(err)), err)
    return o


def gated_norm_bwd(y, z, w, do, eps=1e-6, want_dw=True):
    y, z, do = y.contiguous(), z.to(y.dtype).contiguous(), do.to(y.dtype).contiguous()
    w = w.to(torch.float32).contiguous()
    P, Hv, Dv = _shape(y)
    dy, dz = torch.empty_like(y), torch.empty_like(y)
    dw = torch.empty(Dv, dtype=torch.float32, device=y.device) if want_dw else None
    n = int(load().qb_gdn_gated_norm_workspace_bytes(P, Hv, Dv))
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=y.device)
    err = err_buf()
    _lib.check(load().qb_gdn_gated_norm_bwd(P, Hv, Dv, float(eps), _dtype(y), _ptr(y), _ptr(z), _ptr(w), _ptr(do),
                                            _ptr(dy), _ptr(dz), _ptr(dw), _ptr(ws), n,
                                            ctypes.c_void_p(torch.cuda.current_stream(y.device).cuda_stream), err,
                                            len(err)), err)
    return dy, dz, dw


class _GatedNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, z, w, eps):
        ctx.save_for_backward(y, z, w)
        ctx.eps = eps
        return gated_norm_fwd(y, z, w, eps)

    @staticmethod
    def backward(ctx, do):
        y, z, w = ctx.saved_tensors
        dy, dz, dw = gated_norm_bwd(y, z, w, do, ctx.eps)
        return dy, dz, dw.to(w.dtype), None


def gated_norm(y, z, w, eps=1e-6):
    return _GatedNorm.apply(y, z, w, eps)

"""The recurrence with its norm and gate graph fused in, over the C ABI (qb_gdn_layer_fwd / _bwd).

This is the middle of quotebound's deltanet() (src/deltanet.cpp:94-100, compute_g :22-33) from the conv
outputs to y: q, k are the raw rows, normalised inside as the model does (rms_norm rounded to bf16, times
the bf16 scalar 1/Dk for q and 1/sqrt(Dk) for k); log g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b).
The backward returns the gradients of the raw q, k, v, a, b and the per-head sums of dA_log, ddt_bias
(the reference freezes A_log and dt_bias, src/lora.cpp:19-23; this build also differentiates them).

Runs on the chunked tensor-core path only (bf16 activations, Dk = Dv = 128).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib, checks
from ._lib import err_buf, load
from .deltanet import _cu_pair, _empty_bytes, _prep, _ptr, _stream, make_desc

__all__ = ["gated_delta_layer_fwd", "gated_delta_layer_bwd", "gated_delta_layer"]


def _desc(q, v, cu_dev, cu_host, out_dtype, algo):
    if q.dtype != torch.bfloat16:
        raise ValueError("gated delta layer: q, k, v must be bfloat16")
    return make_desc(q, v, cu_dev, cu_host, torch.bfloat16, out_dtype, algo)


def _ws(d, op, dev):
    err = err_buf()
    n = load().qb_gdn_workspace_bytes(ctypes.byref(d), op, err, len(err))
    if n < 0:
        raise ValueError(err.value.decode())
    return _empty_bytes(n, dev), int(n)


def gated_delta_layer_fwd(q, k, v, a, b, A_log, dt_bias, state=None, *, cu_seqlens=None, save=False,
                          out_dtype=torch.bfloat16, algo=0, check=None):
    """y [B, T, Hv, Dv], final state(s), saved (or None).  ``check`` as in deltanet.gated_delta_fwd."""
    dev = q.device
    q, k, v = _prep(q, torch.bfloat16), _prep(k, torch.bfloat16), _prep(v, torch.bfloat16)
    a, b = _prep(a, torch.float32), _prep(b, torch.float32)
    A_log, dt_bias, state = _prep(A_log, torch.float32), _prep(dt_bias, torch.float32), _prep(state, torch.float32)
    cu_dev, cu_host = _cu_pair(cu_seqlens, dev)
    d = _desc(q, v, cu_dev, cu_host, out_dtype, algo)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    N = B if cu_host is None else cu_host.numel() - 1
    y = torch.empty(B, T, Hv, Dv, dtype=out_dtype, device=dev)
    hT = torch.empty(N, Hv, Dv, Dk, dtype=torch.float32, device=dev)
    saved = None
    if save:
        err = err_buf()
        n = load().qb_gdn_layer_saved_bytes(ctypes.byref(d), err, len(err))
        if n < 0:
            raise ValueError(err.value.decode())
        saved = _empty_bytes(n, dev)
    ws, wsb = _ws(d, _lib.QB_OP_LAYER_FWD, dev)
    err = err_buf()
    rc = load().qb_gdn_layer_fwd(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(A_log),
                                 _ptr(dt_bias), _ptr(state), _ptr(y), _ptr(hT), _ptr(saved), _ptr(ws), wsb,
                                 _stream(dev), err, len(err))
    _lib.check(rc, err)
    if checks.enabled(check):
        checks.require_ok("gated delta layer forward", ws)
        checks.require_finite("gated delta layer forward", y=y, state=hT)
    return y, hT, saved


def gated_delta_layer_bwd(q, k, v, a, b, A_log, dt_bias, state, dy, dstate=None, *, saved=None, cu_seqlens=None,
                          grad_dtype=torch.bfloat16, algo=0, check=None):
    """(dq, dk, dv, da, db, dA_log, ddt_bias, dstate0).  ``check`` as in deltanet.gated_delta_fwd."""
    dev = q.device
    q, k, v, dy = (_prep(t, torch.bfloat16) for t in (q, k, v, dy))
    a, b = _prep(a, torch.float32), _prep(b, torch.float32)
    A_log, dt_bias = _prep(A_log, torch.float32), _prep(dt_bias, torch.float32)
    state, dstate = _prep(state, torch.float32), _prep(dstate, torch.float32)
    cu_dev, cu_host = _cu_pair(cu_seqlens, dev)
    d = _desc(q, v, cu_dev, cu_host, grad_dtype, algo)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    N = B if cu_host is None else cu_host.numel() - 1
    dq = torch.empty(q.shape, dtype=grad_dtype, device=dev)
    dk = torch.empty(k.shape, dtype=grad_dtype, device=dev)
    dv = torch.empty(v.shape, dtype=grad_dtype, device=dev)
    da = torch.empty(a.shape, dtype=torch.float32, device=dev)
    db = torch.empty(b.shape, dtype=torch.float32, device=dev)
    dA = torch.empty(Hv, dtype=torch.float32, device=dev)
    ddt = torch.empty(Hv, dtype=torch.float32, device=dev)
    dh0 = torch.empty(N, Hv, Dv, Dk, dtype=torch.float32, device=dev)
    err = err_buf()
    n = load().qb_gdn_workspace_bytes(ctypes.byref(d), _lib.QB_OP_LAYER_BWD, err, len(err))
    if n < 0:
        raise ValueError(err.value.decode())
    ws = _empty_bytes(n, dev)
    rc = load().qb_gdn_layer_bwd(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(A_log),
                                 _ptr(dt_bias), _ptr(state), _ptr(dy), _ptr(dstate), _ptr(saved), _ptr(dq), _ptr(dk),
                                 _ptr(dv), _ptr(da), _ptr(db), _ptr(dA), _ptr(ddt), _ptr(dh0), _ptr(ws), int(n),
                                 _stream(dev), err, len(err))
    _lib.check(rc, err)
    if checks.enabled(check):
        checks.require_ok("gated delta layer backward", ws)
        checks.require_finite("gated delta layer backward", dq=dq, dk=dk, dv=dv, da=da, db=db, dA_log=dA,
                              ddt_bias=ddt, dstate=dh0)
    return dq, dk, dv, da, db, dA, ddt, dh0


class _Layer(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, a, b, A_log, dt_bias, state, cu_seqlens):
        y, hT, saved = gated_delta_layer_fwd(q, k, v, a, b, A_log, dt_bias, state, cu_seqlens=cu_seqlens, save=True)
        ctx.save_for_backward(q, k, v, a, b, A_log, dt_bias, state if state is not None else torch.empty(0), saved)
        ctx.has_state = state is not None
        ctx.cu = cu_seqlens
        return y, hT

    @staticmethod
    def backward(ctx, dy, dhT):
        q, k, v, a, b, A_log, dt_bias, state, saved = ctx.saved_tensors
        state = state if ctx.has_state else None
        if dy is None:
            dy = torch.zeros(v.shape, dtype=torch.bfloat16, device=v.device)
        dq, dk, dv, da, db, dA, ddt, dh0 = gated_delta_layer_bwd(q, k, v, a, b, A_log, dt_bias, state, dy, dhT,
                                                                 saved=saved, cu_seqlens=ctx.cu)
        return dq, dk, dv, da, db, dA, ddt, (dh0 if ctx.has_state else None), None


def gated_delta_layer(q, k, v, a, b, A_log, dt_bias, state=None, *, cu_seqlens=None):
    """(y, final state) with the library's backward attached."""
    return _Layer.apply(q, k, v, a, b, A_log, dt_bias, state, cu_seqlens)

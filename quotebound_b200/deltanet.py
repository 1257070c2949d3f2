"""Host-side mirror of quotebound's recurrence entry points over the C ABI (torch for memory and streams).

Same names, argument order and meaning as the reference:

* ``gated_delta(q, k, v, g, beta, state, train=False) -> (y, state)``  — src/deltanet.h:17-19
* ``gated_delta_trainable(q, k, v, g, beta, state) -> (y, state)``     — src/delta_grad.h:14-16
* ``gated_delta_vjp([q, k, v, g, beta, state], dy, dstate) -> [dq, dk, dv, dg, dbeta, dstate]``
                                                                          — src/delta_grad.h:18-20

Layouts: q, k [B, T, Hk, Dk]; v [B, T, Hv, Dv]; g, beta [B, T, Hv] float32; state [B, Hv, Dv, Dk]
float32.  y comes back in q's dtype and the state in float32 (src/deltanet.cpp:49-61).  Like the
reference, which feeds the op float32 (src/deltanet.cpp:54-60), inputs of mixed dtypes are computed in
float32; bf16 q, k, v are read as bf16 directly (every bf16 value is exact in float32, so nothing is
lost) and the recurrence itself always runs with a float32 state.

Errors: shape and dtype problems raise ``ValueError`` naming the shapes (src/delta_grad.cpp:164-170);
failures reported by the library raise ``QbError``.  Every call runs on the current CUDA stream.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib, checks
from ._lib import Desc, QbError, err_buf, load

__all__ = ["gated_delta", "gated_delta_trainable", "gated_delta_vjp", "gated_delta_fwd", "gated_delta_bwd",
           "gated_delta_bwd_from_ckpt", "ckpt_bytes", "saved_ckpt", "saved_bytes", "workspace_bytes", "QbError"]


def _dtype_code(t: torch.dtype) -> int:
    if t == torch.bfloat16:
        return _lib.QB_DTYPE_BF16
    if t == torch.float32:
        return _lib.QB_DTYPE_F32
    raise ValueError(f"gated delta: activations must be bfloat16 or float32 (got {t})")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _act_dtype(*xs) -> torch.dtype:
    ds = {x.dtype for x in xs if x is not None}
    return torch.bfloat16 if ds == {torch.bfloat16} else torch.float32


def _prep(x, dtype):
    if x is None:
        return None
    x = x if x.dtype == dtype else x.to(dtype)
    return x.contiguous()


def make_desc(q, v, cu_seqlens=None, cu_host=None, in_dtype=torch.bfloat16, out_dtype=None, algo=0):
    if q.dim() != 4 or v.dim() != 4:
        raise ValueError(f"gated delta: q must be [B, T, Hk, Dk] and v [B, T, Hv, Dv] (q {tuple(q.shape)}, "
                         f"v {tuple(v.shape)})")
    B, T, Hk, Dk = q.shape
    if v.shape[0] != B or v.shape[1] != T:
        raise ValueError(f"gated delta: q {tuple(q.shape)} and v {tuple(v.shape)} disagree on [B, T]")
    d = Desc()
    d.B, d.T, d.Hk, d.Dk = B, T, Hk, Dk
    d.Hv, d.Dv = v.shape[2], v.shape[3]
    d.in_dtype = _dtype_code(in_dtype)
    d.out_dtype = _dtype_code(out_dtype if out_dtype is not None else in_dtype)
    d.algo = algo
    if cu_seqlens is not None:
        d.n_seqs = cu_host.numel() - 1
        d.cu_seqlens = cu_seqlens.data_ptr()
        d.cu_seqlens_host = cu_host.data_ptr()
    return d


def _cu_pair(cu_seqlens, device):
    """(device int32, host int32) copies of the offsets."""
    if cu_seqlens is None:
        return None, None
    if isinstance(cu_seqlens, torch.Tensor):
        host = cu_seqlens.detach().to("cpu", torch.int32).contiguous()
        dev = cu_seqlens.to(device=device, dtype=torch.int32).contiguous()
    else:
        host = torch.tensor(list(cu_seqlens), dtype=torch.int32)
        dev = host.to(device)
    return dev, host


def workspace_bytes(desc: Desc, op: int) -> int:
    err = err_buf()
    n = load().qb_gdn_workspace_bytes(ctypes.byref(desc), op, err, len(err))
    if n < 0:
        raise ValueError(err.value.decode())
    return int(n)


def saved_bytes(desc: Desc) -> int:
    err = err_buf()
    n = load().qb_gdn_saved_bytes(ctypes.byref(desc), err, len(err))
    if n < 0:
        raise ValueError(err.value.decode())
    return int(n)


def _empty_bytes(n, device):
    return torch.empty(max(int(n), 1), dtype=torch.uint8, device=device)


def _check_inputs(q, k, v, g, beta, state, n_seqs):
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    if tuple(k.shape) != tuple(q.shape):
        raise ValueError(f"gated delta: q {tuple(q.shape)} and k {tuple(k.shape)} differ")
    for name, t in (("g", g), ("beta", beta)):
        if tuple(t.shape) != (B, T, Hv):
            raise ValueError(f"gated delta: {name} must be [B, T, Hv] = {(B, T, Hv)} (got {tuple(t.shape)})")
    if state is not None and tuple(state.shape) != (n_seqs, Hv, Dv, Dk):
        raise ValueError(f"gated delta: state must be {(n_seqs, Hv, Dv, Dk)} (got {tuple(state.shape)})")
    if not q.is_cuda:
        raise ValueError("gated delta: tensors must be on a CUDA device (the library has no CPU path)")


def gated_delta_fwd(q, k, v, g, beta, state=None, *, cu_seqlens=None, save=False, out_dtype=None, algo=0,
                    check=None):
    """The forward op.  Returns (y, final_state, saved) — saved is None unless ``save``.

    With ``cu_seqlens`` (N + 1 offsets) the batch is B = 1 and ``state`` is [N, Hv, Dv, Dk].  ``check``
    (default: ``QB_GDN_CHECK``) reads back the device status and checks y and the state for NaN / inf."""
    dev = q.device
    adt = _act_dtype(q, k, v)
    q, k, v = _prep(q, adt), _prep(k, adt), _prep(v, adt)
    g, beta = _prep(g, torch.float32), _prep(beta, torch.float32)
    state = _prep(state, torch.float32)
    cu_dev, cu_host = _cu_pair(cu_seqlens, dev)
    n_seqs = q.shape[0] if cu_host is None else cu_host.numel() - 1
    _check_inputs(q, k, v, g, beta, state, n_seqs)
    y_dtype = out_dtype or q.dtype
    d = make_desc(q, v, cu_dev, cu_host, adt, y_dtype if y_dtype in (torch.bfloat16, torch.float32)
                  else torch.float32, algo)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    y = torch.empty(B, T, Hv, Dv, dtype=torch.bfloat16 if d.out_dtype == _lib.QB_DTYPE_BF16 else torch.float32,
                    device=dev)
    hT = torch.empty(n_seqs, Hv, Dv, Dk, dtype=torch.float32, device=dev)
    saved = _empty_bytes(saved_bytes(d), dev) if save else None
    wsb = workspace_bytes(d, _lib.QB_OP_FWD)
    ws = _empty_bytes(wsb, dev)
    err = err_buf()
    rc = load().qb_gdn_fwd(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(y),
                           _ptr(hT), _ptr(saved), _ptr(ws), wsb, _stream(dev), err, len(err))
    _lib.check(rc, err)
    if checks.enabled(check):
        checks.require_ok("gated delta forward", ws)
        checks.require_finite("gated delta forward", y=y, state=hT)
    if y_dtype != y.dtype:
        y = y.to(y_dtype)
    return y, hT, saved


def gated_delta_bwd(q, k, v, g, beta, state, dy, dstate=None, *, saved=None, cu_seqlens=None, algo=0,
                    grad_dtype=None, check=None):
    """Cotangents (dq, dk, dv, dg, dbeta, dstate0) of the forward given dy and dstate (the final state's)."""
    dev = q.device
    adt = _act_dtype(q, k, v, dy)
    q, k, v, dy = _prep(q, adt), _prep(k, adt), _prep(v, adt), _prep(dy, adt)
    g, beta = _prep(g, torch.float32), _prep(beta, torch.float32)
    state = _prep(state, torch.float32)
    dstate = _prep(dstate, torch.float32)
    cu_dev, cu_host = _cu_pair(cu_seqlens, dev)
    n_seqs = q.shape[0] if cu_host is None else cu_host.numel() - 1
    _check_inputs(q, k, v, g, beta, state, n_seqs)
    if tuple(dy.shape) != tuple(v.shape):
        raise ValueError(f"gated delta: dy must match v {tuple(v.shape)} (got {tuple(dy.shape)})")
    gdt = grad_dtype or adt
    d = make_desc(q, v, cu_dev, cu_host, adt, gdt, algo)
    dq = torch.empty(q.shape, dtype=gdt, device=dev)
    dk = torch.empty(k.shape, dtype=gdt, device=dev)
    dv = torch.empty(v.shape, dtype=gdt, device=dev)
    dg = torch.empty(g.shape, dtype=torch.float32, device=dev)
    dbeta = torch.empty(beta.shape, dtype=torch.float32, device=dev)
    B, T, Hk, Dk = q.shape
    dh0 = torch.empty(n_seqs, v.shape[2], v.shape[3], Dk, dtype=torch.float32, device=dev)
    wsb = workspace_bytes(d, _lib.QB_OP_BWD)
    ws = _empty_bytes(wsb, dev)
    err = err_buf()
    rc = load().qb_gdn_bwd(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(dy),
                           _ptr(dstate), _ptr(saved), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(dbeta), _ptr(dh0),
                           _ptr(ws), wsb, _stream(dev), err, len(err))
    _lib.check(rc, err)
    if checks.enabled(check):
        checks.require_ok("gated delta backward", ws)
        checks.require_finite("gated delta backward", dq=dq, dk=dk, dv=dv, dg=dg, dbeta=dbeta, dstate=dh0)
    return dq, dk, dv, dg, dbeta, dh0


def ckpt_bytes(desc: Desc) -> int:
    err = err_buf()
    n = load().qb_gdn_ckpt_bytes(ctypes.byref(desc), err, len(err))
    if n < 0:
        raise ValueError(err.value.decode())
    return int(n)


def saved_ckpt(saved, q, v, cu_seqlens=None, algo=0):
    """The chunk-start states [N_chunks, Hv, Dv, Dk] float32 at the head of a training forward's saved
    buffer (a view, no copy)."""
    cu_dev, cu_host = _cu_pair(cu_seqlens, q.device)
    d = make_desc(q, v, cu_dev, cu_host, _act_dtype(q, v), None, algo)
    n = ckpt_bytes(d)
    return saved[:n].view(torch.float32).view(-1, v.shape[2], v.shape[3], q.shape[3])


def gated_delta_bwd_from_ckpt(q, k, v, g, beta, dy, ckpt, dstate=None, *, cu_seqlens=None, algo=0, grad_dtype=None,
                              check=None):
    """gated_delta_vjp given the chunk-start states ckpt [N_chunks, Hv, Dv, Dk] float32 (the reference's
    ckpt, src/delta_grad.cpp:172-181): (dq, dk, dv, dg, dbeta, dstate0)."""
    dev = q.device
    adt = _act_dtype(q, k, v, dy)
    q, k, v, dy = _prep(q, adt), _prep(k, adt), _prep(v, adt), _prep(dy, adt)
    g, beta = _prep(g, torch.float32), _prep(beta, torch.float32)
    ckpt, dstate = _prep(ckpt, torch.float32), _prep(dstate, torch.float32)
    cu_dev, cu_host = _cu_pair(cu_seqlens, dev)
    n_seqs = q.shape[0] if cu_host is None else cu_host.numel() - 1
    _check_inputs(q, k, v, g, beta, None, n_seqs)
    gdt = grad_dtype or adt
    d = make_desc(q, v, cu_dev, cu_host, adt, gdt, algo)
    if ckpt.numel() * 4 != ckpt_bytes(d):
        raise ValueError(f"gated delta: ckpt must hold {ckpt_bytes(d) // 4} floats (got {ckpt.numel()})")
    dq, dk = torch.empty(q.shape, dtype=gdt, device=dev), torch.empty(k.shape, dtype=gdt, device=dev)
    dv = torch.empty(v.shape, dtype=gdt, device=dev)
    dg = torch.empty(g.shape, dtype=torch.float32, device=dev)
    dbeta = torch.empty(beta.shape, dtype=torch.float32, device=dev)
    dh0 = torch.empty(n_seqs, v.shape[2], v.shape[3], q.shape[3], dtype=torch.float32, device=dev)
    wsb = workspace_bytes(d, _lib.QB_OP_BWD_CKPT)
    ws = _empty_bytes(wsb, dev)
    err = err_buf()
    rc = load().qb_gdn_bwd_from_ckpt(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), None, _ptr(dy),
                                     _ptr(dstate), _ptr(ckpt), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(dbeta),
                                     _ptr(dh0), _ptr(ws), wsb, _stream(dev), err, len(err))
    _lib.check(rc, err)
    if checks.enabled(check):
        checks.require_ok("gated delta backward from ckpt", ws)
        checks.require_finite("gated delta backward from ckpt", dq=dq, dk=dk, dv=dv, dg=dg, dbeta=dbeta, dstate=dh0)
    return dq, dk, dv, dg, dbeta, dh0


class _GatedDelta(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, state, cu_seqlens, algo):
        y, hT, saved = gated_delta_fwd(q, k, v, g, beta, state, cu_seqlens=cu_seqlens, save=True, algo=algo)
        ctx.save_for_backward(q, k, v, g, beta, state if state is not None else torch.empty(0), saved)
        ctx.has_state = state is not None
        ctx.cu_seqlens = cu_seqlens
        ctx.algo = algo
        return y, hT

    @staticmethod
    def backward(ctx, dy, dhT):
        q, k, v, g, beta, state, saved = ctx.saved_tensors
        state = state if ctx.has_state else None
        if dy is None:
            dy = torch.zeros(v.shape, dtype=v.dtype, device=v.device)
        dq, dk, dv, dg, dbeta, dh0 = gated_delta_bwd(q, k, v, g, beta, state, dy, dhT, saved=saved,
                                                     cu_seqlens=ctx.cu_seqlens, algo=ctx.algo)
        return (dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg.to(g.dtype), dbeta.to(beta.dtype),
                dh0 if ctx.has_state else None, None, None)


def gated_delta_trainable(q, k, v, g, beta, state=None, *, cu_seqlens=None, algo=0):
    """The forward with the library's backward attached (a torch.autograd.Function)."""
    return _GatedDelta.apply(q, k, v, g, beta, state, cu_seqlens, algo)


def gated_delta(q, k, v, g, beta, state=None, train=False, *, cu_seqlens=None, algo=0):
    """y [B, T, Hv, Dv] in q's dtype and the new state [B, Hv, Dv, Dk] float32 (src/deltanet.cpp:49-61)."""
    if train:
        y, s = gated_delta_trainable(q, k, v, g, beta, state, cu_seqlens=cu_seqlens, algo=algo)
        return y.to(q.dtype), s
    y, s, _ = gated_delta_fwd(q, k, v, g, beta, state, cu_seqlens=cu_seqlens, algo=algo)
    return y.to(q.dtype), s


def gated_delta_vjp(primals, dy, dstate, *, cu_seqlens=None, algo=0):
    """[dq, dk, dv, dg, dbeta, dstate] given the primals [q, k, v, g, beta, state] (src/delta_grad.h:18-20)."""
    q, k, v, g, beta, state = primals
    return list(gated_delta_bwd(q, k, v, g, beta, state, dy, dstate, cu_seqlens=cu_seqlens, algo=algo))

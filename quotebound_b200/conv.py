"""The causal depthwise conv1d + SiLU in front of the recurrence, over the C ABI (qb_gdn_conv_*).

quotebound's deltanet() (src/deltanet.cpp:74-93) convolves the projected channels x = in_proj_qkv(h)
[B, T, conv_dim] (q | k | v, conv_dim = 2 Hk Dk + Hv Dv) over time with K taps per channel (Qwen3.5:
K = 4), the K - 1 inputs before a sequence carried in the layer cache's conv state, applies SiLU and
splits the result into q, k, v.  Here the split is fused: the kernel writes contiguous q [B, T, Hk, Dk],
k [B, T, Hk, Dk], v [B, T, Hv, Dv] -- the raw rows quotebound_b200.layer normalises inside the
recurrence.

* ``conv_fwd(x, w, state=None, ...) -> (q, k, v, new_state)``  (the new state: src/deltanet.cpp:75-77)
* ``conv_bwd(...) -> (dx, dw, dstate)``
* ``causal_conv_silu(x, w, state, ...)``  the two as a torch.autograd.Function
* ``conv_verify(x, w, state, ...) -> (q, k, v, states)``  V drafted tokens as V one-token steps, bit for bit,
  every token's conv window kept (deltanet(..., rows), src/deltanet.cpp:79-87)
* ``keep_conv_rows(states, keep)``  the conv state after keep[n] accepted tokens (src/exact.cpp:151-159)
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import ConvDesc, err_buf, load

__all__ = ["conv_fwd", "conv_bwd", "causal_conv_silu", "conv_verify", "keep_conv_rows"]


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _dtype(t):
    if t.dtype == torch.bfloat16:
        return _lib.QB_DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.QB_DTYPE_F32
    raise ValueError(f"gated delta conv: bfloat16 or float32 only (got {t.dtype})")


def _desc(x, w, Hk, Dk, Hv, Dv, cu_dev=None, cu_host=None):
    if x.dim() != 3 or w.dim() != 2:
        raise ValueError(f"gated delta conv: x must be [B, T, conv_dim] and w [conv_dim, K] "
                         f"(x {tuple(x.shape)}, w {tuple(w.shape)})")
    cd = 2 * Hk * Dk + Hv * Dv
    if x.shape[2] != cd or w.shape[0] != cd:
        raise ValueError(f"gated delta conv: conv_dim = 2 Hk Dk + Hv Dv = {cd} (x {tuple(x.shape)}, w {tuple(w.shape)})")
    d = ConvDesc()
    d.B, d.T, d.Hk, d.Hv, d.Dk, d.Dv, d.K = x.shape[0], x.shape[1], Hk, Hv, Dk, Dv, w.shape[1]
    d.dtype = _dtype(x)
    if cu_dev is not None:
        d.n_seqs = cu_host.numel() - 1
        d.cu_seqlens, d.cu_seqlens_host = cu_dev.data_ptr(), cu_host.data_ptr()
    return d


def _cu(cu_seqlens, dev):
    if cu_seqlens is None:
        return None, None
    host = torch.as_tensor(cu_seqlens, dtype=torch.int32).cpu().contiguous()
    return host.to(dev), host


def _ws(d, dev):
    err = err_buf()
    n = load().qb_gdn_conv_workspace_bytes(ctypes.byref(d), err, len(err))
    if n < 0:
        raise ValueError(err.value.decode())
    return torch.empty(int(n), dtype=torch.uint8, device=dev), int(n)


def conv_fwd(x, w, state=None, *, Hk, Dk, Hv, Dv, cu_seqlens=None, want_state=True):
    """(q, k, v, new_state or None).  x [B, T, conv_dim], w [conv_dim, K] (x's dtype), state [N, K-1, conv_dim]."""
    dev = x.device
    x, w = x.contiguous(), w.to(x.dtype).contiguous()
    state = None if state is None else state.to(x.dtype).contiguous()
    cu_dev, cu_host = _cu(cu_seqlens, dev)
    d = _desc(x, w, Hk, Dk, Hv, Dv, cu_dev, cu_host)
    B, T = x.shape[:2]
    N = B if cu_host is None else cu_host.numel() - 1
    q = torch.empty(B, T, Hk, Dk, dtype=x.dtype, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(B, T, Hv, Dv, dtype=x.dtype, device=dev)
    so = torch.empty(N, d.K - 1, x.shape[2], dtype=x.dtype, device=dev) if want_state else None
    ws, n = _ws(d, dev)
    err = err_buf()
    _lib.check(load().qb_gdn_conv_fwd(ctypes.byref(d), _ptr(x), _ptr(w), _ptr(state), _ptr(q), _ptr(k), _ptr(v),
                                      _ptr(so), _ptr(ws), n, _stream(dev), err, len(err)), err)
    return q, k, v, so


def conv_bwd(x, w, state, dq, dk, dv, dstate=None, *, Hk, Dk, Hv, Dv, cu_seqlens=None, want_dw=True,
             want_dstate=True):
    """(dx, dw float32 or None, dstate_in or None)."""
    dev = x.device
    x, w = x.contiguous(), w.to(x.dtype).contiguous()
    state = None if state is None else state.to(x.dtype).contiguous()
    dq, dk, dv = (t.to(x.dtype).contiguous() for t in (dq, dk, dv))
    dstate = None if dstate is None else dstate.to(x.dtype).contiguous()
    cu_dev, cu_host = _cu(cu_seqlens, dev)
    d = _desc(x, w, Hk, Dk, Hv, Dv, cu_dev, cu_host)
    N = x.shape[0] if cu_host is None else cu_host.numel() - 1
    dx = torch.empty_like(x)
    dw = torch.empty(w.shape, dtype=torch.float32, device=dev) if want_dw else None
    dsi = torch.empty(N, d.K - 1, x.shape[2], dtype=x.dtype, device=dev) if want_dstate else None
    ws, n = _ws(d, dev)
    err = err_buf()
    _lib.check(load().qb_gdn_conv_bwd(ctypes.byref(d), _ptr(x), _ptr(w), _ptr(state), _ptr(dq), _ptr(dk), _ptr(dv),
                                      _ptr(dstate), _ptr(dx), _ptr(dw), _ptr(dsi), _ptr(ws), n, _stream(dev), err,
                                      len(err)), err)
    return dx, dw, dsi


class _Conv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, state, Hk, Dk, Hv, Dv, cu_seqlens):
        q, k, v, so = conv_fwd(x, w, state, Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv, cu_seqlens=cu_seqlens)
        ctx.save_for_backward(x, w, state if state is not None else torch.empty(0))
        ctx.meta = (Hk, Dk, Hv, Dv, cu_seqlens, state is not None)
        return q, k, v, so

    @staticmethod
    def backward(ctx, dq, dk, dv, dso):
        x, w, state = ctx.saved_tensors
        Hk, Dk, Hv, Dv, cu, has_state = ctx.meta
        z = lambda t, like: t if t is not None else torch.zeros(like, dtype=x.dtype, device=x.device)
        dq = z(dq, (x.shape[0], x.shape[1], Hk, Dk))
        dk = z(dk, (x.shape[0], x.shape[1], Hk, Dk))
        dv = z(dv, (x.shape[0], x.shape[1], Hv, Dv))
        dx, dw, dsi = conv_bwd(x, w, state if has_state else None, dq, dk, dv, dso, Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv,
                               cu_seqlens=cu, want_dstate=has_state)
        return dx, dw.to(w.dtype), dsi, None, None, None, None, None


def causal_conv_silu(x, w, state=None, *, Hk, Dk, Hv, Dv, cu_seqlens=None):
    """(q, k, v, new_state) with the library's backward attached."""
    return _Conv.apply(x, w, state, Hk, Dk, Hv, Dv, cu_seqlens)


def conv_verify(x, w, state, *, Hk, Dk, Hv, Dv):
    """x [N, V, conv_dim] drafted tokens, state [N, K-1, conv_dim] -> (q, k, v, states [N, V, K-1, conv_dim])."""
    dev = x.device
    x, w, state = x.contiguous(), w.to(x.dtype).contiguous(), state.to(x.dtype).contiguous()
    d = _desc(x, w, Hk, Dk, Hv, Dv)
    N, V = x.shape[:2]
    q = torch.empty(N, V, Hk, Dk, dtype=x.dtype, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(N, V, Hv, Dv, dtype=x.dtype, device=dev)
    states = torch.empty(N, V, d.K - 1, x.shape[2], dtype=x.dtype, device=dev)
    err = err_buf()
    _lib.check(load().qb_gdn_conv_verify(ctypes.byref(d), _ptr(x), _ptr(w), _ptr(state), _ptr(q), _ptr(k), _ptr(v),
                                         _ptr(states), _stream(dev), err, len(err)), err)
    return q, k, v, states


def keep_conv_rows(states, keep, out=None, status=None):
    """state_out[n] = states[n, keep[n] - 1]; keep int32 [N] on the host or device."""
    N, V, K1, cd = states.shape
    keep = torch.as_tensor(keep, dtype=torch.int32).to(states.device)
    out = torch.empty(N, K1, cd, dtype=states.dtype, device=states.device) if out is None else out
    err = err_buf()
    _lib.check(load().qb_gdn_keep_conv_rows(N, V, K1 + 1, cd, _dtype(states), _ptr(states.contiguous()), _ptr(keep),
                                            _ptr(out), _ptr(status), _stream(states.device), err, len(err)), err)
    return out

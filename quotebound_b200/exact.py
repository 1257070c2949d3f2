"""Decode-time recurrence over the C ABI: the one-token step, the exact multi-row verify and keep_rows.

* ``step(q, k, v, g, beta, state)`` — gated_delta on one token with the cached state (the decode path,
  src/deltanet.cpp:118-120 with S = 1).
* ``verify(q, k, v, g, beta, state)`` — V drafted tokens run as V one-token steps, bit for bit equal to
  V calls of ``step``, with every row's state kept (deltanet(..., rows), src/deltanet.cpp:102-117;
  RowStates, src/model.h:84-89).
* ``keep_rows(states, keep)`` — the state after ``keep[n]`` accepted tokens (src/exact.cpp:151-159).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, err_buf, load
from .deltanet import _act_dtype, _dtype_code, _prep, _ptr, _stream


def step(q, k, v, g, beta, state, *, out=None):
    """q, k [N, Hk, Dk]; v [N, Hv, Dv]; g, beta [N, Hv]; state [N, Hv, Dv, Dk] -> (y [N, Hv, Dv], new state).

    ``out`` may be ``state`` itself for an in-place update."""
    adt = _act_dtype(q, k, v)
    q, k, v = _prep(q, adt), _prep(k, adt), _prep(v, adt)
    g, beta, state = _prep(g, torch.float32), _prep(beta, torch.float32), _prep(state, torch.float32)
    N, Hk, Dk = q.shape
    Hv, Dv = v.shape[1], v.shape[2]
    if tuple(state.shape) != (N, Hv, Dv, Dk) or tuple(g.shape) != (N, Hv):
        raise ValueError(f"gated delta step: state {tuple(state.shape)} / g {tuple(g.shape)} do not fit "
                         f"q {tuple(q.shape)}, v {tuple(v.shape)}")
    y = torch.empty(N, Hv, Dv, dtype=adt, device=q.device)
    out = torch.empty_like(state) if out is None else out
    err = err_buf()
    code = _dtype_code(adt)
    rc = load().qb_gdn_step(N, Hk, Hv, Dk, Dv, code, code, _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                            _ptr(state), _ptr(y), _ptr(out), _stream(q.device), err, len(err))
    check(rc, err)
    return y, out


def verify(q, k, v, g, beta, state):
    """q, k [N, V, Hk, Dk]; v [N, V, Hv, Dv]; g, beta [N, V, Hv]; state [N, Hv, Dv, Dk]
    -> (y [N, V, Hv, Dv], states [N, V, Hv, Dv, Dk])."""
    adt = _act_dtype(q, k, v)
    q, k, v = _prep(q, adt), _prep(k, adt), _prep(v, adt)
    g, beta, state = _prep(g, torch.float32), _prep(beta, torch.float32), _prep(state, torch.float32)
    N, V, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    if tuple(state.shape) != (N, Hv, Dv, Dk) or tuple(g.shape) != (N, V, Hv):
        raise ValueError(f"gated delta verify: state {tuple(state.shape)} / g {tuple(g.shape)} do not fit "
                         f"q {tuple(q.shape)}, v {tuple(v.shape)}")
    y = torch.empty(N, V, Hv, Dv, dtype=adt, device=q.device)
    states = torch.empty(N, V, Hv, Dv, Dk, dtype=torch.float32, device=q.device)
    err = err_buf()
    code = _dtype_code(adt)
    rc = load().qb_gdn_verify(N, V, Hk, Hv, Dk, Dv, code, code, _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                              _ptr(state), _ptr(y), _ptr(states), _stream(q.device), err, len(err))
    check(rc, err)
    return y, states


def keep_rows(states, keep, out=None, status=None):
    """state after keep[n] tokens of sequence n: states [N, V, Hv, Dv, Dk], keep int [N] in [1, V]."""
    N, V, Hv, Dv, Dk = states.shape
    keep = keep.to(device=states.device, dtype=torch.int32).contiguous()
    out = torch.empty(N, Hv, Dv, Dk, dtype=torch.float32, device=states.device) if out is None else out
    err = err_buf()
    rc = load().qb_gdn_keep_rows(N, V, Hv, Dk, Dv, _ptr(states.contiguous()), _ptr(keep), _ptr(out), _ptr(status),
                                 _stream(states.device), err, len(err))
    check(rc, err)
    return out

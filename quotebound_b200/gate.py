"""The gate / beta / q-k norm graph around the recurrence, over the C ABI.

Forward (src/deltanet.cpp:94-100, compute_g :22-33):
    qn = q * rsqrt(mean(q^2) + 1e-6) / Dk;   kn = k * rsqrt(mean(k^2) + 1e-6) / sqrt(Dk)
    beta = sigmoid(b);   g = exp(-exp(A_log) * softplus(a + dt_bias))
Backward: the chain rule of all of it, with this call's per-head sums of dA_log and ddt_bias (the
reference freezes A_log and dt_bias, src/lora.cpp:19-23; this build also returns their gradients).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, err_buf, load
from .deltanet import _act_dtype, _dtype_code, _prep, _ptr, _stream


def gate_fwd(q, k, a, b, A_log, dt_bias, *, out_dtype=None):
    """q, k [..., Hk, Dk]; a, b [..., Hv] -> (qn, kn, g, beta)."""
    adt = _act_dtype(q, k)
    odt = out_dtype or adt
    q, k = _prep(q, adt), _prep(k, adt)
    a, b = _prep(a, torch.float32), _prep(b, torch.float32)
    A_log, dt_bias = _prep(A_log, torch.float32), _prep(dt_bias, torch.float32)
    Hk, Dk = q.shape[-2], q.shape[-1]
    Hv = a.shape[-1]
    P = a.numel() // Hv
    qn = torch.empty(q.shape, dtype=odt, device=q.device)
    kn = torch.empty(k.shape, dtype=odt, device=q.device)
    g = torch.empty(a.shape, dtype=torch.float32, device=q.device)
    beta = torch.empty(a.shape, dtype=torch.float32, device=q.device)
    err = err_buf()
    rc = load().qb_gdn_gate_fwd(P, Hk, Hv, Dk, _dtype_code(adt), _dtype_code(odt), _ptr(q), _ptr(k), _ptr(a),
                                _ptr(b), _ptr(A_log), _ptr(dt_bias), _ptr(qn), _ptr(kn), _ptr(g), _ptr(beta),
                                _stream(q.device), err, len(err))
    check(rc, err)
    return qn, kn, g, beta


def gate_bwd(q, k, a, b, A_log, dt_bias, dqn, dkn, dg, dbeta, *, out_dtype=None):
    """-> (dq, dk, da, db, dA_log, ddt_bias); dA_log and ddt_bias are this call's per-head sums."""
    adt = _act_dtype(q, k, dqn, dkn)
    odt = out_dtype or adt
    q, k, dqn, dkn = _prep(q, adt), _prep(k, adt), _prep(dqn, adt), _prep(dkn, adt)
    a, b = _prep(a, torch.float32), _prep(b, torch.float32)
    A_log, dt_bias = _prep(A_log, torch.float32), _prep(dt_bias, torch.float32)
    dg, dbeta = _prep(dg, torch.float32), _prep(dbeta, torch.float32)
    Hk, Dk = q.shape[-2], q.shape[-1]
    Hv = a.shape[-1]
    P = a.numel() // Hv
    dev = q.device
    dq = torch.empty(q.shape, dtype=odt, device=dev)
    dk = torch.empty(k.shape, dtype=odt, device=dev)
    da = torch.empty(a.shape, dtype=torch.float32, device=dev)
    db = torch.empty(a.shape, dtype=torch.float32, device=dev)
    dA = torch.empty(Hv, dtype=torch.float32, device=dev)
    ddt = torch.empty(Hv, dtype=torch.float32, device=dev)
    L = load()
    wsb = int(L.qb_gdn_gate_workspace_bytes(P, Hv))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    err = err_buf()
    rc = L.qb_gdn_gate_bwd(P, Hk, Hv, Dk, _dtype_code(adt), _dtype_code(odt), _ptr(q), _ptr(k), _ptr(a), _ptr(b),
                           _ptr(A_log), _ptr(dt_bias), _ptr(dqn), _ptr(dkn), _ptr(dg), _ptr(dbeta), _ptr(dq),
                           _ptr(dk), _ptr(da), _ptr(db), _ptr(dA), _ptr(ddt), _ptr(ws), wsb, _stream(dev), err,
                           len(err))
    check(rc, err)
    return dq, dk, da, db, dA, ddt

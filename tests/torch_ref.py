"""A float64 torch restatement of the reference's plain-ops recurrence, for cross-checks.

Written from the step equations of tests/gated_delta_ref.h:100-120 (the reference's
``gated_delta_ops``) and the gate/norm graph of src/deltanet.cpp:22-33,94-100.
Autograd through it is the independent check of the oracle's hand-written backward,
as the reference checks its own backward against autodiff through the plain ops
(tests/test_deltanet.cpp:105-137).  Test infrastructure only.
"""
from __future__ import annotations

import math

import torch


def gated_delta_ops(q, k, v, g, beta, state, cu_seqlens=None):
    """q, k [B,T,Hk,Dk]; v [B,T,Hv,Dv]; g, beta [B,T,Hv]; state [N,Hv,Dv,Dk] -> (y, final states)."""
    B, T, Hk, Dk = q.shape
    Hv = v.shape[2]
    r = Hv // Hk
    qr = q.repeat_interleave(r, dim=2) if r > 1 else q
    kr = k.repeat_interleave(r, dim=2) if r > 1 else k
    if cu_seqlens is None:
        segs = [(b, 0, T) for b in range(B)]
    else:
        cu = [int(x) for x in cu_seqlens]
        segs = [(0, cu[n], cu[n + 1]) for n in range(len(cu) - 1)]
    ys = torch.zeros(B, T, Hv, v.shape[3], dtype=q.dtype)
    finals = []
    y_rows = {}
    for n, (b, t0, t1) in enumerate(segs):
        S = state[n]
        for t in range(t0, t1):
            S = S * g[b, t][:, None, None]
            u = (S * kr[b, t][:, None, :]).sum(-1)
            d = (v[b, t] - u) * beta[b, t][:, None]
            S = S + kr[b, t][:, None, :] * d[:, :, None]
            y_rows[(b, t)] = (S * qr[b, t][:, None, :]).sum(-1)
        finals.append(S)
    y = torch.stack([torch.stack([y_rows[(b, t)] if (b, t) in y_rows else torch.zeros_like(ys[0, 0])
                                  for t in range(T)]) for b in range(B)])
    return y, torch.stack(finals)


def gate(q, k, a, b, A_log, dt_bias, eps=1e-6):
    """(qn, kn, g, beta) as src/deltanet.cpp:94-100 computes them, in float64."""
    Dk = q.shape[-1]
    qn = q * torch.rsqrt((q * q).mean(-1, keepdim=True) + eps) * (1.0 / Dk)
    kn = k * torch.rsqrt((k * k).mean(-1, keepdim=True) + eps) * (1.0 / math.sqrt(Dk))
    x = a + dt_bias
    sp = torch.logaddexp(x, torch.zeros_like(x))
    g = torch.exp(-torch.exp(A_log) * sp)
    return qn, kn, g, torch.sigmoid(b)

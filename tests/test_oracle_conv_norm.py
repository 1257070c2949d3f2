"""The oracle's conv + SiLU (src/deltanet.cpp:74-93) and gated RMSNorm (src/deltanet.cpp:35-45, :122)
against float64 torch autograd through a restatement of the same ops (CPU)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle


def torch_conv(x, w, state, Hk, Dk, Hv, Dv, cu=None):
    """(q, k, v, state_out) by torch ops, float64, per sequence."""
    B, T, cd = x.shape
    K = w.shape[1]
    seqs = [(b, 0, T) for b in range(B)] if cu is None else [(0, cu[n], cu[n + 1]) for n in range(len(cu) - 1)]
    outs, states = [], []
    for n, (b, t0, t1) in enumerate(seqs):
        st = state[n] if state is not None else torch.zeros(K - 1, cd, dtype=x.dtype)
        xp = torch.cat([st, x[b, t0:t1]], 0)                       # [L + K - 1, cd]
        if t1 > t0:
            u = F.conv1d(xp.t()[None], w[:, None, :], groups=cd)[0].t()  # [L, cd]
            outs.append(F.silu(u))
        states.append(xp[xp.shape[0] - (K - 1):])
    y = torch.cat(outs, 0).reshape(B, T, cd) if cu is None else torch.cat(outs, 0)[None]
    kd = Hk * Dk
    q = y[..., :kd].reshape(B, T, Hk, Dk)
    k = y[..., kd:2 * kd].reshape(B, T, Hk, Dk)
    v = y[..., 2 * kd:].reshape(B, T, Hv, Dv)
    return q, k, v, torch.stack(states)


@pytest.mark.parametrize("K", [2, 4])
@pytest.mark.parametrize("lengths", [None, [5, 0, 70, 1, 2]])
def test_conv_oracle_against_autograd(K, lengths):
    rng = np.random.default_rng(K)
    Hk, Dk, Hv, Dv = 2, 8, 3, 8
    cd = 2 * Hk * Dk + Hv * Dv
    if lengths is None:
        B, T, cu = 2, 37, None
        N = B
    else:
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        B, T, N = 1, int(cu[-1]), len(lengths)
    x = rng.standard_normal((B, T, cd))
    w = rng.standard_normal((cd, K)) * 0.5
    st = rng.standard_normal((N, K - 1, cd))
    dq, dk = rng.standard_normal((B, T, Hk, Dk)), rng.standard_normal((B, T, Hk, Dk))
    dv, dso = rng.standard_normal((B, T, Hv, Dv)), rng.standard_normal((N, K - 1, cd))
    q, k, v, so = oracle.conv_fwd(x, w, st, Hk, Dk, Hv, Dv, cu_seqlens=cu)
    xs = [torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (x, w, st)]
    tq, tk, tv, tso = torch_conv(*xs, Hk, Dk, Hv, Dv, cu=None if cu is None else list(cu))
    for a, b in ((q, tq), (k, tk), (v, tv), (so, tso)):
        assert np.allclose(a, b.detach().numpy(), rtol=1e-5, atol=1e-5)
    loss = sum((t * torch.tensor(c)).sum() for t, c in ((tq, dq), (tk, dk), (tv, dv), (tso, dso)))
    loss.backward()
    dx, dw, dsi = oracle.conv_bwd(x, w, st, dq, dk, dv, dso, Hk, Dk, Hv, Dv, cu_seqlens=cu)
    for a, t in ((dx, xs[0]), (dw, xs[1]), (dsi, xs[2])):
        assert np.allclose(a, t.grad.numpy(), rtol=1e-4, atol=1e-4)


def test_gated_norm_oracle_against_autograd():
    rng = np.random.default_rng(3)
    P, Hv, Dv, eps = 7, 3, 32, 1e-6
    y, z = rng.standard_normal((P, Hv, Dv)), rng.standard_normal((P, Hv, Dv))
    w, do = 1 + 0.1 * rng.standard_normal(Dv), rng.standard_normal((P, Hv, Dv))
    o = oracle.gated_norm_fwd(y, z, w, eps)
    ty, tz, tw = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (y, z, w))
    to = F.silu(tz) * (ty * torch.rsqrt((ty * ty).mean(-1, keepdim=True) + eps) * tw)
    assert np.allclose(o, to.detach().numpy(), rtol=1e-5, atol=1e-6)
    (to * torch.tensor(do)).sum().backward()
    dy, dz, dw = oracle.gated_norm_bwd(y, z, w, do, eps)
    for a, t in ((dy, ty), (dz, tz), (dw, tw)):
        assert np.allclose(a, t.grad.numpy(), rtol=1e-4, atol=1e-5)

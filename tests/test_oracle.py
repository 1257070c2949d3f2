"""The CPU oracle against independent restatements (CPU only).

The reference cannot run here (MLX + Metal), so the oracle's parity with it is
unpinned; these tests pin the oracle to float64 torch autograd through the
plain-ops recurrence (the reference's own gradient check, tests/test_deltanet.cpp:70-137),
to central finite differences, and to committed golden fixtures.
"""
import math
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from quotebound_b200 import synthetic
import torch_ref

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def worst(a, b):
    """The reference's gradient metric: max |a - b| over max |b| (tests/test_deltanet.cpp:126-128)."""
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def problem_ref_style(B, T, Hk, Hv, Dk, Dv, g_lo, seed):
    """Inputs as the reference's trainable_gradient draws them (tests/test_deltanet.cpp:106-113)."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)
    unit = lambda x, s: x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6) * s
    q = unit(n(B, T, Hk, Dk), 1.0 / Dk)
    k = unit(n(B, T, Hk, Dk), 1.0 / math.sqrt(Dk))
    v = n(B, T, Hv, Dv)
    g = g_lo + (1 - g_lo) * torch.rand(B, T, Hv, generator=gen, dtype=torch.float64)
    beta = torch.rand(B, T, Hv, generator=gen, dtype=torch.float64)
    s0 = n(B, Hv, Dv, Dk) * 0.1
    cy = n(B, T, Hv, Dv)
    cs = n(B, Hv, Dv, Dk)
    return [x.float().double() for x in (q, k, v, g, beta, s0, cy, cs)]


def autodiff(q, k, v, g, beta, s0, cy, cs, cu=None):
    xs = [t.clone().requires_grad_(True) for t in (q, k, v, g, beta, s0)]
    y, s = torch_ref.gated_delta_ops(*xs, cu_seqlens=cu)
    loss = (y * cy).sum() + (s * cs).sum()
    loss.backward()
    return y.detach(), s.detach(), [x.grad for x in xs]


@pytest.mark.parametrize("T,g_lo", [(37, 0.5), (80, 0.99)])
def test_forward_matches_plain_ops(T, g_lo):
    q, k, v, g, beta, s0, _, _ = problem_ref_style(2, T, 4, 8, 32, 16, g_lo, seed=T)
    y_ref, s_ref = torch_ref.gated_delta_ops(q, k, v, g, beta, s0)
    for acc64, tol in ((True, 1e-6), (False, 1e-5)):
        y, s = oracle.gated_delta_fwd(q, k, v, g, beta, s0, acc64=acc64)
        # the reference's agree() bounds: 1e-5 of the max (tests/test_deltanet.cpp:43-44)
        assert np.abs(y - y_ref.numpy()).max() <= tol * np.abs(y_ref.numpy()).max()
        assert np.abs(s - s_ref.numpy()).max() <= tol * np.abs(s_ref.numpy()).max()


def test_state_carry_split():
    """20 + rest steps against one call (tests/test_deltanet.cpp:47-52)."""
    q, k, v, g, beta, s0, _, _ = problem_ref_style(2, 75, 2, 4, 32, 32, 0.9, seed=5)
    y, s = oracle.gated_delta_fwd(q, k, v, g, beta, s0, acc64=False)
    y1, s1 = oracle.gated_delta_fwd(q[:, :20], k[:, :20], v[:, :20], g[:, :20], beta[:, :20], s0, acc64=False)
    y2, s2 = oracle.gated_delta_fwd(q[:, 20:], k[:, 20:], v[:, 20:], g[:, 20:], beta[:, 20:], s1, acc64=False)
    assert np.array_equal(np.concatenate([y1, y2], 1), y)
    assert np.array_equal(s2, s)


# The reference's eight trainable_gradient shapes (tests/test_deltanet.cpp:145-154).
TRAINABLE = [
    (1, 19, 16, 32, 128, 128, 0.5),
    (1, 64, 16, 32, 128, 128, 0.9),
    (2, 150, 16, 32, 128, 128, 0.99),
    (1, 129, 16, 32, 128, 128, 0.9),
    (1, 70, 2, 8, 32, 32, 0.9),
    (2, 33, 4, 4, 64, 64, 0.99),
    (1, 70, 2, 4, 128, 4, 0.9),
    (1, 40, 2, 4, 256, 64, 0.9),
]


@pytest.mark.parametrize("shape", TRAINABLE, ids=lambda s: "B%dT%dHk%dHv%dDk%dDv%d" % s[:6])
def test_backward_matches_autodiff(shape):
    B, T, Hk, Hv, Dk, Dv, g_lo = shape
    q, k, v, g, beta, s0, cy, cs = problem_ref_style(B, T, Hk, Hv, Dk, Dv, g_lo, seed=100 + T)
    _, _, grads = autodiff(q, k, v, g, beta, s0, cy, cs)
    got = oracle.gated_delta_bwd(q, k, v, g, beta, s0, cy, cs, acc64=False)
    for name, a, b in zip(("q", "k", "v", "g", "beta", "state"), got, grads):
        # the reference's bound for its backward: worst max-abs / max ≤ 1e-5 (tests/test_deltanet.cpp:136)
        assert worst(a, b.numpy()) <= 1e-5, name


def test_backward_finite_differences():
    """Central differences of loss = <y, cy> + <S_T, cs> on a tiny float64 case."""
    B, T, Hk, Hv, Dk, Dv = 1, 9, 1, 2, 4, 3
    q, k, v, g, beta, s0, cy, cs = problem_ref_style(B, T, Hk, Hv, Dk, Dv, 0.5, seed=1)
    grads = oracle.gated_delta_bwd(q, k, v, g, beta, s0, cy, cs, acc64=True)

    def loss(xs):
        y, s = torch_ref.gated_delta_ops(*xs)
        return float((y * cy).sum() + (s * cs).sum())

    base = [q, k, v, g, beta, s0]
    rng = np.random.default_rng(0)
    for idx in range(6):
        flat = base[idx].reshape(-1)
        for j in rng.choice(flat.numel(), size=min(5, flat.numel()), replace=False):
            h = 1e-5
            plus = [x.clone() for x in base]; minus = [x.clone() for x in base]
            plus[idx].view(-1)[j] += h; minus[idx].view(-1)[j] -= h
            fd = (loss(plus) - loss(minus)) / (2 * h)
            an = float(np.asarray(grads[idx], np.float64).reshape(-1)[j])
            assert abs(fd - an) <= 1e-5 * max(1.0, abs(fd)), (idx, j, fd, an)


def test_varlen_equals_separate_sequences():
    lengths = [5, 64, 1, 70]
    cu = synthetic.cu_from_lengths(lengths)
    Ttot = cu[-1]
    p = synthetic.make(1, Ttot, 2, 4, 32, 16, seed=3, h0_std=0.05, dhT_std=0.05, cu_seqlens=cu)
    y, hT = oracle.gated_delta_fwd(p.q, p.k, p.v, p.g, p.beta, p.h0, cu_seqlens=cu)
    dq, dk, dv, dg, db, dh0 = oracle.gated_delta_bwd(p.q, p.k, p.v, p.g, p.beta, p.h0, p.dy, p.dhT,
                                                     cu_seqlens=cu)
    for n in range(len(lengths)):
        a, e = cu[n], cu[n + 1]
        sl = lambda x: x[:, a:e]
        ys, hs = oracle.gated_delta_fwd(sl(p.q), sl(p.k), sl(p.v), sl(p.g), sl(p.beta), p.h0[n:n + 1])
        assert np.array_equal(ys, y[:, a:e]) and np.array_equal(hs[0], hT[n])
        gs = oracle.gated_delta_bwd(sl(p.q), sl(p.k), sl(p.v), sl(p.g), sl(p.beta), p.h0[n:n + 1],
                                    sl(p.dy), p.dhT[n:n + 1])
        for full, part in zip((dq, dk, dv, dg, db), gs[:5]):
            assert np.array_equal(full[:, a:e], part)
        assert np.array_equal(dh0[n], gs[5][0])


def test_varlen_against_autodiff():
    cu = [0, 7, 30, 31, 90]
    p = synthetic.make(1, cu[-1], 2, 4, 16, 8, seed=9, h0_std=0.1, dhT_std=0.1, cu_seqlens=cu)
    d = lambda t: t.double()
    _, _, grads = autodiff(d(p.q), d(p.k), d(p.v), d(p.g), d(p.beta), d(p.h0), d(p.dy), d(p.dhT), cu=cu)
    got = oracle.gated_delta_bwd(p.q, p.k, p.v, p.g, p.beta, p.h0, p.dy, p.dhT, cu_seqlens=cu)
    for a, b in zip(got, grads):
        assert worst(a, b.numpy()) <= 1e-5


def test_gate_forward_and_backward():
    gen = torch.Generator().manual_seed(4)
    M, Dk, P, Hv, Hk = 6, 16, 3, 4, 2
    q = torch.randn(P, Hk, Dk, generator=gen, dtype=torch.float64)
    k = torch.randn(P, Hk, Dk, generator=gen, dtype=torch.float64)
    a = torch.randn(P, Hv, generator=gen, dtype=torch.float64)
    b = torch.randn(P, Hv, generator=gen, dtype=torch.float64)
    A_log = torch.log(1 + 15 * torch.rand(Hv, generator=gen, dtype=torch.float64))
    dt = 0.5 * torch.randn(Hv, generator=gen, dtype=torch.float64)
    xs = [t.float().double().requires_grad_(True) for t in (q, k, a, b, A_log, dt)]
    qn, kn, g, beta = torch_ref.gate(*xs)
    got = oracle.gate_fwd(*[x.detach() for x in xs])
    for x, y in zip(got[:4], (qn, kn, g, beta)):
        assert rel(x, y.detach().numpy()) < 1e-6
    cq, ck, cg, cb = [torch.randn(t.shape, generator=gen, dtype=torch.float64) for t in (qn, kn, g, beta)]
    ((qn * cq).sum() + (kn * ck).sum() + (g * cg).sum() + (beta * cb).sum()).backward()
    dq, dk, da, db, dA, ddt = oracle.gate_bwd(*[x.detach() for x in xs], cq, ck, cg, cb)
    for x, t in zip((dq, dk, da, db, dA, ddt), xs):
        assert rel(x, t.grad.numpy()) < 1e-5


def test_golden_fixtures():
    """The oracle against the committed fixtures (made by tests/golden/make_golden.py in float64 torch)."""
    files = sorted(f for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    assert files, "no golden fixtures"
    for f in files:
        z = np.load(os.path.join(GOLDEN, f))
        cu = z["cu_seqlens"] if "cu_seqlens" in z.files else None
        y, hT = oracle.gated_delta_fwd(z["q"], z["k"], z["v"], z["g"], z["beta"], z["h0"], cu_seqlens=cu)
        assert worst(y, z["y"]) <= 1e-5, f
        assert worst(hT, z["hT"]) <= 1e-5, f
        grads = oracle.gated_delta_bwd(z["q"], z["k"], z["v"], z["g"], z["beta"], z["h0"], z["dy"], z["dhT"],
                                       cu_seqlens=cu)
        for name, x in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), grads):
            assert worst(x, z[name]) <= 1e-5, (f, name)

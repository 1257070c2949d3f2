"""The chunked (WY) backward that the kernels implement, restated in float64 numpy and checked against
the CPU oracle (the per-step recurrence of src/delta_grad.cpp:13-18) on the CPU.

This pins the algebra of both backward paths -- the CUDA-core one (gdn_cc.cu) and the tensor-core one
(gdn_chunk_*.cu) -- independently of any GPU: the chunk-start states, the dS carried backwards across
chunks, F = T^T dD, and in particular the gate gradient formed directly as a sum over the gate products
that span each step (dg_t = sum_{i >= t > j} f_ij Gamma_it Gamma_{t-1,j}), which stays accurate where g
is tiny and d log g / g would not.  Test infrastructure only: nothing here is called by the library.
"""
import numpy as np
import pytest

from oracle import oracle

C = 64


def _gammas(g):
    """Ge[i][e] = Gamma_{i, e-1} = g_e ... g_i (e - 1 < i), 1 on e - 1 == i, 0 above; column 0 = gamma_i."""
    n = len(g)
    Ge = np.zeros((n, n + 1))
    for e in range(n + 1):
        j = e - 1
        p = 1.0
        for i in range(n):
            if i > j:
                p *= g[i]
            Ge[i, e] = p if i >= j else 0.0
    return Ge


def chunked_bwd(q, k, v, g, beta, h0, dy, dhT):
    """One value head: q, k [T, Dk]; v, dy [T, Dv]; g, beta [T]; h0, dhT [Dv, Dk]."""
    T, Dk = q.shape
    Dv = v.shape[1]
    # forward: the chunk-start states
    S = h0.copy()
    starts = []
    for t in range(T):
        if t % C == 0:
            starts.append(S.copy())
        S = g[t] * S
        u = S @ k[t]
        d = beta[t] * (v[t] - u)
        S = S + np.outer(d, k[t])
    nc = len(starts)
    dq = np.zeros_like(q); dk = np.zeros_like(k); dv = np.zeros_like(v)
    dg = np.zeros_like(g); dbeta = np.zeros_like(beta)
    dS = dhT.copy()
    for c in reversed(range(nc)):
        t0, t1 = c * C, min(T, c * C + C)
        L = t1 - t0
        pad = lambda x: np.concatenate([x, np.zeros((C - L,) + x.shape[1:])]) if L < C else x
        Q, K, V, dO = pad(q[t0:t1]), pad(k[t0:t1]), pad(v[t0:t1]), pad(dy[t0:t1])
        gg = np.concatenate([g[t0:t1], np.ones(C - L)])
        be = np.concatenate([beta[t0:t1], np.zeros(C - L)])
        S0 = starts[c]
        Ge = _gammas(gg)
        Gam = Ge[:, 1:]                  # Gamma_ij (j <= i)
        gam, lam = Ge[:, 0], Ge[C - 1, 1:]
        KK, QK = K @ K.T, Q @ K.T
        Lm = np.tril(be[:, None] * Gam * KK, -1)
        Tm = np.linalg.inv(np.eye(C) + Lm)
        P = np.tril(Gam * QK)
        KS, QS = K @ S0.T, Q @ S0.T
        E = be[:, None] * (V - gam[:, None] * KS)
        D = Tm @ E
        # the reverse walk's part
        X = K @ dS.T
        dD = P.T @ dO + lam[:, None] * X
        F = Tm.T @ dD
        dv[t0:t1] = (be[:, None] * F)[:L]
        # the gradient kernels' part
        dP, FD = dO @ D.T, F @ D.T
        t2 = np.sum(F * KS, 1); t3 = np.sum(dO * QS, 1); t4 = np.sum(D * X, 1); fv = np.sum(F * V, 1)
        st5 = np.sum(S0 * dS)
        f = np.zeros((C, C + 1))
        f[:, 1:] = np.tril(dP * QK - FD * be[:, None] * KK, -1)
        f[:, 0] = t3 - be * t2
        f[C - 1, 1:] += t4
        f[C - 1, 0] += st5
        for t in range(L):
            A = np.array([f[i, 0] if t == 0 else f[i, :t + 1] @ Ge[t - 1, :t + 1] for i in range(C)])
            dg[t0 + t] = sum(Ge[i, t + 1] * A[i] for i in range(t, C))
        dbeta[t0:t1] = (fv - gam * t2 + np.sum(np.tril(-FD * Gam * KK, -1), 1))[:L]
        dPh = np.tril(Gam * dP)
        dKK = np.tril(-be[:, None] * Gam * FD, -1)
        dq[t0:t1] = (gam[:, None] * (dO @ S0) + dPh @ K)[:L]
        dk[t0:t1] = (dPh.T @ Q + lam[:, None] * (D @ dS) - (be * gam)[:, None] * (F @ S0) + (dKK + dKK.T) @ K)[:L]
        dS = gam[C - 1] * dS + (gam[:, None] * dO).T @ Q - ((be * gam)[:, None] * F).T @ K
    return dq, dk, dv, dg, dbeta, dS


@pytest.mark.parametrize("T,Dk,Dv,g_lo", [(19, 32, 32, 0.5), (64, 32, 16, 0.9), (150, 32, 32, 0.99), (129, 64, 8, 0.9),
                                          (70, 32, 4, 0.9)])
def test_chunked_backward_matches_the_per_step_oracle(T, Dk, Dv, g_lo):
    rng = np.random.default_rng(T + Dk)
    unit = lambda x, s: x / np.sqrt(np.mean(x * x, -1, keepdims=True) + 1e-6) * s
    q = unit(rng.standard_normal((T, Dk)), 1 / Dk)
    k = unit(rng.standard_normal((T, Dk)), 1 / np.sqrt(Dk))
    v = rng.standard_normal((T, Dv))
    g = rng.uniform(g_lo, 1, T)
    beta = rng.uniform(0, 1, T)
    h0 = 0.1 * rng.standard_normal((Dv, Dk))
    dy = rng.standard_normal((T, Dv))
    dhT = rng.standard_normal((Dv, Dk))
    got = chunked_bwd(q, k, v, g, beta, h0, dy, dhT)
    f = lambda x, *s: np.ascontiguousarray(x.reshape(*s), np.float32)
    want = oracle.gated_delta_bwd(f(q, 1, T, 1, Dk), f(k, 1, T, 1, Dk), f(v, 1, T, 1, Dv), f(g, 1, T, 1),
                                  f(beta, 1, T, 1), f(h0, 1, 1, Dv, Dk), f(dy, 1, T, 1, Dv), f(dhT, 1, 1, Dv, Dk),
                                  acc64=True)
    for name, a, w in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), got, want):
        w = w.reshape(a.shape)
        assert np.max(np.abs(a - w)) <= 1e-5 * np.max(np.abs(w)), name


def test_direct_gate_gradient_keeps_tiny_gates_exact():
    """Gates of 1e-30: dg formed from d log g / g loses everything; the direct form keeps full precision
    (checked against the per-step oracle in float64 accumulation)."""
    rng = np.random.default_rng(7)
    T, Dk, Dv = 96, 32, 16
    unit = lambda x, s: x / np.sqrt(np.mean(x * x, -1, keepdims=True) + 1e-6) * s
    q = unit(rng.standard_normal((T, Dk)), 1 / Dk)
    k = unit(rng.standard_normal((T, Dk)), 1 / np.sqrt(Dk))
    v = rng.standard_normal((T, Dv))
    g = rng.uniform(0.5, 1, T)
    g[[3, 40, 70]] = 1e-30
    beta = rng.uniform(0, 1, T)
    h0 = 0.1 * rng.standard_normal((Dv, Dk))
    dy = rng.standard_normal((T, Dv))
    dhT = rng.standard_normal((Dv, Dk))
    dg = chunked_bwd(q, k, v, g, beta, h0, dy, dhT)[3]
    f = lambda x, *s: np.ascontiguousarray(x.reshape(*s), np.float32)
    want = oracle.gated_delta_bwd(f(q, 1, T, 1, Dk), f(k, 1, T, 1, Dk), f(v, 1, T, 1, Dv), f(g, 1, T, 1),
                                  f(beta, 1, T, 1), f(h0, 1, 1, Dv, Dk), f(dy, 1, T, 1, Dv), f(dhT, 1, 1, Dv, Dk),
                                  acc64=True)[3].reshape(T)
    for t in (3, 40, 70):
        assert abs(dg[t] - want[t]) <= 1e-5 * abs(want[t]) + 1e-6, (t, dg[t], want[t])
    assert np.max(np.abs(dg - want)) <= 1e-5 * np.max(np.abs(want))

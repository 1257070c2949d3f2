"""CUDA path against the CPU oracle on the same seeded inputs (GPU only).

Tolerances (the build's contract): rel-L2 <= 1e-5 for float32 activations, <= 2e-3 for bf16
activations; the reference's own recurrence bounds (1e-5 of the max for float32 forward and
gradients, tests/test_deltanet.cpp:43-44,136) are checked on the float32 cases as well.  The
verify rows are checked bit for bit against one-token steps.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from quotebound_b200 import _lib, build, deltanet, exact, gate, synthetic

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROWS, CHUNKED = _lib.QB_ALGO_ROWS, _lib.QB_ALGO_CHUNKED


@pytest.fixture(scope="module", autouse=True)
def lib():
    build.ensure()
    _lib.load()


def rel(a, b):
    a = np.asarray(a.float().cpu() if torch.is_tensor(a) else a, np.float64)
    b = np.asarray(b.float().cpu() if torch.is_tensor(b) else b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def worst(a, b):
    a = np.asarray(a.float().cpu() if torch.is_tensor(a) else a, np.float64)
    b = np.asarray(b.float().cpu() if torch.is_tensor(b) else b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def oracle_all(p, cu=None):
    f = lambda t: None if t is None else t.float().cpu().numpy()
    y, hT = oracle.gated_delta_fwd(f(p.q), f(p.k), f(p.v), f(p.g), f(p.beta), f(p.h0), cu_seqlens=cu)
    grads = oracle.gated_delta_bwd(f(p.q), f(p.k), f(p.v), f(p.g), f(p.beta), f(p.h0), f(p.dy), f(p.dhT),
                                   cu_seqlens=cu)
    return y, hT, grads


def run_gpu(p, algo, cu=None):
    d = p.to("cuda")
    y, hT, saved = deltanet.gated_delta_fwd(d.q, d.k, d.v, d.g, d.beta, d.h0, cu_seqlens=cu, save=True, algo=algo)
    grads = deltanet.gated_delta_bwd(d.q, d.k, d.v, d.g, d.beta, d.h0, d.dy, d.dhT, saved=saved, cu_seqlens=cu,
                                     algo=algo)
    torch.cuda.synchronize()
    return y, hT, grads


def assert_close(p, got, want, tol, names=("dq", "dk", "dv", "dg", "dbeta", "dh0"), ref_worst=False):
    """Every output against the oracle at rel-L2 <= tol, dg directly (both backward paths form the gate
    gradient from the gate products that span each step, so gates near zero -- the bench's
    distribution reaches g ~ 1e-30 -- keep full relative precision)."""
    y, hT, grads = got
    yo, hTo, go = want
    assert rel(y, yo) <= tol, ("y", rel(y, yo))
    assert rel(hT, hTo) <= tol, ("hT", rel(hT, hTo))
    for n, a, b in zip(names, grads, go):
        if n == "dh0" and p.h0 is None and p.dhT is None:
            continue
        assert rel(a, b) <= tol, (n, rel(a, b))
        if ref_worst:
            assert worst(a, b) <= 1e-5, (n, worst(a, b))


# ---- float32: config 0 and the reference's trainable_gradient shapes on the row-parallel path ----
def test_config0_f32():
    p = synthetic.make(**synthetic.CONFIGS[0], seed=0)
    assert_close(p, run_gpu(p, ROWS), oracle_all(p), 1e-5, ref_worst=True)


TRAINABLE = [
    (1, 19, 16, 32, 128, 128, 0.5), (1, 64, 16, 32, 128, 128, 0.9), (2, 150, 16, 32, 128, 128, 0.99),
    (1, 129, 16, 32, 128, 128, 0.9), (1, 70, 2, 8, 32, 32, 0.9), (2, 33, 4, 4, 64, 64, 0.99),
    (1, 70, 2, 4, 128, 4, 0.9), (1, 40, 2, 4, 256, 64, 0.9),
]


@pytest.mark.parametrize("shape", TRAINABLE, ids=lambda s: "B%dT%dHk%dHv%dDk%dDv%d" % s[:6])
def test_trainable_shapes_f32(shape):
    B, T, Hk, Hv, Dk, Dv, g_lo = shape
    p = synthetic.make(B, T, Hk, Hv, Dk, Dv, seed=100 + T, uniform_gate=g_lo, h0_std=0.1, dhT_std=1.0)
    assert_close(p, run_gpu(p, ROWS), oracle_all(p), 1e-5, ref_worst=True)


# ---- the reference's agree() family: B=2, 16/32 heads, T in {37, 300}, g in [g_lo, 1) ----
@pytest.mark.parametrize("T,g_lo", [(37, 0.5), (300, 0.99)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_agree_forward(T, g_lo, dtype):
    p = synthetic.make(2, T, 16, 32, 128, 128, seed=T, uniform_gate=g_lo, h0_std=0.1, dtype=dtype)
    yo, so = oracle.gated_delta_fwd(p.q.float().numpy(), p.k.float().numpy(), p.v.float().numpy(), p.g.numpy(),
                                    p.beta.numpy(), p.h0.numpy())
    d = p.to("cuda")
    algos = [ROWS] if dtype == torch.float32 else [ROWS, 0]
    for algo in algos:
        y, s, _ = deltanet.gated_delta_fwd(d.q, d.k, d.v, d.g, d.beta, d.h0, algo=algo)
        tol = 1e-5 if dtype == torch.float32 else 2e-3
        assert rel(y, yo) <= tol and rel(s, so) <= tol
        if dtype == torch.float32:  # the reference's agree() bounds
            assert worst(y, yo) <= 1e-5 and worst(s, so) <= 1e-5
        # 20 + rest steps against one call (tests/test_deltanet.cpp:47-52)
        y1, s1, _ = deltanet.gated_delta_fwd(d.q[:, :20], d.k[:, :20], d.v[:, :20], d.g[:, :20], d.beta[:, :20],
                                             d.h0, algo=algo)
        y2, s2, _ = deltanet.gated_delta_fwd(d.q[:, 20:], d.k[:, 20:], d.v[:, 20:], d.g[:, 20:], d.beta[:, 20:],
                                             s1, algo=algo)
        assert rel(torch.cat([y1, y2], 1), yo) <= tol and rel(s2, so) <= tol


# ---- bf16 at the production head shape, both paths ----
@pytest.mark.parametrize("T", [64, 200, 1000])
def test_bf16_fwd_bwd(T):
    p = synthetic.make(1, T, 16, 32, 128, 128, seed=T, dtype=torch.bfloat16, h0_std=0.02, dhT_std=0.02)
    want = oracle_all(p)
    for algo in (ROWS, CHUNKED):
        assert_close(p, run_gpu(p, algo), want, 2e-3)


@pytest.mark.parametrize("B,T,Hk,Hv,g_lo", [(2, 150, 16, 32, 0.99), (1, 129, 16, 32, 0.9), (2, 64, 8, 32, 0.5),
                                            (1, 333, 4, 4, 0.9)])
def test_chunked_backward_reference_gates(B, T, Hk, Hv, g_lo):
    """The chunked backward on the reference's own gate family (g ~ U[g_lo, 1),
    tests/test_deltanet.cpp:106-113), dg compared directly."""
    p = synthetic.make(B, T, Hk, Hv, 128, 128, seed=100 + T, dtype=torch.bfloat16, uniform_gate=g_lo,
                       h0_std=0.1, dhT_std=0.1)
    assert_close(p, run_gpu(p, CHUNKED), oracle_all(p), 2e-3)


def test_varlen_matches_oracle():
    lengths = [130, 1, 64, 257, 40]
    cu = synthetic.cu_from_lengths(lengths)
    p = synthetic.make(1, cu[-1], 16, 32, 128, 128, seed=7, dtype=torch.bfloat16, h0_std=0.02, dhT_std=0.02,
                       cu_seqlens=cu)
    want = oracle_all(p, cu)
    for algo in (ROWS, CHUNKED):
        assert_close(p, run_gpu(p, algo, cu), want, 2e-3)
    pf = synthetic.make(1, cu[-1], 2, 4, 32, 32, seed=8, h0_std=0.1, dhT_std=0.1, cu_seqlens=cu)
    assert_close(pf, run_gpu(pf, ROWS, cu), oracle_all(pf, cu), 1e-5, ref_worst=True)


@pytest.mark.parametrize("lengths", [None, [130, 1, 64, 257, 40]])
def test_chunked_fp32_outputs(lengths):
    """bf16 activations with float32 y and gradients on the chunked path (the float32 output tiles and
    their stores), fixed-length and varlen with partial last chunks.  With no bf16 rounding of the
    outputs the error budget is the kernels' own: rel-L2 <= 1e-3."""
    cu = synthetic.cu_from_lengths(lengths) if lengths else None
    T = cu[-1] if cu else 200
    p = synthetic.make(1, T, 16, 32, 128, 128, seed=21, dtype=torch.bfloat16, h0_std=0.02, dhT_std=0.02,
                       cu_seqlens=cu, uniform_gate=0.9)
    d = p.to("cuda")
    y, hT, saved = deltanet.gated_delta_fwd(d.q, d.k, d.v, d.g, d.beta, d.h0, cu_seqlens=cu, save=True,
                                            out_dtype=torch.float32, algo=CHUNKED)
    grads = deltanet.gated_delta_bwd(d.q, d.k, d.v, d.g, d.beta, d.h0, d.dy, d.dhT, saved=saved, cu_seqlens=cu,
                                     algo=CHUNKED, grad_dtype=torch.float32)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and grads[0].dtype == torch.float32 and grads[2].dtype == torch.float32
    assert_close(p, (y, hT, grads), oracle_all(p.to(dtype=torch.float32), cu), 1e-3)


def test_golden_fixtures_through_the_abi():
    for f in sorted(os.listdir(GOLDEN)):
        if not f.endswith(".npz"):
            continue
        z = np.load(os.path.join(GOLDEN, f))
        t = lambda n: torch.from_numpy(z[n]).cuda()
        cu = [int(x) for x in z["cu_seqlens"]] if "cu_seqlens" in z.files else None
        y, hT, saved = deltanet.gated_delta_fwd(t("q"), t("k"), t("v"), t("g"), t("beta"), t("h0"), cu_seqlens=cu,
                                                save=True, algo=ROWS)
        assert worst(y, z["y"]) <= 1e-5 and worst(hT, z["hT"]) <= 1e-5, f
        grads = deltanet.gated_delta_bwd(t("q"), t("k"), t("v"), t("g"), t("beta"), t("h0"), t("dy"), t("dhT"),
                                         saved=saved, cu_seqlens=cu, algo=ROWS)
        for n, a in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), grads):
            assert worst(a, z[n]) <= 1e-5, (f, n)


def test_backward_without_saved_states_recomputes():
    p = synthetic.make(1, 150, 4, 8, 128, 128, seed=3, dtype=torch.bfloat16, h0_std=0.02, dhT_std=0.02)
    d = p.to("cuda")
    for algo in (ROWS, 0):
        y, hT, saved = deltanet.gated_delta_fwd(d.q, d.k, d.v, d.g, d.beta, d.h0, save=True, algo=algo)
        a = deltanet.gated_delta_bwd(d.q, d.k, d.v, d.g, d.beta, d.h0, d.dy, d.dhT, saved=saved, algo=algo)
        b = deltanet.gated_delta_bwd(d.q, d.k, d.v, d.g, d.beta, d.h0, d.dy, d.dhT, saved=None, algo=algo)
        for x, z in zip(a, b):
            assert torch.equal(x, z)


def test_deterministic_bitwise():
    """No atomics: two runs give the same bits (the reference's resume test relies on it,
    tests/test_train.cpp:435-500)."""
    p = synthetic.make(2, 300, 16, 32, 128, 128, seed=11, dtype=torch.bfloat16, h0_std=0.02, dhT_std=0.02)
    for algo in (ROWS, 0):
        a = run_gpu(p, algo)
        b = run_gpu(p, algo)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        for x, z in zip(a[2], b[2]):
            assert torch.equal(x, z)


def test_autograd_function():
    p = synthetic.make(1, 100, 2, 4, 128, 128, seed=12, dtype=torch.bfloat16, h0_std=0.02, uniform_gate=0.8)
    d = p.to("cuda")
    xs = [t.clone().requires_grad_(True) for t in (d.q, d.k, d.v, d.g, d.beta, d.h0)]
    y, s = deltanet.gated_delta(*xs, train=True)
    ((y.float() * d.dy.float()).sum()).backward()
    want = oracle_all(p.to(dtype=torch.float32))
    for x, w in zip(xs, want[2]):
        assert rel(x.grad, w) <= 2e-3


# ---- decode: one-token steps and the exact verify ----
def _decode_inputs(N, V, Hk, Hv, Dk, Dv, dtype, seed):
    p = synthetic.make(N, V, Hk, Hv, Dk, Dv, seed=seed, dtype=dtype, with_dy=False)
    gen = torch.Generator().manual_seed(seed + 1)
    state = torch.randn(N, Hv, Dv, Dk, generator=gen) * 0.05
    return p, state


@pytest.mark.parametrize("V", [1, 2, 3, 6, 9, 16])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_verify_bit_exact_against_steps(V, dtype):
    """tests/test_exact.cpp:80-123's pattern: V rows equal V decode steps, outputs and states."""
    p, state = _decode_inputs(3, V, 16, 32, 128, 128, dtype, seed=V)
    d = p.to("cuda")
    s = state.cuda()
    y, states = exact.verify(d.q, d.k, d.v, d.g, d.beta, s)
    cur = s.clone()
    for j in range(V):
        yj, cur = exact.step(d.q[:, j], d.k[:, j], d.v[:, j], d.g[:, j], d.beta[:, j], cur)
        assert torch.equal(yj, y[:, j]), j
        assert torch.equal(cur, states[:, j]), j
    # and the sequential forward over the same tokens gives the same bits
    for n in range(3):
        yf, sf, _ = deltanet.gated_delta_fwd(d.q[n:n + 1], d.k[n:n + 1], d.v[n:n + 1], d.g[n:n + 1],
                                             d.beta[n:n + 1], s[n:n + 1], algo=ROWS)
        assert torch.equal(yf[0], y[n]) and torch.equal(sf[0], states[n, -1])
    # against the oracle
    yo, so = oracle.gated_delta_fwd(p.q.float().numpy(), p.k.float().numpy(), p.v.float().numpy(), p.g.numpy(),
                                    p.beta.numpy(), state.numpy())
    assert rel(states[:, -1], so) <= 1e-5
    assert rel(y, yo) <= (1e-5 if dtype == torch.float32 else 2e-3)


def test_keep_rows():
    p, state = _decode_inputs(4, 5, 2, 4, 64, 32, torch.bfloat16, seed=3)
    d = p.to("cuda")
    _, states = exact.verify(d.q, d.k, d.v, d.g, d.beta, state.cuda())
    keep = torch.tensor([1, 5, 3, 2], dtype=torch.int32)
    out = exact.keep_rows(states, keep)
    for n in range(4):
        assert torch.equal(out[n], states[n, keep[n] - 1])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    exact.keep_rows(states, torch.tensor([0, 1, 6, 2], dtype=torch.int32), out=out, status=status)
    assert int(status.item()) == 1


# ---- the gate / beta / norm graph ----
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gate_fwd_bwd(dtype):
    gen = torch.Generator().manual_seed(5)
    P, Hk, Hv, Dk = 300, 16, 32, 128
    q = torch.randn(P, Hk, Dk, generator=gen).to(dtype)
    k = torch.randn(P, Hk, Dk, generator=gen).to(dtype)
    a = torch.randn(P, Hv, generator=gen)
    b = torch.randn(P, Hv, generator=gen)
    A_log = torch.log(1 + 15 * torch.rand(Hv, generator=gen))
    dt = 0.5 * torch.randn(Hv, generator=gen)
    dqn = torch.randn(P, Hk, Dk, generator=gen).to(dtype)
    dkn = torch.randn(P, Hk, Dk, generator=gen).to(dtype)
    dg = torch.randn(P, Hv, generator=gen)
    dbeta = torch.randn(P, Hv, generator=gen)
    f = lambda t: t.float().numpy()
    want_f = oracle.gate_fwd(f(q), f(k), f(a), f(b), f(A_log), f(dt))
    want_b = oracle.gate_bwd(f(q), f(k), f(a), f(b), f(A_log), f(dt), f(dqn), f(dkn), f(dg), f(dbeta))
    c = lambda t: t.cuda()
    got_f = gate.gate_fwd(c(q), c(k), c(a), c(b), c(A_log), c(dt), out_dtype=torch.float32)
    got_b = gate.gate_bwd(c(q), c(k), c(a), c(b), c(A_log), c(dt), c(dqn), c(dkn), c(dg), c(dbeta),
                          out_dtype=torch.float32)
    for x, w in zip(got_f, want_f[:4]):
        assert rel(x, w) <= 1e-5
    for x, w in zip(got_b, want_b):
        assert rel(x, w) <= 1e-5


# ---- the chunk-start states as a shared format (qb_gdn_ckpt_bytes, qb_gdn_bwd_from_ckpt) ----
def oracle_ckpt(p, cu=None):
    """The state at the start of every 64-step chunk, by the oracle run chunk by chunk with the state
    carried -- as the reference builds its ckpt (src/delta_grad.cpp:172-181)."""
    f = lambda t: None if t is None else t.float().cpu().numpy()
    q, k, v, g, beta = f(p.q), f(p.k), f(p.v), f(p.g), f(p.beta)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    seqs = [(b, 0, T) for b in range(B)] if cu is None else [(0, cu[n], cu[n + 1]) for n in range(len(cu) - 1)]
    out = []
    for n, (b, t0, t1) in enumerate(seqs):
        s = np.zeros((1, Hv, Dv, Dk), np.float32) if p.h0 is None else f(p.h0)[n:n + 1]
        for c0 in range(t0, t1, 64):
            out.append(s[0])
            c1 = min(t1, c0 + 64)
            sl = lambda a: np.ascontiguousarray(a[b:b + 1, c0:c1])
            _, s = oracle.gated_delta_fwd(sl(q), sl(k), sl(v), sl(g), sl(beta), s)
    return np.stack(out)


@pytest.mark.parametrize("algo,dtype,tol", [(ROWS, torch.float32, 1e-5), (CHUNKED, torch.bfloat16, 2e-3)])
@pytest.mark.parametrize("lengths", [None, [130, 1, 64, 257, 40]])
def test_backward_from_ckpt(algo, dtype, tol, lengths):
    """gated_delta_vjp given the chunk-start states alone: from the oracle's ckpt, and from the head of a
    training forward's saved buffer (the states it stores there match the oracle's)."""
    cu = synthetic.cu_from_lengths(lengths) if lengths else None
    T = cu[-1] if cu else 200
    B = 1 if cu else 2
    Hk, Hv, D = (4, 8, 64) if algo == ROWS else (4, 8, 128)
    p = synthetic.make(B, T, Hk, Hv, D, D, seed=31, dtype=dtype, h0_std=0.1, dhT_std=0.1, cu_seqlens=cu,
                       uniform_gate=0.9)
    want = oracle_all(p, cu)[2]
    ck = oracle_ckpt(p, cu)
    d = p.to("cuda")
    got = deltanet.gated_delta_bwd_from_ckpt(d.q, d.k, d.v, d.g, d.beta, d.dy, torch.from_numpy(ck).cuda(), d.dhT,
                                             cu_seqlens=cu, algo=algo, check=True)
    for n, a, b in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), got, want):
        assert rel(a, b) <= tol, (n, rel(a, b))
    _, _, saved = deltanet.gated_delta_fwd(d.q, d.k, d.v, d.g, d.beta, d.h0, save=True, cu_seqlens=cu, algo=algo)
    head = deltanet.saved_ckpt(saved, d.q, d.v, cu_seqlens=cu, algo=algo)
    assert rel(head, ck) <= (1e-6 if algo == ROWS else 1e-3)  # the tensor-core path stores them tf32-rounded
    again = deltanet.gated_delta_bwd_from_ckpt(d.q, d.k, d.v, d.g, d.beta, d.dy, head.clone(), d.dhT, cu_seqlens=cu,
                                               algo=algo)
    for n, a, b in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), again, want):
        assert rel(a, b) <= tol, (n, rel(a, b))

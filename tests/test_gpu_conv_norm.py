"""The conv + SiLU before the recurrence and the gated RMSNorm after it, on the GPU against the CPU oracle
(GPU only).  Tolerances: rel-L2 <= 1e-5 for float32, <= 2e-3 for bf16 (the oracle rounds what the
reference keeps in bf16).  The conv's verify rows are checked bit for bit against one-token steps."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle
from quotebound_b200 import build, conv, layer, norm, synthetic, _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def lib():
    build.ensure()
    _lib.load()


def rel(a, b):
    a = np.asarray(a.detach().float().cpu() if torch.is_tensor(a) else a, np.float64)
    b = np.asarray(b.detach().float().cpu() if torch.is_tensor(b) else b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _conv_inputs(B, T, Hk, Dk, Hv, Dv, K, N, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    cd = 2 * Hk * Dk + Hv * Dv
    x = torch.randn(B, T, cd, generator=gen).to(dtype)
    w = (torch.randn(cd, K, generator=gen) * 0.5).to(dtype)
    st = torch.randn(N, K - 1, cd, generator=gen).to(dtype)
    dq = torch.randn(B, T, Hk, Dk, generator=gen).to(dtype)
    dk = torch.randn(B, T, Hk, Dk, generator=gen).to(dtype)
    dv = torch.randn(B, T, Hv, Dv, generator=gen).to(dtype)
    dso = torch.randn(N, K - 1, cd, generator=gen).to(dtype)
    return x, w, st, dq, dk, dv, dso


CASES = [  # (B, T, Hk, Dk, Hv, Dv, K, lengths)
    (2, 130, 2, 32, 4, 32, 4, None),
    (1, 2048, 16, 128, 32, 128, 4, None),          # config 1's channels (conv_dim 8192)
    (1, 0, 2, 64, 2, 64, 3, [40, 0, 1, 2, 100]),   # varlen: an empty sequence, sequences shorter than K-1
    (3, 5, 1, 32, 2, 8, 2, None),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B%dT%dHk%dDk%dHv%dDv%dK%d" % c[:7] + ("var" if c[7] else ""))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_state", [True, False])
def test_conv_against_oracle(case, dtype, with_state):
    B, T, Hk, Dk, Hv, Dv, K, lengths = case
    cu = None
    if lengths:
        cu = [0]
        for L in lengths:
            cu.append(cu[-1] + L)
        T = cu[-1]
    N = B if cu is None else len(cu) - 1
    x, w, st, dq, dk, dv, dso = _conv_inputs(B, T, Hk, Dk, Hv, Dv, K, N, dtype, seed=T + K)
    st = st if with_state else None
    f = lambda t: None if t is None else t.float().numpy()
    rb = dtype == torch.bfloat16
    want = oracle.conv_fwd(f(x), f(w), f(st), Hk, Dk, Hv, Dv, round_bf16=rb, cu_seqlens=cu)
    wb = oracle.conv_bwd(f(x), f(w), f(st), f(dq), f(dk), f(dv), f(dso), Hk, Dk, Hv, Dv, round_bf16=rb, cu_seqlens=cu)
    c = lambda t: None if t is None else t.cuda()
    got = conv.conv_fwd(c(x), c(w), c(st), Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv, cu_seqlens=cu)
    gb = conv.conv_bwd(c(x), c(w), c(st), c(dq), c(dk), c(dv), c(dso), Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv, cu_seqlens=cu)
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 2e-3
    for name, a, b in zip(("q", "k", "v", "state"), got, want):
        assert rel(a, b) <= tol, (name, rel(a, b))
    for name, a, b in zip(("dx", "dw", "dstate"), gb, wb):
        if name == "dstate" and not with_state:
            # without a carried state the rows before the start are zeros; their cotangent is still reported
            pass
        assert rel(a, b) <= tol, (name, rel(a, b))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_conv_verify_bit_exact_against_steps(dtype):
    """V drafted tokens at once equal V one-token conv steps, outputs and every kept window; keep_conv_rows
    cuts back to any of them (src/deltanet.cpp:79-87, src/exact.cpp:151-159)."""
    N, V, Hk, Dk, Hv, Dv, K = 32, 8, 16, 128, 32, 128, 4
    x, w, st, *_ = _conv_inputs(N, V, Hk, Dk, Hv, Dv, K, N, dtype, seed=9)
    x, w, st = x.cuda(), w.cuda(), st.cuda()
    q, k, v, states = conv.conv_verify(x, w, st, Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv)
    cur = st.clone()
    for j in range(V):
        qj, kj, vj, cur = conv.conv_fwd(x[:, j:j + 1].contiguous(), w, cur, Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv)
        assert torch.equal(qj[:, 0], q[:, j]) and torch.equal(kj[:, 0], k[:, j]) and torch.equal(vj[:, 0], v[:, j]), j
        assert torch.equal(cur, states[:, j]), j
    # the sequence form over the same tokens gives the same bits as well
    qs, ks, vs, ss = conv.conv_fwd(x, w, st, Hk=Hk, Dk=Dk, Hv=Hv, Dv=Dv)
    assert torch.equal(qs, q) and torch.equal(ks, k) and torch.equal(vs, v) and torch.equal(ss, states[:, -1])
    keep = torch.randint(1, V + 1, (N,), generator=torch.Generator().manual_seed(3), dtype=torch.int32)
    out = conv.keep_conv_rows(states, keep)
    for n in range(N):
        assert torch.equal(out[n], states[n, int(keep[n]) - 1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("Dv", [32, 128])
def test_gated_norm_against_oracle(dtype, Dv):
    gen = torch.Generator().manual_seed(Dv)
    P, Hv, eps = 777, 8, 1e-6
    y = torch.randn(P, Hv, Dv, generator=gen).to(dtype)
    z = torch.randn(P, Hv, Dv, generator=gen).to(dtype)
    w = 1 + 0.1 * torch.randn(Dv, generator=gen)
    do = torch.randn(P, Hv, Dv, generator=gen).to(dtype)
    f = lambda t: t.float().numpy()
    rb = dtype == torch.bfloat16
    o_want = oracle.gated_norm_fwd(f(y), f(z), f(w), eps, round_bf16=rb)
    b_want = oracle.gated_norm_bwd(f(y), f(z), f(w), f(do), eps, round_bf16=rb)
    o = norm.gated_norm_fwd(y.cuda(), z.cuda(), w.cuda(), eps)
    b = norm.gated_norm_bwd(y.cuda(), z.cuda(), w.cuda(), do.cuda(), eps)
    tol = 1e-5 if dtype == torch.float32 else 2e-3
    assert rel(o, o_want) <= tol
    for name, a, c in zip(("dy", "dz", "dw"), b, b_want):
        assert rel(a, c) <= tol, (name, rel(a, c))


def test_layer_chain_conv_recurrence_norm():
    """x -> conv + SiLU -> the fused recurrence layer -> gated norm, forward and backward through the three
    autograd functions, against the oracle's chain at bf16 tolerance (rel-L2 <= 2e-3)."""
    B, T, Hk, Hv, D, K, eps = 1, 200, 2, 4, 128, 4, 1e-6
    gen = torch.Generator().manual_seed(11)
    cd = 2 * Hk * D + Hv * D
    x = (torch.randn(B, T, cd, generator=gen) * 0.5).to(torch.bfloat16)
    w = (torch.randn(cd, K, generator=gen) * 0.5).to(torch.bfloat16)
    p = synthetic.make(B, T, Hk, Hv, D, D, seed=11)
    z = torch.randn(B, T, Hv, D, generator=gen).to(torch.bfloat16)
    nw = 1 + 0.1 * torch.randn(D, generator=gen)
    do = torch.randn(B, T, Hv, D, generator=gen).to(torch.bfloat16)
    # GPU chain
    xs = [t.cuda().requires_grad_(True) for t in (x, w)]
    zz, nww = z.cuda().requires_grad_(True), nw.cuda().requires_grad_(True)
    a_, b_ = p.a.cuda().requires_grad_(True), p.b.cuda().requires_grad_(True)
    q, k, v, _ = conv.causal_conv_silu(xs[0], xs[1], None, Hk=Hk, Dk=D, Hv=Hv, Dv=D)
    y, _ = layer.gated_delta_layer(q, k, v, a_, b_, p.A_log.cuda(), p.dt_bias.cuda())
    o = norm.gated_norm(y, zz, nww, eps)
    (o.float() * do.cuda().float()).sum().backward()
    # oracle chain: the conv's bf16 outputs feed the layer oracle (the same rounding model as the layer tests)
    from test_gpu_layer import oracle_layer
    f = lambda t: t.float().numpy()
    oq, ok, ov, _ = oracle.conv_fwd(f(x), f(w), None, Hk, D, Hv, D, round_bf16=True)
    T_ = lambda a: torch.from_numpy(np.asarray(a, np.float32))
    pz = synthetic.Problem(None, None, None, None, None, None, None, None, None, p.a, p.b, p.A_log, p.dt_bias)
    yo = oracle_layer(pz, T_(oq), T_(ok), T_(ov), torch.zeros(B, T, Hv, D))[0]
    yo = T_(yo).to(torch.bfloat16).float().numpy()
    o_want = oracle.gated_norm_fwd(yo, f(z), f(nw), eps, round_bf16=True)
    assert rel(o, o_want) <= 2e-3
    dy, dz, dnw = oracle.gated_norm_bwd(yo, f(z), f(nw), f(do), eps, round_bf16=True)
    assert rel(zz.grad, dz) <= 2e-3 and rel(nww.grad, dnw) <= 2e-3
    _, _, (dq, dk, dvv, da, db, _, _, _) = oracle_layer(pz, T_(oq), T_(ok), T_(ov), T_(dy))
    dx, dwc, _ = oracle.conv_bwd(f(x), f(w), None, dq, dk, dvv, None, Hk, D, Hv, D, round_bf16=True)
    assert rel(a_.grad, da) <= 5e-3 and rel(b_.grad, db) <= 5e-3
    assert rel(xs[0].grad, dx) <= 5e-3 and rel(xs[1].grad, dwc) <= 5e-3

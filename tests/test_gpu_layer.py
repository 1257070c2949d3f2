"""The fused layer path (qb_gdn_layer_fwd / _bwd: norm + gates + recurrence) against the CPU oracle (GPU only).

The reference computes q^, k^ in bf16 (rms_norm output in the activation dtype, times a bf16 scalar,
src/deltanet.cpp:94-97), so the oracle's recurrence is fed those same bf16-rounded rows; the norm's
chain rule is the straight-through one autodiff applies to the rounding.  Tolerance rel-L2 <= 2e-3.
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle
from quotebound_b200 import _lib, build, layer, synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def lib():
    build.ensure()
    _lib.load()


def rel(a, b):
    a = np.asarray(a.float().cpu() if torch.is_tensor(a) else a, np.float64)
    b = np.asarray(b.float().cpu() if torch.is_tensor(b) else b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def raw_inputs(B, T, Hk, Hv, seed, cu=None):
    p = synthetic.make(B, T, Hk, Hv, 128, 128, seed=seed, h0_std=0.02, dhT_std=0.02, cu_seqlens=cu)
    gen = torch.Generator().manual_seed(seed + 99)
    q = (p.q * math.sqrt(128) * (0.5 + torch.rand(B, T, Hk, 1, generator=gen))).to(torch.bfloat16)
    k = (p.k * (0.5 + torch.rand(B, T, Hk, 1, generator=gen))).to(torch.bfloat16)
    return p, q, k, p.v.to(torch.bfloat16), p.dy.to(torch.bfloat16)


def model_norm(x, scale):
    """rms_norm(x) in fp32 rounded to bf16, times the bf16 scalar, rounded again (the reference's bf16 path)."""
    xf = x.float()
    r = torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)
    s = torch.tensor(scale, dtype=torch.bfloat16).float()
    return ((xf * r).to(torch.bfloat16).float() * s).to(torch.bfloat16).float()


def oracle_layer(p, q, k, v, dy, cu=None):
    f = lambda t: None if t is None else t.float().cpu().numpy()
    qn = model_norm(q, 1.0 / 128)
    kn = model_norm(k, 1.0 / math.sqrt(128))
    _, _, g, beta, _ = oracle.gate_fwd(f(q), f(k), f(p.a), f(p.b), f(p.A_log), f(p.dt_bias))
    y, hT = oracle.gated_delta_fwd(f(qn), f(kn), f(v), g, beta, f(p.h0), cu_seqlens=cu)
    dqn, dkn, dv, dg, dbeta, dh0 = oracle.gated_delta_bwd(f(qn), f(kn), f(v), g, beta, f(p.h0), f(dy), f(p.dhT),
                                                          cu_seqlens=cu)
    dq, dk, da, db, dA, ddt = oracle.gate_bwd(f(q), f(k), f(p.a), f(p.b), f(p.A_log), f(p.dt_bias), dqn, dkn, dg,
                                              dbeta)
    return y, hT, (dq, dk, dv, da, db, dA, ddt, dh0)


def run_layer(p, q, k, v, dy, cu=None):
    c = lambda t: None if t is None else t.cuda()
    y, hT, saved = layer.gated_delta_layer_fwd(c(q), c(k), c(v), c(p.a), c(p.b), c(p.A_log), c(p.dt_bias), c(p.h0),
                                               cu_seqlens=cu, save=True)
    grads = layer.gated_delta_layer_bwd(c(q), c(k), c(v), c(p.a), c(p.b), c(p.A_log), c(p.dt_bias), c(p.h0), c(dy),
                                        c(p.dhT), saved=saved, cu_seqlens=cu)
    torch.cuda.synchronize()
    return y, hT, grads


NAMES = ("dq", "dk", "dv", "da", "db", "dA_log", "ddt_bias", "dh0")


@pytest.mark.parametrize("B,T,Hk,Hv", [(1, 300, 16, 32), (2, 129, 4, 8), (1, 64, 2, 8)])
def test_layer_matches_oracle(B, T, Hk, Hv):
    p, q, k, v, dy = raw_inputs(B, T, Hk, Hv, seed=T)
    y, hT, grads = run_layer(p, q, k, v, dy)
    yo, hTo, go = oracle_layer(p, q, k, v, dy)
    assert rel(y, yo) <= 2e-3 and rel(hT, hTo) <= 2e-3, (rel(y, yo), rel(hT, hTo))
    for n, a, b in zip(NAMES, grads, go):
        assert rel(a, b) <= 2e-3, (n, rel(a, b))


def test_layer_varlen():
    cu = synthetic.cu_from_lengths([100, 1, 64, 200])
    p, q, k, v, dy = raw_inputs(1, cu[-1], 16, 32, seed=5, cu=cu)
    y, hT, grads = run_layer(p, q, k, v, dy, cu)
    yo, hTo, go = oracle_layer(p, q, k, v, dy, cu)
    assert rel(y, yo) <= 2e-3 and rel(hT, hTo) <= 2e-3
    for n, a, b in zip(NAMES, grads, go):
        assert rel(a, b) <= 2e-3, (n, rel(a, b))


def test_layer_recompute_and_determinism():
    p, q, k, v, dy = raw_inputs(1, 200, 16, 32, seed=7)
    c = lambda t: None if t is None else t.cuda()
    args = (c(q), c(k), c(v), c(p.a), c(p.b), c(p.A_log), c(p.dt_bias), c(p.h0))
    _, _, saved = layer.gated_delta_layer_fwd(*args, save=True)
    g1 = layer.gated_delta_layer_bwd(*args, c(dy), c(p.dhT), saved=saved)
    g2 = layer.gated_delta_layer_bwd(*args, c(dy), c(p.dhT), saved=None)
    g3 = layer.gated_delta_layer_bwd(*args, c(dy), c(p.dhT), saved=saved)
    for x, y_, z in zip(g1, g2, g3):
        assert torch.equal(x, y_) and torch.equal(x, z)


def test_layer_autograd():
    p, q, k, v, dy = raw_inputs(1, 100, 2, 4, seed=9)
    xs = [t.cuda().clone().requires_grad_(True) for t in (q, k, v, p.a, p.b, p.A_log, p.dt_bias, p.h0)]
    y, s = layer.gated_delta_layer(*xs)
    ((y.float() * dy.cuda().float()).sum() + (s * p.dhT.cuda()).sum()).backward()
    _, _, go = oracle_layer(p, q, k, v, dy)
    want = dict(zip(NAMES, go))
    for name, x in zip(("dq", "dk", "dv", "da", "db", "dA_log", "ddt_bias", "dh0"), xs):
        assert rel(x.grad, want[name]) <= 2e-3, name


def test_layer_argument_checks():
    """On a GPU (where the chunked path is available) the layer calls refuse null, misaligned and
    short-workspace arguments with the reason, and enqueue nothing."""
    import ctypes
    from quotebound_b200 import deltanet
    L = _lib.load()
    q = torch.zeros(1, 128, 2, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(1, 128, 4, 128, dtype=torch.bfloat16, device="cuda")
    d = deltanet.make_desc(q, v)
    err = _lib.err_buf()
    need = L.qb_gdn_workspace_bytes(ctypes.byref(d), _lib.QB_OP_LAYER_FWD, err, len(err))
    assert need > 0, err.value
    assert L.qb_gdn_layer_saved_bytes(ctypes.byref(d), err, len(err)) > 0
    fake, odd = ctypes.c_void_p(0x10000), ctypes.c_void_p(0x10002)
    assert L.qb_gdn_layer_fwd(ctypes.byref(d), *([None] * 12), need, None, err, len(err)) == -1
    assert b"non-null" in err.value
    args = [fake] * 7 + [None, fake, None, None]  # q k v a b A_log dt_bias, h0, y, hT, saved
    assert L.qb_gdn_layer_fwd(ctypes.byref(d), odd, *args[1:], fake, need, None, err, len(err)) == -1
    assert b"alignment" in err.value
    assert L.qb_gdn_layer_fwd(ctypes.byref(d), *args, fake, need - 1, None, err, len(err)) == -1
    assert b"workspace" in err.value
    need_b = L.qb_gdn_workspace_bytes(ctypes.byref(d), _lib.QB_OP_LAYER_BWD, err, len(err))
    assert need_b > 0
    assert L.qb_gdn_layer_bwd(ctypes.byref(d), *([None] * 20), need_b, None, err, len(err)) == -1
    assert b"non-null" in err.value
    torch.cuda.synchronize()

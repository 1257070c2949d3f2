"""qb_gdn_gate_bwd_noalloc (GPU only): the gate backward for callers that may not allocate device
memory -- code working inside a fixed pre-allocated pool or memory budget, plugins that are handed
only their input and output buffers, hosts that keep cudaMalloc/cudaFree (which synchronise the
device) off the hot path.  Its partial sums live in a fixed array inside the library instead of a
caller workspace.  Checked through the C ABI against qb_gdn_gate_bwd, the entry point with a
workspace, on two calls in a row with different inputs and sizes (the shared array keeps the first
call's contents, which must not leak into the second), and against the CPU oracle's gate backward
with the gate tests' tolerance.

Named to be collected last: a run that stops at the first failure has run every other test first.
"""
import ctypes

import pytest
import torch

from oracle import oracle
from quotebound_b200 import _lib, build

pytestmark = pytest.mark.gpu


def _inputs(P, Hk, Hv, Dk, seed):
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen)
    x = dict(q=r(P, Hk, Dk).to(torch.bfloat16), k=r(P, Hk, Dk).to(torch.bfloat16), a=r(P, Hv), b=r(P, Hv),
             A_log=torch.log(1 + 15 * torch.rand(Hv, generator=gen)), dt=0.5 * r(Hv),
             dqn=r(P, Hk, Dk).to(torch.bfloat16), dkn=r(P, Hk, Dk).to(torch.bfloat16), dg=r(P, Hv), dbeta=r(P, Hv))
    return {n: t.cuda().contiguous() for n, t in x.items()}


def _outputs(P, Hk, Hv, Dk):
    z = lambda *s: torch.full(s, float("nan"), device="cuda")
    return dict(dq=z(P, Hk, Dk), dk=z(P, Hk, Dk), da=z(P, Hv), db=z(P, Hv), dA=z(Hv), ddt=z(Hv))


def _ptrs(x, o):
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    return [p(x[n]) for n in ("q", "k", "a", "b", "A_log", "dt", "dqn", "dkn", "dg", "dbeta")] + \
           [p(o[n]) for n in ("dq", "dk", "da", "db", "dA", "ddt")]


def _with_workspace(L, P, Hk, Hv, Dk, x):
    o = _outputs(P, Hk, Hv, Dk)
    n = int(L.qb_gdn_gate_workspace_bytes(P, Hv))
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    err = _lib.err_buf()
    rc = L.qb_gdn_gate_bwd(P, Hk, Hv, Dk, _lib.QB_DTYPE_BF16, _lib.QB_DTYPE_F32, *_ptrs(x, o),
                           ctypes.c_void_p(ws.data_ptr()), n, None, err, len(err))
    _lib.check(rc, err)
    return o


def _no_alloc(L, P, Hk, Hv, Dk, x):
    o = _outputs(P, Hk, Hv, Dk)
    err = _lib.err_buf()
    rc = L.qb_gdn_gate_bwd_noalloc(P, Hk, Hv, Dk, _lib.QB_DTYPE_BF16, _lib.QB_DTYPE_F32, *_ptrs(x, o), None, err,
                                   len(err))
    _lib.check(rc, err)
    return o


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def test_no_alloc_matches_workspace_entry_on_two_calls():
    build.ensure()
    L = _lib.load()
    # the second call is smaller and has fewer heads, so stale partials of the first would show
    for P, Hk, Hv, Dk, seed in ((4096, 16, 32, 128, 1), (700, 4, 8, 64, 2)):
        x = _inputs(P, Hk, Hv, Dk, seed)
        want = _with_workspace(L, P, Hk, Hv, Dk, x)
        got = _no_alloc(L, P, Hk, Hv, Dk, x)
        torch.cuda.synchronize()
        for n in want:
            assert torch.isfinite(got[n]).all(), n
            # the tolerance of the gate tests (rel-L2 <= 1e-5); the same kernels run, so the bits agree too
            assert _rel(got[n], want[n]) <= 1e-5, n
            assert torch.equal(got[n], want[n]), n
        # and against the oracle (rel-L2 <= 1e-5, as the gate tests bound the entry point with a workspace)
        f = lambda t: t.float().cpu().numpy()
        ref = oracle.gate_bwd(*(f(x[n]) for n in ("q", "k", "a", "b", "A_log", "dt", "dqn", "dkn", "dg", "dbeta")))
        for n, w in zip(("dq", "dk", "da", "db", "dA", "ddt"), ref):
            assert _rel(got[n].cpu(), torch.from_numpy(w)) <= 1e-5, n


def test_no_alloc_refuses_more_heads_than_its_scratch_holds():
    build.ensure()
    L = _lib.load()
    err = _lib.err_buf()
    fake = ctypes.c_void_p(0x10000)
    rc = L.qb_gdn_gate_bwd_noalloc(100, 1, 512, 128, 1, 0, *([fake] * 16), None, err, len(err))
    assert rc == -1 and b"scratch" in err.value

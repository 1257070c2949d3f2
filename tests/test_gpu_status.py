"""The failure path on a B200, without faulting it: a bounded wait made to run out on a normal input.

The test hook qb_gdn_set_wait_limit(code, 1) makes the wait with that code give up after one poll, as a
lost arrival would.  The call must still return (no hang, no trap), report the code through
qb_gdn_status, and leave the context usable: the next call, hook off, matches a clean run bit for bit.
Also the host-side finite check of the reference's training step (src/train.cpp:266-271)."""
import math

import pytest
import torch

from quotebound_b200 import _lib, checks, layer, synthetic
from quotebound_b200._lib import QbError

pytestmark = pytest.mark.gpu


def _inputs(seed=0, T=200):
    p = synthetic.make(1, T, 2, 4, 128, 128, seed=seed, device="cuda", with_dy=True)
    gen = torch.Generator(device="cuda").manual_seed(seed + 1)
    q = (p.q * math.sqrt(128) * torch.rand(1, T, 2, 1, generator=gen, device="cuda").add_(0.5)).to(torch.bfloat16)
    k = (p.k * torch.rand(1, T, 2, 1, generator=gen, device="cuda").add_(0.5)).to(torch.bfloat16)
    return q, k, p.v.to(torch.bfloat16), p.a, p.b, p.A_log, p.dt_bias, p.dy.to(torch.bfloat16)


def _pass(x, check=False):
    q, k, v, a, b, A, dtb, dy = x
    y, hT, saved = layer.gated_delta_layer_fwd(q, k, v, a, b, A, dtb, None, save=True, check=check)
    g = layer.gated_delta_layer_bwd(q, k, v, a, b, A, dtb, None, dy, None, saved=saved, check=check)
    torch.cuda.synchronize()
    return (y, hT) + tuple(g[:7])


@pytest.mark.parametrize("code,where", [(1, "forward"), (11, "forward"), (12, "forward"), (22, "backward"),
                                        (34, "backward")])
def test_a_wait_that_runs_out_is_reported_and_the_next_call_is_clean(code, where):
    x = _inputs()
    clean = _pass(x, check=True)
    assert all(bool(torch.isfinite(t.float()).all()) for t in clean)
    hits = 0
    try:
        _lib.set_wait_limit(code, 1)
        for _ in range(3):  # one poll is almost always too few; a wait whose data had already landed passes
            with _Expect() as e:
                _pass(x, check=True)
            if e.error is not None:
                assert f"device wait {code} gave up" in str(e.error) and where in str(e.error), str(e.error)
                hits += 1
    finally:
        _lib.set_wait_limit(0, 1)
    assert hits >= 1, f"wait {code} never ran out in three calls"
    again = _pass(x, check=True)
    for a_, b_ in zip(clean, again):
        assert torch.equal(a_, b_)


class _Expect:
    """Catches a QbError from the block (None when the block raised nothing)."""

    def __enter__(self):
        self.error = None
        return self

    def __exit__(self, et, ev, tb):
        if et is not None and issubclass(et, QbError):
            self.error = ev
            return True
        return False


def test_status_is_zero_after_a_normal_call():
    q, k, v, a, b, A, dtb, dy = _inputs(seed=3)
    d = layer._desc(q, v, None, None, torch.bfloat16, 0)
    ws, n = layer._ws(d, _lib.QB_OP_LAYER_FWD, q.device)
    ws.fill_(0xFF)  # whatever the workspace held before, the call clears its status block
    import ctypes
    y = torch.empty_like(v)
    hT = torch.empty(1, 4, 128, 128, device="cuda")
    err = _lib.err_buf()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = _lib.load().qb_gdn_layer_fwd(ctypes.byref(d), P(q), P(k), P(v), P(a), P(b), P(A), P(dtb), None, P(y), P(hT),
                                      None, P(ws), n, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                      err, len(err))
    assert rc == 0, err.value
    assert _lib.status(ws, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0


def test_count_nonfinite_counts_nan_and_inf():
    for dt in (torch.float32, torch.bfloat16):
        t = torch.randn(100_003, device="cuda").to(dt)
        assert checks.nonfinite(t) == 0
        t[5] = float("nan")
        t[77_777] = float("inf")
        t[100_002] = -float("inf")
        assert checks.nonfinite(t) == 3
    assert checks.nonfinite(torch.empty(0, device="cuda")) == 0


def test_a_nan_input_is_reported_by_the_finite_check():
    """A NaN in q propagates through the recurrence (as in the reference); the opt-in check names the
    non-finite outputs instead of handing them on."""
    x = list(_inputs(seed=5))
    x[0] = x[0].clone()
    x[0][0, 17, 1, 3] = float("nan")
    with pytest.raises(QbError, match="not finite: y"):
        _pass(tuple(x), check=True)
    y = _pass(tuple(x), check=False)[0]  # unchecked, the NaN reaches the outputs from step 17 on
    assert not bool(torch.isfinite(y[0, 17:].float()).all()) and bool(torch.isfinite(y[0, :17].float()).all())

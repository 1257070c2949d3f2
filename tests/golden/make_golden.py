"""Writes the golden fixtures of tests/golden/ (run: python tests/golden/make_golden.py).

The reference's recurrence cannot run here (MLX + Metal) and stores no vectors of its
own, so these fixtures are computed by float64 torch autograd through a restatement of
the reference's plain-ops recurrence (tests/gated_delta_ref.h:100-120): an
implementation independent of both the C oracle and the CUDA kernels.  Inputs are
stored as the float32 values fed to every implementation; outputs are the float64
results rounded to float32.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, os.path.dirname(HERE))

from quotebound_b200 import synthetic  # noqa: E402
import torch_ref  # noqa: E402

CASES = {
    # B=1, T=64, Hk=2, Hv=4, Dk=Dv=32, zero initial state, seed 0
    "config0": dict(B=1, T=64, Hk=2, Hv=4, Dk=32, Dv=32, seed=0),
    # across a chunk boundary with a last chunk of one step, initial state and final-state cotangent
    "chunks_h0": dict(B=2, T=129, Hk=2, Hv=4, Dk=32, Dv=16, seed=1, h0_std=0.05, dhT_std=0.05),
    # GQA ratio 4, slow decay (g in [0.99, 1))
    "gqa4_slow": dict(B=1, T=70, Hk=1, Hv=4, Dk=64, Dv=32, seed=2, uniform_gate=0.99, h0_std=0.1),
    # varlen, with a one-step sequence
    "varlen": dict(B=1, T=0, Hk=2, Hv=4, Dk=32, Dv=32, seed=3, h0_std=0.02, dhT_std=0.02,
                   cu_seqlens=[0, 40, 41, 140, 203]),
}


def make(name, spec):
    spec = dict(spec)
    cu = spec.get("cu_seqlens")
    if cu is not None:
        spec["T"] = cu[-1]
    p = synthetic.make(**spec)
    NS = p.q.shape[0] if cu is None else len(cu) - 1
    Hv, Dv, Dk = p.v.shape[2], p.v.shape[3], p.q.shape[3]
    h0 = p.h0 if p.h0 is not None else torch.zeros(NS, Hv, Dv, Dk)
    dhT = p.dhT if p.dhT is not None else torch.zeros(NS, Hv, Dv, Dk)
    xs = [t.double().requires_grad_(True) for t in (p.q, p.k, p.v, p.g, p.beta, h0)]
    y, hT = torch_ref.gated_delta_ops(*xs, cu_seqlens=cu)
    ((y * p.dy.double()).sum() + (hT * dhT.double()).sum()).backward()
    out = dict(q=p.q, k=p.k, v=p.v, g=p.g, beta=p.beta, h0=h0, dy=p.dy, dhT=dhT, y=y.detach(),
               hT=hT.detach(), dq=xs[0].grad, dk=xs[1].grad, dv=xs[2].grad, dg=xs[3].grad, dbeta=xs[4].grad,
               dh0=xs[5].grad)
    arrays = {k: v.detach().float().numpy() for k, v in out.items()}
    if cu is not None:
        arrays["cu_seqlens"] = np.asarray(cu, np.int32)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


if __name__ == "__main__":
    for name, spec in CASES.items():
        make(name, spec)
        print("wrote", name)

"""Seeded synthetic inputs for the Gated DeltaNet path.

No public dataset is involved: every workload is random data with the shapes and
value distributions of the configurations this package is measured on.

* q, k, v ~ N(0, 1); q and k are L2-normalised per head and q is scaled by
  1/sqrt(Dk) (the model's rms_norm * 1/Dk and * 1/sqrt(Dk), src/deltanet.cpp:94-97,
  give the same vectors up to the norm's 1e-6 epsilon).
* a ~ N(0, 1), dt_bias ~ N(0, 0.5), A_log = log U(1, 16) per value head;
  g = exp(-exp(A_log) * softplus(a + dt_bias)) (src/deltanet.cpp:22-33), beta = sigmoid(b), b ~ N(0, 1).
* dO ~ N(0, 1).

The reference's own recurrence tests draw g ~ U[g_lo, 1) instead
(tests/test_deltanet.cpp:145-154); ``uniform_gate`` reproduces that family.
"""
from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass
class Problem:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    g: torch.Tensor
    beta: torch.Tensor
    h0: torch.Tensor | None
    dy: torch.Tensor | None
    dhT: torch.Tensor | None
    cu_seqlens: torch.Tensor | None = None
    # raw gate parameters (present when the gates were drawn from them)
    a: torch.Tensor | None = None
    b: torch.Tensor | None = None
    A_log: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None

    def to(self, device=None, dtype=None):
        """Move every tensor; `dtype` applies to q, k, v, dy only (g, beta, states stay float32)."""
        out = {}
        for f in dataclasses.fields(self):
            t = getattr(self, f.name)
            if t is None:
                out[f.name] = None
                continue
            if dtype is not None and f.name in ("q", "k", "v", "dy"):
                t = t.to(dtype)
            out[f.name] = t.to(device) if device is not None else t
        return Problem(**out)


def _unit(x: torch.Tensor) -> torch.Tensor:
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12)


def make(B: int, T: int, Hk: int, Hv: int, Dk: int, Dv: int, *, seed: int = 0, device="cpu",
         dtype=torch.float32, h0_std: float = 0.0, dhT_std: float = 0.0, with_dy: bool = True,
         uniform_gate: float | None = None, cu_seqlens=None) -> Problem:
    """One seeded problem.  `dtype` is the activation dtype of q, k, v, dy (g, beta, states float32)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)

    def randn(*shape, std=1.0):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std

    q = _unit(randn(B, T, Hk, Dk)) / math.sqrt(Dk)
    k = _unit(randn(B, T, Hk, Dk))
    v = randn(B, T, Hv, Dv)
    a = randn(B, T, Hv)
    b = randn(B, T, Hv)
    dt_bias = randn(Hv, std=0.5)
    A_log = torch.log(torch.rand(Hv, generator=gen, device=device) * 15.0 + 1.0)
    if uniform_gate is not None:
        g = uniform_gate + (1.0 - uniform_gate) * torch.rand(B, T, Hv, generator=gen, device=device)
    else:
        g = torch.exp(-torch.exp(A_log) * torch.nn.functional.softplus(a + dt_bias))
    beta = torch.sigmoid(b)
    NS = B if cu_seqlens is None else len(cu_seqlens) - 1
    h0 = randn(NS, Hv, Dv, Dk, std=h0_std) if h0_std > 0 else None
    dy = randn(B, T, Hv, Dv) if with_dy else None
    dhT = randn(NS, Hv, Dv, Dk, std=dhT_std) if dhT_std > 0 else None
    cu = None
    if cu_seqlens is not None:
        cu = torch.as_tensor(cu_seqlens, dtype=torch.int32, device=device)
    p = Problem(q, k, v, g, beta, h0, dy, dhT, cu, a, b, A_log, dt_bias)
    if dtype != torch.float32:
        p = p.to(dtype=dtype)
    return p


def varlen_lengths(n: int, lo: int, hi: int, seed: int = 0) -> list[int]:
    """n sequence lengths drawn uniformly from [lo, hi] (seeded)."""
    gen = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=gen)]


def cu_from_lengths(lengths) -> list[int]:
    cu = [0]
    for L in lengths:
        cu.append(cu[-1] + int(L))
    return cu


# The measured configurations (shapes only; see the module docstring for the distributions).
CONFIGS = {
    0: dict(B=1, T=64, Hk=2, Hv=4, Dk=32, Dv=32),            # CPU-runnable, float32
    1: dict(B=1, T=2048, Hk=16, Hv=32, Dk=128, Dv=128),      # Qwen3.5-4B layer, bf16 activations
    2: dict(B=8, T=4096, Hk=16, Hv=64, Dk=128, Dv=128),      # batched, sharded over GPUs
    3: dict(N=16, lo=128, hi=4096, Hk=16, Hv=32, Dk=128, Dv=128),   # varlen
    4: dict(N=32, V=8, Hk=16, Hv=32, Dk=128, Dv=128),        # speculative verify
}

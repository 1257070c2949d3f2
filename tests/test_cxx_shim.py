"""A compiled C++ host over the C ABI: tests/cxx/shim_config0.cpp includes include/qb_gdn.h, links
libqb_gdn.so and runs the gated_delta / gated_delta_vjp shim of INTEGRATION.md -- the binding a
maintainer of quotebound's C++ code would add -- on config 0 (B=1, T=64, Hk=2, Hv=4, Dk=Dv=32,
float32).  Built here with g++ (no GPU needed); run on the GPU and compared with the CPU oracle at
the float32 bound (rel-L2 <= 1e-5)."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle
from quotebound_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
SRC = os.path.join(ROOT, "tests", "cxx", "shim_config0.cpp")


def _build(out_dir):
    lib = build.ensure()
    exe = os.path.join(out_dir, "shim_config0")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Werror", "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA, "include"), SRC, "-o", exe, "-L" + os.path.dirname(lib), "-lqb_gdn",
           "-Wl,-rpath," + os.path.dirname(lib), "-L" + os.path.join(CUDA, "lib64"), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cxx_shim_compiles_and_links(tmp_path):
    exe = _build(str(tmp_path))
    assert os.path.exists(exe)



@pytest.mark.gpu
def test_cxx_shim_runs_config0_against_the_oracle(tmp_path):
    exe = _build(str(tmp_path))
    rng = np.random.default_rng(0)
    B, T, Hk, Hv, Dk, Dv = 1, 64, 2, 4, 32, 32
    from quotebound_b200 import synthetic
    p = synthetic.make(B, T, Hk, Hv, Dk, Dv, seed=0)
    f = lambda t: t.float().numpy().astype(np.float32)
    q, k, v, g, beta, dy = f(p.q), f(p.k), f(p.v), f(p.g), f(p.beta), f(p.dy)
    h0 = (0.1 * rng.standard_normal((B, Hv, Dv, Dk))).astype(np.float32)
    dhT = rng.standard_normal((B, Hv, Dv, Dk)).astype(np.float32)
    inp, outp = str(tmp_path / "in.bin"), str(tmp_path / "out.bin")
    with open(inp, "wb") as fh:
        np.array([B, T, Hk, Hv, Dk, Dv], np.int32).tofile(fh)
        for a in (q, k, v, g, beta, h0, dy, dhT):
            a.tofile(fh)
    r = subprocess.run([exe, inp, outp], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    raw = np.fromfile(outp, np.float32)
    shapes = [v.shape, h0.shape, q.shape, k.shape, v.shape, g.shape, g.shape, h0.shape]
    got, off = [], 0
    for s in shapes:
        n = int(np.prod(s))
        got.append(raw[off:off + n].reshape(s))
        off += n
    assert off == raw.size
    yo, hTo = oracle.gated_delta_fwd(q, k, v, g, beta, h0)
    go = oracle.gated_delta_bwd(q, k, v, g, beta, h0, dy, dhT)
    rel = lambda a, b: float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
    for name, a, w in zip(("y", "state", "dq", "dk", "dv", "dg", "dbeta", "dstate0"), got, (yo, hTo) + tuple(go)):
        assert rel(a, w) <= 1e-5, (name, rel(a, w))

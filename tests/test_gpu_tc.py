"""The tcgen05 building blocks the chunked kernels are made of (GPU only): one MMA tile through the
shared-memory layouts, descriptors, TMEM allocation and loads of quotebound_b200/csrc/tc_sm100.cuh,
for bf16 and tf32 operands, M in {64, 128}, every operand majorness, against float64 matmul of the
same rounded operands."""
import ctypes
import itertools
import os
import subprocess

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SO = os.path.join(HERE, "_build", "libtcprobe.so")


def build_probe():
    if not os.path.exists(SO):
        os.makedirs(os.path.dirname(SO), exist_ok=True)
        nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-shared",
                        "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "quotebound_b200", "csrc"),
                        os.path.join(HERE, "tc_probe.cu"), "-o", SO], check=True)
    L = ctypes.CDLL(SO)
    L.tc_probe_gemm.argtypes = [ctypes.c_int] * 6 + [ctypes.c_void_p] * 4 + [ctypes.c_int]
    return L


def tf32(x):
    u = x.contiguous().view(torch.int32)
    return ((u + 0x1000) & ~0x1FFF).view(torch.float32)


CASES = list(itertools.product((1, 2), (64, 128), (32, 64, 128), (64, 128), (0, 1), (0, 1)))


@pytest.fixture(scope="module")
def L():
    return build_probe()


def _tile(L, kind, M, N, K, a_mn, b_mn, lane_off=0):
    gen = torch.Generator(device="cuda").manual_seed(M * 1000 + N * 10 + K + a_mn + 2 * b_mn + kind)
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(N, K, device="cuda", generator=gen)
    D = torch.full((M, N), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.tc_probe_gemm(M, N, K, kind, a_mn, b_mn, A.data_ptr(), B.data_ptr(), D.data_ptr(), err.data_ptr(),
                         lane_off)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0, "mbarrier wait timed out"
    if kind == 1:
        Ar, Br = A.to(torch.bfloat16).double(), B.to(torch.bfloat16).double()
    else:
        Ar, Br = tf32(A).double(), tf32(B).double()
    want = Ar @ Br.T
    rel = ((D.double() - want).norm() / want.norm()).item()
    assert rel < 1e-5, rel


@pytest.mark.parametrize("kind,M,N,K,a_mn,b_mn", CASES,
                         ids=lambda v: str(v))
def test_mma_tile(L, kind, M, N, K, a_mn, b_mn):
    _tile(L, kind, M, N, K, a_mn, b_mn)


@pytest.mark.parametrize("kind,N,a_mn,b_mn", [(1, 32, 0, 1), (1, 64, 1, 1), (2, 32, 0, 1), (2, 64, 1, 0)])
def test_mma_m64_upper_half_lanes(L, kind, N, a_mn, b_mn):
    """An M = 64 accumulator addressed at lane 16: rows 16w..16w+15 land in lanes 32w+16..32w+31, so two
    M = 64 accumulators can share TMEM columns (lower and upper half of every subpartition)."""
    _tile(L, kind, 64, N, 64, a_mn, b_mn, lane_off=16)


def _expect_offsets(kind):
    """Byte offset of element (row k, column r) of a 64 x 32 fp32 box in the layout tc_sm100.cuh uses:
    kind 'k' = K-major 128-byte swizzle (16-byte chunks by row & 7), 'mn' = MN-major tf32 (32-byte
    granules by row & 3)."""
    off = {}
    for k in range(64):
        for r in range(32):
            b = r * 4
            if kind == "k":
                off[(k, r)] = k * 128 + (((b >> 4) ^ (k & 7)) << 4) + (b & 15)
            else:
                off[(k, r)] = k * 128 + (((b >> 5) ^ (k & 3)) << 5) + (b & 31)
    return off


@pytest.mark.parametrize("swizzle,kind", [(3, "k"), (4, "mn")])
@pytest.mark.parametrize("col0", [0, 32])
def test_tma_box_layout(swizzle, kind, col0):
    L = build_probe()
    L.tc_probe_tma.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, ctypes.c_void_p]
    rows = 256
    src = torch.arange(rows * 64, dtype=torch.float32, device="cuda").reshape(rows, 64)
    out = torch.full((2048,), -1.0, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.tc_probe_tma(src.data_ptr(), rows, 64, col0, swizzle, out.data_ptr(), err.data_ptr()) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.cpu()
    for (k, r), o in _expect_offsets(kind).items():
        assert got[o // 4].item() == src[64 + k, col0 + r].item(), (k, r)

"""The C ABI without a GPU: the library loads, exports every symbol the header declares, and
rejects bad shapes, dtypes, offsets and pointers on the host before launching anything."""
import ctypes
import os
import re

import pytest
import torch

from quotebound_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def L():
    build.ensure()
    return _lib.load()


def declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"\b(qb_gdn_\w+)\s*\(", text))
    return names


def test_exports_every_declared_symbol(L):
    names = declared_symbols()
    assert names, "no declarations found"
    for n in names:
        assert hasattr(L, n), n
    assert names == set(_lib.SYMBOLS)


def test_no_torch_in_the_library():
    """The shared library is plain C ABI: it links no torch or python library."""
    import subprocess
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    names = [line.split()[0] for line in out.splitlines() if line.strip()]
    assert not any("torch" in n or "python" in n or "c10" in n for n in names), names


def test_version(L):
    assert "sm_100a" in _lib.version()


def desc(**kw):
    d = _lib.Desc()
    d.B, d.T, d.Hk, d.Hv, d.Dk, d.Dv = 1, 128, 2, 4, 128, 128
    d.in_dtype = d.out_dtype = _lib.QB_DTYPE_BF16
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def ws_or_err(L, d, op=_lib.QB_OP_BWD):
    err = _lib.err_buf()
    n = L.qb_gdn_workspace_bytes(ctypes.byref(d), op, err, len(err))
    return n, err.value.decode()


@pytest.mark.parametrize("bad,msg", [
    (dict(Dk=48), "Dk in"),
    (dict(Hk=3), "multiple of key heads"),
    (dict(in_dtype=7), "dtypes"),
    (dict(B=0), "bad shape"),
    (dict(algo=9), "unknown algo"),
])
def test_shape_errors(L, bad, msg):
    n, e = ws_or_err(L, desc(**bad))
    assert n == -1 and msg in e


def test_chunked_needs_its_shape(L):
    n, e = ws_or_err(L, desc(Dk=64, Dv=64, algo=_lib.QB_ALGO_CHUNKED))
    assert n == -1 and "chunked path" in e


def _cu(host):
    h = torch.tensor(host, dtype=torch.int32)
    return h


@pytest.mark.parametrize("cu,msg", [
    ([1, 64, 128], "cu_seqlens[0] must be 0"),
    ([0, 70, 64, 128], "non-decreasing"),
    ([0, 64, 100], "must equal T"),
])
def test_cu_seqlens_errors(L, cu, msg):
    h = _cu(cu)
    d = desc(n_seqs=len(cu) - 1, cu_seqlens=h.data_ptr(), cu_seqlens_host=h.data_ptr())
    n, e = ws_or_err(L, d)
    assert n == -1 and msg in e


def test_varlen_needs_batch_one(L):
    h = _cu([0, 128])
    n, e = ws_or_err(L, desc(B=2, n_seqs=1, cu_seqlens=h.data_ptr(), cu_seqlens_host=h.data_ptr()))
    assert n == -1 and "B == 1" in e


def test_null_and_misaligned_pointers(L):
    d = desc()
    err = _lib.err_buf()
    rc = L.qb_gdn_fwd(ctypes.byref(d), None, None, None, None, None, None, None, None, None, None, 0, None, err,
                      len(err))
    assert rc == -1 and b"non-null" in err.value
    fake = ctypes.c_void_p(0x1000)
    odd = ctypes.c_void_p(0x1002)
    rc = L.qb_gdn_fwd(ctypes.byref(d), odd, fake, fake, fake, fake, None, fake, None, None, None, 0, None, err,
                      len(err))
    assert rc == -1 and b"alignment" in err.value



def test_gated_norm_refuses_misaligned_rows(L):
    """Each lane of the gated norm moves its Dv / 32 elements of a row as one vector, so the rows' base
    pointers must be aligned to min(16, Dv / 32 x element size) bytes; a misaligned one is refused on the
    host, before anything is launched."""
    err = _lib.err_buf()
    fake, odd = 0x1000, 0x1008  # 0x1008: 8-byte aligned, not 16 (Dv = 128 in float32 needs 16)
    rc = L.qb_gdn_gated_norm_fwd(4, 2, 128, 1e-6, _lib.QB_DTYPE_F32, odd, fake, fake, fake, None, err, len(err))
    assert rc == -1 and b"alignment" in err.value
    rc = L.qb_gdn_gated_norm_bwd(4, 2, 128, 1e-6, _lib.QB_DTYPE_BF16, fake, fake, fake, fake, fake, 0x1004, None,
                                 None, 0, None, err, len(err))
    assert rc == -1 and b"alignment" in err.value  # bf16 at Dv = 128: 8 bytes


def test_workspace_too_small_is_refused(L):
    d = desc()
    need, _ = ws_or_err(L, d, _lib.QB_OP_BWD)
    assert need > 0
    fake = ctypes.c_void_p(0x10000)
    err = _lib.err_buf()
    rc = L.qb_gdn_bwd(ctypes.byref(d), fake, fake, fake, fake, fake, None, fake, None, None, fake, fake, fake, fake,
                      fake, None, fake, need - 1, None, err, len(err))
    assert rc == -1 and b"workspace" in err.value


def test_error_text_is_cut_to_errlen(L):
    d = desc(Dk=48)
    err = ctypes.create_string_buffer(16)
    assert L.qb_gdn_workspace_bytes(ctypes.byref(d), 0, err, 16) == -1
    assert len(err.value) == 15


def test_step_verify_gate_validation(L):
    err = _lib.err_buf()
    assert L.qb_gdn_step(1, 3, 4, 128, 128, 1, 1, *([None] * 8), None, err, len(err)) == -1
    assert b"multiple of key heads" in err.value
    assert L.qb_gdn_verify(1, 0, 2, 4, 128, 128, 1, 1, *([None] * 8), None, err, len(err)) == -1
    assert L.qb_gdn_gate_fwd(10, 2, 4, 100, 1, 1, *([None] * 10), None, err, len(err)) == -1
    assert L.qb_gdn_keep_rows(1, 2, 4, 128, 128, None, None, None, None, None, err, len(err)) == -1


@pytest.mark.parametrize("bad", [dict(Dk=64, Dv=64), dict(in_dtype=_lib.QB_DTYPE_F32), dict(algo=_lib.QB_ALGO_ROWS)])
def test_layer_path_refuses_what_the_chunked_kernels_cannot_take(L, bad):
    """The fused norm/gate path runs on the chunked kernels only: other shapes, float32 activations or
    the row-parallel algo are refused (workspace, saved-buffer and both calls alike), before any launch."""
    d = desc(**bad)
    err = _lib.err_buf()
    for op in (_lib.QB_OP_LAYER_FWD, _lib.QB_OP_LAYER_BWD):
        assert L.qb_gdn_workspace_bytes(ctypes.byref(d), op, err, len(err)) == -1
        assert b"fused norm/gate path" in err.value
    assert L.qb_gdn_layer_saved_bytes(ctypes.byref(d), err, len(err)) == -1
    fake = ctypes.c_void_p(0x10000)
    assert L.qb_gdn_layer_fwd(ctypes.byref(d), *([fake] * 12), 1 << 30, None, err, len(err)) == -1
    assert L.qb_gdn_layer_bwd(ctypes.byref(d), *([fake] * 20), 1 << 30, None, err, len(err)) == -1
    assert b"fused norm/gate path" in err.value


def test_unknown_op_is_refused(L):
    n, e = ws_or_err(L, desc(), 9)
    assert n == -1 and "unknown op" in e


def test_status_and_checks_reject_bad_arguments(L):
    """qb_gdn_status, qb_gdn_set_wait_limit and qb_gdn_count_nonfinite validate on the host."""
    err = _lib.err_buf()
    code = ctypes.c_int32(7)
    assert L.qb_gdn_status(None, ctypes.byref(code), None, err, len(err)) == -1
    assert b"non-null" in err.value and code.value == 7
    assert L.qb_gdn_status(ctypes.c_void_p(4096 + 16), ctypes.byref(code), None, err, len(err)) == -1
    assert b"alignment" in err.value
    assert L.qb_gdn_set_wait_limit(-1, 1, err, len(err)) == -1
    assert L.qb_gdn_set_wait_limit(1, 0, err, len(err)) == -1
    assert L.qb_gdn_count_nonfinite(None, 10, _lib.QB_DTYPE_F32, None, None, err, len(err)) == -1
    assert L.qb_gdn_count_nonfinite(None, -1, _lib.QB_DTYPE_F32, None, None, err, len(err)) == -1
    assert L.qb_gdn_count_nonfinite(None, 1, 9, None, None, err, len(err)) == -1


@pytest.mark.parametrize("op", [_lib.QB_OP_FWD, _lib.QB_OP_BWD, _lib.QB_OP_LAYER_FWD, _lib.QB_OP_LAYER_BWD])
@pytest.mark.parametrize("dk,dt", [(128, _lib.QB_DTYPE_BF16), (32, _lib.QB_DTYPE_F32)])
def test_every_workspace_holds_the_status_block(L, op, dk, dt):
    """Every recurrence call's workspace opens with the 256-byte status block, even when the kernels
    need no scratch (the row-parallel forward)."""
    d = desc(Dk=dk, Dv=dk, in_dtype=dt, out_dtype=dt)
    err = _lib.err_buf()
    n = L.qb_gdn_workspace_bytes(ctypes.byref(d), op, err, len(err))
    if op in (_lib.QB_OP_LAYER_FWD, _lib.QB_OP_LAYER_BWD):
        # the fused layer path needs the tensor-core shape and, for its tensor maps, a CUDA driver
        assert n == -1 if dk != 128 else (n == -1 and b"chunked" in err.value) or n >= 256
    else:
        assert n >= 256, err.value

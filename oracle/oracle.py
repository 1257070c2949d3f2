"""ctypes binding of the CPU oracle (oracle/gdn_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference leg as the checker; the product path in
quotebound_b200/ never imports it.

Parity status: unpinned against the reference's bits (the reference's forward is
MLX's closed op ``mx::fast::gated_delta_update`` and its backward a Metal kernel,
src/delta_grad.cpp:23-145; neither runs on Linux and no golden vectors for the
recurrence exist).  The oracle restates tests/gated_delta_ref.h:100-120 (forward)
and src/delta_grad.cpp:13-18,97-141 (backward), and is cross-checked against
float64 torch autograd and finite differences in tests/test_oracle.py.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libgdn_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-C", _HERE, "-B" if force else "all"], check=True,
                       stdout=subprocess.DEVNULL)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        i, p, ip = ctypes.c_int, _f32p, _i32p
        L.gdn_oracle_fwd.argtypes = [i, i, i, i, i, i, ip, i, p, p, p, p, p, p, p, p, i, i]
        L.gdn_oracle_bwd.argtypes = [i, i, i, i, i, i, ip, i, p, p, p, p, p, p, p, p,
                                     p, p, p, p, p, p, i, i]
        i64 = ctypes.c_int64
        L.gdn_oracle_gate_fwd.argtypes = [i64, i, i64, i, p, p, p, p, p, p, p, p, p, p, p]
        L.gdn_oracle_gate_bwd.argtypes = [i64, i, i64, i, p, p, p, p, p, p, p, p, p, p,
                                          p, p, p, p, p, p]
        L.gdn_oracle_conv_fwd.argtypes = [i, i, ip, i, i, i, i, i, p, p, p, p, p, p, p]
        L.gdn_oracle_conv_bwd.argtypes = [i, i, ip, i, i, i, i, i, p, p, p, p, p, p, p, p, p, p]
        f = ctypes.c_float
        L.gdn_oracle_gated_norm_fwd.argtypes = [i64, i, f, i, p, p, p, p]
        L.gdn_oracle_gated_norm_bwd.argtypes = [i64, i, f, i, p, p, p, p, p, p, p]
        L.gdn_oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _f(x):
    if x is None:
        return None, None
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return a, a.ctypes.data_as(_f32p)


def _cu(cu):
    if cu is None:
        return None, None, 0
    a = np.ascontiguousarray(np.asarray(cu, dtype=np.int32))
    return a, a.ctypes.data_as(_i32p), len(a) - 1


def max_threads() -> int:
    return lib().gdn_oracle_max_threads()


def gated_delta_fwd(q, k, v, g, beta, h0=None, cu_seqlens=None, acc64=True, threads=0):
    """y [B,T,Hv,Dv] float32 and the final state(s) [N,Hv,Dv,Dk] of the recurrence."""
    q, qp = _f(q); k, kp = _f(k); v, vp = _f(v); g, gp = _f(g); beta, bp = _f(beta)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    cua, cup, N = _cu(cu_seqlens)
    NS = N if cua is not None else B
    h0a, h0p = _f(h0)
    y = np.zeros((B, T, Hv, Dv), np.float32)
    hT = np.zeros((NS, Hv, Dv, Dk), np.float32)
    rc = lib().gdn_oracle_fwd(B, T, Hk, Hv, Dk, Dv, cup, N, qp, kp, vp, gp, bp, h0p,
                              y.ctypes.data_as(_f32p), hT.ctypes.data_as(_f32p), int(acc64), threads)
    if rc:
        raise ValueError(f"oracle fwd failed ({rc})")
    return y, hT


def gated_delta_bwd(q, k, v, g, beta, h0, dy, dhT=None, cu_seqlens=None, acc64=True, threads=0):
    """Cotangents (dq, dk, dv, dg, dbeta, dh0) given dy and the final-state cotangent dhT."""
    q, qp = _f(q); k, kp = _f(k); v, vp = _f(v); g, gp = _f(g); beta, bp = _f(beta)
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    cua, cup, N = _cu(cu_seqlens)
    NS = N if cua is not None else B
    h0a, h0p = _f(h0)
    dya, dyp = _f(dy)
    dhTa, dhTp = _f(dhT)
    dq = np.zeros_like(q); dk = np.zeros_like(k); dv = np.zeros_like(v)
    dg = np.zeros_like(g); dbeta = np.zeros_like(beta)
    dh0 = np.zeros((NS, Hv, Dv, Dk), np.float32)
    P = lambda a: a.ctypes.data_as(_f32p)
    rc = lib().gdn_oracle_bwd(B, T, Hk, Hv, Dk, Dv, cup, N, qp, kp, vp, gp, bp, h0p, dyp, dhTp,
                              P(dq), P(dk), P(dv), P(dg), P(dbeta), P(dh0), int(acc64), threads)
    if rc:
        raise ValueError(f"oracle bwd failed ({rc})")
    return dq, dk, dv, dg, dbeta, dh0


def gate_fwd(q, k, a, b, A_log, dt_bias):
    """(qn, kn, g, beta, log g): the q/k norm and the gates of src/deltanet.cpp:94-100, :22-33."""
    q, qp = _f(q); k, kp = _f(k); a, ap = _f(a); b, bp = _f(b)
    A_log, Ap = _f(A_log); dt_bias, dp = _f(dt_bias)
    Dk = q.shape[-1]; Hv = a.shape[-1]
    M = q.size // Dk; Pn = a.size // Hv
    qn = np.zeros_like(q); kn = np.zeros_like(k); g = np.zeros_like(a); beta = np.zeros_like(a)
    lg = np.zeros_like(a)
    P = lambda x: x.ctypes.data_as(_f32p)
    lib().gdn_oracle_gate_fwd(M, Dk, Pn, Hv, qp, kp, ap, bp, Ap, dp, P(qn), P(kn), P(g), P(beta), P(lg))
    return qn, kn, g, beta, lg


def gate_bwd(q, k, a, b, A_log, dt_bias, dqn, dkn, dg, dbeta):
    """(dq, dk, da, db, dA_log, ddt_bias) through the norm and the gates."""
    q, qp = _f(q); k, kp = _f(k); a, ap = _f(a); b, bp = _f(b)
    A_log, Ap = _f(A_log); dt_bias, dp = _f(dt_bias)
    dqn, dqp = _f(dqn); dkn, dkp = _f(dkn); dg, dgp = _f(dg); dbeta, dbp = _f(dbeta)
    Dk = q.shape[-1]; Hv = a.shape[-1]
    M = q.size // Dk; Pn = a.size // Hv
    dq = np.zeros_like(q); dk = np.zeros_like(k); da = np.zeros_like(a); db = np.zeros_like(a)
    dA = np.zeros(Hv, np.float32); ddt = np.zeros(Hv, np.float32)
    P = lambda x: x.ctypes.data_as(_f32p)
    lib().gdn_oracle_gate_bwd(M, Dk, Pn, Hv, qp, kp, ap, bp, Ap, dp, dqp, dkp, dgp, dbp,
                              P(dq), P(dk), P(da), P(db), P(dA), P(ddt))
    return dq, dk, da, db, dA, ddt


def _cu_conv(cu_seqlens):
    if cu_seqlens is None:
        return None, None
    c = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int32))
    return c, c.ctypes.data_as(_i32p)


def conv_fwd(x, w, state_in, Hk, Dk, Hv, Dv, round_bf16=False, cu_seqlens=None):
    """The causal depthwise conv1d + SiLU split into (q, k, v, state_out) (src/deltanet.cpp:74-93).
    x [B, T, conv_dim]; w [conv_dim, K]; state_in [N, K - 1, conv_dim] or None."""
    x, xp = _f(x); w, wp = _f(w); state_in, sp = _f(state_in)
    B, T, cd = x.shape
    K = w.shape[1]
    cu, cup = _cu_conv(cu_seqlens)
    N = B if cu is None else len(cu) - 1
    kd, vd = Hk * Dk, Hv * Dv
    q = np.zeros((B, T, Hk, Dk), np.float32); k = np.zeros_like(q); v = np.zeros((B, T, Hv, Dv), np.float32)
    so = np.zeros((N, K - 1, cd), np.float32)
    P = lambda a: a.ctypes.data_as(_f32p)
    lib().gdn_oracle_conv_fwd(B, T, cup, N, kd, vd, K, int(round_bf16), xp, wp, sp, P(q), P(k), P(v), P(so))
    return q, k, v, so


def conv_bwd(x, w, state_in, dq, dk, dv, dstate_out, Hk, Dk, Hv, Dv, round_bf16=False, cu_seqlens=None):
    """(dx, dw, dstate_in) of conv_fwd given the cotangents of q, k, v and of the new state."""
    x, xp = _f(x); w, wp = _f(w); state_in, sp = _f(state_in)
    dq, dqp = _f(dq); dk, dkp = _f(dk); dv, dvp = _f(dv); dstate_out, dsp = _f(dstate_out)
    B, T, cd = x.shape
    K = w.shape[1]
    cu, cup = _cu_conv(cu_seqlens)
    N = B if cu is None else len(cu) - 1
    dx = np.zeros_like(x); dw = np.zeros_like(w); dsi = np.zeros((N, K - 1, cd), np.float32)
    P = lambda a: a.ctypes.data_as(_f32p)
    lib().gdn_oracle_conv_bwd(B, T, cup, N, Hk * Dk, Hv * Dv, K, int(round_bf16), xp, wp, sp, dqp, dkp, dvp, dsp,
                              P(dx), P(dw), P(dsi))
    return dx, dw, dsi


def gated_norm_fwd(y, z, w, eps, round_bf16=False):
    """o = silu(z) rms_norm(y, w, eps) per row of Dv (src/deltanet.cpp:35-45, :122)."""
    y, yp = _f(y); z, zp = _f(z); w, wp = _f(w)
    Dv = y.shape[-1]
    o = np.zeros_like(y)
    lib().gdn_oracle_gated_norm_fwd(y.size // Dv, Dv, float(eps), int(round_bf16), yp, zp, wp, o.ctypes.data_as(_f32p))
    return o


def gated_norm_bwd(y, z, w, dout, eps, round_bf16=False):
    """(dy, dz, dw) of gated_norm_fwd."""
    y, yp = _f(y); z, zp = _f(z); w, wp = _f(w); dout, dp = _f(dout)
    Dv = y.shape[-1]
    dy = np.zeros_like(y); dz = np.zeros_like(y); dw = np.zeros_like(w)
    P = lambda a: a.ctypes.data_as(_f32p)
    lib().gdn_oracle_gated_norm_bwd(y.size // Dv, Dv, float(eps), int(round_bf16), yp, zp, wp, dp, P(dy), P(dz), P(dw))
    return dy, dz, dw

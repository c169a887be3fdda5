"""ORACLE — test infrastructure only.

ctypes wrapper over ``oracle/lib/libkattn_oracle.so``, the plain-C restatement
of kerr-engine's CPU causal self-attention (forward: src/pipeline.rs:305-347;
backward: src/backend.rs:344-373 -> src/backward.rs:464-514).  Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm may use
it, and only as the checker or the timed CPU reference.  PARITY UNPINNED: the
reference ships no golden vectors for attention; see kattn_oracle.h.

Arrays are numpy float32.  A batch is q, k, v of shape [B, T, ld] (row stride
ld >= C, head h in columns h*hd..(h+1)*hd), exactly the reference's per-sequence
``[T][n_embd]`` rows stacked over the batch.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "lib", "libkattn_oracle.so")
_lib = None

_f = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.kattn_oracle_forward_batch.argtypes = [
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            _f, _f, _f, ctypes.c_long, _f, ctypes.c_long, _f, _f, ctypes.c_int]
        L.kattn_oracle_forward_batch.restype = None
        L.kattn_oracle_backward_batch.argtypes = [
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            _f, ctypes.c_long, _f, _f, _f, ctypes.c_long, _f,
            _f, _f, _f, ctypes.c_long, ctypes.c_int]
        L.kattn_oracle_backward_batch.restype = None
        L.kattn_oracle_default_threads.argtypes = [ctypes.c_int]
        L.kattn_oracle_default_threads.restype = ctypes.c_int
        L.kproj_oracle_forward.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f, _f,
                                           _f, ctypes.c_long, ctypes.c_int]
        L.kproj_oracle_forward.restype = None
        L.kproj_oracle_backward_dx.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f,
                                               _f, ctypes.c_long, ctypes.c_int]
        L.kproj_oracle_backward_dx.restype = None
        L.kproj_oracle_backward_dw.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f,
                                               ctypes.c_long, _f, _f, ctypes.c_int]
        L.kproj_oracle_backward_dw.restype = None
        L.kln_oracle_forward.argtypes = [ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f, _f, _f, ctypes.c_long]
        L.kln_oracle_forward.restype = None
        L.kln_oracle_backward.argtypes = [ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f, ctypes.c_long, _f, _f,
                                          ctypes.c_long, _f, _f, ctypes.c_int]
        L.kln_oracle_backward.restype = None
        L.kode_oracle_forward.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f, _f,
                                          ctypes.c_float, ctypes.c_float, _f, ctypes.c_long, ctypes.c_int]
        L.kode_oracle_forward.restype = None
        L.kode_oracle_backward.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _f, ctypes.c_long, _f,
                                           ctypes.c_long, _f, _f, ctypes.c_float, ctypes.c_float, _f, ctypes.c_long,
                                           _f, _f, _f, ctypes.c_int]
        L.kode_oracle_backward.restype = None
        _lib = L
    return _lib


def _ptr(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f)


def _view(a, C):
    """Return (base array, row stride) for a [B, T, >=C] float32 view whose rows
    may be a column slice of a wider contiguous buffer."""
    assert a.dtype == np.float32 and a.ndim == 3 and a.strides[2] == 4
    ld = a.strides[1] // 4
    assert a.strides[0] == a.shape[1] * a.strides[1]
    return a, ld


def _addr(a):
    return ctypes.cast(ctypes.c_void_p(a.__array_interface__["data"][0]), _f)


def default_threads(B: int) -> int:
    return lib().kattn_oracle_default_threads(B)


def forward(q, k, v, n_head: int, want_att: bool = True, threads: int = 0):
    """Reference forward.  q, k, v: [B, T, C] float32 (may be strided column
    slices of one [B, T, 3C] qkv buffer, as the reference splits it).
    Returns (out [B,T,C], att [B,H,T,T] or None, lse [B,H,T])."""
    B, T, C = q.shape
    _, ld = _view(q, C)
    assert k.strides == q.strides and v.strides == q.strides
    out = np.empty((B, T, C), np.float32)
    att = np.empty((B, n_head, T, T), np.float32) if want_att else None
    lse = np.empty((B, n_head, T), np.float32)
    lib().kattn_oracle_forward_batch(B, T, C, n_head, _addr(q), _addr(k), _addr(v), ld,
                                     _ptr(out), C, _ptr(att), _ptr(lse), threads)
    return out, att, lse


def backward(d_out, q, k, v, att, n_head: int, threads: int = 0):
    """Reference backward from the cached post-softmax weights.
    d_out: [B,T,C] contiguous; q,k,v as in forward(); att: [B,H,T,T].
    Returns (dq, dk, dv), each [B,T,C]."""
    B, T, C = q.shape
    _, ld = _view(q, C)
    d_out = np.ascontiguousarray(d_out, np.float32)
    att = np.ascontiguousarray(att, np.float32)
    dq = np.empty((B, T, C), np.float32)
    dk = np.empty((B, T, C), np.float32)
    dv = np.empty((B, T, C), np.float32)
    lib().kattn_oracle_backward_batch(B, T, C, n_head, _ptr(d_out), C, _addr(q), _addr(k), _addr(v),
                                      ld, _ptr(att), _ptr(dq), _ptr(dk), _ptr(dv), C, threads)
    return dq, dk, dv


# ---------------------------------------------------------------- linear layers
# The attention projections (c_attn, c_proj): src/backend.rs:240-247, :508-520
# (forward), src/backward.rs:48-60 (dx), src/backend.rs:320-342 (dw, db).
# x / dy are [M, in] / [M, out] float32 rows (positions); w is [out, in].

def linear_forward(x, w, b=None, threads=0):
    """y[m, n] = b[n] + sum_k w[n, k] x[m, k]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    M, K = x.shape
    N = w.shape[0]
    assert w.shape == (N, K)
    y = np.empty((M, N), np.float32)
    bb = None if b is None else np.ascontiguousarray(b, np.float32)
    lib().kproj_oracle_forward(M, N, K, _ptr(x), K, _ptr(w), _ptr(bb), _ptr(y), N, threads)
    return y


def linear_backward_dx(dy, w, threads=0):
    """dx[m, k] = sum_n dy[m, n] w[n, k]."""
    dy = np.ascontiguousarray(dy, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    M, N = dy.shape
    K = w.shape[1]
    dx = np.empty((M, K), np.float32)
    lib().kproj_oracle_backward_dx(M, N, K, _ptr(dy), N, _ptr(w), _ptr(dx), K, threads)
    return dx


def linear_backward_dw(dy, x, threads=0):
    """(dw, db): dw[n, k] = sum_m dy[m, n] x[m, k], db[n] = sum_m dy[m, n]."""
    dy = np.ascontiguousarray(dy, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    M, N = dy.shape
    K = x.shape[1]
    dw = np.zeros((N, K), np.float32)
    db = np.zeros(N, np.float32)
    lib().kproj_oracle_backward_dw(M, N, K, _ptr(dy), N, _ptr(x), K, _ptr(dw), _ptr(db), threads)
    return dw, db


def layernorm_forward(x, w, b):
    """LayerNorm of each row of x [M, N] (src/backend.rs:258-267)."""
    x = np.ascontiguousarray(x, np.float32)
    M, N = x.shape
    y = np.empty((M, N), np.float32)
    lib().kln_oracle_forward(M, N, _ptr(x), N, _ptr(np.ascontiguousarray(w, np.float32)),
                             _ptr(np.ascontiguousarray(b, np.float32)), _ptr(y), N)
    return y


def layernorm_backward(dy, x, w, dw=None, db=None):
    """(dx, dw, db) of LayerNorm (src/backward.rs:93-128, src/backend.rs:195-206);
    dw / db given: the column sums are added to copies of them."""
    dy = np.ascontiguousarray(dy, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    M, N = x.shape
    dx = np.empty((M, N), np.float32)
    acc = dw is not None
    dw_o = np.array(dw, np.float32) if acc else np.empty(N, np.float32)
    db_o = np.array(db, np.float32) if db is not None else np.empty(N, np.float32)
    lib().kln_oracle_backward(M, N, _ptr(dy), N, _ptr(x), N, _ptr(np.ascontiguousarray(w, np.float32)), _ptr(dx), N,
                              _ptr(dw_o), _ptr(db_o), int(acc))
    return dx, dw_o, db_o



def kerr_ode_forward(x, gamma_raw, omega, alpha, beta, n_steps, threads=0):
    """Kerr-ODE of each row of x [M, 2*nb] (interleaved r, s bands):
    kerr_ode_cpu, src/backend.rs:387-417, mapped over the rows."""
    x = np.ascontiguousarray(x, np.float32)
    M, n = x.shape
    nb = n // 2
    y = np.empty((M, n), np.float32)
    lib().kode_oracle_forward(M, nb, int(n_steps), _ptr(x), n, _ptr(np.ascontiguousarray(gamma_raw, np.float32)),
                              _ptr(np.ascontiguousarray(omega, np.float32)), float(alpha), float(beta), _ptr(y), n,
                              threads)
    return y


def kerr_ode_backward(dy, x, gamma_raw, omega, alpha, beta, n_steps, threads=1):
    """(dx, d_gamma_raw, d_omega, d_alpha, d_beta) of the Kerr-ODE over the rows
    of x: kerr_ode_backward_batch's default, src/backend.rs:147-176.  With
    threads=1 the parameter sums run over the positions in the reference's
    order."""
    dy = np.ascontiguousarray(dy, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    M, n = x.shape
    nb = n // 2
    dx = np.empty((M, n), np.float32)
    dgr = np.empty(nb, np.float32)
    dom = np.empty(nb, np.float32)
    dab = np.empty(2, np.float32)
    lib().kode_oracle_backward(M, nb, int(n_steps), _ptr(dy), n, _ptr(x), n,
                               _ptr(np.ascontiguousarray(gamma_raw, np.float32)),
                               _ptr(np.ascontiguousarray(omega, np.float32)), float(alpha), float(beta), _ptr(dx), n,
                               _ptr(dgr), _ptr(dom), _ptr(dab), threads)
    return dx, dgr, dom, float(dab[0]), float(dab[1])

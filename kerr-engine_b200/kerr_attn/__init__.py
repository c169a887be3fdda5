"""Python binding of libkerr_attn.so (the C ABI declared in include/kerr_attn.h).

The library is the product: sm_100a CUDA kernels for kerr-engine's causal
self-attention forward (src/pipeline.rs:305-347) and backward
(ComputeBackend::attention_backward, src/backend.rs:223-231).  This module only
marshals tensors into the C ABI; it has no compute path of its own and raises
if the library is missing.

Tensors: torch float32, CUDA for :func:`fwd` / :func:`bwd` (device pointers)
and CPU (pinned or pageable) for :func:`fwd_host` / :func:`bwd_host`.  q, k, v,
dq, dk, dv are [B, T, H*d] views whose last dimension is contiguous and whose
rows may be strided (e.g. the q|k|v column blocks of one [B, T, 3C] buffer).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_DIR, "lib", "libkerr_attn.so")

KATTN_OK = 0
KATTN_ERR_INVALID_ARGUMENT = 1
KATTN_ERR_UNSUPPORTED = 2
KATTN_ERR_MISALIGNED = 3
KATTN_ERR_DEVICE = 4
KATTN_ERR_CUDA = 5
KATTN_ERR_OUT_OF_MEMORY = 6
KATTN_ERR_DEVICE_TIMEOUT = 7

PATH_AUTO = 0
PATH_FFMA = 1
PATH_TENSOR = 2

# Every function include/kerr_attn.h declares.
EXPORTED_SYMBOLS = (
    "kattn_version", "kattn_strerror", "kattn_last_error", "kattn_create", "kattn_destroy",
    "kattn_set_path", "kattn_check_device", "kattn_set_wait_limit", "kattn_test_withhold_next_load",
    "kattn_set_deterministic",
    "kattn_fwd", "kattn_bwd", "kattn_fwd_host", "kattn_bwd_host", "kattn_last_launch_count",
    "kattn_bwd_noalloc",
    "kattn_linear_fwd", "kattn_linear_bwd_dx", "kattn_linear_bwd_dw",
    "kattn_saved_create", "kattn_saved_destroy", "kattn_fwd_host_save", "kattn_bwd_host_saved",
    "kattn_layernorm_fwd", "kattn_layernorm_bwd",
    "kattn_kerr_ode_fwd", "kattn_kerr_ode_bwd", "kattn_kerr_ode_fwd_host", "kattn_kerr_ode_bwd_host",
    "kattn_block_create", "kattn_block_destroy", "kattn_block_fwd", "kattn_block_bwd",
)

# Widest row kattn_layernorm_fwd / _bwd accept (KATTN_LN_MAX_N).
LN_MAX_N = 1536
# Most bands kattn_kerr_ode_fwd / _bwd accept (KATTN_KODE_MAX_BANDS).
KODE_MAX_BANDS = 1024

# Largest B*H*T that kattn_bwd_noalloc accepts (KATTN_NOALLOC_MAX_ROWS).
NOALLOC_MAX_ROWS = 1 << 20


class KattnError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: {detail} (status {status})")
        self.status = status


_lib = None
_p = ctypes.c_void_p
_l = ctypes.c_long
_i = ctypes.c_int
_fl = ctypes.c_float


def build() -> str:
    """Compile libkerr_attn.so in-tree with the package Makefile."""
    subprocess.run(["make", "-s", "-C", _PKG_DIR], check=True)
    return LIB_PATH


def lib():
    """Load libkerr_attn.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {_PKG_DIR}`")
    L = ctypes.CDLL(LIB_PATH)
    L.kattn_version.restype = _i
    L.kattn_strerror.argtypes = [_i]
    L.kattn_strerror.restype = ctypes.c_char_p
    L.kattn_last_error.restype = ctypes.c_char_p
    L.kattn_last_launch_count.restype = _i
    L.kattn_create.argtypes = [_i, ctypes.POINTER(_p)]
    L.kattn_create.restype = _i
    L.kattn_destroy.argtypes = [_p]
    L.kattn_destroy.restype = _i
    L.kattn_set_path.argtypes = [_p, _i]
    L.kattn_set_path.restype = _i
    L.kattn_check_device.argtypes = [_p]
    L.kattn_check_device.restype = _i
    L.kattn_set_wait_limit.argtypes = [_p, ctypes.c_ulonglong]
    L.kattn_set_wait_limit.restype = _i
    L.kattn_set_deterministic.argtypes = [_p, _i]
    L.kattn_set_deterministic.restype = _i
    L.kattn_test_withhold_next_load.argtypes = [_p]
    L.kattn_test_withhold_next_load.restype = _i
    fwd_args = [_p, _p, _p, _p, _l, _p, _l, _p, _i, _i, _i, _i, _fl, _i]
    bwd_args = [_p, _p, _p, _p, _l, _p, _p, _l, _p, _p, _p, _p, _l, _i, _i, _i, _i, _fl, _i]
    L.kattn_fwd.argtypes = fwd_args + [_p]
    L.kattn_fwd.restype = _i
    L.kattn_bwd.argtypes = bwd_args + [_p]
    L.kattn_bwd.restype = _i
    L.kattn_bwd_noalloc.argtypes = bwd_args + [_p]
    L.kattn_bwd_noalloc.restype = _i
    L.kattn_fwd_host.argtypes = fwd_args
    L.kattn_fwd_host.restype = _i
    L.kattn_bwd_host.argtypes = bwd_args
    L.kattn_bwd_host.restype = _i
    L.kattn_saved_create.argtypes = [_p, ctypes.POINTER(_p)]
    L.kattn_saved_create.restype = _i
    L.kattn_block_create.argtypes = [_p, _i, _i, _i, _i, _i, ctypes.POINTER(_p)]
    L.kattn_block_create.restype = _i
    L.kattn_block_destroy.argtypes = [_p]
    L.kattn_block_destroy.restype = _i
    L.kattn_block_fwd.argtypes = [_p, _p, ctypes.POINTER(BlockParams), _p, _p, _p]
    L.kattn_block_fwd.restype = _i
    L.kattn_block_bwd.argtypes = [_p, _p, _p, _p, ctypes.POINTER(BlockGrads), _i, _p]
    L.kattn_block_bwd.restype = _i
    L.kattn_saved_destroy.argtypes = [_p]
    L.kattn_saved_destroy.restype = _i
    L.kattn_fwd_host_save.argtypes = [_p, _p] + fwd_args[1:]
    L.kattn_fwd_host_save.restype = _i
    L.kattn_bwd_host_saved.argtypes = [_p, _p, _p, _l, _p, _p, _p, _l]
    L.kattn_bwd_host_saved.restype = _i
    L.kattn_layernorm_fwd.argtypes = [_p, _p, _l, _p, _p, _p, _l, _i, _i, _p]
    L.kattn_layernorm_fwd.restype = _i
    L.kattn_layernorm_bwd.argtypes = [_p, _p, _l, _p, _l, _p, _p, _l, _p, _p, _i, _i, _i, _p]
    L.kattn_layernorm_bwd.restype = _i
    L.kattn_linear_fwd.argtypes = [_p, _p, _l, _p, _p, _p, _l, _i, _i, _i, _p]
    L.kattn_linear_fwd.restype = _i
    L.kattn_linear_bwd_dx.argtypes = [_p, _p, _l, _p, _p, _l, _i, _i, _i, _p]
    L.kattn_linear_bwd_dx.restype = _i
    L.kattn_linear_bwd_dw.argtypes = [_p, _p, _l, _p, _l, _p, _p, _i, _i, _i, _i, _p]
    L.kattn_linear_bwd_dw.restype = _i
    L.kattn_kerr_ode_fwd.argtypes = [_p, _p, _l, _p, _l, _p, _p, _p, _i, _i, _i, _p]
    L.kattn_kerr_ode_fwd.restype = _i
    L.kattn_kerr_ode_bwd.argtypes = [_p, _p, _l, _p, _l, _p, _p, _p, _p, _l, _p, _p, _p, _i, _i, _i, _i, _p]
    L.kattn_kerr_ode_bwd.restype = _i
    L.kattn_kerr_ode_fwd_host.argtypes = [_p, _p, _l, _p, _l, _p, _p, _fl, _fl, _i, _i, _i]
    L.kattn_kerr_ode_fwd_host.restype = _i
    L.kattn_kerr_ode_bwd_host.argtypes = [_p, _p, _l, _p, _l, _p, _p, _fl, _fl, _p, _l, _p, _p, _p, _i, _i, _i, _i]
    L.kattn_kerr_ode_bwd_host.restype = _i
    _lib = L
    return L


def strerror(status: int) -> str:
    return lib().kattn_strerror(status).decode()


def last_error() -> str:
    return lib().kattn_last_error().decode()


def last_launch_count() -> int:
    return lib().kattn_last_launch_count()


def _check(status: int, what: str):
    if status != KATTN_OK:
        raise KattnError(status, what, f"{strerror(status)}: {last_error()}")


class Context:
    """One kattn_ctx on a CUDA device (kattn_create / kattn_destroy)."""

    def __init__(self, device: int = 0):
        h = _p()
        _check(lib().kattn_create(device, ctypes.byref(h)), "kattn_create")
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    def set_path(self, path: int):
        """Kernel family for later calls: PATH_AUTO, PATH_FFMA or PATH_TENSOR."""
        _check(lib().kattn_set_path(self._h, path), "kattn_set_path")

    def check_device(self):
        """Synchronise the device; raise if a kernel gave up a bounded wait."""
        _check(lib().kattn_check_device(self._h), "kattn_check_device")

    def set_wait_limit(self, ns: int):
        """Wall-time limit of the tensor-core kernels' bounded waits (0: one second)."""
        _check(lib().kattn_set_wait_limit(self._h, int(ns)), "kattn_set_wait_limit")

    def set_deterministic(self, on: bool = True):
        """dQ by per-key-tile slices summed in a fixed order (same inputs, same bits)."""
        _check(lib().kattn_set_deterministic(self._h, 1 if on else 0), "kattn_set_deterministic")

    def test_withhold_next_load(self):
        """Diagnostic: the next tensor-core forward withholds its first key-tile
        copy, so its bounded waits run out (kattn_test_withhold_next_load)."""
        _check(lib().kattn_test_withhold_next_load(self._h), "kattn_test_withhold_next_load")

    def close(self):
        if self._h is not None and self._h.value:
            _check(lib().kattn_destroy(self._h), "kattn_destroy")
        self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _rows(t, name):
    """(pointer, row stride) of a [B, T, C] float32 view with unit inner stride."""
    import torch

    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32")
    if t.dim() != 3 or t.stride(2) != 1 or t.stride(0) != t.shape[1] * t.stride(1):
        raise ValueError(f"{name} must be a [B, T, C] view with contiguous rows stacked over the batch")
    return ctypes.c_void_p(t.data_ptr()), t.stride(1)


def _vec(t, name):
    import torch

    if t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous float32 tensor")
    return ctypes.c_void_p(t.data_ptr())


def _stream_ptr(stream, device):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream(device)
    return ctypes.c_void_p(s.cuda_stream)


def fwd(ctx: Context, q, k, v, o, lse, n_head: int, causal: bool = True, scale: float | None = None,
        stream=None) -> int:
    """Enqueue the forward on `stream` (default: torch's current stream).
    q, k, v, o: [B, T, C] CUDA views; lse: [B, H, T].  Returns kernels launched."""
    B, T, C = q.shape
    d = C // n_head
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    pq, ld = _rows(q, "q")
    pk, ldk = _rows(k, "k")
    pv, ldv = _rows(v, "v")
    po, ldo = _rows(o, "o")
    if not (ld == ldk == ldv):
        raise ValueError("q, k, v must share one row stride")
    st = lib().kattn_fwd(ctx.handle, pq, pk, pv, ld, po, ldo, _vec(lse, "lse"), B, T, n_head, d, sc,
                         int(causal), _stream_ptr(stream, q.device))
    _check(st, "kattn_fwd")
    return last_launch_count()


def bwd(ctx: Context, q, k, v, o, dout, lse, dq, dk, dv, n_head: int, causal: bool = True,
        scale: float | None = None, stream=None) -> int:
    """Enqueue the backward on `stream`.  dq, dk, dv are overwritten.
    Returns kernels launched."""
    B, T, C = q.shape
    d = C // n_head
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    pq, ld = _rows(q, "q")
    pk, ldk = _rows(k, "k")
    pv, ldv = _rows(v, "v")
    po, ldo = _rows(o, "o")
    pdo, ldd_o = _rows(dout, "dout")
    pdq, ldg = _rows(dq, "dq")
    pdk, ldgk = _rows(dk, "dk")
    pdv, ldgv = _rows(dv, "dv")
    if not (ld == ldk == ldv) or ldo != ldd_o or not (ldg == ldgk == ldgv):
        raise ValueError("stride groups (q,k,v), (o,dout), (dq,dk,dv) must each share one row stride")
    st = lib().kattn_bwd(ctx.handle, pq, pk, pv, ld, po, pdo, ldo, _vec(lse, "lse"), pdq, pdk, pdv, ldg,
                         B, T, n_head, d, sc, int(causal), _stream_ptr(stream, q.device))
    _check(st, "kattn_bwd")
    return last_launch_count()


def bwd_noalloc(ctx: Context, q, k, v, o, dout, lse, dq, dk, dv, n_head: int, causal: bool = True,
                scale: float | None = None, stream=None) -> int:
    """kattn_bwd_noalloc: the backward for callers that cannot allocate device
    memory; its workspace is the library's fixed device array (B*H*T up to
    NOALLOC_MAX_ROWS; calls that overlap on the GPU race on it)."""
    B, T, C = q.shape
    d = C // n_head
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    pq, ld = _rows(q, "q")
    pk, ldk = _rows(k, "k")
    pv, ldv = _rows(v, "v")
    po, ldo = _rows(o, "o")
    pdo, ldd_o = _rows(dout, "dout")
    pdq, ldg = _rows(dq, "dq")
    pdk, ldgk = _rows(dk, "dk")
    pdv, ldgv = _rows(dv, "dv")
    if not (ld == ldk == ldv) or ldo != ldd_o or not (ldg == ldgk == ldgv):
        raise ValueError("stride groups (q,k,v), (o,dout), (dq,dk,dv) must each share one row stride")
    st = lib().kattn_bwd_noalloc(ctx.handle, pq, pk, pv, ld, po, pdo, ldo, _vec(lse, "lse"), pdq, pdk, pdv, ldg,
                                 B, T, n_head, d, sc, int(causal), _stream_ptr(stream, q.device))
    _check(st, "kattn_bwd_noalloc")
    return last_launch_count()


def fwd_host(ctx: Context, q, k, v, o, lse, n_head: int, causal: bool = True, scale: float | None = None) -> int:
    """Synchronous forward on host (CPU) tensors through kattn_fwd_host."""
    B, T, C = q.shape
    d = C // n_head
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    pq, ld = _rows(q, "q")
    pk, _ = _rows(k, "k")
    pv, _ = _rows(v, "v")
    po, ldo = _rows(o, "o")
    st = lib().kattn_fwd_host(ctx.handle, pq, pk, pv, ld, po, ldo, _vec(lse, "lse"), B, T, n_head, d, sc,
                              int(causal))
    _check(st, "kattn_fwd_host")
    return last_launch_count()


def bwd_host(ctx: Context, q, k, v, o, dout, lse, dq, dk, dv, n_head: int, causal: bool = True,
             scale: float | None = None) -> int:
    """Synchronous backward on host (CPU) tensors through kattn_bwd_host."""
    B, T, C = q.shape
    d = C // n_head
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    pq, ld = _rows(q, "q")
    pk, _ = _rows(k, "k")
    pv, _ = _rows(v, "v")
    po, ldo = _rows(o, "o")
    pdo, _ = _rows(dout, "dout")
    pdq, ldg = _rows(dq, "dq")
    pdk, _ = _rows(dk, "dk")
    pdv, _ = _rows(dv, "dv")
    st = lib().kattn_bwd_host(ctx.handle, pq, pk, pv, ld, po, pdo, ldo, _vec(lse, "lse"), pdq, pdk, pdv, ldg,
                              B, T, n_head, d, sc, int(causal))
    _check(st, "kattn_bwd_host")
    return last_launch_count()


class Saved:
    """Device-resident state of one forward (the reference's AttnCache,
    src/pipeline.rs:157-164): q/k/v, o and lse, for :func:`bwd_host_saved`."""

    def __init__(self, ctx: Context):
        h = ctypes.c_void_p()
        _check(lib().kattn_saved_create(ctx.handle, ctypes.byref(h)), "kattn_saved_create")
        self._h = h
        self.ctx = ctx

    @property
    def handle(self):
        if self._h is None:
            raise RuntimeError("saved state is closed")
        return self._h

    def close(self):
        if self._h is not None:
            st = lib().kattn_saved_destroy(self._h)
            self._h = None
            _check(st, "kattn_saved_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def fwd_host_save(ctx: Context, saved: Saved, q, k, v, o, lse, n_head: int, causal: bool = True,
                  scale: float | None = None) -> int:
    """fwd_host, keeping q/k/v, o and lse on the device in `saved`."""
    B, T, C = q.shape
    d = C // n_head
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    pq, ld = _rows(q, "q")
    pk, _ = _rows(k, "k")
    pv, _ = _rows(v, "v")
    po, ldo = _rows(o, "o")
    st = lib().kattn_fwd_host_save(ctx.handle, saved.handle, pq, pk, pv, ld, po, ldo, _vec(lse, "lse"), B, T,
                                   n_head, d, sc, int(causal))
    _check(st, "kattn_fwd_host_save")
    return last_launch_count()


def bwd_host_saved(ctx: Context, saved: Saved, dout, dq, dk, dv) -> int:
    """Backward of the forward held in `saved`, host tensors dout in and dq/dk/dv out."""
    pdo, ldo = _rows(dout, "dout")
    pdq, ldg = _rows(dq, "dq")
    pdk, _ = _rows(dk, "dk")
    pdv, _ = _rows(dv, "dv")
    st = lib().kattn_bwd_host_saved(ctx.handle, saved.handle, pdo, ldo, pdq, pdk, pdv, ldg)
    _check(st, "kattn_bwd_host_saved")
    return last_launch_count()


def split_qkv(qkv, n_embd: int):
    """q, k, v column-block views of a [B, T, 3C] buffer (src/pipeline.rs:296-302)."""
    return qkv[..., :n_embd], qkv[..., n_embd:2 * n_embd], qkv[..., 2 * n_embd:]


# ---------------------------------------------------------------- projections
# c_attn / c_proj as dense layers (include/kerr_attn.h, kattn_linear_*).  Rows
# are positions: x / y / dy / dx are [..., features] float32 CUDA views whose
# leading dimensions flatten to M rows with one row stride; w is [out, in]
# contiguous (the reference's layout), b / db [out] contiguous.

def _mat(t, name):
    """(pointer, row stride, rows, cols) of a float32 CUDA view whose rows
    (all leading dimensions) share one stride and have unit inner stride."""
    import torch

    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit inner stride")
    cols = t.shape[-1]
    rows = t.numel() // cols if cols else 0
    if t.dim() == 1:
        return ctypes.c_void_p(t.data_ptr()), cols, 1, cols
    ld = t.stride(-2)
    expect = ld
    for dim in range(t.dim() - 2, 0, -1):
        expect *= t.shape[dim]
        if t.shape[dim - 1] > 1 and t.stride(dim - 1) != expect:
            raise ValueError(f"{name} rows must be evenly strided over the leading dimensions")
    return ctypes.c_void_p(t.data_ptr()), ld, rows, cols


def linear_fwd(ctx: Context, x, w, b, y, stream=None) -> int:
    """y = x w^T + b (b may be None).  Returns this library's kernels launched."""
    px, ldx, M, K = _mat(x, "x")
    py, ldy, My, N = _mat(y, "y")
    if My != M or tuple(w.shape) != (N, K):
        raise ValueError("shapes: x [M, K], w [N, K], y [M, N]")
    st = lib().kattn_linear_fwd(ctx.handle, px, ldx, _vec(w, "w"), None if b is None else _vec(b, "b"), py, ldy,
                                M, N, K, _stream_ptr(stream, x.device))
    _check(st, "kattn_linear_fwd")
    return last_launch_count()


def linear_bwd_dx(ctx: Context, dy, w, dx, stream=None) -> int:
    """dx = dy w."""
    pd, ldd, M, N = _mat(dy, "dy")
    px, ldx, Mx, K = _mat(dx, "dx")
    if Mx != M or tuple(w.shape) != (N, K):
        raise ValueError("shapes: dy [M, N], w [N, K], dx [M, K]")
    st = lib().kattn_linear_bwd_dx(ctx.handle, pd, ldd, _vec(w, "w"), px, ldx, M, N, K,
                                   _stream_ptr(stream, dy.device))
    _check(st, "kattn_linear_bwd_dx")
    return last_launch_count()


def linear_bwd_dw(ctx: Context, dy, x, dw, db, accumulate: bool = True, stream=None) -> int:
    """dw (+)= dy^T x and db (+)= colsum(dy) (db may be None)."""
    pd, ldd, M, N = _mat(dy, "dy")
    px, ldx, Mx, K = _mat(x, "x")
    if Mx != M or tuple(dw.shape) != (N, K):
        raise ValueError("shapes: dy [M, N], x [M, K], dw [N, K]")
    st = lib().kattn_linear_bwd_dw(ctx.handle, pd, ldd, px, ldx, _vec(dw, "dw"), None if db is None else _vec(db, "db"),
                                   M, N, K, int(accumulate), _stream_ptr(stream, dy.device))
    _check(st, "kattn_linear_bwd_dw")
    return last_launch_count()


# ---------------------------------------------------------------- layer norm

def layernorm_fwd(ctx: Context, x, w, b, y, stream=None) -> int:
    """y = LayerNorm(x) w + b over the last dimension (eps 1e-5).  Returns kernels launched."""
    px, ldx, M, N = _mat(x, "x")
    py, ldy, My, Ny = _mat(y, "y")
    if (My, Ny) != (M, N) or tuple(w.shape) != (N,) or tuple(b.shape) != (N,):
        raise ValueError("shapes: x [.., N], y like x, w [N], b [N]")
    st = lib().kattn_layernorm_fwd(ctx.handle, px, ldx, _vec(w, "w"), _vec(b, "b"), py, ldy, M, N,
                                   _stream_ptr(stream, x.device))
    _check(st, "kattn_layernorm_fwd")
    return last_launch_count()


def layernorm_bwd(ctx: Context, dy, x, w, dx, dw, db, accumulate: bool = True, stream=None) -> int:
    """dx of LayerNorm; dw / db (either may be None) receive the column sums
    (added when `accumulate`).  Returns kernels launched."""
    pdy, lddy, M, N = _mat(dy, "dy")
    px, ldx, Mx, Nx = _mat(x, "x")
    pdx, lddx, Md, Nd = _mat(dx, "dx")
    if (Mx, Nx) != (M, N) or (Md, Nd) != (M, N) or tuple(w.shape) != (N,):
        raise ValueError("shapes: dy, x, dx [.., N], w [N]")
    st = lib().kattn_layernorm_bwd(ctx.handle, pdy, lddy, px, ldx, _vec(w, "w"), pdx, lddx,
                                   None if dw is None else _vec(dw, "dw"), None if db is None else _vec(db, "db"),
                                   M, N, int(accumulate), _stream_ptr(stream, dy.device))
    _check(st, "kattn_layernorm_bwd")
    return last_launch_count()



# ---------------------------------------------------------------- Kerr-ODE
# The FFN's ODE core (include/kerr_attn.h, kattn_kerr_ode_*): rows of x / y /
# dy / dx are positions of 2 * n_bands interleaved (r, s) floats; gamma_raw and
# omega are [n_bands], alpha_beta is [alpha, beta]; all float32 CUDA tensors.

def kerr_ode_fwd(ctx: Context, x, gamma_raw, omega, alpha_beta, y, n_steps: int, stream=None) -> int:
    """y = Kerr-ODE(x) per row (kerr_ode_cpu, src/backend.rs:387-417).  Returns kernels launched."""
    px, ldx, M, n = _mat(x, "x")
    py, ldy, My, ny = _mat(y, "y")
    nb = n // 2
    if (My, ny) != (M, n) or tuple(gamma_raw.shape) != (nb,) or tuple(omega.shape) != (nb,) \
            or tuple(alpha_beta.shape) != (2,):
        raise ValueError("shapes: x [.., 2 nb], y like x, gamma_raw [nb], omega [nb], alpha_beta [2]")
    st = lib().kattn_kerr_ode_fwd(ctx.handle, px, ldx, py, ldy, _vec(gamma_raw, "gamma_raw"), _vec(omega, "omega"),
                                  _vec(alpha_beta, "alpha_beta"), M, nb, int(n_steps), _stream_ptr(stream, x.device))
    _check(st, "kattn_kerr_ode_fwd")
    return last_launch_count()


def kerr_ode_bwd(ctx: Context, dy, x, gamma_raw, omega, alpha_beta, dx, d_gamma_raw, d_omega, d_alpha_beta,
                 n_steps: int, accumulate: bool = True, stream=None) -> int:
    """dx of the Kerr-ODE; the parameter gradients summed over the rows go into
    d_gamma_raw / d_omega / d_alpha_beta (added when `accumulate`).  Returns kernels launched."""
    pdy, lddy, M, n = _mat(dy, "dy")
    px, ldx, Mx, nx = _mat(x, "x")
    pdx, lddx, Md, nd = _mat(dx, "dx")
    nb = n // 2
    if (Mx, nx) != (M, n) or (Md, nd) != (M, n):
        raise ValueError("shapes: dy, x, dx [.., 2 nb]")
    for t, name, shape in ((gamma_raw, "gamma_raw", (nb,)), (omega, "omega", (nb,)), (alpha_beta, "alpha_beta", (2,)),
                           (d_gamma_raw, "d_gamma_raw", (nb,)), (d_omega, "d_omega", (nb,)),
                           (d_alpha_beta, "d_alpha_beta", (2,))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}")
    st = lib().kattn_kerr_ode_bwd(ctx.handle, pdy, lddy, px, ldx, _vec(gamma_raw, "gamma_raw"), _vec(omega, "omega"),
                                  _vec(alpha_beta, "alpha_beta"), pdx, lddx, _vec(d_gamma_raw, "d_gamma_raw"),
                                  _vec(d_omega, "d_omega"), _vec(d_alpha_beta, "d_alpha_beta"), M, nb, int(n_steps),
                                  int(accumulate), _stream_ptr(stream, dy.device))
    _check(st, "kattn_kerr_ode_bwd")
    return last_launch_count()


def kerr_ode_fwd_host(ctx: Context, x, gamma_raw, omega, alpha: float, beta: float, y, n_steps: int) -> int:
    """Synchronous Kerr-ODE forward on host (CPU) float32 tensors: rows of x / y
    are positions; gamma_raw / omega host vectors; alpha, beta floats."""
    px, ldx, M, n = _mat(x, "x")
    py, ldy, My, ny = _mat(y, "y")
    nb = n // 2
    if (My, ny) != (M, n) or tuple(gamma_raw.shape) != (nb,) or tuple(omega.shape) != (nb,):
        raise ValueError("shapes: x [.., 2 nb], y like x, gamma_raw [nb], omega [nb]")
    st = lib().kattn_kerr_ode_fwd_host(ctx.handle, px, ldx, py, ldy, _vec(gamma_raw, "gamma_raw"),
                                       _vec(omega, "omega"), float(alpha), float(beta), M, nb, int(n_steps))
    _check(st, "kattn_kerr_ode_fwd_host")
    return last_launch_count()


def kerr_ode_bwd_host(ctx: Context, dy, x, gamma_raw, omega, alpha: float, beta: float, dx, d_gamma_raw, d_omega,
                      d_alpha_beta, n_steps: int, accumulate: bool = True) -> int:
    """Synchronous Kerr-ODE backward on host float32 tensors (see kerr_ode_bwd)."""
    pdy, lddy, M, n = _mat(dy, "dy")
    px, ldx, Mx, nx = _mat(x, "x")
    pdx, lddx, Md, nd = _mat(dx, "dx")
    nb = n // 2
    if (Mx, nx) != (M, n) or (Md, nd) != (M, n):
        raise ValueError("shapes: dy, x, dx [.., 2 nb]")
    for t, name, shape in ((gamma_raw, "gamma_raw", (nb,)), (omega, "omega", (nb,)),
                           (d_gamma_raw, "d_gamma_raw", (nb,)), (d_omega, "d_omega", (nb,)),
                           (d_alpha_beta, "d_alpha_beta", (2,))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}")
    st = lib().kattn_kerr_ode_bwd_host(ctx.handle, pdy, lddy, px, ldx, _vec(gamma_raw, "gamma_raw"),
                                       _vec(omega, "omega"), float(alpha), float(beta), pdx, lddx,
                                       _vec(d_gamma_raw, "d_gamma_raw"), _vec(d_omega, "d_omega"),
                                       _vec(d_alpha_beta, "d_alpha_beta"), M, nb, int(n_steps), int(accumulate))
    _check(st, "kattn_kerr_ode_bwd_host")
    return last_launch_count()


# Parameter / gradient tables of kattn_block_fwd / _bwd (kattn_block_params /
# kattn_block_grads in include/kerr_attn.h), in declaration order.
BLOCK_FIELDS = ("ln1_w", "ln1_b", "w_attn", "b_attn", "w_proj", "b_proj", "ln2_w", "ln2_b", "gamma_raw", "omega",
                "alpha_beta")


class BlockParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in BLOCK_FIELDS]


class BlockGrads(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in BLOCK_FIELDS]


def _table(cls, tensors: dict, ffn: bool):
    t = cls()
    for n in BLOCK_FIELDS:
        x = tensors.get(n)
        if x is None:
            if ffn or n in BLOCK_FIELDS[:6]:
                raise ValueError(f"{n} is required")
            continue
        if not (x.is_cuda and x.dtype == _f32() and x.is_contiguous()):
            raise ValueError(f"{n} must be a contiguous float32 CUDA tensor")
        setattr(t, n, x.data_ptr())
    return t


def _f32():
    import torch
    return torch.float32


class Block:
    """Device-resident transformer block (kattn_block_*): LN1, c_attn,
    causal attention, c_proj and the residual, then, with rk4_n_steps > 0,
    LN2 and the Kerr-ODE FFN core with its residual; every intermediate stays
    on the device between :meth:`fwd` and :meth:`bwd` (the reference's
    forward_backward_batch, src/pipeline.rs:764-1222, per block)."""

    def __init__(self, ctx: Context, B: int, T: int, C: int, n_head: int, rk4_n_steps: int = 0):
        h = ctypes.c_void_p()
        _check(lib().kattn_block_create(ctx.handle, B, T, C, n_head, rk4_n_steps, ctypes.byref(h)),
               "kattn_block_create")
        self._h = h
        self.ctx = ctx
        self.shape = (B, T, C)
        self.ffn = rk4_n_steps > 0
        self._keep = None

    @property
    def handle(self):
        if self._h is None:
            raise RuntimeError("block is closed")
        return self._h

    def _rows(self, x, name):
        B, T, C = self.shape
        if not (x.is_cuda and x.dtype == _f32() and x.is_contiguous() and x.numel() == B * T * C):
            raise ValueError(f"{name} must be a contiguous float32 CUDA tensor of {B * T * C} elements")
        return x.data_ptr()

    def fwd(self, params: dict, h, h_out, stream=None) -> int:
        """h_out = block(h); h and params must stay unchanged until :meth:`bwd`."""
        t = _table(BlockParams, params, self.ffn)
        self._keep = (params, h)  # the backward reads them
        st = lib().kattn_block_fwd(self.ctx.handle, self.handle, ctypes.byref(t), self._rows(h, "h"),
                                   self._rows(h_out, "h_out"), _stream_ptr(stream, h.device))
        _check(st, "kattn_block_fwd")
        return last_launch_count()

    def bwd(self, dh_out, dh, grads: dict, accumulate: bool = False, stream=None) -> int:
        """dh = d(loss)/dh from dh_out (dh may be dh_out); parameter gradients into `grads`."""
        t = _table(BlockGrads, grads, self.ffn)
        st = lib().kattn_block_bwd(self.ctx.handle, self.handle, self._rows(dh_out, "dh_out"), self._rows(dh, "dh"),
                                   ctypes.byref(t), int(accumulate), _stream_ptr(stream, dh.device))
        _check(st, "kattn_block_bwd")
        return last_launch_count()

    def close(self):
        if self._h is not None:
            st = lib().kattn_block_destroy(self._h)
            self._h = None
            _check(st, "kattn_block_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

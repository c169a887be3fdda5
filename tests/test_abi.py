"""CPU checks of the C ABI boundary: the library loads, exports exactly what
include/kerr_attn.h declares, and rejects bad arguments before it touches a
device (these calls make no compute call and need no GPU)."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

import kerr_attn
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "kerr_attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const char\s*\*)\s*(kattn_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(kerr_attn.LIB_PATH):
        kerr_attn.build()
    return kerr_attn.lib()


def test_header_declares_the_binding_surface():
    assert declared_functions() == sorted(kerr_attn.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(L):
    out = subprocess.run(["nm", "-D", "--defined-only", kerr_attn.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(L, name)
    # Nothing but the C ABI is visible.
    assert exported == set(declared_functions())


def test_strerror_and_version(L):
    assert L.kattn_version() >= 100
    names = {kerr_attn.strerror(s) for s in range(7)}
    assert len(names) == 7
    assert kerr_attn.strerror(0) == "ok"
    assert kerr_attn.strerror(99) == "unknown status"


def _fake_ctx():
    # A non-NULL handle: every call below fails validation before reading it.
    return ctypes.c_void_p(0x10)


def _fwd(L, ctx, q=0x1000, ld=128, o=0x2000, ld_o=128, lse=0x3000, B=1, T=8, H=4, d=32, scale=0.17, causal=1):
    return L.kattn_fwd(ctx, ctypes.c_void_p(q), ctypes.c_void_p(q + 512), ctypes.c_void_p(q + 1024), ld,
                       ctypes.c_void_p(o), ld_o, ctypes.c_void_p(lse), B, T, H, d, scale, causal, None)


def test_argument_validation(L):
    ctx = _fake_ctx()
    assert _fwd(L, None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert _fwd(L, ctx, d=48, H=2) == kerr_attn.KATTN_ERR_UNSUPPORTED
    assert "head_dim 48" in kerr_attn.last_error()
    assert _fwd(L, ctx, B=-1) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert _fwd(L, ctx, H=0) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert _fwd(L, ctx, causal=2) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert _fwd(L, ctx, scale=float("nan")) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert _fwd(L, ctx, ld=64) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT  # ld < H*d
    assert _fwd(L, ctx, q=0x1004) == kerr_attn.KATTN_ERR_MISALIGNED
    assert _fwd(L, ctx, ld=130) == kerr_attn.KATTN_ERR_MISALIGNED
    assert _fwd(L, ctx, o=0) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert _fwd(L, ctx, lse=0x3002) == kerr_attn.KATTN_ERR_MISALIGNED


def test_empty_problem_launches_nothing(L):
    ctx = _fake_ctx()
    assert _fwd(L, ctx, B=0, q=0, o=0, lse=0) == kerr_attn.KATTN_OK
    assert kerr_attn.last_launch_count() == 0
    assert _fwd(L, ctx, T=0, q=0, o=0, lse=0) == kerr_attn.KATTN_OK
    st = L.kattn_bwd(ctx, None, None, None, 0, None, None, 0, None, None, None, None, 0, 4, 0, 2, 64, 0.125, 1,
                     None)
    assert st == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0


def test_bwd_validation(L):
    ctx = _fake_ctx()
    p = [ctypes.c_void_p(0x1000 * (i + 1)) for i in range(9)]
    args = [ctx, p[0], p[1], p[2], 128, p[3], p[4], 128, p[5], p[6], p[7], p[8], 128]
    bad = list(args)
    bad[9] = ctypes.c_void_p(0x9008)  # dq misaligned
    assert L.kattn_bwd(*bad, 1, 8, 4, 32, 0.17, 1, None) == kerr_attn.KATTN_ERR_MISALIGNED
    bad = list(args)
    bad[12] = 100  # ld_dqkv < H*d
    assert L.kattn_bwd(*bad, 1, 8, 4, 32, 0.17, 1, None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT


def test_linear_validation(L):
    # The projection entry points reject bad arguments before touching a device.
    ctx = _fake_ctx()
    P = ctypes.c_void_p
    x, w, b, y = P(0x10000), P(0x20000), P(0x30000), P(0x40000)

    def fwd(c=ctx, x=x, ldx=128, w=w, b=b, y=y, ldy=384, M=256, N=384, K=128):
        return L.kattn_linear_fwd(c, x, ldx, w, b, y, ldy, M, N, K, None)

    assert fwd(c=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(M=-1) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(x=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(ldx=64) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT      # ld < K
    assert fwd(x=P(0x10008)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(ldy=386) == kerr_attn.KATTN_ERR_MISALIGNED           # stride not a multiple of 4
    assert fwd(K=126, ldx=128) == kerr_attn.KATTN_ERR_MISALIGNED    # width not a multiple of 4
    assert fwd(b=P(0x30002)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(M=0, x=None, y=None) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0
    assert L.kattn_linear_bwd_dx(ctx, y, 384, w, P(0x50004), 128, 256, 384, 128, None) == \
        kerr_attn.KATTN_ERR_MISALIGNED
    assert L.kattn_linear_bwd_dw(ctx, y, 384, x, 128, None, b, 256, 384, 128, 1, None) == \
        kerr_attn.KATTN_ERR_INVALID_ARGUMENT                         # dw is NULL
    assert L.kattn_linear_bwd_dw(ctx, y, 384, x, 128, P(0x60000), b, 256, 0, 128, 1, None) == kerr_attn.KATTN_OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_create_without_device_fails_cleanly(L):
    with pytest.raises(kerr_attn.KattnError) as e:
        kerr_attn.Context(0)
    assert e.value.status == kerr_attn.KATTN_ERR_DEVICE


def test_saved_state_validation(L):
    # The saved-state calls reject bad arguments and an empty state before
    # touching a device; creating and destroying an unused state needs none.
    ctx, other = _fake_ctx(), ctypes.c_void_p(0x20)  # two distinct handles; neither is dereferenced
    P = ctypes.c_void_p
    out = P()
    assert L.kattn_saved_create(None, ctypes.byref(out)) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert L.kattn_saved_create(ctx, None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert L.kattn_saved_create(ctx, ctypes.byref(out)) == kerr_attn.KATTN_OK and out.value
    h = P(0x10000)
    # No forward has run into it yet.
    assert L.kattn_bwd_host_saved(ctx, out, h, 64, h, h, h, 192) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert "no completed forward" in kerr_attn.last_error()
    assert L.kattn_bwd_host_saved(ctx, None, h, 64, h, h, h, 192) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert L.kattn_bwd_host_saved(None, out, h, 64, h, h, h, 192) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    # A state belongs to the context that created it.
    assert L.kattn_bwd_host_saved(other, out, h, 64, h, h, h, 192) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert L.kattn_fwd_host_save(other, out, h, h, h, 192, h, 64, h, 2, 8, 1, 64, 0.125, 1) == \
        kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert L.kattn_fwd_host_save(ctx, None, h, h, h, 192, h, 64, h, 2, 8, 1, 64, 0.125, 1) == \
        kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    # The forward's own argument checks apply (head_dim 48 is unsupported).
    assert L.kattn_fwd_host_save(ctx, out, h, h, h, 144, h, 48, h, 2, 8, 1, 48, 0.125, 1) == \
        kerr_attn.KATTN_ERR_UNSUPPORTED
    assert L.kattn_saved_destroy(out) == kerr_attn.KATTN_OK
    assert L.kattn_saved_destroy(None) == kerr_attn.KATTN_OK


def test_layernorm_validation(L):
    # The LayerNorm entry points reject bad arguments before touching a device.
    ctx = _fake_ctx()
    P = ctypes.c_void_p
    x, w, b, y = P(0x10000), P(0x20000), P(0x30000), P(0x40000)

    def fwd(c=ctx, x=x, ldx=768, w=w, b=b, y=y, ldy=768, M=64, N=768):
        return L.kattn_layernorm_fwd(c, x, ldx, w, b, y, ldy, M, N, None)

    assert fwd(c=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(M=-1) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(N=kerr_attn.LN_MAX_N + 4, ldx=4096, ldy=4096) == kerr_attn.KATTN_ERR_UNSUPPORTED
    assert fwd(x=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(ldx=764) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT      # ld < N
    assert fwd(x=P(0x10008)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(N=766, ldx=768, ldy=768) == kerr_attn.KATTN_ERR_MISALIGNED  # width not a multiple of 4
    assert fwd(w=P(0x20004)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(b=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(M=0) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0

    def bwd(dw=P(0x50000), db=P(0x60000), M=64, acc=1, dx=P(0x70000)):
        return L.kattn_layernorm_bwd(ctx, y, 768, x, 768, w, dx, 768, dw, db, M, 768, acc, None)

    assert bwd(dx=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert bwd(dw=P(0x50004)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert bwd(M=0, acc=1) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0


def test_kerr_ode_validation(L):
    # The Kerr-ODE entry points reject bad arguments before touching a device.
    ctx = _fake_ctx()
    P = ctypes.c_void_p
    x, y, g, o, ab = P(0x10000), P(0x20000), P(0x30000), P(0x40000), P(0x50000)

    def fwd(c=ctx, x=x, ldx=768, y=y, ldy=768, g=g, o=o, ab=ab, M=64, nb=384, steps=8):
        return L.kattn_kerr_ode_fwd(c, x, ldx, y, ldy, g, o, ab, M, nb, steps, None)

    assert fwd(c=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(M=-1) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(nb=0) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(steps=0) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(nb=382, ldx=764, ldy=764) == kerr_attn.KATTN_ERR_UNSUPPORTED  # n_embd not a multiple of 8
    assert fwd(nb=kerr_attn.KODE_MAX_BANDS + 4, ldx=4096, ldy=4096) == kerr_attn.KATTN_ERR_UNSUPPORTED
    assert fwd(nb=1024, ldx=2048, ldy=2048, steps=64) == kerr_attn.KATTN_ERR_UNSUPPORTED  # states exceed shared memory
    assert "shared memory" in kerr_attn.last_error()
    assert fwd(x=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(ldx=764) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT      # ld < 2 nb
    assert fwd(ldy=770) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(x=P(0x10008)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(g=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(ab=P(0x50002)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert fwd(M=0) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0

    def bwd(dx=P(0x60000), dg=P(0x70000), do=P(0x80000), dab=P(0x90000), M=64, acc=1):
        return L.kattn_kerr_ode_bwd(ctx, y, 768, x, 768, g, o, ab, dx, 768, dg, do, dab, M, 384, 8, acc, None)

    assert bwd(dx=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert bwd(dg=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert bwd(dab=P(0x90001)) == kerr_attn.KATTN_ERR_MISALIGNED
    assert bwd(M=0, acc=1) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0


def test_kerr_ode_host_validation(L):
    # The host-buffer Kerr-ODE entry points check their arguments before any
    # device call (host arrays carry no alignment requirement).
    ctx = _fake_ctx()
    P = ctypes.c_void_p
    x, y, g, o = P(0x10004), P(0x20004), P(0x30004), P(0x40004)

    def fwd(c=ctx, x=x, ldx=768, y=y, ldy=768, g=g, o=o, M=64, nb=384, steps=8):
        return L.kattn_kerr_ode_fwd_host(c, x, ldx, y, ldy, g, o, 0.1, 0.1, M, nb, steps)

    assert fwd(c=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(g=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(x=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(ldy=700) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(nb=382, ldx=764, ldy=764) == kerr_attn.KATTN_ERR_UNSUPPORTED
    assert fwd(steps=0) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert fwd(M=0) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0

    def bwd(dx=P(0x50004), dg=P(0x60004), M=64, acc=1):
        return L.kattn_kerr_ode_bwd_host(ctx, y, 768, x, 768, g, o, 0.1, 0.1, dx, 768, dg, P(0x70004), P(0x80004),
                                         M, 384, 8, acc)

    assert bwd(dx=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert bwd(dg=None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert bwd(M=0, acc=1) == kerr_attn.KATTN_OK and kerr_attn.last_launch_count() == 0
    # No positions and accumulate=0: the host gradients are set to zero.
    dgr = (ctypes.c_float * 384)(*([5.0] * 384))
    dom = (ctypes.c_float * 384)(*([5.0] * 384))
    dab = (ctypes.c_float * 2)(5.0, 5.0)
    st = L.kattn_kerr_ode_bwd_host(ctx, y, 768, x, 768, g, o, 0.1, 0.1, P(0x50004), 768, dgr, dom, dab, 0, 384, 8, 0)
    assert st == kerr_attn.KATTN_OK
    assert not any(dgr) and not any(dom) and not any(dab)

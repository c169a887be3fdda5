"""kattn_bwd_noalloc: the backward for callers that cannot allocate device memory.

A framework that routes every device byte through its own caching allocator,
or a runtime that reserves all device memory up front, cannot let the library
take memory from the device's stream-ordered pool the way kattn_bwd does for
its [B][H][T] workspace.  kattn_bwd_noalloc uses a fixed array in the
library's device image instead.  These tests call it through the C ABI and
compare it with kattn_bwd on the same inputs, twice in a row (the array keeps
the previous call's contents), for both kernel families, and check that sizes
beyond the fixed array are refused.  The file is collected last so that a run
stopping at the first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

import kerr_attn
from conftest import make_inputs, rel_err

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3  # the gradient tolerance of every parity test


def _setup(B, T, H, d, seed):
    dev = torch.device("cuda", 0)
    qkv, dout = make_inputs(B, T, H, d, seed=seed)
    C = H * d
    x = torch.from_numpy(qkv).to(dev)
    q, k, v = kerr_attn.split_qkv(x, C)
    o = torch.empty(B, T, C, device=dev)
    lse = torch.empty(B, H, T, device=dev)
    return q, k, v, o, lse, torch.from_numpy(dout).to(dev)


def _grads(fn, ctx, q, k, v, o, dout, lse, H):
    g = torch.full((q.shape[0], q.shape[1], 3 * q.shape[2]), float("nan"), device=q.device)
    dq, dk, dv = kerr_attn.split_qkv(g, q.shape[2])
    n = fn(ctx, q, k, v, o, dout, lse, dq, dk, dv, H)
    torch.cuda.synchronize()
    return n, g.cpu().numpy()


@pytest.mark.parametrize("B,T,H,d,path", [(16, 256, 12, 64, kerr_attn.PATH_AUTO),   # tensor-core kernels
                                          (3, 130, 2, 64, kerr_attn.PATH_AUTO),     # ragged
                                          (4, 64, 4, 32, kerr_attn.PATH_AUTO),      # FFMA kernels
                                          (2, 200, 3, 64, kerr_attn.PATH_FFMA)])
def test_noalloc_matches_bwd_twice(B, T, H, d, path):
    with kerr_attn.Context(0) as ctx:
        ctx.set_path(path)
        q, k, v, o, lse, dout = _setup(B, T, H, d, seed=B * 100 + T)
        kerr_attn.fwd(ctx, q, k, v, o, lse, H)
        n_ref, ref = _grads(kerr_attn.bwd, ctx, q, k, v, o, dout, lse, H)
        for _ in range(2):
            n, got = _grads(kerr_attn.bwd_noalloc, ctx, q, k, v, o, dout, lse, H)
            assert n == n_ref
            assert np.all(np.isfinite(got))
            assert rel_err(got, ref) < GRAD_TOL
        ctx.check_device()


def test_noalloc_calls_queued_back_to_back():
    # Two calls on one stream with no host synchronisation between them, on
    # different shapes and inputs: the second call's kernels may start while
    # the first call's drain (programmatic dependent launch), and both use the
    # one fixed array.  Each result must still match kattn_bwd on its inputs.
    with kerr_attn.Context(0) as ctx:
        cases = [(16, 256, 12, 64, 7), (3, 130, 2, 64, 8)]
        runs = []
        for B, T, H, d, seed in cases:
            q, k, v, o, lse, dout = _setup(B, T, H, d, seed=seed)
            kerr_attn.fwd(ctx, q, k, v, o, lse, H)
            runs.append((H, q, k, v, o, lse, dout))
        torch.cuda.synchronize()
        refs = [_grads(kerr_attn.bwd, ctx, q, k, v, o, dout, lse, H)[1] for H, q, k, v, o, lse, dout in runs]
        outs = []
        for H, q, k, v, o, lse, dout in runs:  # queued, no synchronisation in between
            g = torch.full((q.shape[0], q.shape[1], 3 * q.shape[2]), float("nan"), device=q.device)
            dq, dk, dv = kerr_attn.split_qkv(g, q.shape[2])
            kerr_attn.bwd_noalloc(ctx, q, k, v, o, dout, lse, dq, dk, dv, H)
            outs.append(g)
        torch.cuda.synchronize()
        for g, ref in zip(outs, refs):
            got = g.cpu().numpy()
            assert np.all(np.isfinite(got))
            assert rel_err(got, ref) < GRAD_TOL
        ctx.check_device()


def test_noalloc_takes_no_device_memory():
    # The entry point's promise: no device memory is allocated by the call.
    # After one call (which loads the kernels), three more calls leave the
    # device's free memory unchanged, while kattn_bwd on the same fresh
    # context (whose workspace pool starts empty) visibly reserves some.  The
    # FFMA kernels are the ones with a [B][H][T] workspace.
    with kerr_attn.Context(0) as ctx:
        ctx.set_path(kerr_attn.PATH_FFMA)
        H = 5
        q, k, v, o, lse, dout = _setup(6, 190, H, 64, seed=11)
        kerr_attn.fwd(ctx, q, k, v, o, lse, H)
        g = torch.empty((6, 190, 3 * H * 64), device=q.device)
        dq, dk, dv = kerr_attn.split_qkv(g, H * 64)
        kerr_attn.bwd_noalloc(ctx, q, k, v, o, dout, lse, dq, dk, dv, H)
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        for _ in range(3):
            kerr_attn.bwd_noalloc(ctx, q, k, v, o, dout, lse, dq, dk, dv, H)
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0
        kerr_attn.bwd(ctx, q, k, v, o, dout, lse, dq, dk, dv, H)
        torch.cuda.synchronize()
        free2, _ = torch.cuda.mem_get_info()
        assert free2 < free1  # the measurement sees a pool allocation
        ctx.check_device()


def test_noalloc_refuses_oversized_problem():
    with kerr_attn.Context(0) as ctx:
        H, d = 1, 32
        T = kerr_attn.NOALLOC_MAX_ROWS // 4 + 1  # B*H*T just above the fixed array with B=4
        dev = torch.device("cuda", 0)
        x = torch.zeros(4, T, 3 * H * d, device=dev)
        q, k, v = kerr_attn.split_qkv(x, H * d)
        o = torch.zeros(4, T, H * d, device=dev)
        lse = torch.zeros(4, H, T, device=dev)
        with pytest.raises(kerr_attn.KattnError) as e:
            kerr_attn.bwd_noalloc(ctx, q, k, v, o, o, lse, q, k, v, H)
        assert e.value.status == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
        assert "fixed workspace" in str(e.value)

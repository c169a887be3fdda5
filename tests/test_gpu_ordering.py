"""Stream ordering between this library's kernels under programmatic
dependent launch.

Every kernel lets the grid behind it launch early and waits for the grid
before it (griddepcontrol.wait) before it reads global memory, with one
exception: attn_bwd_tc64 stages its first key tiles before its own wait,
relying on attn_bwd_rowdot, launched just before it, to release it only after
rowdot's own wait.  The case that needs that order is a backward queued right
behind one of this library's kernels that writes the backward's q, k, v (the
c_attn projection recomputing qkv, as activation recomputation does), with
no host synchronisation in between.  Here qkv is first filled with NaN, then
rewritten by kattn_linear_fwd and read by kattn_bwd at once, on one stream;
in deterministic mode the gradients must equal, bit for bit, those of the
same backward run after a device synchronise.  A read of K or V ahead of the
projection's writes would show as NaN or as differing gradients.
"""
import numpy as np
import pytest
import torch

import kerr_attn

pytestmark = pytest.mark.gpu


# (B, T, H): small problems, whose few CTAs fit beside the projection's.
@pytest.mark.parametrize("B,T,H", [(1, 64, 2), (1, 130, 2), (2, 256, 4)])
def test_backward_right_after_projection_writes_qkv(B, T, H):
    d = 64
    C = H * d
    M = B * T
    rng = np.random.default_rng(11)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(rng.standard_normal((M, C)).astype(np.float32)).to(dev)
    w = torch.from_numpy((rng.standard_normal((3 * C, C)) / np.sqrt(C) / 8).astype(np.float32)).to(dev)
    b = torch.from_numpy((rng.standard_normal(3 * C) * 0.01).astype(np.float32)).to(dev)
    dout = torch.from_numpy(rng.standard_normal((B, T, C)).astype(np.float32)).to(dev)
    qkv = torch.empty(B, T, 3 * C, device=dev)
    o = torch.empty(B, T, C, device=dev)
    lse = torch.empty(B, H, T, device=dev)
    grads = torch.empty(B, T, 3 * C, device=dev)

    def views(t):
        return t[..., :C], t[..., C:2 * C], t[..., 2 * C:]

    with kerr_attn.Context(0) as ctx:
        ctx.set_deterministic(True)
        kerr_attn.linear_fwd(ctx, x, w, b, qkv.view(M, 3 * C))
        torch.cuda.synchronize()
        kerr_attn.fwd(ctx, *views(qkv), o, lse, H)
        torch.cuda.synchronize()
        kerr_attn.bwd(ctx, *views(qkv), o, dout, lse, *views(grads), H)
        torch.cuda.synchronize()
        ref = grads.clone()
        assert torch.isfinite(ref).all()
        for _ in range(20):
            grads.fill_(float("nan"))
            qkv.fill_(float("nan"))
            kerr_attn.linear_fwd(ctx, x, w, b, qkv.view(M, 3 * C))
            kerr_attn.bwd(ctx, *views(qkv), o, dout, lse, *views(grads), H)
            torch.cuda.synchronize()
            assert torch.equal(grads, ref)
        ctx.check_device()

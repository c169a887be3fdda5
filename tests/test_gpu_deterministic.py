"""The deterministic dQ mode (kattn_set_deterministic).

By default the backward adds each key tile's dQ contribution into dq with
floating-point reductions whose order depends on scheduling.  In the
deterministic mode every key tile stores its contribution into its own
slice of a workspace, and one more kernel adds the slices in key-tile order
(the reference's dQ is a sequential sum over keys, src/backward.rs:508-512).
Checked here, on both kernel families and with and without the causal mask:
repeated calls give bitwise-identical dq (and dk, dv); dq matches the oracle
(causal) at the parity tolerance and the reduction path closely; the
allocation-free entry point refuses the mode.  The mode's bitwise
reproducibility also checks that the tensor-core backward's two row-load
paths (rows on 32-byte boundaries or not) agree.
"""
import numpy as np
import pytest
import torch

import kerr_attn
from conftest import make_inputs
from test_gpu_parity import assert_parity, oracle_fwd_bwd

pytestmark = pytest.mark.gpu

PATHS = {"tensor": kerr_attn.PATH_TENSOR, "ffma": kerr_attn.PATH_FFMA}


def run(ctx, qkv, dout, H, causal):
    B, T, C3 = qkv.shape
    C = C3 // 3
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(qkv).to(dev)
    q, k, v = kerr_attn.split_qkv(x, C)
    o = torch.empty(B, T, C, device=dev)
    lse = torch.empty(B, H, T, device=dev)
    kerr_attn.fwd(ctx, q, k, v, o, lse, H, causal=causal)
    g = torch.from_numpy(dout).to(dev)
    dqkv = torch.full_like(x, float("nan"))
    dq, dk, dv = kerr_attn.split_qkv(dqkv, C)
    n = kerr_attn.bwd(ctx, q, k, v, o, g, lse, dq, dk, dv, H, causal=causal)
    torch.cuda.synchronize()
    ctx.check_device()
    return n, tuple(t.cpu().numpy() for t in (o, lse, dq, dk, dv))


# (B, T, H, d, path): the 768-dim headline's head shape on the tensor cores
# (ragged T: the last key tile partly past T), two key tiles and more, head_dim
# 32 on the tensor cores, and the FFMA kernels at head_dim 32 and 64.
CASES = [(2, 300, 2, 64, "tensor"), (1, 513, 3, 64, "tensor"), (2, 200, 2, 32, "tensor"), (2, 200, 2, 32, "ffma"),
         (1, 130, 2, 64, "ffma")]


@pytest.mark.parametrize("B,T,H,d,path", CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_deterministic_dq(oracle_lib, B, T, H, d, path, causal):
    qkv, dout = make_inputs(B, T, H, d, seed=91)
    with kerr_attn.Context(0) as ctx:
        ctx.set_path(PATHS[path])
        n_red, red = run(ctx, qkv, dout, H, causal)
        ctx.set_deterministic(True)
        n1, a = run(ctx, qkv, dout, H, causal)
        n2, b = run(ctx, qkv, dout, H, causal)
        ctx.set_deterministic(False)
    assert n1 == n2 == n_red + 1  # the ordered sum is one more kernel
    for x, y in zip(a, b):
        assert np.array_equal(x, y)  # bit for bit
    for i in (0, 1, 3, 4):  # o, lse, dk, dv do not depend on the mode
        assert np.array_equal(a[i], red[i])
    dq_a, dq_r = a[2], red[2]
    assert np.isfinite(dq_a).all()
    rel = np.linalg.norm(dq_a - dq_r) / np.linalg.norm(dq_r)
    assert rel < 1e-6, rel  # only the order of the f32 additions differs
    if causal:
        assert_parity(a, oracle_fwd_bwd(oracle_lib, qkv, dout, H), case=f"deterministic {path} d={d}")


def test_noalloc_refuses_deterministic_mode():
    B, T, H, d = 1, 64, 2, 64
    qkv, dout = make_inputs(B, T, H, d, seed=5)
    C = H * d
    dev = torch.device("cuda", 0)
    with kerr_attn.Context(0) as ctx:
        x = torch.from_numpy(qkv).to(dev)
        q, k, v = kerr_attn.split_qkv(x, C)
        o = torch.empty(B, T, C, device=dev)
        lse = torch.empty(B, H, T, device=dev)
        kerr_attn.fwd(ctx, q, k, v, o, lse, H)
        g = torch.from_numpy(dout).to(dev)
        dq, dk, dv = kerr_attn.split_qkv(torch.empty_like(x), C)
        ctx.set_deterministic(True)
        with pytest.raises(kerr_attn.KattnError) as e:
            kerr_attn.bwd_noalloc(ctx, q, k, v, o, g, lse, dq, dk, dv, H)
        assert e.value.status == kerr_attn.KATTN_ERR_UNSUPPORTED
        ctx.set_deterministic(False)
        kerr_attn.bwd_noalloc(ctx, q, k, v, o, g, lse, dq, dk, dv, H)
        torch.cuda.synchronize()


def test_set_deterministic_argument_checks():
    assert kerr_attn.lib().kattn_set_deterministic(None, 1) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("causal", [True, False])
def test_row_alignment_paths_agree(causal):
    """The tensor-core backward loads rows with 256-bit loads when q, k, v
    and dout rows all start on 32-byte boundaries, and with 128-bit loads
    otherwise.  The same inputs placed 16 bytes off a 32-byte boundary (one
    spare float before each buffer's first row) take the second path; in the
    deterministic mode both give bitwise-identical results."""
    B, T, H, d = 2, 200, 2, 64
    qkv, dout = make_inputs(B, T, H, d, seed=17)
    C = H * d
    dev = torch.device("cuda", 0)

    def place(a, shift):
        """a (contiguous [B, T, W]) as a view `shift` floats into a larger buffer."""
        flat = torch.empty(a.size + 8, device=dev)
        v = flat[shift:shift + a.size].view(a.shape)
        v.copy_(torch.from_numpy(a))
        return v

    def run_at(ctx, shift):
        x = place(qkv, shift)
        g = place(dout, shift)
        assert (x.data_ptr() % 32 == 0) == (shift == 0)
        q, k, v = kerr_attn.split_qkv(x, C)
        o = torch.empty(B, T, C, device=dev)
        lse = torch.empty(B, H, T, device=dev)
        kerr_attn.fwd(ctx, q, k, v, o, lse, H, causal=causal)
        dqkv = torch.full((B, T, 3 * C), float("nan"), device=dev)
        dq, dk, dv = kerr_attn.split_qkv(dqkv, C)
        kerr_attn.bwd(ctx, q, k, v, o, g, lse, dq, dk, dv, H, causal=causal)
        torch.cuda.synchronize()
        ctx.check_device()
        return dqkv.cpu()

    with kerr_attn.Context(0) as ctx:
        ctx.set_path(kerr_attn.PATH_TENSOR)
        ctx.set_deterministic(True)
        a = run_at(ctx, 0)
        b = run_at(ctx, 4)
    assert torch.isfinite(a).all()
    assert torch.equal(a, b)

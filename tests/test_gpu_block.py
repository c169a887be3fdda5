"""The device-resident block pipeline (kattn_block_*) against the oracle.

One block of the reference's batched pipeline as far as this library covers
it (src/pipeline.rs:236-360 forward, :670-750 backward):

    x1 = LN1(h); qkv = c_attn(x1); o = causal_attention(qkv); h1 = h + c_proj(o)
    h_out = h1 + KerrODE(LN2(h1))        (with the FFN; h_out = h1 without)

run as two C-ABI calls with every intermediate on the device, and on the
oracle's CPU restatements of each operation (the same composition as the
loss-curve harness, tests/train_stack.py).  Tolerances: h_out within 1e-4
and every gradient within 1e-3 norm-wise relative error (the attention
parity tolerances), on the tensor-core path (head_dim 64) and the FFMA path
(head_dim 32 at these sizes), with and without the FFN.
"""
import numpy as np
import pytest
import torch

import kerr_attn
import train_stack
from conftest import rel_err

pytestmark = pytest.mark.gpu

RK4 = 8


def oracle_block(p, h, dh_out, H, ffn):
    from oracle import oracle

    B, T, C = h.shape
    M = B * T
    hm = h.reshape(M, C)
    x1 = oracle.layernorm_forward(hm, p["ln1_w"], p["ln1_b"])
    qkv = oracle.linear_forward(x1, p["wa"], p["ba"]).reshape(B, T, 3 * C)
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, _ = oracle.forward(q, k, v, H)
    o = o.reshape(M, C)
    h1 = hm + oracle.linear_forward(o, p["wp"], p["bp"])
    g = {}
    dy = dh_out.reshape(M, C)
    if ffn:
        ab = p["alpha_beta"]
        x2 = oracle.layernorm_forward(h1, p["ln2_w"], p["ln2_b"])
        h_out = h1 + oracle.kerr_ode_forward(x2, p["gamma_raw"], p["omega"], ab[0], ab[1], RK4)
        dx2, g["gamma_raw"], g["omega"], da, db = oracle.kerr_ode_backward(dy, x2, p["gamma_raw"], p["omega"], ab[0],
                                                                           ab[1], RK4)
        g["alpha_beta"] = np.array([da, db], np.float32)
        dln2, g["ln2_w"], g["ln2_b"] = oracle.layernorm_backward(dx2, h1, p["ln2_w"])
        dh1 = dy + dln2
    else:
        h_out = h1
        dh1 = dy
    d_o = oracle.linear_backward_dx(dh1, p["wp"])
    g["w_proj"], g["b_proj"] = oracle.linear_backward_dw(dh1, o)
    dq, dk, dv = oracle.backward(d_o.reshape(B, T, C), q, k, v, att, H)
    dqkv = np.concatenate([dq, dk, dv], axis=-1).reshape(M, 3 * C)
    dx1 = oracle.linear_backward_dx(dqkv, p["wa"])
    g["w_attn"], g["b_attn"] = oracle.linear_backward_dw(dqkv, x1)
    dln1, g["ln1_w"], g["ln1_b"] = oracle.layernorm_backward(dx1, hm, p["ln1_w"])
    dh = dh1 + dln1
    return h_out.reshape(B, T, C), dh.reshape(B, T, C), g


NAMES = {"ln1_w": "ln1_w", "ln1_b": "ln1_b", "w_attn": "wa", "b_attn": "ba", "w_proj": "wp", "b_proj": "bp",
         "ln2_w": "ln2_w", "ln2_b": "ln2_b", "gamma_raw": "gamma_raw", "omega": "omega", "alpha_beta": "alpha_beta"}


# (B, T, C, H): head_dim 64 (tensor cores, ragged T) and head_dim 32 (FFMA at
# this size).
@pytest.mark.parametrize("B,T,C,H", [(2, 130, 128, 2), (2, 64, 128, 4)])
@pytest.mark.parametrize("ffn", [False, True])
def test_block_matches_oracle(oracle_lib, B, T, C, H, ffn):
    blocks, h0, _ = train_stack.init(B, T, C, H, 1, seed=7)
    p = blocks[0]
    rng = np.random.default_rng(8)
    dh_out = rng.standard_normal((B, T, C)).astype(np.float32)
    ref_out, ref_dh, ref_g = oracle_block(p, h0, dh_out, H, ffn)

    dev = torch.device("cuda", 0)
    P = {n: torch.from_numpy(p[k]).to(dev) for n, k in NAMES.items()}
    G = {n: torch.full_like(P[n], float("nan")) for n in NAMES}
    h = torch.from_numpy(h0).to(dev)
    h_out = torch.empty_like(h)
    dh = torch.from_numpy(dh_out).to(dev)  # the backward writes dh over dh_out (aliasing allowed)
    with kerr_attn.Context(0) as ctx, kerr_attn.Block(ctx, B, T, C, H, RK4 if ffn else 0) as blk:
        nf = blk.fwd(P, h, h_out)
        nb = blk.bwd(dh, dh, G)
        torch.cuda.synchronize()
        ctx.check_device()
    assert nf > 0 and nb > 0
    assert rel_err(h_out.cpu().numpy(), ref_out) < 1e-4
    assert rel_err(dh.cpu().numpy(), ref_dh) < 1e-3
    for n in (NAMES if ffn else list(NAMES)[:6]):
        got = G[n].cpu().numpy()
        assert np.isfinite(got).all(), n
        assert rel_err(got, ref_g[n] if n in ref_g else ref_g[NAMES[n]]) < 1e-3, n


def test_block_accumulates_and_reuses(oracle_lib):
    """Two forward/backward rounds on one block object with accumulate = 1
    give twice the gradients of one round (same inputs)."""
    B, T, C, H = 1, 96, 128, 2
    blocks, h0, _ = train_stack.init(B, T, C, H, 1, seed=3)
    dev = torch.device("cuda", 0)
    P = {n: torch.from_numpy(blocks[0][k]).to(dev) for n, k in NAMES.items()}
    G1 = {n: torch.zeros_like(P[n]) for n in NAMES}
    G2 = {n: torch.zeros_like(P[n]) for n in NAMES}
    h = torch.from_numpy(h0).to(dev)
    h_out = torch.empty_like(h)
    dy = torch.ones_like(h)
    with kerr_attn.Context(0) as ctx, kerr_attn.Block(ctx, B, T, C, H, RK4) as blk:
        dh = torch.empty_like(h)
        blk.fwd(P, h, h_out)
        blk.bwd(dy, dh, G1)
        for _ in range(2):
            blk.fwd(P, h, h_out)
            blk.bwd(dy, dh, G2, accumulate=True)
        torch.cuda.synchronize()
        ctx.check_device()
    for n in NAMES:
        a, b = G1[n].cpu().numpy(), G2[n].cpu().numpy()
        assert rel_err(b, 2 * a) < 1e-5, n


def test_block_argument_checks():
    lib = kerr_attn.lib()
    with kerr_attn.Context(0) as ctx:
        with pytest.raises(kerr_attn.KattnError):
            kerr_attn.Block(ctx, 1, 64, 100, 2)  # C not a multiple of 8
        with pytest.raises(kerr_attn.KattnError):
            kerr_attn.Block(ctx, 1, 64, 96, 2)  # head_dim 48
        with kerr_attn.Block(ctx, 1, 64, 128, 2) as blk:
            dev = torch.device("cuda", 0)
            x = torch.zeros(1, 64, 128, device=dev)
            with pytest.raises(kerr_attn.KattnError):  # no forward yet
                blk.bwd(x, x, {n: torch.zeros(4, device=dev) for n in NAMES})
    assert lib.kattn_block_destroy(None) == kerr_attn.KATTN_OK

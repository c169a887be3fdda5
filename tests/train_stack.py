"""A small training loop over the rebuilt path, written twice: once on the
oracle's CPU restatements (numpy) and once on this library's CUDA kernels
through the C ABI (torch tensors on the device).  Both run the same blocks
of the reference's per-block pipeline as far as this path covers it
(src/pipeline.rs:236-360 forward, :670-750 backward):

    x1 = LN1(h);  qkv = c_attn(x1);  o = causal_attention(qkv);  h1 = h + c_proj(o)
    x2 = LN2(h1); h2 = h1 + KerrODE(x2)

(the FFN's maestro and out_proj layers are dense layers outside this path and
are left out), with the mean squared error against a fixed target as the
loss and plain SGD as the update (the Kerr-ODE's alpha and beta, whose
gradients are orders of magnitude larger than the rest, take a 1/100 step).
The tests compare the two loss curves step by step.  Inputs stand in for the embeddings: seeded h0 ~ N(0,1);
weights follow the reference's initialisation (src/init.rs:9-16, :18-23,
:50-61): linear U(+-1/sqrt(fan_in)) with zero bias, LayerNorm 1 / 0,
KerrWeights gamma_raw = softplus^-1(0.1), omega_k = (k+1)/nb, alpha = beta =
0.1."""
import math

import numpy as np


def init(B, T, C, H, n_blocks, seed):
    rng = np.random.default_rng(seed)
    nb = C // 2

    def lin(n_out, n_in):
        lim = 1.0 / math.sqrt(n_in)
        return rng.uniform(-lim, lim, (n_out, n_in)).astype(np.float32), np.zeros(n_out, np.float32)

    blocks = []
    for _ in range(n_blocks):
        wa, ba = lin(3 * C, C)
        wp, bp = lin(C, C)
        blocks.append({
            "ln1_w": np.ones(C, np.float32), "ln1_b": np.zeros(C, np.float32),
            "wa": wa, "ba": ba, "wp": wp, "bp": bp,
            "ln2_w": np.ones(C, np.float32), "ln2_b": np.zeros(C, np.float32),
            "gamma_raw": np.full(nb, np.log(np.expm1(0.1)), np.float32),
            "omega": ((np.arange(nb) + 1) / nb).astype(np.float32),
            "alpha_beta": np.array([0.1, 0.1], np.float32),
        })
    h0 = rng.standard_normal((B, T, C)).astype(np.float32)
    target = rng.standard_normal((B, T, C)).astype(np.float32)
    return blocks, h0, target


# Step size of each parameter relative to the learning rate.
LR_SCALE = {"alpha_beta": 0.01}


def train_oracle(blocks, h0, target, H, n_steps, lr, rk4_steps=8):
    """Loss per step on the oracle (CPU, f32)."""
    from oracle import oracle

    blocks = [{k: v.copy() for k, v in b.items()} for b in blocks]
    B, T, C = h0.shape
    M = B * T
    losses = []
    for _ in range(n_steps):
        h = h0.reshape(M, C)
        caches = []
        for p in blocks:
            x1 = oracle.layernorm_forward(h, p["ln1_w"], p["ln1_b"])
            qkv = oracle.linear_forward(x1, p["wa"], p["ba"]).reshape(B, T, 3 * C)
            q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
            o, att, _ = oracle.forward(q, k, v, H)
            o = o.reshape(M, C)
            h1 = h + oracle.linear_forward(o, p["wp"], p["bp"])
            x2 = oracle.layernorm_forward(h1, p["ln2_w"], p["ln2_b"])
            ab = p["alpha_beta"]
            h2 = h1 + oracle.kerr_ode_forward(x2, p["gamma_raw"], p["omega"], ab[0], ab[1], rk4_steps)
            caches.append((h, x1, qkv, att, o, h1, x2))
            h = h2
        diff = h - target.reshape(M, C)
        losses.append(float(np.mean(np.float64(diff) ** 2) / 2))
        dh = (diff / diff.size).astype(np.float32)
        grads = []
        for p, (hin, x1, qkv, att, o, h1, x2) in zip(reversed(blocks), reversed(caches)):
            g = {}
            ab = p["alpha_beta"]
            dx2, g["gamma_raw"], g["omega"], da, db = oracle.kerr_ode_backward(
                dh, x2, p["gamma_raw"], p["omega"], ab[0], ab[1], rk4_steps)
            g["alpha_beta"] = np.array([da, db], np.float32)
            dln2, g["ln2_w"], g["ln2_b"] = oracle.layernorm_backward(dx2, h1, p["ln2_w"])
            dh1 = dh + dln2
            d_o = oracle.linear_backward_dx(dh1, p["wp"])
            g["wp"], g["bp"] = oracle.linear_backward_dw(dh1, o)
            q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
            dq, dk, dv = oracle.backward(d_o.reshape(B, T, C), q, k, v, att, H)
            dqkv = np.concatenate([dq, dk, dv], axis=-1).reshape(M, 3 * C)
            dx1 = oracle.linear_backward_dx(dqkv, p["wa"])
            g["wa"], g["ba"] = oracle.linear_backward_dw(dqkv, x1)
            dln1, g["ln1_w"], g["ln1_b"] = oracle.layernorm_backward(dx1, hin, p["ln1_w"])
            dh = dh1 + dln1
            grads.append(g)
        for p, g in zip(reversed(blocks), grads):
            for k in g:
                p[k] = (p[k] - np.float32(lr * LR_SCALE.get(k, 1.0)) * g[k]).astype(np.float32)
    return losses


def train_gpu(blocks, h0, target, H, n_steps, lr, rk4_steps=8, device=0):
    """Loss per step on this library's kernels (every LayerNorm, linear,
    attention and Kerr-ODE call goes through the C ABI; residual adds, the
    loss and the SGD update are torch elementwise ops)."""
    import torch

    import kerr_attn

    dev = torch.device("cuda", device)
    B, T, C = h0.shape
    M = B * T
    nb = C // 2
    P = [{k: torch.from_numpy(v.copy()).to(dev) for k, v in b.items()} for b in blocks]
    h0d = torch.from_numpy(h0).to(dev).reshape(M, C)
    tgt = torch.from_numpy(target).to(dev).reshape(M, C)
    ctx = kerr_attn.Context(device)
    e = lambda *s: torch.empty(*s, device=dev)  # noqa: E731
    losses = []
    try:
        for _ in range(n_steps):
            h = h0d
            caches = []
            for p in P:
                x1 = e(M, C)
                kerr_attn.layernorm_fwd(ctx, h, p["ln1_w"], p["ln1_b"], x1)
                qkv = e(B, T, 3 * C)
                kerr_attn.linear_fwd(ctx, x1, p["wa"], p["ba"], qkv.view(M, 3 * C))
                q, k, v = kerr_attn.split_qkv(qkv, C)
                o, lse = e(B, T, C), e(B, H, T)
                kerr_attn.fwd(ctx, q, k, v, o, lse, H)
                a = e(M, C)
                kerr_attn.linear_fwd(ctx, o.view(M, C), p["wp"], p["bp"], a)
                h1 = h + a
                x2, f = e(M, C), e(M, C)
                kerr_attn.layernorm_fwd(ctx, h1, p["ln2_w"], p["ln2_b"], x2)
                kerr_attn.kerr_ode_fwd(ctx, x2, p["gamma_raw"], p["omega"], p["alpha_beta"], f, rk4_steps)
                caches.append((h, x1, qkv, o, lse, h1, x2))
                h = h1 + f
            diff = h - tgt
            losses.append(float((diff.double() ** 2).mean().item() / 2))
            dh = diff / diff.numel()
            grads = []
            for p, (hin, x1, qkv, o, lse, h1, x2) in zip(reversed(P), reversed(caches)):
                g = {k: torch.empty_like(v) for k, v in p.items()}
                dx2 = e(M, C)
                kerr_attn.kerr_ode_bwd(ctx, dh, x2, p["gamma_raw"], p["omega"], p["alpha_beta"], dx2,
                                       g["gamma_raw"], g["omega"], g["alpha_beta"], rk4_steps, accumulate=False)
                dln2 = e(M, C)
                kerr_attn.layernorm_bwd(ctx, dx2, h1, p["ln2_w"], dln2, g["ln2_w"], g["ln2_b"], accumulate=False)
                dh1 = dh + dln2
                d_o = e(B, T, C)
                kerr_attn.linear_bwd_dx(ctx, dh1, p["wp"], d_o.view(M, C))
                kerr_attn.linear_bwd_dw(ctx, dh1, o.view(M, C), g["wp"], g["bp"], accumulate=False)
                q, k, v = kerr_attn.split_qkv(qkv, C)
                dqkv = e(B, T, 3 * C)
                dq, dk, dv = kerr_attn.split_qkv(dqkv, C)
                kerr_attn.bwd(ctx, q, k, v, o, d_o, lse, dq, dk, dv, H)
                dx1 = e(M, C)
                kerr_attn.linear_bwd_dx(ctx, dqkv.view(M, 3 * C), p["wa"], dx1)
                kerr_attn.linear_bwd_dw(ctx, dqkv.view(M, 3 * C), x1, g["wa"], g["ba"], accumulate=False)
                dln1 = e(M, C)
                kerr_attn.layernorm_bwd(ctx, dx1, hin, p["ln1_w"], dln1, g["ln1_w"], g["ln1_b"], accumulate=False)
                dh = dh1 + dln1
                grads.append(g)
            for p, g in zip(reversed(P), grads):
                for k in g:
                    p[k] -= float(np.float32(lr * LR_SCALE.get(k, 1.0))) * g[k]
        torch.cuda.synchronize(dev)
        ctx.check_device()
    finally:
        ctx.close()
    assert nb == P[0]["omega"].numel()
    return losses


def train_gpu_native(blocks, h0, target, H, n_steps, lr, rk4_steps=8, device=0):
    """train_gpu on the device-resident block pipeline: each block's forward
    and backward are one kattn_block_fwd / kattn_block_bwd call (every
    intermediate stays in the library's block object); the loss and the SGD
    update are torch elementwise ops."""
    import torch

    import kerr_attn

    dev = torch.device("cuda", device)
    B, T, C = h0.shape
    names = {"ln1_w": "ln1_w", "ln1_b": "ln1_b", "w_attn": "wa", "b_attn": "ba", "w_proj": "wp", "b_proj": "bp",
             "ln2_w": "ln2_w", "ln2_b": "ln2_b", "gamma_raw": "gamma_raw", "omega": "omega",
             "alpha_beta": "alpha_beta"}
    P = [{n: torch.from_numpy(b[k].copy()).to(dev) for n, k in names.items()} for b in blocks]
    G = [{n: torch.empty_like(v) for n, v in p.items()} for p in P]
    tgt = torch.from_numpy(target).to(dev)
    hs = [torch.from_numpy(h0).to(dev)] + [torch.empty(B, T, C, device=dev) for _ in blocks]
    dh = torch.empty(B, T, C, device=dev)
    ctx = kerr_attn.Context(device)
    objs = [kerr_attn.Block(ctx, B, T, C, H, rk4_steps) for _ in blocks]
    losses = []
    try:
        for _ in range(n_steps):
            for i, o in enumerate(objs):
                o.fwd(P[i], hs[i], hs[i + 1])
            diff = hs[-1] - tgt
            losses.append(float((diff.double() ** 2).mean().item() / 2))
            dh.copy_(diff / diff.numel())
            for i in reversed(range(len(objs))):
                objs[i].bwd(dh, dh, G[i])
            for p, g in zip(P, G):
                for n in g:
                    p[n] -= float(np.float32(lr * LR_SCALE.get(names[n], 1.0))) * g[n]
        torch.cuda.synchronize(dev)
        ctx.check_device()
    finally:
        for o in objs:
            o.close()
        ctx.close()
    return losses

"""CPU checks of the oracle (the C restatement of the reference's attention).

The reference ships no attention golden vectors (parity unpinned), so the
oracle is checked (1) against an independent float64 autograd computation of
causal softmax attention, (2) against algebraic known answers of the
reference's formulas, and (3) against the committed fixtures it generated
(tests/golden/make_golden.py), which pins it against accidental change.
"""
import os

import numpy as np
import pytest
import torch

from conftest import make_inputs, rel_err

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def torch_reference(q, k, v, dout, H, causal=True):
    """float64 autograd reference (independent of the oracle's loop order)."""
    B, T, C = q.shape
    d = C // H
    Q, K, V = (torch.tensor(np.ascontiguousarray(x), dtype=torch.float64, requires_grad=True) for x in (q, k, v))

    def heads(x):
        return x.view(B, T, H, d).transpose(1, 2)

    s = heads(Q) @ heads(K).transpose(-1, -2) / np.sqrt(d)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    lse = torch.logsumexp(s, -1)
    O = (s.softmax(-1) @ heads(V)).transpose(1, 2).reshape(B, T, C)
    O.backward(torch.tensor(dout, dtype=torch.float64))
    return O.detach().numpy(), lse.detach().numpy(), Q.grad.numpy(), K.grad.numpy(), V.grad.numpy()


@pytest.mark.parametrize("B,T,H,d", [(1, 1, 1, 8), (2, 2, 2, 8), (1, 63, 4, 32), (2, 65, 2, 32),
                                     (1, 130, 3, 64), (4, 64, 4, 32)])
def test_oracle_matches_float64_autograd(oracle_lib, B, T, H, d):
    qkv, dout = make_inputs(B, T, H, d, seed=T * 7 + d)
    C = H * d
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, lse = oracle_lib.forward(q, k, v, H)
    dq, dk, dv = oracle_lib.backward(dout, q, k, v, att, H)
    ro, rlse, rdq, rdk, rdv = torch_reference(q, k, v, dout, H)
    assert rel_err(o, ro) < 1e-5
    assert rel_err(lse, rlse) < 1e-5
    for g, r in ((dq, rdq), (dk, rdk), (dv, rdv)):
        assert rel_err(g, r) < 1e-4


def test_single_position_known_answer(oracle_lib):
    # T = 1: the only weight is 1, so o = v, dv = dout, dq = dk = 0
    # (src/pipeline.rs:326-345, src/backward.rs:488-515 with pos = 0).
    qkv, dout = make_inputs(3, 1, 4, 32, seed=1)
    C = 128
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, _ = oracle_lib.forward(q, k, v, 4)
    assert np.array_equal(o, np.ascontiguousarray(v))
    assert np.all(att == 1.0)
    dq, dk, dv = oracle_lib.backward(dout, q, k, v, att, 4)
    assert np.array_equal(dv, dout)
    assert np.all(dq == 0) and np.all(dk == 0)


def test_equal_keys_give_running_mean(oracle_lib):
    # All keys equal: every causal row is uniform, o[t] = mean(v[0..t]).
    B, T, H, d = 1, 40, 2, 32
    C = H * d
    qkv, _ = make_inputs(B, T, H, d, seed=3)
    qkv[..., C:2 * C] = qkv[:, :1, C:2 * C]
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, _ = oracle_lib.forward(q, k, v, H)
    mean = np.cumsum(v.astype(np.float64), axis=1) / np.arange(1, T + 1)[None, :, None]
    assert rel_err(o, mean) < 1e-6
    for t in range(T):
        assert np.allclose(att[0, :, t, : t + 1], 1.0 / (t + 1), rtol=1e-6)


def test_att_cache_layout(oracle_lib):
    # AttnCache.att_weights rows sum to one on ki <= qi and stay -inf above the
    # diagonal, as the reference copies its -inf-initialised scratch row.
    qkv, _ = make_inputs(2, 17, 3, 8, seed=5)
    C = 24
    _, att, _ = oracle_lib.forward(qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:], 3)
    T = 17
    upper = np.triu(np.ones((T, T), bool), 1)
    assert np.all(np.isneginf(att[..., upper]))
    lower = np.where(upper, 0.0, att)
    assert np.allclose(lower.sum(-1), 1.0, atol=1e-6)


def test_strided_qkv_equals_packed(oracle_lib):
    qkv, dout = make_inputs(2, 33, 2, 32, seed=9)
    C = 64
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o1, a1, l1 = oracle_lib.forward(q, k, v, 2)
    qc, kc, vc = (np.ascontiguousarray(x) for x in (q, k, v))
    o2, a2, l2 = oracle_lib.forward(qc, kc, vc, 2)
    assert np.array_equal(o1, o2) and np.array_equal(a1, a2) and np.array_equal(l1, l2)
    g1 = oracle_lib.backward(dout, q, k, v, a1, 2)
    g2 = oracle_lib.backward(dout, qc, kc, vc, a2, 2)
    for x, y in zip(g1, g2):
        assert np.array_equal(x, y)


def test_thread_count_does_not_change_results(oracle_lib):
    qkv, dout = make_inputs(5, 20, 2, 16, seed=11)
    C = 32
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    r1 = oracle_lib.forward(q, k, v, 2, threads=1)
    r4 = oracle_lib.forward(q, k, v, 2, threads=4)
    for x, y in zip(r1, r4):
        assert np.array_equal(x, y)
    g1 = oracle_lib.backward(dout, q, k, v, r1[1], 2, threads=1)
    g3 = oracle_lib.backward(dout, q, k, v, r1[1], 2, threads=3)
    for x, y in zip(g1, g3):
        assert np.array_equal(x, y)


def golden_cases():
    return sorted(f for f in os.listdir(GOLDEN) if f.endswith(".npz"))


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_reproduces_golden(oracle_lib, name):
    z = np.load(os.path.join(GOLDEN, name))
    H = int(z["n_head"])
    C = z["qkv"].shape[-1] // 3
    qkv = z["qkv"]
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, lse = oracle_lib.forward(q, k, v, H)
    assert np.array_equal(o, z["o"])
    assert np.array_equal(lse, z["lse"])
    dq, dk, dv = oracle_lib.backward(z["dout"], q, k, v, att, H)
    assert np.array_equal(dq, z["dq"]) and np.array_equal(dk, z["dk"]) and np.array_equal(dv, z["dv"])


@pytest.mark.parametrize("M,N,K", [(1, 4, 4), (37, 29, 41), (64, 384, 128)])
def test_linear_oracle_against_float64(M, N, K):
    # The projection layers' restatement (oracle/kproj_oracle.c) against float64.
    from oracle import oracle

    rng = np.random.default_rng(M * 31 + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    x64, w64, dy64 = x.astype(np.float64), w.astype(np.float64), dy.astype(np.float64)
    y = oracle.linear_forward(x, w, b)
    assert np.abs(y - (x64 @ w64.T + b)).max() < 1e-5 * max(1.0, np.abs(y).max())
    dx = oracle.linear_backward_dx(dy, w)
    assert np.abs(dx - dy64 @ w64).max() < 1e-5 * max(1.0, np.abs(dx).max())
    dw, db = oracle.linear_backward_dw(dy, x)
    assert np.abs(dw - dy64.T @ x64).max() < 1e-5 * max(1.0, np.abs(dw).max()) * np.sqrt(M)
    assert np.abs(db - dy64.sum(0)).max() < 1e-5 * max(1.0, np.abs(db).max()) * np.sqrt(M)


def test_layernorm_oracle_against_float64():
    # The LayerNorm restatement (src/backend.rs:258-267, src/backward.rs:93-128)
    # against a float64 evaluation of the same formulas, rows of 768 and 100.
    from oracle import oracle

    rng = np.random.default_rng(5)
    for M, N in ((37, 768), (9, 100)):
        x = (rng.standard_normal((M, N)) * 2 + 0.5).astype(np.float32)
        w = rng.standard_normal(N).astype(np.float32)
        b = rng.standard_normal(N).astype(np.float32)
        dy = rng.standard_normal((M, N)).astype(np.float32)
        xd = x.astype(np.float64)
        mean = xd.mean(1, keepdims=True)
        rstd = 1.0 / np.sqrt(((xd - mean) ** 2).mean(1, keepdims=True) + 1e-5)
        xh = (xd - mean) * rstd
        y = oracle.layernorm_forward(x, w, b)
        assert rel_err(y, xh * w + b) < 1e-6
        g = dy * w
        dx_ref = rstd / N * (N * g - g.sum(1, keepdims=True) - xh * (g * xh).sum(1, keepdims=True))
        dw0 = rng.standard_normal(N).astype(np.float32)
        dx, dw, db = oracle.layernorm_backward(dy, x, w, dw=dw0, db=dw0)
        assert rel_err(dx, dx_ref) < 1e-6
        assert rel_err(dw, dw0 + (dy * xh).sum(0)) < 1e-5
        assert rel_err(db, dw0 + dy.sum(0)) < 1e-5


# ---------------------------------------------------------------- Kerr-ODE

@pytest.mark.parametrize("M,nb,n_steps,seed", [(6, 64, 8, 1), (3, 384, 8, 2), (2, 20, 16, 3), (4, 4, 1, 4)])
def test_kerr_ode_oracle_against_float64_autograd(oracle_lib, M, nb, n_steps, seed):
    # The restatement of kerr_ode_cpu / kerr_ode_backward_batch against an
    # independent float64 autograd of the same ODE (the reference's own
    # check of its Kerr backward, src/grad_test.rs:50-174).
    import kerr_ode_f64

    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, 2 * nb)).astype(np.float32)
    dy = rng.standard_normal((M, 2 * nb)).astype(np.float32)
    gr, om, al, be = kerr_ode_f64.init_params(nb, seed=seed)
    y = oracle_lib.kerr_ode_forward(x, gr, om, al, be, n_steps)
    dx, dgr, dom, da, db = oracle_lib.kerr_ode_backward(dy, x, gr, om, al, be, n_steps)
    ry, rdx, rdgr, rdom, rda, rdb = kerr_ode_f64.forward_backward(x, dy, gr, om, al, be, n_steps)
    assert rel_err(y, ry) < 1e-6
    assert rel_err(dx, rdx) < 1e-5
    assert rel_err(dgr, rdgr) < 1e-5
    assert rel_err(dom, rdom) < 1e-5
    assert abs(da - rda) <= 1e-5 * max(abs(rda), 1e-30) + 1e-6
    assert abs(db - rdb) <= 1e-5 * max(abs(rdb), 1e-30) + 1e-6


def test_kerr_ode_oracle_known_answers(oracle_lib):
    # Algebraic known answers of the reference's ODE (src/model.rs:778-843):
    # a zero state stays zero; with alpha = beta = 0 every band is the linear
    # rotation-with-decay (r + i s)' = (-gamma + i omega)(r + i s), whose RK4
    # step multiplies by the degree-4 Taylor polynomial of exp(z dt).
    nb, n_steps = 16, 8
    gr = np.linspace(-2, 1, nb).astype(np.float32)
    om = np.linspace(0.1, 2, nb).astype(np.float32)
    zero = np.zeros((2, 2 * nb), np.float32)
    assert not oracle_lib.kerr_ode_forward(zero, gr, om, 0.1, 0.1, n_steps).any()
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 2 * nb)).astype(np.float32)
    y = oracle_lib.kerr_ode_forward(x, gr, om, 0.0, 0.0, n_steps)
    gamma = np.log1p(np.exp(gr.astype(np.float64)))
    z = (-gamma + 1j * om.astype(np.float64)) / n_steps
    g = (1 + z + z ** 2 / 2 + z ** 3 / 6 + z ** 4 / 24) ** n_steps
    c = (x[:, 0::2] + 1j * x[:, 1::2]) * g
    want = np.stack([c.real, c.imag], axis=2).reshape(x.shape)
    assert rel_err(y, want) < 1e-6


def test_kerr_ode_oracle_threads_keep_forward_bits(oracle_lib):
    import kerr_ode_f64

    rng = np.random.default_rng(8)
    x = rng.standard_normal((9, 128)).astype(np.float32)
    gr, om, al, be = kerr_ode_f64.init_params(64)
    a = oracle_lib.kerr_ode_forward(x, gr, om, al, be, 8, threads=1)
    b = oracle_lib.kerr_ode_forward(x, gr, om, al, be, 8, threads=4)
    assert np.array_equal(a, b)


def test_training_loop_on_the_oracle_descends(oracle_lib):
    # The CPU half of the loss-curve comparison (tests/test_gpu_train.py):
    # the oracle's layers compose into a trainable stack whose loss falls.
    import train_stack

    blocks, h0, target = train_stack.init(2, 32, 64, 2, 2, seed=3)
    losses = train_stack.train_oracle(blocks, h0, target, 2, 8, 0.03)
    assert all(np.isfinite(losses))
    assert all(b < a for a, b in zip(losses, losses[1:]))


def test_model128_harness_on_the_oracle(oracle_lib):
    # The oracle arm of the 128-dim model's training run (tests/model128.py):
    # the reference's initialisation draws every weight inside its limit, the
    # first loss is near ln 65 (uniform over the symbols) and a few Adam
    # steps lower it.
    import math

    import model128

    blocks, top = model128.init_model(42)
    lim = 1 / math.sqrt(model128.N_EMBD)
    assert np.abs(blocks[0]["wa"]).max() <= lim and np.abs(top["lm_head"]).max() <= lim
    assert np.abs(blocks[0]["band_w"]).max() <= 1 / math.sqrt(2) and "band_w" not in blocks[1]
    assert model128.active_bands(0) == 8 and model128.active_bands(998) == 8 and model128.active_bands(999) == 24
    losses = model128.train_oracle(4)
    assert abs(losses[0] - math.log(model128.VOCAB)) < 0.5
    assert losses[-1] < losses[0]

"""GPU parity: the sm_100a kernels (through the C ABI) against the oracle.

Tolerances (f32): forward output and lse within 1e-4, gradients
within 1e-3, both as norm-wise relative error max|x - ref| / max|ref|.
Small and ragged shapes run against the oracle; the full 768-dim and micro-
benchmark batches run against the oracle too (seconds on the host threads);
size-independent identities of softmax attention are checked at full size.
"""
import os

import numpy as np
import pytest
import torch

import kerr_attn
from conftest import elem_rel_err, make_inputs, record_errors, rel_err

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
FWD_TOL = 1e-4
GRAD_TOL = 1e-3


@pytest.fixture(scope="module")
def module_ctx():
    c = kerr_attn.Context(0)
    yield c
    c.close()


@pytest.fixture
def ctx(module_ctx):
    module_ctx.set_path(kerr_attn.PATH_AUTO)
    yield module_ctx
    module_ctx.check_device()


PATHS = {"ffma": kerr_attn.PATH_FFMA, "tensor": kerr_attn.PATH_TENSOR}


def gpu_fwd_bwd(ctx, qkv, dout, H, causal=True, stream=None, path="auto"):
    B, T, C3 = qkv.shape
    C = C3 // 3
    if path == "tensor" and C // H not in (32, 64):
        pytest.skip("the tensor-core path covers head_dim 32 (forward) and 64")
    ctx.set_path(PATHS.get(path, kerr_attn.PATH_AUTO))
    dev = torch.device("cuda", 0)
    qkv_d = torch.from_numpy(qkv).to(dev)
    q, k, v = kerr_attn.split_qkv(qkv_d, C)
    o = torch.empty(B, T, C, device=dev)
    lse = torch.empty(B, H, T, device=dev)
    n_f = kerr_attn.fwd(ctx, q, k, v, o, lse, H, causal=causal, stream=stream)
    dout_d = torch.from_numpy(dout).to(dev)
    dqkv = torch.full_like(qkv_d, float("nan"))
    dq, dk, dv = kerr_attn.split_qkv(dqkv, C)
    n_b = kerr_attn.bwd(ctx, q, k, v, o, dout_d, lse, dq, dk, dv, H, causal=causal, stream=stream)
    torch.cuda.synchronize()
    ctx.check_device()
    assert n_f == 1 and n_b == 2
    return (o.cpu().numpy(), lse.cpu().numpy(), dq.cpu().numpy(), dk.cpu().numpy(), dv.cpu().numpy())


def oracle_fwd_bwd(oracle_lib, qkv, dout, H):
    C = qkv.shape[-1] // 3
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, lse = oracle_lib.forward(q, k, v, H)
    dq, dk, dv = oracle_lib.backward(dout, q, k, v, att, H)
    return o, lse, dq, dk, dv


def assert_parity(got, ref, case=""):
    """Norm-wise relative error (the tolerance measure) of each output, with
    the elementwise relative error (absolute floor 1e-3 of the largest
    element) reported beside it and recorded."""
    names = ("o", "lse", "dq", "dk", "dv")
    errs = {n: rel_err(g, r) for n, g, r in zip(names, got, ref)}
    elem = {f"elem_{n}": elem_rel_err(g, r) for n, g, r in zip(names, got, ref)}
    record_errors(case, {**errs, **elem})
    for n in names:
        assert np.all(np.isfinite(got[names.index(n)])), n
    assert errs["o"] < FWD_TOL and errs["lse"] < FWD_TOL, (errs, elem)
    assert errs["dq"] < GRAD_TOL and errs["dk"] < GRAD_TOL and errs["dv"] < GRAD_TOL, (errs, elem)
    return errs


SHAPES = [
    (4, 64, 4, 32),     # the 128-dim model's attention (C=128, 4 heads, seq 64, batch 4)
    (1, 1, 1, 32),      # single position
    (2, 2, 2, 64),
    (1, 63, 4, 32),     # ragged: one short tile
    (2, 65, 2, 64),     # ragged: one row into the second tile
    (1, 127, 3, 128),
    (3, 130, 2, 32),
    (2, 256, 4, 32),    # micro-benchmark shape, 2 sequences
    (2, 256, 12, 64),   # 768-dim model shape, 2 sequences
    (1, 300, 2, 64),
    (1, 1024, 2, 64),   # long-context shape
]


@pytest.mark.parametrize("path", ["ffma", "tensor"])
@pytest.mark.parametrize("B,T,H,d", SHAPES)
def test_parity_with_oracle(ctx, oracle_lib, B, T, H, d, path):
    qkv, dout = make_inputs(B, T, H, d, seed=B * 1000 + T + d)
    assert_parity(gpu_fwd_bwd(ctx, qkv, dout, H, path=path), oracle_fwd_bwd(oracle_lib, qkv, dout, H),
                  case=f"shape B={B} T={T} H={H} d={d} {path}")


@pytest.mark.parametrize("path", ["ffma", "tensor"])
@pytest.mark.parametrize("name", sorted(f for f in os.listdir(GOLDEN) if f.endswith(".npz")))
def test_parity_with_golden(ctx, name, path):
    z = np.load(os.path.join(GOLDEN, name))
    got = gpu_fwd_bwd(ctx, z["qkv"], z["dout"], int(z["n_head"]), path=path)
    assert_parity(got, (z["o"], z["lse"], z["dq"], z["dk"], z["dv"]), case=f"golden {name} {path}")


@pytest.mark.parametrize("path", ["ffma", "tensor"])
@pytest.mark.parametrize("B,T,H,d,sigma", [(64, 256, 4, 32, None), (16, 256, 12, 64, None),
                                           (16, 256, 12, 64, 1.0)])
def test_full_size_against_oracle(ctx, oracle_lib, B, T, H, d, sigma, path):
    # The attention micro-benchmark (B=64, H=4, T=256, d=32) and the 768-dim
    # model's per-layer batch (B=16, H=12, T=256, d=64) at full size; sigma=1
    # gives sharper softmax rows than the 1/sqrt(d) default.
    qkv, dout = make_inputs(B, T, H, d, seed=2024, qkv_sigma=sigma)
    assert_parity(gpu_fwd_bwd(ctx, qkv, dout, H, path=path), oracle_fwd_bwd(oracle_lib, qkv, dout, H),
                  case=f"full B={B} T={T} H={H} d={d} sigma={sigma} {path}")


def torch_f64(qkv, dout, H, causal):
    B, T, C3 = qkv.shape
    C = C3 // 3
    d = C // H
    x = torch.tensor(qkv, dtype=torch.float64, device="cuda", requires_grad=True)

    def heads(t):
        return t.reshape(B, T, H, d).transpose(1, 2)

    q, k, v = heads(x[..., :C]), heads(x[..., C:2 * C]), heads(x[..., 2 * C:])
    s = q @ k.transpose(-1, -2) / np.sqrt(d)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    o = (s.softmax(-1) @ v).transpose(1, 2).reshape(B, T, C)
    o.backward(torch.tensor(dout, dtype=torch.float64, device="cuda"))
    g = x.grad
    return (o.detach().cpu().numpy(), torch.logsumexp(s, -1).detach().cpu().numpy(),
            g[..., :C].cpu().numpy(), g[..., C:2 * C].cpu().numpy(), g[..., 2 * C:].cpu().numpy())


@pytest.mark.parametrize("path", ["ffma", "tensor"])
@pytest.mark.parametrize("B,T,H,d", [(2, 64, 2, 32), (1, 100, 2, 64), (2, 200, 1, 128), (1, 300, 3, 64)])
def test_non_causal_against_float64(ctx, B, T, H, d, path):
    qkv, dout = make_inputs(B, T, H, d, seed=77 + T)
    assert_parity(gpu_fwd_bwd(ctx, qkv, dout, H, causal=False, path=path), torch_f64(qkv, dout, H, causal=False))


@pytest.mark.parametrize("path", ["ffma", "tensor"])
def test_long_context_against_float64(ctx, path):
    # Long-context sweep shape (H=12, d=64) at T=2048 for one sequence,
    # q, k, v ~ N(0, 1)/8.
    qkv, dout = make_inputs(1, 2048, 12, 64, seed=5, qkv_sigma=1.0 / 8)
    assert_parity(gpu_fwd_bwd(ctx, qkv, dout, 12, path=path), torch_f64(qkv, dout, 12, causal=True))


@pytest.mark.parametrize("path", ["ffma", "tensor"])
def test_full_size_identities(ctx, path):
    # Size-independent identities of causal softmax attention at the 768-dim
    # layer size: sum_t dV[t] = sum_t dO[t] and sum_t dK[t] = 0 per (b, h)
    # (softmax rows sum to one); constant values give o = v; adding one vector
    # to every key leaves the output unchanged (row-constant score shift).
    B, T, H, d = 16, 256, 12, 64
    C = H * d
    qkv, dout = make_inputs(B, T, H, d, seed=99)
    o, lse, dq, dk, dv = gpu_fwd_bwd(ctx, qkv, dout, H, path=path)
    sdv = dv.astype(np.float64).reshape(B, T, H, d).sum(1)
    sdo = dout.astype(np.float64).reshape(B, T, H, d).sum(1)
    assert rel_err(sdv, sdo) < 1e-4
    sdk = np.abs(dk.astype(np.float64).reshape(B, T, H, d).sum(1)).max()
    assert sdk < 1e-3 * np.abs(dk).max() * np.sqrt(T)

    const = qkv.copy()
    const[..., 2 * C:] = qkv[:, :1, 2 * C:]
    o_c = gpu_fwd_bwd(ctx, const, dout, H, path=path)[0]
    assert rel_err(o_c, np.broadcast_to(qkv[:, :1, 2 * C:], o_c.shape)) < 1e-5

    shifted = qkv.copy()
    rng = np.random.default_rng(3)
    shifted[..., C:2 * C] += (rng.standard_normal((1, 1, C)) * 0.1).astype(np.float32)
    o_s = gpu_fwd_bwd(ctx, shifted, dout, H, path=path)[0]
    assert rel_err(o_s, o) < 1e-4


def test_host_entry_points_match_device(ctx, oracle_lib):
    # kattn_fwd_host / kattn_bwd_host: host buffers in and out, as the
    # reference's trait call is made (src/pipeline.rs:707-714).
    B, T, H, d = 3, 96, 4, 32
    C = H * d
    qkv, dout = make_inputs(B, T, H, d, seed=123)
    qkv_t = torch.from_numpy(qkv).pin_memory()
    q, k, v = kerr_attn.split_qkv(qkv_t, C)
    o = torch.empty(B, T, C).pin_memory()
    lse = torch.empty(B, H, T).pin_memory()
    kerr_attn.fwd_host(ctx, q, k, v, o, lse, H)
    dqkv = torch.empty(B, T, 3 * C)  # pageable output is accepted too
    dq, dk, dv = kerr_attn.split_qkv(dqkv, C)
    kerr_attn.bwd_host(ctx, q, k, v, o, torch.from_numpy(dout), lse, dq, dk, dv, H)
    got = (o.numpy(), lse.numpy(), dq.numpy(), dk.numpy(), dv.numpy())
    assert_parity(got, oracle_fwd_bwd(oracle_lib, qkv, dout, H))
    # Separate (non-fused) host q/k/v arrays take the strided-copy path.
    qs, ks, vs = (x.contiguous() for x in (q, k, v))
    o2 = torch.empty(B, T, C)
    lse2 = torch.empty(B, H, T)
    kerr_attn.fwd_host(ctx, qs, ks, vs, o2, lse2, H)
    assert torch.equal(o2, o) and torch.equal(lse2, lse)


def _host_fwd_bwd(ctx, qkv, dout, H, saved=None, split_grads=False):
    """Forward + backward through the host-buffer calls (fwd_host / bwd_host,
    or fwd_host_save / bwd_host_saved when `saved` is given)."""
    B, T, C3 = qkv.shape
    C = C3 // 3
    qkv_t = torch.from_numpy(qkv).pin_memory()
    q, k, v = kerr_attn.split_qkv(qkv_t, C)
    o = torch.empty(B, T, C).pin_memory()
    lse = torch.empty(B, H, T).pin_memory()
    dout_t = torch.from_numpy(dout).pin_memory()
    if split_grads:
        dq, dk, dv = (torch.empty(B, T, C).pin_memory() for _ in range(3))
    else:
        dq, dk, dv = kerr_attn.split_qkv(torch.empty(B, T, 3 * C).pin_memory(), C)
    if saved is None:
        kerr_attn.fwd_host(ctx, q, k, v, o, lse, H)
        kerr_attn.bwd_host(ctx, q, k, v, o, dout_t, lse, dq, dk, dv, H)
    else:
        kerr_attn.fwd_host_save(ctx, saved, q, k, v, o, lse, H)
        kerr_attn.bwd_host_saved(ctx, saved, dout_t, dq, dk, dv)
    return (o.numpy(), lse.numpy(), dq.numpy(), dk.numpy(), dv.numpy())


def test_host_paths_pipelined_and_saved(ctx):
    # At the 768-dim shape with B=10 the host calls split the batch into
    # chunks (4/4/2 sequences for the forward and the saved-state backward,
    # five of 2 for the plain backward), overlapping each chunk's copies with
    # its neighbours' kernels.  Results must equal the device-pointer path's: the
    # forward bit for bit, the gradients up to dQ's run-dependent summation
    # order.  The saved-state pair (kattn_fwd_host_save / kattn_bwd_host_saved,
    # the reference's AttnCache) must give the same results as the plain pair.
    B, T, H, d = 10, 256, 12, 64
    qkv, dout = make_inputs(B, T, H, d, seed=77)
    ref = gpu_fwd_bwd(ctx, qkv, dout, H)

    def check(got):
        assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1])
        for g, r in zip(got[2:], ref[2:]):
            assert rel_err(g, r) < 1e-6

    check(_host_fwd_bwd(ctx, qkv, dout, H))
    with kerr_attn.Saved(ctx) as saved:
        check(_host_fwd_bwd(ctx, qkv, dout, H, saved=saved))
        # Reused for a smaller forward; separate dq / dk / dv host arrays take
        # the strided download path.
        qkv2, dout2 = make_inputs(3, 100, H, d, seed=78)
        ref2 = gpu_fwd_bwd(ctx, qkv2, dout2, H)
        got2 = _host_fwd_bwd(ctx, qkv2, dout2, H, saved=saved, split_grads=True)
        assert np.array_equal(got2[0], ref2[0]) and np.array_equal(got2[1], ref2[1])
        for g, r in zip(got2[2:], ref2[2:]):
            assert rel_err(g, r) < 1e-6


def test_side_stream_and_reuse(ctx, oracle_lib):
    qkv, dout = make_inputs(2, 128, 2, 64, seed=8)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        got = gpu_fwd_bwd(ctx, qkv, dout, 2, stream=s)
    ref = oracle_fwd_bwd(oracle_lib, qkv, dout, 2)
    assert_parity(got, ref)
    again = gpu_fwd_bwd(ctx, qkv, dout, 2)
    assert np.array_equal(again[0], got[0]) and np.array_equal(again[1], got[1])
    assert rel_err(again[2], got[2]) < 1e-6  # dQ sums in a run-dependent order


def test_device_errors_are_reported(ctx):
    dev = torch.device("cuda", 0)
    buf = torch.zeros(1, 8, 3 * 130, device=dev)
    q, k, v = buf[..., 1:129], buf[..., 130:258], buf[..., 259:387]
    o = torch.empty(1, 8, 128, device=dev)
    lse = torch.empty(1, 4, 8, device=dev)
    with pytest.raises(kerr_attn.KattnError) as e:
        kerr_attn.fwd(ctx, q, k, v, o, lse, 4)
    assert e.value.status == kerr_attn.KATTN_ERR_MISALIGNED
    with pytest.raises(kerr_attn.KattnError) as e:
        kerr_attn.fwd(ctx, o[..., :96], o[..., :96], o[..., :96], o[..., :96], lse, 2)  # head_dim 48
    assert e.value.status == kerr_attn.KATTN_ERR_UNSUPPORTED

"""GPU parity of the Kerr-ODE (kattn_kerr_ode_fwd / _bwd, through the C ABI)
against the oracle's restatement of the reference's CPU path
(kerr_ode_cpu, src/backend.rs:387-417; kerr_ode_backward_batch,
src/backend.rs:147-176 -> src/backward.rs:382-458).

Tolerances (norm-wise, max|x - ref| / max|ref|): 1e-5 for the forward (the
kernels contract a*b+c into fused multiply-adds, the reference does not),
1e-4 for dx and the per-band parameter gradients, 1e-3 (the gradient
tolerance) for the two scalar sums d_alpha and d_beta, which add hundreds of
thousands of terms in a different order.  On the reference's own GPU check
inputs the reference's bar applies as well: max absolute difference < 1e-4
(src/gpu_validate.rs:100, :151, :201).
"""
import numpy as np
import pytest
import torch

import kerr_attn
import kerr_ode_f64
from conftest import rel_err

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-5
BWD_TOL = 1e-4
SCALAR_TOL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = kerr_attn.Context(0)
    yield c
    c.check_device()
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).cuda()


def gpu_forward(ctx, x, gr, om, al, be, n_steps):
    y = torch.full(x.shape, float("nan"), device="cuda")
    assert kerr_attn.kerr_ode_fwd(ctx, dev(x), dev(gr), dev(om), dev([al, be]), y, n_steps) == 1
    torch.cuda.synchronize()
    return y.cpu().numpy()


def gpu_backward(ctx, dy, x, gr, om, al, be, n_steps):
    M, n = x.shape
    nb = n // 2
    dx = torch.full((M, n), float("nan"), device="cuda")
    dgr = torch.full((nb,), float("nan"), device="cuda")
    dom = torch.full((nb,), float("nan"), device="cuda")
    dab = torch.full((2,), float("nan"), device="cuda")
    assert kerr_attn.kerr_ode_bwd(ctx, dev(dy), dev(x), dev(gr), dev(om), dev([al, be]), dx, dgr, dom, dab, n_steps,
                                  accumulate=False) == 2
    torch.cuda.synchronize()
    ab = dab.cpu().numpy()
    return dx.cpu().numpy(), dgr.cpu().numpy(), dom.cpu().numpy(), float(ab[0]), float(ab[1])


def check_backward(got, ref):
    dx, dgr, dom, da, db = got
    rdx, rdgr, rdom, rda, rdb = ref
    assert rel_err(dx, rdx) < BWD_TOL
    assert rel_err(dgr, rdgr) < BWD_TOL
    assert rel_err(dom, rdom) < BWD_TOL
    assert abs(da - rda) <= SCALAR_TOL * abs(rda) + 1e-6
    assert abs(db - rdb) <= SCALAR_TOL * abs(rdb) + 1e-6


@pytest.mark.parametrize("case", kerr_ode_f64.reference_cases(), ids=lambda c: c[0])
def test_reference_gpu_check_inputs(ctx, oracle_lib, case):
    # The inputs of the reference's own GPU-vs-CPU Kerr-ODE checks.
    _, x, gr, om, al, be, n_steps = case
    y = gpu_forward(ctx, x, gr, om, al, be, n_steps)
    y_ref = oracle_lib.kerr_ode_forward(x, gr, om, al, be, n_steps)
    assert np.abs(y - y_ref).max() < 1e-4
    assert rel_err(y, y_ref) < FWD_TOL
    dy = np.random.default_rng(len(x)).standard_normal(x.shape).astype(np.float32)
    check_backward(gpu_backward(ctx, dy, x, gr, om, al, be, n_steps),
                   oracle_lib.kerr_ode_backward(dy, x, gr, om, al, be, n_steps))


# (M positions, n_bands, n_steps): the 128-dim model (B=4, T=64), the 768-dim
# model (B=16, T=256) and the 1280-dim model (B=32, T=512) at rk4_n_steps 8;
# 16 steps (src/gpu_validate.rs:122); a single step; a band count that is not
# a multiple of the 128 bands of a warp (196); the fewest bands (one live
# thread) and the most bands supported.
SHAPES = [(256, 64, 8), (4096, 384, 8), (16384, 640, 8), (300, 384, 16), (64, 128, 1), (45, 196, 8),
          (33, 4, 8), (40, kerr_attn.KODE_MAX_BANDS, 8)]


@pytest.mark.parametrize("M,nb,n_steps", SHAPES)
def test_parity_with_oracle(ctx, oracle_lib, M, nb, n_steps):
    rng = np.random.default_rng(M + nb + n_steps)
    x = rng.standard_normal((M, 2 * nb)).astype(np.float32)
    dy = rng.standard_normal((M, 2 * nb)).astype(np.float32)
    gr, om, al, be = kerr_ode_f64.init_params(nb, seed=nb)
    y = gpu_forward(ctx, x, gr, om, al, be, n_steps)
    assert rel_err(y, oracle_lib.kerr_ode_forward(x, gr, om, al, be, n_steps)) < FWD_TOL
    check_backward(gpu_backward(ctx, dy, x, gr, om, al, be, n_steps),
                   oracle_lib.kerr_ode_backward(dy, x, gr, om, al, be, n_steps, threads=0))


def test_against_float64_autograd(ctx):
    # The 768-dim shape against the independent float64 autograd ODE.
    M, nb, n_steps = 1024, 384, 8
    rng = np.random.default_rng(3)
    x = rng.standard_normal((M, 2 * nb)).astype(np.float32)
    dy = rng.standard_normal((M, 2 * nb)).astype(np.float32)
    gr, om, al, be = kerr_ode_f64.init_params(nb, seed=7)
    ry, rdx, rdgr, rdom, rda, rdb = kerr_ode_f64.forward_backward(x, dy, gr, om, al, be, n_steps)
    assert rel_err(gpu_forward(ctx, x, gr, om, al, be, n_steps), ry) < FWD_TOL
    check_backward(gpu_backward(ctx, dy, x, gr, om, al, be, n_steps), (rdx, rdgr, rdom, rda, rdb))


def test_strided_in_place_accumulate_and_deterministic(ctx, oracle_lib):
    M, nb, n_steps = 512, 384, 8
    n = 2 * nb
    rng = np.random.default_rng(11)
    x = rng.standard_normal((M, n)).astype(np.float32)
    dy = rng.standard_normal((M, n)).astype(np.float32)
    gr, om, al, be = kerr_ode_f64.init_params(nb, seed=2)
    g, o, ab = dev(gr), dev(om), dev([al, be])
    y_ref = oracle_lib.kerr_ode_forward(x, gr, om, al, be, n_steps)
    # Rows at a stride of 3n inside a wider buffer; nothing outside them written.
    buf = torch.full((M, 3 * n), float("nan"), device="cuda")
    buf[:, n:2 * n] = dev(x)
    out = torch.full((M, 2 * n), float("nan"), device="cuda")
    kerr_attn.kerr_ode_fwd(ctx, buf[:, n:2 * n], g, o, ab, out[:, :n], n_steps)
    assert rel_err(out[:, :n].cpu().numpy(), y_ref) < FWD_TOL
    assert torch.isnan(out[:, n:]).all() and torch.isnan(buf[:, :n]).all()
    # In place: y = x.
    xi = dev(x)
    kerr_attn.kerr_ode_fwd(ctx, xi, g, o, ab, xi, n_steps)
    assert rel_err(xi.cpu().numpy(), y_ref) < FWD_TOL
    # Accumulation into existing parameter gradients (src/pipeline.rs:627-632),
    # and dx = dy in place.
    rdx, rdgr, rdom, rda, rdb = oracle_lib.kerr_ode_backward(dy, x, gr, om, al, be, n_steps, threads=0)
    g0 = rng.standard_normal(nb).astype(np.float32)
    o0 = rng.standard_normal(nb).astype(np.float32)
    ab0 = np.array([0.5, -0.25], np.float32)
    dgr, dom, dab = dev(g0), dev(o0), dev(ab0)
    d = dev(dy)
    assert kerr_attn.kerr_ode_bwd(ctx, d, dev(x), g, o, ab, d, dgr, dom, dab, n_steps, accumulate=True) == 2
    assert rel_err(d.cpu().numpy(), rdx) < BWD_TOL
    assert rel_err(dgr.cpu().numpy(), g0 + rdgr) < BWD_TOL
    assert rel_err(dom.cpu().numpy(), o0 + rdom) < BWD_TOL
    got_ab = dab.cpu().numpy()
    assert abs(got_ab[0] - (ab0[0] + rda)) <= SCALAR_TOL * abs(ab0[0] + rda)
    assert abs(got_ab[1] - (ab0[1] + rdb)) <= SCALAR_TOL * abs(ab0[1] + rdb)
    # Fixed-order sums: two runs give the same bits.
    runs = []
    for _ in range(2):
        dx = torch.empty(M, n, device="cuda")
        gs = [torch.empty(nb, device="cuda"), torch.empty(nb, device="cuda"), torch.empty(2, device="cuda")]
        kerr_attn.kerr_ode_bwd(ctx, dev(dy), dev(x), g, o, ab, dx, *gs, n_steps, accumulate=False)
        runs.append([dx] + gs)
    assert all(torch.equal(a, b) for a, b in zip(*runs))


def test_empty(ctx):
    nb = 64
    g = torch.zeros(nb, device="cuda")
    ab = torch.zeros(2, device="cuda")
    x = torch.empty(0, 2 * nb, device="cuda")
    assert kerr_attn.kerr_ode_fwd(ctx, x, g, g, ab, torch.empty(0, 2 * nb, device="cuda"), 8) == 0
    # No positions and accumulate=0: the parameter gradients are zero.
    dgr = torch.full((nb,), 5.0, device="cuda")
    dom = torch.full((nb,), 5.0, device="cuda")
    dab = torch.full((2,), 5.0, device="cuda")
    kerr_attn.kerr_ode_bwd(ctx, x, x, g, g, ab, torch.empty(0, 2 * nb, device="cuda"), dgr, dom, dab, 8,
                           accumulate=False)
    torch.cuda.synchronize()
    assert torch.count_nonzero(dgr).item() == 0 and torch.count_nonzero(dom).item() == 0
    assert torch.count_nonzero(dab).item() == 0


@pytest.mark.parametrize("pinned", [True, False])
def test_host_buffer_calls(ctx, oracle_lib, pinned):
    # kattn_kerr_ode_fwd_host / _bwd_host (the trait's host-slice boundary):
    # the same results as the device calls, positions split into chunks.
    M, nb, n_steps = 3001, 384, 8
    n = 2 * nb
    rng = np.random.default_rng(21)
    x = rng.standard_normal((M, n)).astype(np.float32)
    dy = rng.standard_normal((M, n)).astype(np.float32)
    gr, om, al, be = kerr_ode_f64.init_params(nb, seed=4)

    def host(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
        return t.pin_memory() if pinned else t.clone()

    hy = host(np.full((M, n), np.nan))
    assert kerr_attn.kerr_ode_fwd_host(ctx, host(x), host(gr), host(om), al, be, hy, n_steps) >= 1
    y_dev = gpu_forward(ctx, x, gr, om, al, be, n_steps)
    assert np.array_equal(hy.numpy(), y_dev)  # positions are independent: same bits
    hdx = host(np.full((M, n), np.nan))
    g0 = rng.standard_normal(nb).astype(np.float32)
    hdg, hdo, hdab = host(g0), host(np.zeros(nb)), host(np.array([1.0, 2.0]))
    launches = kerr_attn.kerr_ode_bwd_host(ctx, host(dy), host(x), host(gr), host(om), al, be, hdx, hdg, hdo, hdab,
                                           n_steps, accumulate=True)
    assert launches >= 2
    dx_dev, dgr_dev, dom_dev, da_dev, db_dev = gpu_backward(ctx, dy, x, gr, om, al, be, n_steps)
    assert np.array_equal(hdx.numpy(), dx_dev)
    assert rel_err(hdg.numpy(), g0 + dgr_dev) < 1e-5
    assert rel_err(hdo.numpy(), dom_dev) < 1e-5
    assert abs(hdab[0].item() - (1.0 + da_dev)) <= 1e-4 * abs(1.0 + da_dev)
    assert abs(hdab[1].item() - (2.0 + db_dev)) <= 1e-4 * abs(2.0 + db_dev)
    rdx, rdgr, rdom, rda, rdb = oracle_lib.kerr_ode_backward(dy, x, gr, om, al, be, n_steps, threads=0)
    assert rel_err(hdx.numpy(), rdx) < BWD_TOL
    assert rel_err(hdg.numpy() - g0, rdgr) < BWD_TOL

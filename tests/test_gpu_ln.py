"""GPU parity of LayerNorm LN1 / LN2 (kattn_layernorm_fwd / _bwd, through the
C ABI) against the oracle's restatement of the reference
(src/backend.rs:258-267; src/backward.rs:93-128; src/backend.rs:195-206).

Tolerances (norm-wise, max|x - ref| / max|ref|): the kernels sum in a
different order than the reference's left-to-right loops, so results differ
in the last bits: 1e-5 for y, 1e-4 for dx (its formula cancels n*g against
the row sums) and for the column sums dw, db over thousands of rows.
"""
import numpy as np
import pytest
import torch

import kerr_attn
from conftest import rel_err

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-5
BWD_TOL = 1e-4


@pytest.fixture(scope="module")
def ctx():
    c = kerr_attn.Context(0)
    yield c
    c.check_device()
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def inputs(M, N, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((M, N)) * 1.5 + 0.3).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    return x, w, b, dy


# (M, N): the 128-dim model (B=4, T=64), the 768-dim model (B=16, T=256), the
# 1280-dim model (B=32, T=512), rows not a multiple of a block's 64, a row
# width that leaves lanes idle, and the widest row supported.
SHAPES = [(256, 128), (4096, 768), (16384, 1280), (1000, 768), (77, 100), (130, kerr_attn.LN_MAX_N)]


@pytest.mark.parametrize("M,N", SHAPES)
def test_layernorm_parity_with_oracle(ctx, oracle_lib, M, N):
    from oracle import oracle

    x, w, b, dy = inputs(M, N, seed=M + N)
    y = torch.full((M, N), float("nan"), device="cuda")
    assert kerr_attn.layernorm_fwd(ctx, dev(x), dev(w), dev(b), y) == 1
    dx = torch.full((M, N), float("nan"), device="cuda")
    dw = torch.full((N,), float("nan"), device="cuda")
    db = torch.full((N,), float("nan"), device="cuda")
    assert kerr_attn.layernorm_bwd(ctx, dev(dy), dev(x), dev(w), dx, dw, db, accumulate=False) == 2
    torch.cuda.synchronize()
    y_ref = oracle.layernorm_forward(x, w, b)
    dx_ref, dw_ref, db_ref = oracle.layernorm_backward(dy, x, w)
    assert rel_err(y.cpu().numpy(), y_ref) < FWD_TOL
    assert rel_err(dx.cpu().numpy(), dx_ref) < BWD_TOL
    assert rel_err(dw.cpu().numpy(), dw_ref) < BWD_TOL
    assert rel_err(db.cpu().numpy(), db_ref) < BWD_TOL


def test_layernorm_strided_accumulate_and_deterministic(ctx, oracle_lib):
    from oracle import oracle

    M, N = 512, 768
    x, w, b, dy = inputs(M, N, seed=9)
    # Rows at a stride of 3N inside a wider buffer (e.g. one block of a
    # [M][3C] activation), outputs into another strided buffer.
    xbuf = torch.zeros(M, 3 * N, device="cuda")
    xbuf[:, N:2 * N] = dev(x)
    ybuf = torch.full((M, 2 * N), float("nan"), device="cuda")
    kerr_attn.layernorm_fwd(ctx, xbuf[:, N:2 * N], dev(w), dev(b), ybuf[:, :N])
    assert rel_err(ybuf[:, :N].cpu().numpy(), oracle.layernorm_forward(x, w, b)) < FWD_TOL
    assert torch.isnan(ybuf[:, N:]).all()  # nothing written outside the rows
    # Accumulation into existing dw / db (the += of src/pipeline.rs:747-750);
    # db may be omitted.
    dw0 = np.random.default_rng(1).standard_normal(N).astype(np.float32)
    dw = dev(dw0)
    dx = torch.empty(M, N, device="cuda")
    kerr_attn.layernorm_bwd(ctx, dev(dy), xbuf[:, N:2 * N], dev(w), dx, dw, None, accumulate=True)
    dx_ref, dw_ref, _ = oracle.layernorm_backward(dy, x, w, dw=dw0)
    assert rel_err(dx.cpu().numpy(), dx_ref) < BWD_TOL
    assert rel_err(dw.cpu().numpy(), dw_ref) < BWD_TOL
    # Fixed-order column sums: a second run gives the same bits.
    dw_a, db_a = torch.empty(N, device="cuda"), torch.empty(N, device="cuda")
    dw_b, db_b = torch.empty(N, device="cuda"), torch.empty(N, device="cuda")
    dx_b = torch.empty(M, N, device="cuda")
    kerr_attn.layernorm_bwd(ctx, dev(dy), dev(x), dev(w), dx, dw_a, db_a, accumulate=False)
    kerr_attn.layernorm_bwd(ctx, dev(dy), dev(x), dev(w), dx_b, dw_b, db_b, accumulate=False)
    assert torch.equal(dw_a, dw_b) and torch.equal(db_a, db_b) and torch.equal(dx, dx_b)


def test_layernorm_empty(ctx):
    N = 768
    w = torch.ones(N, device="cuda")
    x = torch.empty(0, N, device="cuda")
    assert kerr_attn.layernorm_fwd(ctx, x, w, w, torch.empty(0, N, device="cuda")) == 0
    # No rows and accumulate=0: the column sums are zero.
    dw = torch.full((N,), 5.0, device="cuda")
    kerr_attn.layernorm_bwd(ctx, x, x, w, torch.empty(0, N, device="cuda"), dw, None, accumulate=False)
    torch.cuda.synchronize()
    assert torch.count_nonzero(dw).item() == 0

"""GPU parity of the attention projections (kattn_linear_*, through the C
ABI) against the oracle's restatement of the reference's linear layers
(src/backend.rs:240-247, :508-520; src/backward.rs:48-60;
src/backend.rs:320-342).

Tolerances: the products are formed in bf16 hi/lo pairs (~1e-5 relative);
every result must be within 1e-4 (norm-wise, max|x - ref| / max|ref|) of the
f32 oracle, the forward tolerance of the path.
"""
import numpy as np
import pytest
import torch

import kerr_attn
from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.fixture(scope="module")
def ctx():
    c = kerr_attn.Context(0)
    yield c
    c.check_device()
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    return x, w, b, dy


# (M, N, K): the 128-dim model's c_attn and c_proj (B=4, T=64), its maestro
# squeeze / process_1 (maestro_dim 16) and padded lm_head (68 rows), the
# 768-dim model's c_attn and c_proj (B=16, T=256), the 1280-dim model's
# c_attn (B=32, T=512), and ragged shapes (edges of the 128 x 256 x 64 GEMM
# tiles on every side, single rows, K below one stage).
SHAPES = [(256, 384, 128), (256, 128, 128), (256, 16, 128), (256, 128, 16), (256, 68, 128),
          (4096, 2304, 768), (4096, 768, 768), (16384, 3840, 1280),
          (100, 52, 36), (1, 4, 4), (3, 8, 260), (300, 260, 68)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_parity_with_oracle(ctx, oracle_lib, M, N, K):
    from oracle import oracle

    x, w, b, dy = inputs(M, N, K, seed=M + N + K)
    y = torch.full((M, N), float("nan"), device="cuda")
    kerr_attn.linear_fwd(ctx, dev(x), dev(w), dev(b), y)
    dx = torch.full((M, K), float("nan"), device="cuda")
    kerr_attn.linear_bwd_dx(ctx, dev(dy), dev(w), dx)
    dw = torch.full((N, K), float("nan"), device="cuda")
    db = torch.full((N,), float("nan"), device="cuda")
    kerr_attn.linear_bwd_dw(ctx, dev(dy), dev(x), dw, db, accumulate=False)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.linear_forward(x, w, b)) < TOL
    assert rel_err(dx.cpu().numpy(), oracle.linear_backward_dx(dy, w)) < TOL
    dw_ref, db_ref = oracle.linear_backward_dw(dy, x)
    assert rel_err(dw.cpu().numpy(), dw_ref) < TOL
    assert rel_err(db.cpu().numpy(), db_ref) < TOL


def test_strided_rows_and_accumulation(ctx, oracle_lib):
    # c_attn writes q|k|v straight into a [B*T][3C] buffer and reads the
    # gradient back out of one, and gradients accumulate over calls as the
    # reference's bg += (src/pipeline.rs:701-704, :733-736).
    from oracle import oracle

    M, C = 512, 128
    x, w, b, dy = inputs(M, 3 * C, C, seed=5)
    wide = torch.zeros(M, 3 * C + 64, device="cuda")   # row stride 3C + 64
    y = wide[:, 32:32 + 3 * C]
    kerr_attn.linear_fwd(ctx, dev(x), dev(w), dev(b), y)
    assert rel_err(y.cpu().numpy(), oracle.linear_forward(x, w, b)) < TOL
    assert float(wide[:, :32].abs().max()) == 0.0 and float(wide[:, 32 + 3 * C:].abs().max()) == 0.0

    dw = torch.zeros(3 * C, C, device="cuda")
    db = torch.zeros(3 * C, device="cuda")
    for rep in range(2):
        kerr_attn.linear_bwd_dw(ctx, dev(dy), dev(x), dw, db, accumulate=True)
    dw_ref, db_ref = oracle.linear_backward_dw(dy, x)
    assert rel_err(dw.cpu().numpy(), 2 * dw_ref) < TOL
    assert rel_err(db.cpu().numpy(), 2 * db_ref) < TOL

    # No bias, and a zero-row problem that launches nothing.
    y2 = torch.empty(M, 3 * C, device="cuda")
    kerr_attn.linear_fwd(ctx, dev(x), dev(w), None, y2)
    assert rel_err(y2.cpu().numpy(), oracle.linear_forward(x, w, None)) < TOL
    assert kerr_attn.linear_fwd(ctx, torch.empty(0, C, device="cuda"), dev(w), dev(b),
                                torch.empty(0, 3 * C, device="cuda")) == 0

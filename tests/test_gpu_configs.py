"""GPU parity at the remaining workload configurations of the path, through
the C ABI:

- the 1280-dim model's attention layer (B=32 per GPU, H=20, d=64, T=512)
  against the oracle at full size, plus the softmax identities;
- the long-context sweep (B=8, H=12, d=64, T = 1024, 2048, 4096): the whole
  batch against the oracle at T = 1024 and 2048, the first and the last
  sequence at T = 4096 (the oracle's scalar loops take tens of seconds per
  sequence there); the last sequence also against float64 torch; the
  identities over the whole batch.

Tolerances as in test_gpu_parity: forward 1e-4, gradients 1e-3 (norm-wise).
"""
import numpy as np
import pytest

import kerr_attn
from conftest import make_inputs, rel_err
from test_gpu_parity import assert_parity, gpu_fwd_bwd, oracle_fwd_bwd, torch_f64

pytestmark = pytest.mark.gpu


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


def check_identities(qkv, dout, got, H):
    """Size-independent identities of causal softmax attention, per (b, h):
    sum_t dV[t] = sum_t dO[t] (softmax rows sum to one) and sum_t dK[t] = 0
    (a shift of every key by one vector leaves the scores' softmax unchanged)."""
    B, T, C3 = qkv.shape
    C = C3 // 3
    d = C // H
    _, _, _, dk, dv = got
    sdv = dv.astype(np.float64).reshape(B, T, H, d).sum(1)
    sdo = dout.astype(np.float64).reshape(B, T, H, d).sum(1)
    assert rel_err(sdv, sdo) < 1e-4
    sdk = np.abs(dk.astype(np.float64).reshape(B, T, H, d).sum(1)).max()
    assert sdk < 1e-3 * np.abs(dk).max() * np.sqrt(T)


def test_1280dim_layer_against_oracle(ctx, oracle_lib):
    B, T, H, d = 32, 512, 20, 64
    qkv, dout = make_inputs(B, T, H, d, seed=1280)
    got = gpu_fwd_bwd(ctx, qkv, dout, H, path="tensor")
    assert_parity(got, oracle_fwd_bwd(oracle_lib, qkv, dout, H), case="1280-dim layer B=32 T=512 H=20")
    check_identities(qkv, dout, got, H)


@pytest.mark.parametrize("T", [1024, 2048, 4096])
def test_long_context_sweep(ctx, oracle_lib, T):
    B, H, d = 8, 12, 64
    qkv, dout = make_inputs(B, T, H, d, seed=T, qkv_sigma=1.0 / 8)
    got = gpu_fwd_bwd(ctx, qkv, dout, H, path="tensor")
    check_identities(qkv, dout, got, H)
    seqs = list(range(B)) if T <= 2048 else [0, B - 1]
    ref = oracle_fwd_bwd(oracle_lib, np.ascontiguousarray(qkv[seqs]), np.ascontiguousarray(dout[seqs]), H)
    assert_parity(tuple(g[seqs] for g in got), ref, case=f"long context T={T} oracle, sequences {seqs}")
    # The last sequence against float64 as well.
    ref = torch_f64(qkv[-1:], dout[-1:], H, causal=True)
    assert_parity(tuple(g[-1:] for g in got), ref, case=f"long context T={T} float64, last sequence")

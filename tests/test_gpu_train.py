"""Loss curves of a 50-step training run on this library's kernels against the
same run on the oracle (tests/train_stack.py): LN1, c_attn, causal attention,
c_proj, LN2 and the Kerr-ODE per block, four blocks, SGD.  Every forward and
backward op of the path goes through the C ABI on the GPU side.

Tolerance: each step's loss within 1e-3 relative of the oracle's (the
gradient tolerance); the two runs differ only by rounding (bf16x3 products
and fused multiply-adds on the GPU, the reference's f32 loop order on the
CPU), which the 50 SGD steps carry forward."""
import numpy as np
import pytest

import train_stack

pytestmark = pytest.mark.gpu

STEPS = 50
LR = 0.03


# (B, T, C, H): the 128-dim model's shapes (B=4, T=64, head_dim 32, the FFMA
# attention path) and a head_dim 64 stack (the tensor-core path).
@pytest.mark.parametrize("B,T,C,H", [(4, 64, 128, 4), (2, 128, 256, 4)])
def test_loss_curve_matches_oracle(oracle_lib, B, T, C, H):
    blocks, h0, target = train_stack.init(B, T, C, H, 4, seed=42)
    ref = train_stack.train_oracle(blocks, h0, target, H, STEPS, LR)
    got = train_stack.train_gpu(blocks, h0, target, H, STEPS, LR)
    ref, got = np.array(ref), np.array(got)
    assert np.isfinite(got).all()
    assert ref[-1] < 0.6 * ref[0]  # the run learns
    rel = np.abs(got - ref) / ref
    assert rel.max() < 1e-3, f"worst step {rel.argmax()}: {got[rel.argmax()]} vs {ref[rel.argmax()]}"

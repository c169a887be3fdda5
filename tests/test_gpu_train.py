"""Loss curves of 50-step training runs on this library's kernels against the
same runs on the oracle:

- the reference's 128-dim model as it trains (tests/model128.py): xorshift64
  initialisation with seed 42 in the reference's order, frozen harmonic and
  positional embeddings, four blocks (PerBandLinear FFN in block 0,
  KerrMaestroAdd in blocks 1-3), ln_f, lm_head, cross-entropy over 65
  symbols, global-norm clipping at 1.0 and Adam at lr 3e-4, batches of 4 x
  64 tokens from a seeded Zipf(1.0) stream drawn as the reference samples;
- a stack of the path's own layers (tests/train_stack.py): LN1, c_attn,
  causal attention, c_proj, LN2 and the Kerr-ODE per block, four blocks, SGD
  on an MSE target, at the 128-dim shapes (head_dim 32) and at head_dim 64,
  once composed call by call and once through the device-resident block
  pipeline (kattn_block_fwd / _bwd).

Every forward and backward op of the path goes through the C ABI on the GPU
side.

Tolerance: each step's loss within 1e-3 relative of the oracle's (the
gradient tolerance); the two runs differ only by rounding (bf16x3 products
and fused multiply-adds on the GPU, the reference's f32 loop order on the
CPU), which the 50 steps carry forward."""
import math

import numpy as np
import pytest

import model128
import train_stack

pytestmark = pytest.mark.gpu

STEPS = 50
LR = 0.03


# (B, T, C, H): the 128-dim model's shapes (B=4, T=64, head_dim 32: the FFMA
# kernels at this size) and a head_dim 64 stack (the tensor-core kernels).
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


def test_loss_curve_native_block_pipeline(oracle_lib):
    """The same 50-step run with each block as one kattn_block_fwd /
    kattn_block_bwd pair (the device-resident pipeline), head_dim 64."""
    B, T, C, H = 2, 128, 256, 4
    blocks, h0, target = train_stack.init(B, T, C, H, 4, seed=42)
    ref = np.array(train_stack.train_oracle(blocks, h0, target, H, STEPS, LR))
    got = np.array(train_stack.train_gpu_native(blocks, h0, target, H, STEPS, LR))
    assert np.isfinite(got).all()
    rel = np.abs(got - ref) / ref
    assert rel.max() < 1e-3, f"worst step {rel.argmax()}: {got[rel.argmax()]} vs {ref[rel.argmax()]}"


def test_reference_128dim_model_loss_curve(oracle_lib):
    ref = np.array(model128.train_oracle(STEPS))
    got = np.array(model128.train_gpu(STEPS))
    assert np.isfinite(got).all()
    assert abs(ref[0] - math.log(model128.VOCAB)) < 0.5  # starts near uniform over 65 symbols
    assert ref[-5:].mean() < 0.9 * ref[:5].mean()  # and learns
    rel = np.abs(got - ref) / ref
    assert rel.max() < 1e-3, f"worst step {rel.argmax()}: {got[rel.argmax()]} vs {ref[rel.argmax()]}"

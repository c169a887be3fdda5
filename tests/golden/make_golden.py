"""Generate the committed attention fixtures in tests/golden/ from the oracle.

The reference (Rust) cannot be built here and ships no attention golden
vectors, so these fixtures are oracle outputs: they pin the oracle and let the
GPU tests compare against fixed bytes.  Inputs: numpy PCG64 seeded streams,
q, k, v ~ N(0, 1) / sqrt(head_dim) in one [B, T, 3C] qkv buffer, dout ~ N(0, 1).

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402

CASES = [
    # name, B, T, H, d, seed
    ("model128_b1_t64_h4_d32", 1, 64, 4, 32, 1337),   # the 128-dim model's attention shape
    ("ragged_b1_t70_h2_d64", 1, 70, 2, 64, 42),       # T not a multiple of the 64-row tile
    ("tiny_b2_t5_h1_d32", 2, 5, 1, 32, 7),
]


def main():
    oracle.build()
    for name, B, T, H, d, seed in CASES:
        rng = np.random.default_rng(seed)
        C = H * d
        qkv = (rng.standard_normal((B, T, 3 * C)) / np.sqrt(d)).astype(np.float32)
        dout = rng.standard_normal((B, T, C)).astype(np.float32)
        q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
        o, att, lse = oracle.forward(q, k, v, H)
        dq, dk, dv = oracle.backward(dout, q, k, v, att, H)
        np.savez(os.path.join(HERE, name + ".npz"), n_head=np.int32(H), qkv=qkv, dout=dout,
                 o=o, lse=lse, dq=dq, dk=dk, dv=dv)
        print(name, "written")


if __name__ == "__main__":
    main()

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kerr-engine_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


def rel_err(x, ref) -> float:
    """Norm-wise relative error max|x - ref| / max|ref| (the tolerance measure
    of every parity test: 1e-4 for the forward, 1e-3 for gradients)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max() if ref.size else 0.0
    num = np.abs(x - ref).max() if ref.size else 0.0
    return float(num / den) if den > 0 else float(num)


def make_inputs(B, T, H, d, seed=42, qkv_sigma=None):
    """Seeded synthetic inputs: one [B, T, 3C] qkv buffer with q, k, v ~ N(0, 1)
    scaled by 1/sqrt(d) (the attention microbenchmark's distribution) and
    dout ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    C = H * d
    sig = (1.0 / np.sqrt(d)) if qkv_sigma is None else qkv_sigma
    qkv = (rng.standard_normal((B, T, 3 * C)) * sig).astype(np.float32)
    dout = rng.standard_normal((B, T, C)).astype(np.float32)
    return qkv, dout


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle

    oracle.build()
    return oracle

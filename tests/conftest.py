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


def elem_rel_err(x, ref, floor: float = 1e-3) -> float:
    """Elementwise relative error with an absolute floor:
    max_i |x_i - ref_i| / (|ref_i| + floor * max|ref|).  Reported beside
    rel_err: it shows how well small outputs are reproduced, which the
    norm-wise figure does not (an element far below the largest one can be
    off by a large fraction of itself and still pass rel_err)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    if not ref.size:
        return 0.0
    scale = np.abs(ref).max()
    den = np.abs(ref) + floor * scale
    den = np.where(den > 0, den, 1.0)
    return float((np.abs(x - ref) / den).max())


def record_errors(case: str, errs: dict) -> None:
    """Appends one JSON line {case, errors} to the file named by the
    KATTN_PARITY_LOG environment variable (nothing when it is unset), so a run
    can keep every measured error, not only the failures."""
    path = os.environ.get("KATTN_PARITY_LOG")
    if not path:
        return
    import json

    with open(path, "a") as f:
        f.write(json.dumps({"case": case, "errors": {k: float(v) for k, v in errs.items()}}) + "\n")


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

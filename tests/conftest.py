import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# ---- parity helpers shared by the GPU tests --------------------------------
MAX_ABS = 2e-3      # task tolerance for attention outputs
MIN_COS = 0.99999


def parity(out, ref, max_abs=MAX_ABS, min_cos=MIN_COS):
    """Assert max-abs and cosine parity of two arrays (float64 comparison)."""
    a = np.asarray(out, dtype=np.float64).ravel()
    b = np.asarray(ref, dtype=np.float64).ravel()
    assert np.all(np.isfinite(a)), "non-finite output"
    err = np.max(np.abs(a - b)) if a.size else 0.0
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    cos = 1.0 if na == 0 and nb == 0 else float(a @ b / max(na * nb, 1e-30))
    assert err <= max_abs, f"max-abs error {err:.3e} > {max_abs:.1e} (cos {cos:.7f})"
    assert cos >= min_cos, f"cosine {cos:.7f} < {min_cos} (max-abs {err:.3e})"
    return err, cos

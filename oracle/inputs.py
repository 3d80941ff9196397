"""Seeded synthetic inputs for the task configs (test infrastructure only).

Distributions follow the task's configs[0]: Q and K are drawn N(0,1) per head
vector, normalised to RMS 1, then multiplied by one per-dim weight vector
w = 1 + 0.1*N(0,1) (one for Q, one for K, shared by all heads; this mimics the
q_norm/k_norm weights applied at engine/gemma4_multilayer.cpp:182-183).
V is N(0,1). All draws come from numpy.random.default_rng(seed) in the fixed
order below, so the oracle and every test see identical inputs.
"""
from __future__ import annotations

import numpy as np


def _rms_normalise(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    rms = np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True))
    return (x / rms.astype(np.float32) * w).astype(np.float32)


def make_layer(seed: int, H: int, Hkv: int, D: int, N: int, batch: int = 1,
               n_new: int = 1) -> dict:
    """One decode step's tensors for `batch` sequences.

    Returns fp32 arrays: q (B, H, D); k, v (B, Hkv, N, D) (the cached tokens);
    k_new, v_new (B, Hkv, n_new, D) (the tokens appended this step).
    """
    rng = np.random.default_rng(seed)
    wq = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wk = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    q = _rms_normalise(rng.standard_normal((batch, H, D), dtype=np.float32), wq)
    k = _rms_normalise(rng.standard_normal((batch, Hkv, N, D), dtype=np.float32), wk)
    v = rng.standard_normal((batch, Hkv, N, D), dtype=np.float32)
    k_new = _rms_normalise(rng.standard_normal((batch, Hkv, n_new, D), dtype=np.float32), wk)
    v_new = rng.standard_normal((batch, Hkv, n_new, D), dtype=np.float32)
    return dict(q=q, k=k, v=v, k_new=k_new, v_new=v_new, wq=wq, wk=wk)


# Shapes of the task configs (BASELINE configs[0..4]).
CONFIGS = {
    0: dict(H=32, Hkv=16, D=128, N=1024, seed=0, scale=1.0, window=0),
    1: dict(H=32, Hkv=16, D=128, N=(1024, 4096, 8192, 16384, 32768), seeds=(1, 2, 3, 4, 5),
            scale=1.0, window=(1024, 0)),
    2: dict(H=32, Hkv=16, D=128, N=8192, seed=7, scale=1.0, batch=64, chunk=512),
    3: dict(H=32, Hkv=16, D=128, N=4096, seed=11, scale=1.0, qjl_m=256),
    4: dict(H=32, Hkv=8, D=256, N=262144, seed=13, scale=1.0),
}

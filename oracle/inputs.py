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


def make_config2(seed: int = 7, H: int = 32, Hkv: int = 16, D: int = 128, N0: int = 8192,
                 batch: int = 64, chunk: int = 512) -> dict:
    """Config 2's tensors, fp32: the cache's N0 tokens k, v (Hkv, N0, D), the
    prefill chunk's own keys/values k_chunk, v_chunk (Hkv, chunk, D), the
    batched-decode queries q_batched (batch, H, D) and the chunk's queries
    q_chunk (chunk, H, D). Distributions as make_layer (RMS-1 Q/K with one
    per-dim weight each, V ~ N(0,1))."""
    rng = np.random.default_rng(seed)
    wq = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wk = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    k = _rms_normalise(rng.standard_normal((Hkv, N0, D), dtype=np.float32), wk)
    v = rng.standard_normal((Hkv, N0, D), dtype=np.float32)
    kc = _rms_normalise(rng.standard_normal((Hkv, chunk, D), dtype=np.float32), wk)
    vc = rng.standard_normal((Hkv, chunk, D), dtype=np.float32)
    qb = _rms_normalise(rng.standard_normal((batch, H, D), dtype=np.float32), wq)
    qc = _rms_normalise(rng.standard_normal((chunk, H, D), dtype=np.float32), wq)
    return dict(k=k, v=v, k_chunk=kc, v_chunk=vc, q_batched=qb, q_chunk=qc)


def make_long_layer(seed: int, H: int, Hkv: int, D: int, N: int, quantize) -> dict:
    """A long single-sequence layer built one KV head at a time, so that only
    one head's fp32 K/V exist at once (config 4: 262144 tokens x 8 heads x
    D=256 is 4.3 GB in fp32). `quantize(x)` maps (N, D) fp32 to (codes,
    scales, biases). Returns q (1, H, D) fp32, k_new/v_new (1, Hkv, 1, D) fp32
    and the quantized cache kq, ks, kb, vq, vs, vb with shapes (1, Hkv, N, .)."""
    rng = np.random.default_rng(seed)
    wq = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wk = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    q = _rms_normalise(rng.standard_normal((1, H, D), dtype=np.float32), wq)
    out = {}
    for h in range(Hkv):
        k = _rms_normalise(rng.standard_normal((N, D), dtype=np.float32), wk)
        kq = quantize(k)
        del k
        v = rng.standard_normal((N, D), dtype=np.float32)
        vq = quantize(v)
        del v
        for name, arr in zip(("kq", "ks", "kb", "vq", "vs", "vb"), (*kq, *vq)):
            if name not in out:
                out[name] = np.empty((1, Hkv) + arr.shape, arr.dtype)
            out[name][0, h] = arr
    out["q"] = q
    out["k_new"] = _rms_normalise(rng.standard_normal((1, Hkv, 1, D), dtype=np.float32), wk)
    out["v_new"] = rng.standard_normal((1, Hkv, 1, D), dtype=np.float32)
    return out

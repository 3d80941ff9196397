"""Generate the golden fixtures in this directory from the CPU oracle.

    python tests/golden/make_golden.py

Each fixture stores the case's sizes and seed, the sha256 of the packed int4
cache the quantizer must produce from the seeded inputs (bit-exact target),
and the fp64 oracle output of dequantize + SDPA (the reference's baseline
path, engine/gemma4_multilayer.cpp:307-308,349). Small cases also store the
packed K codes. The reference itself has no golden vectors and cannot run
here (Metal/MLX), so these pin the oracle, not the reference.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import inputs, oracle as O  # noqa: E402

CASES = [
    # name, seed, H, Hkv, D, N, window, scales fp16?, store codes?
    ("config0", 0, 32, 16, 128, 1024, 0, 1, 0),
    ("ref_test_shape", 1, 16, 16, 256, 10, 0, 1, 1),
    ("config1_sliding_4k", 1, 32, 16, 128, 4096, 1024, 1, 0),
    ("gqa4_d512_f32scales", 2, 8, 2, 512, 300, 0, 0, 0),
    ("gqa8_d256_ragged", 3, 16, 2, 256, 77, 50, 1, 1),
]


def make(name, seed, H, Hkv, D, N, window, sb_f16, store_codes):
    L = inputs.make_layer(seed, H, Hkv, D, N)
    sb = np.float16 if sb_f16 else np.float32
    kq, ks, kb = O.quantize(L["k"], sb)
    vq, vs, vb = O.quantize(L["v"], sb)
    assert all(np.array_equal(a.view(np.uint8), b.view(np.uint8))
               for a, b in zip((kq, ks, kb), O.quantize_np(L["k"], sb)))
    h = hashlib.sha256()
    for a in (kq, ks, kb, vq, vs, vb):
        h.update(np.ascontiguousarray(a).tobytes())
    out = O.sdpa_int4(L["q"].astype(np.float16), kq, ks, kb, vq, vs, vb, window=window, f64=True)
    d = dict(seed=seed, H=H, Hkv=Hkv, D=D, N=N, window=window, sb_f16=sb_f16,
             cache_sha256=h.hexdigest(), out_f64=out)
    if store_codes:
        d["k_codes"] = kq
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
    return h.hexdigest()


def make_polar(name="polar_cfg3_small", seed=11, Hkv=2, N=40, D=128, H=4, block=128, m=256):
    """PolarQuant + QJL of config-3-shaped keys (7 levels of 16-entry uniform
    codebooks, Gaussian S from default_rng(seed)): packed indices, radii,
    sign bits and residual norms the encoders must reproduce."""
    import math
    k = inputs.make_layer(seed, H, Hkv, D, N)["k"][0]
    c = np.arange(16) + 0.5
    cb = np.stack([c * (2 * math.pi / 16)] + [c * (math.pi / 2 / 16)] * 6).astype(np.float32)
    _, pk, rad = O.polar_encode(k, block, cb)
    kh = O.polar_decode(pk, rad, D, block, cb)
    S = np.random.default_rng(seed).standard_normal((m, D)).astype(np.float32)
    signs, rn = O.qjl_encode(k, kh, S)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), seed=seed, Hkv=Hkv, N=N, D=D, H=H,
                        block=block, m=m, packed=pk, radii=rad.view(np.uint16), signs=signs,
                        rnorm=rn.view(np.uint16))
    return name


if __name__ == "__main__":
    for c in CASES:
        print(c[0], make(*c))
    print(make_polar())

"""CPU tests of the oracle itself: known-answer tests derived from the task's
quantization spec and from the attention definition, numpy vs C agreement,
and the committed golden fixtures. No GPU."""
import os
from fractions import Fraction

import numpy as np
import pytest

from oracle import inputs, oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _kat_quantize_group(x, sb=np.float16):
    """Independent restatement of the spec with exact rationals: scale and
    bias rounded to `sb`, code = round-half-even((x-b)/s) clamped to 0..15."""
    x32 = np.asarray(x, np.float32)
    mn, mx = x32.min(), x32.max()
    scale = np.float32((mx - mn) / np.float32(15))
    s = Fraction(float(np.asarray(scale).astype(sb).astype(np.float64)))
    b = Fraction(float(np.asarray(mn).astype(sb).astype(np.float64)))
    codes = []
    for v in x32:
        if s == 0:
            codes.append(0)
            continue
        # IEEE fp32 (v - b) then fp32 division, exactly as the spec's fp32 compute
        diff = np.float32(np.float32(v) - np.float32(float(b)))
        q = np.float32(diff / np.float32(float(s)))
        r = Fraction(float(q))
        fl = r.numerator // r.denominator
        frac = r - fl
        c = fl + (1 if frac > Fraction(1, 2) or (frac == Fraction(1, 2) and fl % 2 == 1) else 0)
        codes.append(min(15, max(0, c)))
    return codes, float(s), float(b)


def _unpack_row(words):
    return [(int(w) >> (4 * j)) & 0xF for w in words for j in range(8)]


@pytest.mark.parametrize("case", ["ramp", "ties", "constant", "negative", "random"])
def test_quantize_known_answers(case):
    rng = np.random.default_rng(123)
    if case == "ramp":
        x = np.arange(64, dtype=np.float32)
    elif case == "ties":
        # min 0, max 15 -> scale 1, bias 0: x = k + 0.5 ties to the even code
        x = np.concatenate([[0.0, 15.0], np.arange(62) % 15 + 0.5]).astype(np.float32)
    elif case == "constant":
        x = np.full(64, 3.25, np.float32)
    elif case == "negative":
        x = -np.linspace(0.1, 7.7, 64).astype(np.float32)
    else:
        x = rng.standard_normal(64).astype(np.float32)
    codes, s, b = _kat_quantize_group(x)
    w, sc, bi = O.quantize_np(x[None, :].repeat(2, 0).reshape(1, 128)[:, :128])
    # first group of the row is x
    assert _unpack_row(w[0][:8]) == codes
    assert float(sc[0, 0]) == s and float(bi[0, 0]) == b
    if case == "constant":
        assert s == 0.0 and codes == [0] * 64 and b == 3.25
    if case == "ties":
        assert codes[2] == 0 and codes[3] == 2 and codes[4] == 2 and codes[5] == 4


def test_nibble_order_low_first():
    # element 8w+j at bits 4j..4j+3 (lib/turboquant.metal:796-799)
    x = np.zeros((1, 128), np.float32)
    x[0, :64] = np.arange(64) % 16  # min 0, max 15 -> scale 1, codes = values
    w, s, b = O.quantize_np(x)
    assert float(s[0, 0]) == 1.0 and float(b[0, 0]) == 0.0
    assert int(w[0, 0]) == 0x76543210 and int(w[0, 1]) == 0xFEDCBA98


@pytest.mark.parametrize("sb", [np.float16, np.float32])
def test_quantize_numpy_matches_c(sb):
    L = inputs.make_layer(3, 8, 4, 256, 200)
    for x in (L["k"], L["v"], L["k"] * 1000.0, L["v"] * 1e-3):
        a = O.quantize_np(x, sb)
        c = O.quantize(x, sb)
        for u, v in zip(a, c):
            assert np.array_equal(u.view(np.uint8), v.view(np.uint8))


def test_dequantize_roundtrip_error_bound():
    L = inputs.make_layer(4, 8, 4, 128, 300)
    codes, s, b = O.quantize_np(L["v"])
    xh = O.dequantize_np(codes, s, b)
    sc = np.repeat(s.astype(np.float32), 64, -1)
    # half a step plus the fp16 rounding of scale/bias (max 16 steps' worth)
    bound = 0.5 * sc + 16 * np.abs(sc) * 2.0 ** -11 + np.abs(np.repeat(b.astype(np.float32), 64, -1)) * 2.0 ** -11
    assert np.all(np.abs(xh - L["v"]) <= bound + 1e-6)


def _cache(L, sb=np.float16):
    kq, ks, kb = O.quantize_np(L["k"], sb)
    vq, vs, vb = O.quantize_np(L["v"], sb)
    return kq, ks, kb, vq, vs, vb


def test_sdpa_kat_single_token_returns_v():
    L = inputs.make_layer(5, 4, 2, 128, 1)
    c = _cache(L)
    out = O.sdpa_int4(L["q"], *c, f64=True)
    vh = O.dequantize_np(c[3], c[4], c[5])
    for h in range(4):
        np.testing.assert_allclose(out[0, h], vh[0, h // 2, 0], rtol=0, atol=1e-6)


def test_sdpa_kat_equal_keys_average_values():
    L = inputs.make_layer(6, 4, 2, 128, 37)
    L["k"][:] = L["k"][:, :, :1]  # every key identical -> uniform softmax
    c = _cache(L)
    out = O.sdpa_int4(L["q"], *c, f64=True)
    vh = O.dequantize_np(c[3], c[4], c[5])
    np.testing.assert_allclose(out[0, 0], vh[0, 0].mean(0), rtol=0, atol=1e-5)


def test_sdpa_window_and_empty():
    L = inputs.make_layer(7, 4, 2, 128, 50)
    c = _cache(L)
    vh = O.dequantize_np(c[3], c[4], c[5])
    out = O.sdpa_int4(L["q"], *c, window=1, f64=True)  # only token N-1 visible
    np.testing.assert_allclose(out[0, 3], vh[0, 1, 49], rtol=0, atol=1e-6)
    out0 = O.sdpa_int4(L["q"], *c, n_tokens=[0], f64=True)
    assert np.all(out0 == 0)
    # window rule (N-1-t) >= W masked == explicit slice of the last W tokens
    w = 17
    full = O.sdpa_np(L["q"], O.dequantize_np(*c[:3]), vh, window=w)
    sl = O.sdpa_np(L["q"], O.dequantize_np(*c[:3])[:, :, -w:], vh[:, :, -w:])
    np.testing.assert_allclose(full, sl, rtol=0, atol=1e-6)


def test_sdpa_f32_matches_f64_and_numpy():
    L = inputs.make_layer(0, 32, 16, 128, 1024)
    c = _cache(L)
    q16 = L["q"].astype(np.float16)
    o32 = O.sdpa_int4(q16, *c)
    o64 = O.sdpa_int4(q16, *c, f64=True)
    onp = O.sdpa_np(q16.astype(np.float32), O.dequantize_np(*c[:3]), O.dequantize_np(*c[3:]))
    assert np.max(np.abs(o32 - o64)) < 1e-4
    assert np.max(np.abs(onp - o64)) < 1e-6


def test_reference_kernel_order_close_to_oracle():
    """Oracle B (the reference kernel's arithmetic order,
    lib/turboquant.metal:723-889) sits well inside the 2e-3 tolerance of
    oracle A (dequantize + fp32 SDPA) at config 0 and at the reference's own
    test shape (tests/test_sdpa_int4.cpp:13)."""
    for (H, Hkv, D, N, seed) in [(32, 16, 128, 1024, 0), (16, 16, 256, 10, 1)]:
        L = inputs.make_layer(seed, H, Hkv, D, N)
        c = _cache(L, np.float32)
        q = L["q"][0]
        a = O.sdpa_int4(q[None], *c, f64=True)[0]
        bk = O.reference_kernel(q, *(x[0] for x in c), H // Hkv)
        assert np.max(np.abs(a - bk)) < 1e-4


def test_lse_merge_equals_full_attention():
    L = inputs.make_layer(9, 8, 2, 128, 333)
    kh = O.dequantize_np(*O.quantize_np(L["k"]))[0]
    vh = O.dequantize_np(*O.quantize_np(L["v"]))[0]
    q = L["q"][0]
    full = O.sdpa_np(q[None], kh[None], vh[None])[0]
    bounds = [(0, 100), (100, 100), (100, 250), (250, 333)]  # includes an empty part
    parts = O.split_partials_np(q, kh, vh, bounds)
    np.testing.assert_allclose(O.lse_merge_np(parts, 8, 128), full, rtol=0, atol=1e-6)
    np.testing.assert_allclose(O.lse_merge(parts, 8, 128), full, rtol=0, atol=1e-6)
    empty = O.split_partials_np(q, kh, vh, [(5, 5), (7, 7)])
    assert np.all(O.lse_merge(empty, 8, 128) == 0)


def test_golden_fixtures():
    """Committed fixtures (tests/golden/make_golden.py) still reproduce."""
    files = sorted(f for f in os.listdir(GOLDEN) if f.endswith(".npz") and not f.startswith("polar"))
    assert files, "no golden fixtures committed"
    for f in files:
        g = np.load(os.path.join(GOLDEN, f))
        meta = {k: g[k] for k in g.files}
        L = inputs.make_layer(int(meta["seed"]), int(meta["H"]), int(meta["Hkv"]), int(meta["D"]),
                              int(meta["N"]))
        sb = np.float16 if int(meta["sb_f16"]) else np.float32
        kq, ks, kb = O.quantize(L["k"], sb)
        vq, vs, vb = O.quantize(L["v"], sb)
        import hashlib
        h = hashlib.sha256()
        for a in (kq, ks, kb, vq, vs, vb):
            h.update(np.ascontiguousarray(a).tobytes())
        assert h.hexdigest() == str(meta["cache_sha256"]), f
        out = O.sdpa_int4(L["q"].astype(np.float16), kq, ks, kb, vq, vs, vb,
                          window=int(meta["window"]), f64=True)
        np.testing.assert_allclose(out, meta["out_f64"], rtol=0, atol=1e-6, err_msg=f)
        if "k_codes" in meta:
            assert np.array_equal(meta["k_codes"], kq)

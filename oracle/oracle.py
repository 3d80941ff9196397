"""CPU oracle for the int4 KV-cache attention path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and the
`--impl reference` arm) may import this module; the product library never does.

Two restatements of the same spec are kept and cross-checked:
  * numpy functions (`*_np`) -- vectorised, used for golden fixtures and
    small cases;
  * the C library oracle/liboracle.so (OpenMP) -- used at full sizes and as
    the timed CPU baseline.

PARITY UNPINNED against the reference's own outputs (Metal/MLX cannot run
here and the reference has no golden vectors); see oracle/tq_oracle.c.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build_oracle

F32, F16, BF16 = 0, 1, 2
_NP_SB = {F32: np.float32, F16: np.float16}

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_oracle.LIB
        if not os.path.exists(path):
            build_oracle.build()
        L = ctypes.CDLL(path)
        P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        L.tqo_quantize_rows.argtypes = [P, I, I64, I, I, P, P, P]
        L.tqo_dequantize_rows.argtypes = [P, P, P, I, I64, I, P]
        L.tqo_sdpa_dense.argtypes = [P, P, P, I, I, I, I, I, P, F, I, I, P]
        L.tqo_sdpa_int4.argtypes = [P, I, P, P, P, P, P, P, I, I, I, I, I, I, P, F, I, I, P, P, P]
        L.tqo_reference_kernel.argtypes = [P, P, P, P, P, P, P, I, I, I, I, F, I, P]
        L.tqo_lse_merge.argtypes = [P, I, I, I, P]
        L.tqo_num_threads.restype = I
        L.tqo_set_num_threads.argtypes = [I]
        L.tqo_f32_to_f16.restype = ctypes.c_uint16
        L.tqo_f32_to_f16.argtypes = [F]
        L.tqo_f32_to_bf16.restype = ctypes.c_uint16
        L.tqo_f32_to_bf16.argtypes = [F]
        _register_polar(L)
        _lib = L
    return _lib


def _register_polar(L):
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    L.tqo_atan2.restype = F
    L.tqo_atan2.argtypes = [F, F]
    L.tqo_polar_encode.argtypes = [P, I64, I, I, P, P, P, P, P]
    L.tqo_polar_decode.argtypes = [P, P, P, I64, I, I, P, P]
    L.tqo_qjl_encode.argtypes = [P, P, I64, I, P, I, P, P]
    L.tqo_compressed_score.argtypes = [P, I, I, I, I, I, I, P, P, P, P, P, P, I, F, P]
    L.tqo_compressed_sdpa.argtypes = [P, I, I, I, I, I, I, P, P, P, P, P, P, I, F, P, P, P, I, P]


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _sb_code(dtype) -> int:
    dt = np.dtype(dtype)
    if dt == np.float32:
        return F32
    if dt == np.float16:
        return F16
    raise ValueError(f"unsupported scale/bias dtype {dt}")


# ---------------------------------------------------------------- quantizer --

def quantize_np(x: np.ndarray, sb_dtype=np.float16):
    """Affine group-64 4-bit quantize of the last axis (MLX quantize(x, 64, 4)
    call sites: engine/gemma4_multilayer.cpp:228-229, tests/test_sdpa_int4.cpp:25-26).

    scale = (max-min)/15, bias = min, rounded to `sb_dtype`; codes from the
    rounded values, ties to even, clamped to 0..15; scale 0 -> codes 0.
    Returns (codes uint32 [..., D/8], scales [..., D/64], biases [..., D/64]).
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, D = x.shape
    assert D % 64 == 0
    g = x.reshape(-1, D // 64, 64)
    mn = g.min(axis=-1)
    mx = g.max(axis=-1)
    scale_f = ((mx - mn) / np.float32(15.0)).astype(np.float32)
    s_st = scale_f.astype(sb_dtype)
    b_st = mn.astype(sb_dtype)
    s = s_st.astype(np.float32)[..., None]
    b = b_st.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        c = np.rint((g - b) / s)
    c = np.where(s == 0, 0.0, np.clip(c, 0.0, 15.0)).astype(np.uint32)
    c = c.reshape(-1, D // 8, 8)
    shifts = (4 * np.arange(8, dtype=np.uint32))
    words = np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)
    return (words.reshape(*lead, D // 8), s_st.reshape(*lead, D // 64),
            b_st.reshape(*lead, D // 64))


def quantize_signed_edge_np(x: np.ndarray, sb_dtype=np.float16):
    """A cache of the kind MLX's affine quantizer is published to write
    (ml-explore/mlx `quantize(x, 64, 4)`, unpinned: the reference clones it at
    HEAD and no reference test fixes its outputs). Per group of 64:
    delta = (max - min)/15; the edge is the extreme of larger magnitude
    (min if |min| > |max|, else max) and the scale carries its sign
    (+delta for the min edge, -delta for the max edge); q0 = round(edge/scale);
    when q0 != 0 the scale becomes edge/q0 (so that 0.0 is exactly
    representable) and the bias is the edge, otherwise the bias is 0. Codes
    round((x - bias)/scale) clamped to 0..15. Arithmetic in fp32, scale and
    bias rounded to `sb_dtype` before the codes are taken (what a reader of
    the cache sees). So half of the groups carry NEGATIVE scales and a bias
    at the group MAXIMUM -- the cases this repo's own quantizer never
    writes. Same return layout as quantize_np."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, D = x.shape
    assert D % 64 == 0
    g = x.reshape(-1, D // 64, 64)
    mn = g.min(axis=-1)
    mx = g.max(axis=-1)
    delta = np.maximum((mx - mn) / np.float32(15.0), np.float32(1e-7)).astype(np.float32)
    use_min = np.abs(mn) > np.abs(mx)
    scale = np.where(use_min, delta, -delta).astype(np.float32)
    edge = np.where(use_min, mn, mx).astype(np.float32)
    q0 = np.rint(edge / scale)
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.where(q0 != 0, edge / np.where(q0 != 0, q0, 1), scale).astype(np.float32)
    bias = np.where(q0 != 0, edge, 0.0).astype(np.float32)
    s_st = scale.astype(sb_dtype)
    b_st = bias.astype(sb_dtype)
    s = s_st.astype(np.float32)[..., None]
    b = b_st.astype(np.float32)[..., None]
    c = np.clip(np.rint((g - b) / s), 0.0, 15.0).astype(np.uint32).reshape(-1, D // 8, 8)
    shifts = (4 * np.arange(8, dtype=np.uint32))
    words = np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)
    return (words.reshape(*lead, D // 8), s_st.reshape(*lead, D // 64),
            b_st.reshape(*lead, D // 64))


def random_affine_cache(rng, lead, D: int, sb_dtype=np.float16, s_lo=0.02, s_hi=0.5,
                        b_sigma=1.0):
    """Arbitrary affine parameters: uniform random codes, scales of random
    sign with log-uniform magnitude in [s_lo, s_hi], biases N(0, b_sigma^2)
    unrelated to the codes (no group minimum or maximum). Returns
    (codes uint32 (*lead, D/8), scales, biases (*lead, D/64))."""
    lead = tuple(lead)
    codes = rng.integers(0, 1 << 32, size=lead + (D // 8,), dtype=np.uint64).astype(np.uint32)
    mag = np.exp(rng.uniform(np.log(s_lo), np.log(s_hi), size=lead + (D // 64,)))
    sign = np.where(rng.random(lead + (D // 64,)) < 0.5, -1.0, 1.0)
    scales = (sign * mag).astype(sb_dtype)
    biases = (rng.standard_normal(lead + (D // 64,)) * b_sigma).astype(sb_dtype)
    return codes, scales, biases


def unpack_np(codes: np.ndarray) -> np.ndarray:
    """uint32 words -> uint8 nibbles, element 8w+j at bits 4j..4j+3."""
    shifts = (4 * np.arange(8, dtype=np.uint32))
    c = (codes[..., None] >> shifts) & np.uint32(0xF)
    return c.reshape(*codes.shape[:-1], codes.shape[-1] * 8).astype(np.uint8)


def dequantize_np(codes, scales, biases) -> np.ndarray:
    """value = scale * code + bias in fp32 (lib/turboquant.metal:718-720)."""
    c = unpack_np(codes).astype(np.float32)
    *lead, D = c.shape
    s = np.repeat(scales.astype(np.float32), 64, axis=-1)
    b = np.repeat(biases.astype(np.float32), 64, axis=-1)
    return (s * c + b).astype(np.float32)


def quantize(x: np.ndarray, sb_dtype=np.float16):
    """C-oracle quantizer (same spec as quantize_np)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, D = x.shape
    rows = int(np.prod(lead)) if lead else 1
    codes = np.zeros((rows, D // 8), np.uint32)
    scales = np.zeros((rows, D // 64), sb_dtype)
    biases = np.zeros((rows, D // 64), sb_dtype)
    lib().tqo_quantize_rows(_ptr(x), F32, rows, D, _sb_code(sb_dtype), _ptr(codes), _ptr(scales),
                            _ptr(biases))
    return (codes.reshape(*lead, D // 8), scales.reshape(*lead, D // 64),
            biases.reshape(*lead, D // 64))


# --------------------------------------------------------------- attention --

def sdpa_np(q, k, v, scale=1.0, window=0, n_tokens=None, f64=True):
    """Single-query SDPA over dense K/V. q (B,H,D); k,v (B,Hkv,N,D).
    GQA head map kv = h // (H/Hkv) (lib/turboquant.metal:745); window rule
    (N-1-t) >= W -> masked (lib/turboquant.metal:779); empty -> 0."""
    dt = np.float64 if f64 else np.float32
    B, H, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    G = H // Hkv
    out = np.zeros((B, H, D), np.float32)
    for b in range(B):
        n = N if n_tokens is None else int(n_tokens[b])
        t0 = max(0, n - window) if window > 0 else 0
        if n - t0 <= 0:
            continue
        kk = k[b, :, t0:n].astype(dt)
        vv = v[b, :, t0:n].astype(dt)
        qq = (q[b].astype(dt) * dt(scale)).reshape(Hkv, G, D)
        s = np.einsum("hgd,htd->hgt", qq, kk)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        o = np.einsum("hgt,htd->hgd", p, vv) / p.sum(axis=-1, keepdims=True)
        out[b] = o.reshape(H, D).astype(np.float32)
    return out


def sdpa_int4(q, kq, ks, kb, vq, vs, vb, scale=1.0, window=0, n_tokens=None, f64=False,
              q_dtype=F32):
    """The reference's baseline path on the CPU, C oracle: dequantize the int4
    cache to fp32 (engine/gemma4_multilayer.cpp:307-308) then SDPA (:349).
    q (B,H,D); cache arrays (B,Hkv,cap,D/8) and (B,Hkv,cap,D/64)."""
    q = np.ascontiguousarray(q)
    B, H, D = q.shape
    Hkv, cap = kq.shape[1], kq.shape[2]
    if n_tokens is None:
        n_tokens = [cap] * B
    nt = np.ascontiguousarray(np.asarray(n_tokens, dtype=np.int32))
    sb = _sb_code(ks.dtype)
    arrs = [np.ascontiguousarray(a) for a in (kq, ks, kb, vq, vs, vb)]
    sk = np.empty((B, Hkv, cap, D), np.float32)
    sv = np.empty((B, Hkv, cap, D), np.float32)
    out = np.empty((B, H, D), np.float32)
    qd = {np.dtype(np.float32): F32, np.dtype(np.float16): F16}[q.dtype]
    lib().tqo_sdpa_int4(_ptr(q), qd, *[_ptr(a) for a in arrs], sb, B, H, Hkv, cap, D, _ptr(nt),
                        float(scale), int(window), int(bool(f64)), _ptr(sk), _ptr(sv), _ptr(out))
    return out


class Int4Baseline:
    """Reusable CPU baseline runner (fixed shapes, preallocated temporaries):
    dequantize then fp32 SDPA, OpenMP over all host threads."""

    def __init__(self, q, kq, ks, kb, vq, vs, vb, scale=1.0, window=0, n_tokens=None):
        self.q = np.ascontiguousarray(q)
        self.B, self.H, self.D = q.shape
        self.Hkv, self.cap = kq.shape[1], kq.shape[2]
        nt = [self.cap] * self.B if n_tokens is None else n_tokens
        self.nt = np.ascontiguousarray(np.asarray(nt, dtype=np.int32))
        self.arrs = [np.ascontiguousarray(a) for a in (kq, ks, kb, vq, vs, vb)]
        self.sb = _sb_code(ks.dtype)
        self.sk = np.empty((self.B, self.Hkv, self.cap, self.D), np.float32)
        self.sv = np.empty_like(self.sk)
        self.out = np.empty((self.B, self.H, self.D), np.float32)
        self.qd = {np.dtype(np.float32): F32, np.dtype(np.float16): F16}[self.q.dtype]
        self.scale, self.window = float(scale), int(window)

    def __call__(self):
        lib().tqo_sdpa_int4(_ptr(self.q), self.qd, *[_ptr(a) for a in self.arrs], self.sb, self.B,
                            self.H, self.Hkv, self.cap, self.D, _ptr(self.nt), self.scale,
                            self.window, 0, _ptr(self.sk), _ptr(self.sv), _ptr(self.out))
        return self.out


def reference_kernel(q, kq, ks, kb, vq, vs, vb, gqa, scale=1.0, window=0):
    """'Oracle B': the reference Metal kernel's own arithmetic order
    (lib/turboquant.metal:723-889), fp32 scales/biases. q (H,D); cache
    (Hkv,N,D/8), (Hkv,N,D/64)."""
    q = np.ascontiguousarray(q, np.float32)
    H, D = q.shape
    N = kq.shape[1]
    arrs = [np.ascontiguousarray(a) for a in (kq, ks.astype(np.float32), kb.astype(np.float32),
                                              vq, vs.astype(np.float32), vb.astype(np.float32))]
    out = np.empty((H, D), np.float32)
    lib().tqo_reference_kernel(_ptr(q), *[_ptr(a) for a in arrs], H, gqa, N, D, float(scale),
                               int(window), _ptr(out))
    return out


# ------------------------------------------------------------------- merge --

def split_partials_np(q, k, v, bounds, scale=1.0):
    """Partial (m, l, o) of single-query attention over token ranges `bounds`
    [(t0, t1), ...]; returns array (P, H*(D+2)) in the merge layout
    (o (H,D) then ml (H,2)); m in natural-log units, o unnormalised. q (H,D);
    k, v (Hkv,N,D)."""
    H, D = q.shape
    Hkv = k.shape[0]
    G = H // Hkv
    out = []
    for (t0, t1) in bounds:
        o = np.zeros((H, D), np.float64)
        ml = np.zeros((H, 2), np.float64)
        ml[:, 0] = -np.inf
        if t1 > t0:
            qq = q.astype(np.float64).reshape(Hkv, G, D) * scale
            s = np.einsum("hgd,htd->hgt", qq, k[:, t0:t1].astype(np.float64))
            m = s.max(axis=-1)
            p = np.exp(s - m[..., None])
            o = np.einsum("hgt,htd->hgd", p, v[:, t0:t1].astype(np.float64)).reshape(H, D)
            ml[:, 0] = m.reshape(H)
            ml[:, 1] = p.sum(axis=-1).reshape(H)
        out.append(np.concatenate([o.reshape(-1), ml.reshape(-1)]).astype(np.float32))
    return np.stack(out)


def lse_merge_np(parts: np.ndarray, H: int, D: int) -> np.ndarray:
    P = parts.shape[0]
    o = parts[:, : H * D].reshape(P, H, D).astype(np.float64)
    ml = parts[:, H * D:].reshape(P, H, 2).astype(np.float64)
    m, l = ml[..., 0], ml[..., 1]
    bad = np.isnan(m).any(axis=0) | np.isnan(l).any(axis=0)  # a NaN state poisons its head
    m = np.where(np.isnan(m), -np.inf, m)
    M = m.max(axis=0)
    ok = np.isfinite(M)
    e = np.where(ok[None], np.exp(m - np.where(ok, M, 0.0)[None]), 0.0)
    L = (e * l).sum(axis=0)
    num = (np.where(e[..., None] == 0, 0.0, e[..., None] * o)).sum(axis=0)
    L = np.where(bad, np.nan, L)
    # the reference's rule: an empty softmax (sum 0) gives 0, a NaN sum stays
    # NaN (lib/turboquant.metal:886)
    with np.errstate(invalid="ignore", divide="ignore"):
        out = np.where((L == 0)[:, None], 0.0, num / np.where(L == 0, 1.0, L)[:, None])
    return out.astype(np.float32)


def lse_merge(parts: np.ndarray, H: int, D: int) -> np.ndarray:
    parts = np.ascontiguousarray(parts, np.float32)
    out = np.empty((H, D), np.float32)
    lib().tqo_lse_merge(_ptr(parts), parts.shape[0], H, D, _ptr(out))
    return out


def num_threads() -> int:
    return lib().tqo_num_threads()


def set_num_threads(n: int) -> None:
    lib().tqo_set_num_threads(int(n))


# ------------------------------------------------------ PolarQuant + QJL --
# (restated in oracle/tq_oracle_polar.c; lib/turboquant.metal:8-224,424-704)

def atan2(y: float, x: float) -> float:
    return float(lib().tqo_atan2(float(y), float(x)))


def polar_encode(y: np.ndarray, block: int, codebooks: np.ndarray, cb_sizes=None):
    """y (..., D) f32 -> (angles uint8 (..., D/block, block-1) level-major,
    packed uint8 (..., D/block, block/2), radii fp16 (..., D/block))."""
    y = np.ascontiguousarray(y, np.float32)
    D = y.shape[-1]
    rows = y.size // D
    nb = D // block
    levels = int(np.log2(block))
    cb = np.zeros((7, 16), np.float32)
    cb[:codebooks.shape[0]] = codebooks
    sizes = np.array(cb_sizes if cb_sizes is not None else [16] * 7, np.int32)
    ang = np.empty(y.shape[:-1] + (nb, block - 1), np.uint8)
    pk = np.empty(y.shape[:-1] + (nb, block // 2), np.uint8)
    rad = np.empty(y.shape[:-1] + (nb,), np.float16)
    lib().tqo_polar_encode(_ptr(y), rows, D, block, _ptr(cb), _ptr(sizes), _ptr(ang), _ptr(pk),
                           _ptr(rad))
    assert levels <= 7
    return ang, pk, rad


def polar_decode(packed: np.ndarray, radii: np.ndarray, D: int, block: int,
                 codebooks: np.ndarray, angles: np.ndarray = None) -> np.ndarray:
    rows = radii.size // (D // block)
    cb = np.zeros((7, 16), np.float32)
    cb[:codebooks.shape[0]] = codebooks
    out = np.empty(radii.shape[:-1] + (D,), np.float32)
    a = None if angles is None else np.ascontiguousarray(angles, np.uint8)
    p = None if angles is not None else np.ascontiguousarray(packed, np.uint8)
    lib().tqo_polar_decode(_ptr(a) if a is not None else None, _ptr(p) if p is not None else None,
                           _ptr(np.ascontiguousarray(radii, np.float16)), rows, D, block, _ptr(cb),
                           _ptr(out))
    return out


def qjl_encode(y: np.ndarray, yhat: np.ndarray, S: np.ndarray):
    """signs uint32 (..., m/32) with bit i = (S (y - yhat))_i >= 0; |y - yhat| fp16."""
    y = np.ascontiguousarray(y, np.float32)
    yhat = np.ascontiguousarray(yhat, np.float32)
    S = np.ascontiguousarray(S, np.float32)
    m, D = S.shape
    rows = y.size // D
    signs = np.empty(y.shape[:-1] + (m // 32,), np.uint32)
    rn = np.empty(y.shape[:-1], np.float16)
    lib().tqo_qjl_encode(_ptr(y), _ptr(yhat), rows, D, _ptr(S), m, _ptr(signs), _ptr(rn))
    return signs, rn


def compressed_score(q, packed, radii, codebooks, block, scale=1.0, signs=None, rnorm=None,
                     S=None, q_dtype=F32):
    """q (H, D) preconditioned; keys packed (Hkv, N, D/block, block/2) ->
    scores (H, N) f32 (fp64 sums)."""
    q = np.ascontiguousarray(q)
    H, D = q.shape
    Hkv, N = radii.shape[0], radii.shape[1]
    cb = np.zeros((7, 16), np.float32)
    cb[:codebooks.shape[0]] = codebooks
    out = np.empty((H, N), np.float32)
    m = 0 if S is None else S.shape[0]
    lib().tqo_compressed_score(
        _ptr(q), q_dtype, H, Hkv, D, N, block, _ptr(np.ascontiguousarray(packed, np.uint8)),
        _ptr(np.ascontiguousarray(radii, np.float16)), _ptr(cb),
        _ptr(signs) if signs is not None else None, _ptr(rnorm) if rnorm is not None else None,
        _ptr(np.ascontiguousarray(S, np.float32)) if S is not None else None, m, float(scale),
        _ptr(out))
    return out


def compressed_sdpa(q, packed, radii, codebooks, block, vq, vs, vb, scale=1.0, signs=None,
                    rnorm=None, S=None, q_dtype=F32):
    q = np.ascontiguousarray(q)
    H, D = q.shape
    Hkv, N = radii.shape[0], radii.shape[1]
    cb = np.zeros((7, 16), np.float32)
    cb[:codebooks.shape[0]] = codebooks
    out = np.empty((H, D), np.float32)
    m = 0 if S is None else S.shape[0]
    Sc = np.ascontiguousarray(S, np.float32) if S is not None else None
    lib().tqo_compressed_sdpa(
        _ptr(q), q_dtype, H, Hkv, D, N, block, _ptr(np.ascontiguousarray(packed, np.uint8)),
        _ptr(np.ascontiguousarray(radii, np.float16)), _ptr(cb),
        _ptr(signs) if signs is not None else None, _ptr(rnorm) if rnorm is not None else None,
        _ptr(Sc) if Sc is not None else None, m, float(scale),
        _ptr(np.ascontiguousarray(vq)), _ptr(np.ascontiguousarray(vs)),
        _ptr(np.ascontiguousarray(vb)), 1 if vs.dtype == np.float32 else 0, _ptr(out))
    return out


def sdpa_multi_f64(q, k, v, scale=1.0, causal=False, pos0=0, window=0, n_tokens=None,
                   rows=64):
    """sdpa_multi_np with BLAS matrix products, `rows` queries at a time (for
    config-2 sizes: 512 queries x 32 heads x 8.7K tokens). Same masks and
    fp64 arithmetic: q (n_q, H, D), k, v (Hkv, N, D) dense."""
    nq, H, D = q.shape
    Hkv = k.shape[0]
    N = k.shape[1] if n_tokens is None else n_tokens
    G = H // Hkv
    out = np.zeros((nq, H, D), np.float32)
    t = np.arange(N)
    for hk in range(Hkv):
        kk = k[hk, :N].astype(np.float64)
        vv = v[hk, :N].astype(np.float64)
        for r0 in range(0, nq, rows):
            r1 = min(nq, r0 + rows)
            qq = q[r0:r1, hk * G:(hk + 1) * G].astype(np.float64).reshape(-1, D) * scale
            s = qq @ kk.T                                    # ((r1-r0)*G, N)
            pos = (pos0 + np.arange(r0, r1)) if causal else np.full(r1 - r0, N - 1)
            vis = t[None, :] <= pos[:, None]
            if window > 0:
                vis &= (pos[:, None] - t[None, :]) < window
            vis = np.repeat(vis, G, axis=0)
            s = np.where(vis, s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            p = np.where(vis, np.exp(s - np.where(np.isfinite(m), m, 0.0)), 0.0)
            l = p.sum(axis=1, keepdims=True)
            o = (p @ vv) / np.where(l == 0, 1.0, l)
            o = np.where(l == 0, 0.0, o)
            out[r0:r1, hk * G:(hk + 1) * G] = o.reshape(r1 - r0, G, D).astype(np.float32)
    return out


def sdpa_multi_np(q, k, v, scale=1.0, causal=False, pos0=0, window=0, n_tokens=None):
    """Many queries against one dense K/V (fp64): q (n_q, H, D), k, v (Hkv, N, D).
    causal: query i at position pos0 + i sees t <= pos0 + i; otherwise every
    query sits at the last token. window > 0 also masks pos - t >= window (the
    masks the engine builds for prefill, engine/gemma4_multilayer.cpp:347-367,
    441-464, and lib/turboquant.metal:779 for decode)."""
    nq, H, D = q.shape
    Hkv = k.shape[0]
    N = k.shape[1] if n_tokens is None else n_tokens
    G = H // Hkv
    qq = q.astype(np.float64).reshape(nq, Hkv, G, D) * scale
    s = np.einsum("qhgd,htd->qhgt", qq, k[:, :N].astype(np.float64))
    t = np.arange(N)
    pos = (pos0 + np.arange(nq)) if causal else np.full(nq, N - 1)
    vis = t[None, :] <= pos[:, None]
    if window > 0:
        vis &= (pos[:, None] - t[None, :]) < window
    s = np.where(vis[:, None, None, :], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.where(np.isfinite(s), np.exp(s - np.where(np.isfinite(m), m, 0)), 0.0)
    l = p.sum(axis=-1, keepdims=True)
    o = np.einsum("qhgt,htd->qhgd", p, v[:, :N].astype(np.float64))
    out = np.where(l == 0, 0.0, o / np.where(l == 0, 1, l))
    return out.reshape(nq, H, D).astype(np.float32)

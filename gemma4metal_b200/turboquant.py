"""Python host mirror of the reference's `turboquant` API over the C ABI.

Same names, argument order and defaults as lib/turboquant.h (MLX arrays become
torch CUDA tensors; torch is only the device-memory/stream plumbing here):

    set_metallib_path(path)                                  lib/turboquant.h:209
    sdpa_int4(queries, k_quant, k_scales, k_biases,
              v_quant, v_scales, v_biases, gqa_factor,
              scale=1.0, sliding_window=0, s=None)           lib/turboquant.h:202-207
    quantize(x, group_size=64, bits=4)                       MLX quantize, engine/gemma4_multilayer.cpp:228
    dequantize(w, scales, biases, group_size=64, bits=4)     MLX dequantize, engine/gemma4_multilayer.cpp:307

plus the pieces the reference does with whole-cache copies or does not have:
`quantize_append` (replaces quantize + concatenate, engine/gemma4_multilayer.cpp:228-240),
`sdpa_int4_partial` / `lse_merge` (sequence-split across GPUs) and `KVCache`
(a preallocated int4 cache). Errors raise RuntimeError, as the reference's
primitives throw std::runtime_error (lib/turboquant.cpp:363-365).

The CUDA library is mandatory: importing this module without
libturboquant_b200.so raises; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libturboquant_b200.so")

F32, F16, BF16 = 0, 1, 2
_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
_TORCH_DT = {v: k for k, v in _DT.items()}

_lib = None


def load_library() -> ctypes.CDLL:
    """Load libturboquant_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m gemma4metal_b200.build` "
            "(the int4 attention path has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, I, I64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    L.tq_last_error.restype = ctypes.c_char_p
    L.tq_version.restype = ctypes.c_char_p
    L.tq_set_metallib_path.argtypes = [ctypes.c_char_p]
    L.tq_quantize.argtypes = [P, I, I64, I, P, P, P, I, P]
    L.tq_dequantize.argtypes = [P, P, P, I, I64, I, P, I, P]
    L.tq_quantize_append.argtypes = [P, P, I, I, I, I, I, P, P, P, P, P, P, I, I, I, P, P]
    L.tq_sdpa_int4_workspace_size.restype = SZ
    L.tq_sdpa_int4_workspace_size.argtypes = [I, I, I, I, I, I]
    L.tq_workspace_init.argtypes = [P, SZ, P]
    L.tq_sdpa_int4.argtypes = [P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I, P, P, I, P, SZ, P]
    L.tq_peer_buffer_bytes.restype = SZ
    L.tq_peer_buffer_bytes.argtypes = [I, I, I, I]
    L.tq_peer_buffer_alloc.argtypes = [SZ, ctypes.POINTER(ctypes.c_void_p)]
    L.tq_peer_buffer_free.argtypes = [P]
    L.tq_ipc_handle.argtypes = [P, P]
    L.tq_ipc_open.argtypes = [P, ctypes.POINTER(ctypes.c_void_p)]
    L.tq_ipc_close.argtypes = [P]
    L.tq_peer_merge.argtypes = [P, P, I, I, I, I, I, P, I, I, P]
    L.tq_sdpa_int4_append_at.argtypes = [P, I, P, P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I,
                                         I, P, I, P, SZ, P]
    L.tq_sdpa_int4_append.argtypes = [P, I, P, P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I,
                                      P, P, I, P, SZ, P]
    L.tq_sdpa_int4_partial.argtypes = [P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I, I, I, P,
                                       P, SZ, P]
    L.tq_sdpa_int4_partial_publish.argtypes = [P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I,
                                               I, I, P, P, I, P, I, I, P, SZ, P]
    L.tq_peer_merge_published.argtypes = [P, I, I, I, I, I, P, I, I, P]
    L.tq_peer_gather_published.argtypes = [P, I, I, I, I, I, P, I, I, P]
    L.tq_lse_merge.argtypes = [P, I, I, I, I, P, I, P]
    L.tq_device_error.argtypes = [P, ctypes.POINTER(ctypes.c_uint32)]
    _register_extra(L)
    _lib = L
    return L


def _register_extra(L) -> None:
    """Bind the PolarQuant / QJL entry points."""
    P, I, I64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    L.tq_polar_encode.argtypes = [P, I64, I, I, P, P, P, P, P, P]
    L.tq_polar_decode.argtypes = [P, P, P, I64, I, I, P, P, P]
    L.tq_qjl_encode.argtypes = [P, P, I64, I, P, I, P, P, P]
    L.tq_compressed_score.argtypes = [P, I, P, P, P, P, P, I, I, I, I, I, I, P, F, P, P]
    L.tq_compressed_sdpa_workspace_size.restype = SZ
    L.tq_compressed_sdpa_workspace_size.argtypes = [I, I, I, I]
    L.tq_compressed_sdpa.argtypes = [P, I, P, P, P, P, P, I, I, I, I, I, I, P, F, P, P, P, I, P, I,
                                     P, SZ, P]
    L.tq_decode_step_create.argtypes = [I, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I,
                                        ctypes.POINTER(ctypes.c_void_p)]
    L.tq_decode_step_buffers.argtypes = [P, ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.POINTER(ctypes.c_void_p)]
    L.tq_decode_step_run.argtypes = [P, P, P, P, ctypes.POINTER(ctypes.c_int32), P]
    L.tq_decode_step_run_at.argtypes = [P, P, P, P, ctypes.POINTER(ctypes.c_int32),
                                        ctypes.POINTER(ctypes.c_int32), P]
    L.tq_sdpa_int4_append_slots.argtypes = [P, I, P, P, I, P, P, P, P, P, P, I, I, F, I, I, I, I,
                                            I, I, P, P, P, I, P, SZ, P]
    L.tq_decode_step_destroy.argtypes = [P]
    L.tq_read_probe.argtypes = [P, SZ, I, I, P, P]
    L.tq_wait_selftest.argtypes = [I, P, P]
    L.tq_sdpa_int4_multi_workspace_size.restype = SZ
    L.tq_sdpa_int4_multi_workspace_size.argtypes = [I, I, I, I, I]
    L.tq_sdpa_int4_multi.argtypes = [P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I, I, I, P, I,
                                     P, SZ, P]


def _check(rc: int) -> None:
    if rc != 0:
        msg = load_library().tq_last_error().decode()
        raise RuntimeError(f"turboquant error {rc}: {msg}")


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("turboquant tensors must live on a CUDA device")
    if not t.is_contiguous():
        raise RuntimeError("turboquant tensors must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


def _stream(s) -> ctypes.c_void_p:
    if s is None:
        s = torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _dt(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise RuntimeError(f"unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def version() -> str:
    return load_library().tq_version().decode()


def set_metallib_path(path: str) -> None:
    """Kept for source compatibility (lib/turboquant.h:209); kernels are linked in."""
    load_library().tq_set_metallib_path(path.encode())


# -------------------------------------------------------------- quantizer --

def quantize(x: torch.Tensor, group_size: int = 64, bits: int = 4,
             scales_dtype: torch.dtype = torch.float16, s=None):
    """Affine group-64 4-bit quantization of the last axis (MLX quantize
    semantics of the task spec). Returns (codes uint32 [..., D/8],
    scales [..., D/64], biases [..., D/64])."""
    if group_size != 64 or bits != 4:
        raise RuntimeError("only group_size=64, bits=4 is implemented")
    D = x.shape[-1]
    lead = x.shape[:-1]
    rows = int(torch.tensor(lead).prod().item()) if len(lead) else 1
    codes = torch.empty(*lead, D // 8, dtype=torch.int32, device=x.device)
    scales = torch.empty(*lead, D // 64, dtype=scales_dtype, device=x.device)
    biases = torch.empty_like(scales)
    xc = x.contiguous()  # kept alive until the launch is enqueued
    _check(load_library().tq_quantize(_ptr(xc), _dt(x), rows, D, _ptr(codes),
                                      _ptr(scales), _ptr(biases), _dt(scales), _stream(s)))
    return codes, scales, biases


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4, dtype: torch.dtype = torch.float32, s=None) -> torch.Tensor:
    """value = scale * code + bias (lib/turboquant.metal:718-720)."""
    if group_size != 64 or bits != 4:
        raise RuntimeError("only group_size=64, bits=4 is implemented")
    D = w.shape[-1] * 8
    lead = w.shape[:-1]
    rows = int(torch.tensor(lead).prod().item()) if len(lead) else 1
    out = torch.empty(*lead, D, dtype=dtype, device=w.device)
    _check(load_library().tq_dequantize(_ptr(w), _ptr(scales), _ptr(biases), _dt(scales), rows, D,
                                        _ptr(out), _dt(out), _stream(s)))
    return out


# --------------------------------------------------------------- KV cache --

class KVCache:
    """Preallocated int4 KV cache of one attention layer:
    codes (B, Hkv, capacity, D/8) int32 (uint32 bit patterns) and scales/biases
    (B, Hkv, capacity, D/64), the reference's (nkv, N, D/8) layout
    (lib/turboquant.h:197-200) with a fixed capacity instead of a growing
    concatenation (engine/gemma4_multilayer.cpp:230-236)."""

    def __init__(self, batch: int, num_kv_heads: int, head_dim: int, capacity: int,
                 device=None, scales_dtype: torch.dtype = torch.float16):
        if capacity % 4:
            raise RuntimeError("capacity must be a multiple of 4")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.batch, self.num_kv_heads, self.head_dim, self.capacity = batch, num_kv_heads, head_dim, capacity
        shp = (batch, num_kv_heads, capacity)
        self.k_quant = torch.zeros(*shp, head_dim // 8, dtype=torch.int32, device=dev)
        self.v_quant = torch.zeros_like(self.k_quant)
        self.k_scales = torch.zeros(*shp, head_dim // 64, dtype=scales_dtype, device=dev)
        self.k_biases = torch.zeros_like(self.k_scales)
        self.v_scales = torch.zeros_like(self.k_scales)
        self.v_biases = torch.zeros_like(self.k_scales)
        self.length = 0

    def tensors(self):
        return (self.k_quant, self.k_scales, self.k_biases, self.v_quant, self.v_scales,
                self.v_biases)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, pos: Optional[int] = None,
               positions: Optional[torch.Tensor] = None, s=None) -> None:
        """Quantize (B, Hkv, n_new, D) new tokens into slots pos.. (default: the
        current length) and advance the length."""
        if k_new.dim() == 3:
            k_new, v_new = k_new.unsqueeze(0), v_new.unsqueeze(0)
        n_new = k_new.shape[2]
        p = self.length if pos is None else pos
        quantize_append(k_new, v_new, *self.tensors(), pos=p, positions=positions, s=s)
        if positions is None:
            self.length = max(self.length, p + n_new)


class RingKVCache(KVCache):
    """int4 KV cache of a sliding-window layer as a ring of `window` slots
    (batch 1): token t lives in slot t % window, so the cache holds exactly
    the last `window` tokens -- the set the window rule (N-1-t) < W keeps
    (lib/turboquant.metal:779) -- with no copy. The reference keeps the same
    set by concatenating every new token onto the cache and slicing the
    oldest off the front (engine/gemma4_multilayer.cpp:228-249). Attention
    does not depend on the tokens' order, so decode runs over the filled
    slots unmasked."""

    def __init__(self, num_kv_heads: int, head_dim: int, window: int, device=None,
                 scales_dtype: torch.dtype = torch.float16):
        # any window: the token axis is the window rounded up to 4 (16-byte
        # aligned rows per KV head); slots past the window stay unused
        super().__init__(1, num_kv_heads, head_dim, (window + 3) // 4 * 4, device=device,
                         scales_dtype=scales_dtype)
        self.window = window
        self.total = 0  # tokens appended so far (the layer's position)

    @property
    def n_valid(self) -> int:
        return min(self.total, self.window)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, s=None) -> None:  # type: ignore[override]
        """Append (1, Hkv, n, D) tokens at the ring positions (wrapping)."""
        if k_new.dim() == 3:
            k_new, v_new = k_new.unsqueeze(0), v_new.unsqueeze(0)
        n = k_new.shape[2]
        if n > self.window:  # only the last `window` tokens can survive
            k_new, v_new = k_new[:, :, n - self.window:], v_new[:, :, n - self.window:]
            self.total += n - self.window
            n = self.window
        slot = self.total % self.window
        first = min(n, self.window - slot)
        quantize_append(k_new[:, :, :first], v_new[:, :, :first], *self.tensors(), pos=slot, s=s)
        if n > first:
            quantize_append(k_new[:, :, first:], v_new[:, :, first:], *self.tensors(), pos=0, s=s)
        self.total += n
        self.length = self.n_valid

    def decode(self, queries: torch.Tensor, gqa_factor: int, scale: float = 1.0, *,
               out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
               ws: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
        """Decode attention over the window (the ring's filled slots)."""
        return sdpa_int4(queries, *self.tensors(), gqa_factor, scale, 0, s, n_tokens=self.n_valid,
                         out=out, out_dtype=out_dtype, ws=ws)

    def decode_step(self, queries: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                    gqa_factor: int, scale: float = 1.0, *, out: Optional[torch.Tensor] = None,
                    out_dtype: Optional[torch.dtype] = None, ws: Optional[torch.Tensor] = None,
                    s=None) -> torch.Tensor:
        """One decode step in one launch: the new token's K/V (1, Hkv, D) go to
        slot total % window inside the decode kernel, then attention over the
        window."""
        squeeze = queries.dim() == 2
        q = queries.unsqueeze(0) if squeeze else queries
        B, H, D = q.shape
        slot = self.total % self.window
        n = min(self.total + 1, self.window)
        od = out_dtype or q.dtype
        if out is None:
            out = torch.empty(B, H, D, dtype=od, device=q.device)
        nbytes = sdpa_int4_workspace_size(B, H, self.num_kv_heads, D, n, 0)
        if ws is None:
            ws = workspace(q.device, nbytes, s)
        qc, kc, vc = q.contiguous(), k_new.contiguous(), v_new.contiguous()
        _check(load_library().tq_sdpa_int4_append_at(
            _ptr(qc), _dt(q), _ptr(kc), _ptr(vc), _dt(kc), *[_ptr(c) for c in self.tensors()],
            _dt(self.k_scales), int(gqa_factor), float(scale), B, self.num_kv_heads, D, n,
            self.capacity, slot, _ptr(out), _dt(out), _ptr(ws), 0 if ws is None else ws.numel(),
            _stream(s)))
        self.total += 1
        self.length = self.n_valid
        return out[0] if squeeze else out

    def chronological(self):
        """The six cache arrays cut to the valid tokens, oldest first (the
        reference's layout, (1, Hkv, n, ...)), as new tensors."""
        n = self.n_valid
        start = self.total % self.window if self.total > self.window else 0
        idx = (torch.arange(n, device=self.k_quant.device) + start) % self.window
        return tuple(t.index_select(2, idx) for t in self.tensors())


def quantize_append(k_new: torch.Tensor, v_new: torch.Tensor, k_quant, k_scales, k_biases,
                    v_quant, v_scales, v_biases, pos: int = 0,
                    positions: Optional[torch.Tensor] = None, s=None) -> None:
    """Quantize-on-append into a preallocated cache (B, Hkv, capacity, ...).
    k_new, v_new: (B, Hkv, n_new, D)."""
    if k_new.dim() == 3:
        k_new, v_new = k_new.unsqueeze(0), v_new.unsqueeze(0)
    B, Hkv, n_new, D = k_new.shape
    cap = k_quant.shape[-2]
    # contiguous copies of sliced inputs must stay referenced until the launch
    # is enqueued: a temporary freed early could hand its memory to the next one
    kc, vc = k_new.contiguous(), v_new.contiguous()
    _check(load_library().tq_quantize_append(
        _ptr(kc), _ptr(vc), _dt(k_new), B, Hkv, D, n_new,
        _ptr(k_quant), _ptr(k_scales), _ptr(k_biases), _ptr(v_quant), _ptr(v_scales),
        _ptr(v_biases), _dt(k_scales), cap, int(pos), _ptr(positions), _stream(s)))


# -------------------------------------------------------------- attention --

_WS = {}


def workspace(device: torch.device, nbytes: int, s=None) -> Optional[torch.Tensor]:
    """Per-device cached, zero-initialised workspace of at least nbytes."""
    if nbytes == 0:
        return None
    key = (device.index if device.index is not None else torch.cuda.current_device())
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _check(load_library().tq_workspace_init(_ptr(ws), ws.numel(), _stream(s)))
        _WS[key] = ws
    return ws


def sdpa_int4_workspace_size(batch: int, num_heads: int, num_kv_heads: int, head_dim: int,
                             n_tokens: int, sliding_window: int = 0) -> int:
    return int(load_library().tq_sdpa_int4_workspace_size(batch, num_heads, num_kv_heads, head_dim,
                                                          n_tokens, sliding_window))


def sdpa_int4(queries: torch.Tensor, k_quant: torch.Tensor, k_scales: torch.Tensor,
              k_biases: torch.Tensor, v_quant: torch.Tensor, v_scales: torch.Tensor,
              v_biases: torch.Tensor, gqa_factor: int, scale: float = 1.0,
              sliding_window: int = 0, s=None, *, n_tokens: Optional[int] = None,
              seq_lens: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              out_dtype: Optional[torch.dtype] = None,
              ws: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused int4 decode attention (lib/turboquant.h:202-207).

    queries (H, D) with a cache of (Hkv, N, D/8) -- the reference's shapes --
    or batched: queries (B, H, D) with a cache of (B, Hkv, capacity, D/8).
    n_tokens defaults to the cache's token axis. Returns (…, H, D) in
    out_dtype (default: the query dtype)."""
    squeeze = queries.dim() == 2
    q = queries.unsqueeze(0) if squeeze else queries
    cache = [k_quant, k_scales, k_biases, v_quant, v_scales, v_biases]
    if k_quant.dim() == 3:
        cache = [c.unsqueeze(0) for c in cache]
    B, H, D = q.shape
    _, Hkv, cap, _ = cache[0].shape
    n = cap if n_tokens is None else int(n_tokens)
    od = out_dtype or q.dtype
    if out is None:
        out = torch.empty(B, H, D, dtype=od, device=q.device)
    nbytes = sdpa_int4_workspace_size(B, H, Hkv, D, n, sliding_window)
    if ws is None:
        ws = workspace(q.device, nbytes, s)
    qc = q.contiguous()
    _check(load_library().tq_sdpa_int4(
        _ptr(qc), _dt(q), *[_ptr(c) for c in cache], _dt(cache[1]), int(gqa_factor),
        float(scale), int(sliding_window), B, Hkv, D, n, cap, _ptr(seq_lens), _ptr(out), _dt(out),
        _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))
    return out[0] if squeeze else out


def sdpa_int4_append(queries: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                     k_quant, k_scales, k_biases, v_quant, v_scales, v_biases, gqa_factor: int,
                     scale: float = 1.0, sliding_window: int = 0, s=None, *, n_tokens: int,
                     seq_lens: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                     out_dtype: Optional[torch.dtype] = None,
                     ws: Optional[torch.Tensor] = None,
                     slots: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decode step: quantize-on-append of the new token's K/V (B, Hkv, D)
    (or (B, Hkv, 1, D)) into slot n - 1 of a (B, Hkv, capacity, ...) cache,
    then fused int4 decode attention over the n tokens (n = n_tokens, or
    seq_lens[b]); one launch with the tensor-core decode kernel. Same result
    as quantize_append(pos = n - 1) followed by sdpa_int4. slots (device
    int32, one per sequence) puts sequence b's new row at slots[b] instead
    (tq_sdpa_int4_append_slots: ring caches at different positions)."""
    squeeze = queries.dim() == 2
    q = queries.unsqueeze(0) if squeeze else queries
    cache = [k_quant, k_scales, k_biases, v_quant, v_scales, v_biases]
    if k_quant.dim() == 3:
        cache = [c.unsqueeze(0) for c in cache]
    B, H, D = q.shape
    _, Hkv, cap, _ = cache[0].shape
    n = int(n_tokens)
    od = out_dtype or q.dtype
    if out is None:
        out = torch.empty(B, H, D, dtype=od, device=q.device)
    nbytes = sdpa_int4_workspace_size(B, H, Hkv, D, n, sliding_window)
    if ws is None:
        ws = workspace(q.device, nbytes, s)
    # contiguous copies stay referenced until the launch is enqueued
    qc, kc, vc = q.contiguous(), k_new.contiguous(), v_new.contiguous()
    if slots is not None:
        _check(load_library().tq_sdpa_int4_append_slots(
            _ptr(qc), _dt(q), _ptr(kc), _ptr(vc), _dt(kc), *[_ptr(c) for c in cache], _dt(cache[1]),
            int(gqa_factor), float(scale), int(sliding_window), B, Hkv, D, n, cap, _ptr(seq_lens),
            _ptr(slots), _ptr(out), _dt(out), _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))
        return out[0] if squeeze else out
    _check(load_library().tq_sdpa_int4_append(
        _ptr(qc), _dt(q), _ptr(kc), _ptr(vc), _dt(kc), *[_ptr(c) for c in cache], _dt(cache[1]),
        int(gqa_factor), float(scale), int(sliding_window), B, Hkv, D, n, cap, _ptr(seq_lens),
        _ptr(out), _dt(out), _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))
    return out[0] if squeeze else out


class HostDecodeStep:
    """One decode step of one layer from host memory in one call
    (tq_decode_step_*): the host's query and new K/V row go up, the new row is
    quantized into slot n - 1 of `cache` inside the decode kernel, and the
    output comes back to the host -- one CUDA graph launch (H2D copy, fused
    step kernel, D2H copy) and one synchronisation per step. The reference's
    engine makes the same per-token call against unified memory
    (engine/gemma4_multilayer.cpp:222-236).

    Staging buffers (pinned host tensors) are `queries` (B, H, D), `k_new` and
    `v_new` (B, Hkv, D) and `out` (B, H, D): write inputs there and pass
    nothing to run() to skip the host copies, or pass host tensors/arrays.
    A RingKVCache (sliding layer) works too: each run() writes the next
    token at slot total % window and attends over the window."""

    def __init__(self, cache: KVCache, num_heads: int, scale: float = 1.0,
                 sliding_window: int = 0, q_dtype: torch.dtype = torch.float16,
                 new_dtype: torch.dtype = torch.float16,
                 out_dtype: Optional[torch.dtype] = None):
        self.ring = isinstance(cache, RingKVCache)
        if self.ring and sliding_window:
            raise ValueError("a ring cache holds exactly its window: pass sliding_window=0")
        if num_heads % cache.num_kv_heads:
            raise ValueError("num_heads must be a multiple of the cache's kv heads")
        L = load_library()
        self._L = L
        self.cache = cache  # the step holds the cache's device pointers
        self.batch, self.num_heads = cache.batch, num_heads
        od = out_dtype or q_dtype
        handle = ctypes.c_void_p()
        _check(L.tq_decode_step_create(
            _DT[q_dtype], _DT[new_dtype], *[_ptr(t) for t in cache.tensors()], _dt(cache.k_scales),
            num_heads // cache.num_kv_heads, float(scale), int(sliding_window), cache.batch,
            cache.num_kv_heads, cache.head_dim, cache.capacity, _DT[od], ctypes.byref(handle)))
        self._h = handle
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        _check(L.tq_decode_step_buffers(handle, *[ctypes.byref(x) for x in ptrs]))
        B, H, Hkv, D = cache.batch, num_heads, cache.num_kv_heads, cache.head_dim

        def pinned(ptr, shape, dt):
            n = 1
            for x in shape:
                n *= x
            nbytes = n * torch.empty((), dtype=dt).element_size()
            raw = (ctypes.c_char * nbytes).from_address(ptr.value)
            return torch.frombuffer(raw, dtype=torch.uint8).view(dt).view(shape)

        self.queries = pinned(ptrs[0], (B, H, D), q_dtype)
        self.k_new = pinned(ptrs[1], (B, Hkv, D), new_dtype)
        self.v_new = pinned(ptrs[2], (B, Hkv, D), new_dtype)
        self.out = pinned(ptrs[3], (B, H, D), od)
        self._n = (ctypes.c_int32 * B)()
        self._slots = (ctypes.c_int32 * B)()
        self._like = (self.queries, self.k_new, self.v_new, self.out)
        self._seen = [None] * 4
        self._seen_ptr = [0] * 4

    def _host_ptr(self, x, slot: int):
        """Host address of x, checked against staging buffer `slot` (a torch
        tensor already checked in this slot, at the same address, is not
        checked again)."""
        if x is None:
            return None
        like = self._like[slot]
        if isinstance(x, torch.Tensor):
            p = x.data_ptr()
            if x is self._seen[slot] and p == self._seen_ptr[slot]:
                return p
            if x.is_cuda or x.dtype != like.dtype or x.numel() != like.numel() or not x.is_contiguous():
                raise ValueError(f"expected a contiguous host tensor of {like.numel()} {like.dtype}")
            self._seen[slot], self._seen_ptr[slot] = x, p
            return p
        import numpy as np  # numpy arrays of the same element size and count
        if not isinstance(x, np.ndarray) or not x.flags["C_CONTIGUOUS"] or \
                x.size != like.numel() or x.itemsize != like.element_size():
            raise ValueError(f"expected a C-contiguous array of {like.numel()} {like.dtype}")
        return x.ctypes.data

    def run(self, n_tokens=None, queries=None, k_new=None, v_new=None, out=None, slots=None):
        """One step: n_tokens (int, or one per sequence) counts the tokens
        including the new one (default: the cache's length + 1; for a ring
        cache min(total + 1, window)); slots (one per sequence) says where the
        new rows go (default: n - 1; for a ring cache total % window).
        Returns `out` (default: the staging tensor, overwritten by the next
        step)."""
        c = self.cache
        ring_step = self.ring and n_tokens is None and slots is None
        if ring_step:
            n_tokens, slots = min(c.total + 1, c.window), c.total % c.window
        elif n_tokens is None:
            n_tokens = c.length + 1
        if isinstance(n_tokens, int):
            for b in range(self.batch):
                self._n[b] = n_tokens
            n_max = n_tokens
        else:
            if len(n_tokens) != self.batch:
                raise ValueError("n_tokens needs one entry per sequence")
            for b, n in enumerate(n_tokens):
                self._n[b] = int(n)
            n_max = max(int(n) for n in n_tokens)
        args = (self._h, self._host_ptr(queries, 0), self._host_ptr(k_new, 1),
                self._host_ptr(v_new, 2), self._n)
        if slots is None:
            _check(self._L.tq_decode_step_run(*args, self._host_ptr(out, 3)))
        else:
            sl = [slots] * self.batch if isinstance(slots, int) else list(slots)
            if len(sl) != self.batch:
                raise ValueError("slots needs one entry per sequence")
            for b, x in enumerate(sl):
                self._slots[b] = int(x)
            _check(self._L.tq_decode_step_run_at(*args, self._slots, self._host_ptr(out, 3)))
        if ring_step:
            c.total += 1
            c.length = c.n_valid
        elif n_max > c.length:
            c.length = n_max
        return self.out if out is None else out

    def close(self) -> None:
        if self._h:
            _check(self._L.tq_decode_step_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _shard_args(queries, cache, n_local, token_offset, n_total, sliding_window, ws, s):
    q = queries.unsqueeze(0) if queries.dim() == 2 else queries
    cache = list(cache)
    if cache[0].dim() == 3:
        cache = [c.unsqueeze(0) for c in cache]
    B, H, D = q.shape
    _, Hkv, cap, _ = cache[0].shape
    nl = cap if n_local is None else int(n_local)
    nt = token_offset + nl if n_total is None else int(n_total)
    if ws is None:
        ws = workspace(q.device, sdpa_int4_workspace_size(B, H, Hkv, D, nl, sliding_window), s)
    return q, q.contiguous(), cache, B, H, D, Hkv, cap, nl, nt, ws


def sdpa_int4_partial(queries: torch.Tensor, k_quant, k_scales, k_biases, v_quant, v_scales,
                      v_biases, gqa_factor: int, scale: float = 1.0, sliding_window: int = 0,
                      *, n_local: Optional[int] = None, token_offset: int = 0,
                      n_total: Optional[int] = None, part_out: Optional[torch.Tensor] = None,
                      ws: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
    """Partial softmax state of a sequence shard, returned as (B, H*(D+2))
    fp32 in the tq_lse_merge layout."""
    q, qc, cache, B, H, D, Hkv, cap, nl, nt, ws = _shard_args(
        queries, (k_quant, k_scales, k_biases, v_quant, v_scales, v_biases), n_local,
        token_offset, n_total, sliding_window, ws, s)
    if part_out is None:
        part_out = torch.empty(B, H * (D + 2), dtype=torch.float32, device=q.device)
    _check(load_library().tq_sdpa_int4_partial(
        _ptr(qc), _dt(q), *[_ptr(c) for c in cache], _dt(cache[1]), int(gqa_factor),
        float(scale), int(sliding_window), B, Hkv, D, nl, cap, int(token_offset), nt,
        _ptr(part_out), _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))
    return part_out


def sdpa_int4_partial_publish(queries: torch.Tensor, cache, gqa_factor: int, scale: float,
                              sliding_window: int, peer_bufs: torch.Tensor, world: int,
                              rank: int, *, n_local: Optional[int] = None, token_offset: int = 0,
                              n_total: Optional[int] = None, ws: Optional[torch.Tensor] = None,
                              k_new: Optional[torch.Tensor] = None,
                              v_new: Optional[torch.Tensor] = None, s=None) -> None:
    """The shard's partial state, stored by the decode kernel straight into
    every rank's exchange buffer (peer_bufs: device int64 array of the
    world's buffer pointers); tq_peer_merge_published merges it. k_new and
    v_new ((B, Hkv, D), optional) are quantized into slot n_local - 1 in the
    same launch (the rank that holds the sequence's end)."""
    q, qc, cache, B, H, D, Hkv, cap, nl, nt, ws = _shard_args(
        queries, cache, n_local, token_offset, n_total, sliding_window, ws, s)
    kn = None if k_new is None else k_new.contiguous()
    vn = None if v_new is None else v_new.contiguous()
    _check(load_library().tq_sdpa_int4_partial_publish(
        _ptr(qc), _dt(q), *[_ptr(c) for c in cache], _dt(cache[1]), int(gqa_factor),
        float(scale), int(sliding_window), B, Hkv, D, nl, cap, int(token_offset), nt,
        _ptr(kn), _ptr(vn), 0 if kn is None else _dt(kn), peer_bufs.data_ptr(), int(world),
        int(rank), _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))


def lse_merge(parts: torch.Tensor, num_heads: int, head_dim: int,
              out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
              s=None) -> torch.Tensor:
    """Merge partial states parts (P, B, H*(D+2)) into (B, H, D)."""
    if parts.dim() == 2:
        parts = parts.unsqueeze(1)
    P, B, _ = parts.shape
    if out is None:
        out = torch.empty(B, num_heads, head_dim, dtype=out_dtype, device=parts.device)
    _check(load_library().tq_lse_merge(_ptr(parts), P, B, num_heads, head_dim, _ptr(out), _dt(out),
                                       _stream(s)))
    return out


def device_error(s=None) -> int:
    """Read and clear the device error word (0 = no kernel reported an error)."""
    code = ctypes.c_uint32(0)
    _check(load_library().tq_device_error(_stream(s), ctypes.byref(code)))
    return int(code.value)


# ------------------------------------------------------ PolarQuant + QJL --
# The reference's polar_quantize / polar_dequantize / compressed_score /
# compressed_sdpa (lib/turboquant.h:52-165) over the C ABI, generalised to
# blocks of 2^L values, plus the QJL residual sketch. Codebooks and the QJL
# matrix are caller inputs (the reference ships no generator); the helpers
# below give the build's defaults.

def uniform_codebooks(levels: int, device=None) -> torch.Tensor:
    """(levels, 16) fp32 bin centres: level 1 on [0, 2*pi), deeper levels on
    [0, pi/2] (their angles come from non-negative radii)."""
    import math
    c = torch.arange(16, dtype=torch.float64) + 0.5
    rows = [c * (2 * math.pi / 16)] + [c * (math.pi / 2 / 16)] * (levels - 1)
    return torch.stack(rows).float().to(device or "cuda")


def qjl_matrix(m: int, head_dim: int, seed: int, device=None) -> torch.Tensor:
    """Seeded Gaussian JL matrix S (m, head_dim), entries N(0, 1), drawn on the
    host with numpy's default_rng(seed) so every process gets the same S."""
    import numpy as np
    S = np.random.default_rng(seed).standard_normal((m, head_dim)).astype(np.float32)
    return torch.from_numpy(S).to(device or "cuda")


def _cb_host(codebooks: torch.Tensor) -> torch.Tensor:
    """(7, 16) fp32 host copy of the codebooks: the C ABI reads them on the
    host to build the kernels' codebook and cos/sin tables."""
    cb = torch.zeros(7, 16, dtype=torch.float32)
    cb[:codebooks.shape[0]] = codebooks.detach().float().cpu()
    return cb.contiguous()


def _host_ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def polar_quantize(vectors: torch.Tensor, block_size: int, codebooks: torch.Tensor,
                   cb_sizes=None, precondition: Optional[torch.Tensor] = None, s=None):
    """PolarQuant encode of the last axis (lib/turboquant.h:52-59): y = x P^T
    when a preconditioner is given, then per block of block_size values the
    level-major angle indices. Returns (angles uint8 (..., D/block, block-1),
    packed uint8 (..., D/block, block/2), radii fp16 (..., D/block))."""
    y = vectors.float()
    if precondition is not None:
        y = y @ precondition.float().t()
    y = y.contiguous()
    D = y.shape[-1]
    rows = y.numel() // D
    nb = D // block_size
    lead = tuple(y.shape[:-1])
    angles = torch.empty(lead + (nb, block_size - 1), dtype=torch.uint8, device=y.device)
    packed = torch.empty(lead + (nb, block_size // 2), dtype=torch.uint8, device=y.device)
    radii = torch.empty(lead + (nb,), dtype=torch.float16, device=y.device)
    cb = _cb_host(codebooks)
    sizes = None
    if cb_sizes is not None:
        import numpy as np
        sizes = np.ascontiguousarray(np.asarray(cb_sizes, np.int32))
    _check(load_library().tq_polar_encode(
        _ptr(y), rows, D, block_size, _host_ptr(cb),
        sizes.ctypes.data_as(ctypes.c_void_p) if sizes is not None else None,
        _ptr(angles), _ptr(packed), _ptr(radii), _stream(s)))
    return angles, packed, radii


def polar_dequantize(packed: Optional[torch.Tensor], radii: torch.Tensor, head_dim: int,
                     block_size: int, codebooks: torch.Tensor, angles: Optional[torch.Tensor] = None,
                     precondition: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
    """Inverse PolarQuant (lib/turboquant.h:61-72,96-106): (..., head_dim) fp32;
    multiplied by the preconditioner when given (x = y P)."""
    lead = tuple(radii.shape[:-1])
    rows = radii.numel() // (head_dim // block_size)
    y = torch.empty(lead + (head_dim,), dtype=torch.float32, device=radii.device)
    cb = _cb_host(codebooks)
    _check(load_library().tq_polar_decode(
        _ptr(angles) if angles is not None else None, _ptr(packed) if angles is None else None,
        _ptr(radii), rows, head_dim, block_size, _host_ptr(cb), _ptr(y), _stream(s)))
    if precondition is not None:
        y = y @ precondition.float()
    return y


def qjl_encode(y: torch.Tensor, y_hat: torch.Tensor, S: torch.Tensor, s=None):
    """QJL sketch of the residual r = y - y_hat: (sign bits uint32 (..., m/32)
    as int32 bit patterns, |r| fp16 (...))."""
    yc, yh, Sc = y.float().contiguous(), y_hat.float().contiguous(), S.float().contiguous()
    m, D = Sc.shape
    rows = yc.numel() // D
    lead = tuple(yc.shape[:-1])
    signs = torch.empty(lead + (m // 32,), dtype=torch.int32, device=y.device)
    rnorm = torch.empty(lead, dtype=torch.float16, device=y.device)
    _check(load_library().tq_qjl_encode(_ptr(yc), _ptr(yh), rows, D, _ptr(Sc), m, _ptr(signs),
                                        _ptr(rnorm), _stream(s)))
    return signs, rnorm


def compressed_score(queries: torch.Tensor, packed: torch.Tensor, radii: torch.Tensor,
                     codebooks: torch.Tensor, block_size: int, scale: float = 1.0,
                     signs: Optional[torch.Tensor] = None, rnorm: Optional[torch.Tensor] = None,
                     S: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
    """Scores (H, N) of queries (H, D) (preconditioned) against compressed keys
    packed (Hkv, N, D/block, block/2) (lib/turboquant.h:154-162, with GQA and
    the optional QJL correction)."""
    H, D = queries.shape
    Hkv, N = radii.shape[0], radii.shape[1]
    scores = torch.empty(H, N, dtype=torch.float32, device=queries.device)
    qc = queries.contiguous()
    Sc = S.float().contiguous() if S is not None else None
    cb = _cb_host(codebooks)
    _check(load_library().tq_compressed_score(
        _ptr(qc), _dt(qc), _ptr(packed), _ptr(radii), _ptr(signs), _ptr(rnorm), _ptr(Sc),
        0 if Sc is None else Sc.shape[0], H, Hkv, D, N, block_size, _host_ptr(cb),
        float(scale), _ptr(scores), _stream(s)))
    return scores


def compressed_sdpa(queries: torch.Tensor, packed: torch.Tensor, radii: torch.Tensor,
                    codebooks: torch.Tensor, v_quant: torch.Tensor, v_scales: torch.Tensor,
                    v_biases: torch.Tensor, block_size: int, scale: float = 0.0884,
                    signs: Optional[torch.Tensor] = None, rnorm: Optional[torch.Tensor] = None,
                    S: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                    out: Optional[torch.Tensor] = None, ws: Optional[torch.Tensor] = None,
                    s=None) -> torch.Tensor:
    """Compressed-key attention (lib/turboquant.h:129-142): softmax of the
    compressed scores . int4 V (v_quant (Hkv, N, D/8), scales/biases
    (Hkv, N, D/64)). Returns (H, D)."""
    H, D = queries.shape
    Hkv, N = radii.shape[0], radii.shape[1]
    od = out_dtype or queries.dtype
    if out is None:
        out = torch.empty(H, D, dtype=od, device=queries.device)
    nbytes = int(load_library().tq_compressed_sdpa_workspace_size(H, Hkv, D, N))
    if ws is None:
        ws = workspace(queries.device, nbytes, s)
    qc = queries.contiguous()
    Sc = S.float().contiguous() if S is not None else None
    cb = _cb_host(codebooks)
    _check(load_library().tq_compressed_sdpa(
        _ptr(qc), _dt(qc), _ptr(packed), _ptr(radii), _ptr(signs), _ptr(rnorm), _ptr(Sc),
        0 if Sc is None else Sc.shape[0], H, Hkv, D, N, block_size, _host_ptr(cb),
        float(scale), _ptr(v_quant), _ptr(v_scales), _ptr(v_biases), _dt(v_scales), _ptr(out),
        _dt(out), _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))
    return out


# ------------------------------------------- many queries per KV head (tcgen05) --

def sdpa_int4_multi(queries: torch.Tensor, k_quant, k_scales, k_biases, v_quant, v_scales,
                    v_biases, gqa_factor: int, scale: float = 1.0, sliding_window: int = 0, *,
                    n_tokens: Optional[int] = None, causal: bool = False, pos0: int = 0,
                    out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                    ws: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
    """Attention of n_q queries (n_q, H, D) against one int4 cache (Hkv, cap, D/8)
    on the tensor cores: batched decode of many sequences over a shared cache
    (causal=False) or a causal prefill chunk whose query i sits at position
    pos0 + i (causal=True)."""
    cache = [k_quant, k_scales, k_biases, v_quant, v_scales, v_biases]
    if k_quant.dim() == 4:
        cache = [c[0] for c in cache]
    nq, H, D = queries.shape
    Hkv, cap, _ = cache[0].shape
    n = cap if n_tokens is None else int(n_tokens)
    od = out_dtype or queries.dtype
    if out is None:
        out = torch.empty(nq, H, D, dtype=od, device=queries.device)
    nbytes = int(load_library().tq_sdpa_int4_multi_workspace_size(nq, H, Hkv, D, n))
    if ws is None:
        ws = workspace(queries.device, nbytes, s)
    qc = queries.contiguous()
    _check(load_library().tq_sdpa_int4_multi(
        _ptr(qc), _dt(qc), *[_ptr(c) for c in cache], _dt(cache[1]), int(gqa_factor), float(scale),
        int(sliding_window), Hkv, D, nq, n, cap, 1 if causal else 0, int(pos0), _ptr(out),
        _dt(out), _ptr(ws), 0 if ws is None else ws.numel(), _stream(s)))
    return out

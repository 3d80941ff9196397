"""int4 KV caches on disk in the reference engine's format, so a prompt cache
written by one engine loads in the other: one safetensors file holding
`cache_offset` (int32 [1]) and, for every layer L that has a cache,
`l{L}.kq, l{L}.ks, l{L}.kb, l{L}.vq, l{L}.vs, l{L}.vb`
(engine/gemma4_multilayer.cpp:113-144): codes (1, Hkv, T, D/8) uint32 and
scales/biases (1, Hkv, T, D/64) in the cache's float type, T tokens oldest
first (a sliding layer's file holds its last `window` tokens, as the
engine's front trim leaves them, engine/gemma4_multilayer.cpp:242-249).

safetensors layout (written and read here, no dependency): an 8-byte
little-endian header length, a JSON header {name: {dtype, shape,
data_offsets [begin, end)}} padded with spaces to a multiple of 8 bytes, then
the tensors' bytes back to back.
"""
from __future__ import annotations

import json
import struct
from typing import Dict, Mapping, Optional, Tuple, Union

import numpy as np
import torch

from .turboquant import KVCache, RingKVCache

_TO_ST = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.int32: "I32",
          torch.int64: "I64", torch.uint8: "U8", torch.int8: "I8", torch.int16: "I16",
          torch.float64: "F64", torch.bool: "BOOL"}
_FROM_ST = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "I32": torch.int32,
            "U32": torch.int32, "I64": torch.int64, "U8": torch.uint8, "I8": torch.int8,
            "I16": torch.int16, "F64": torch.float64, "BOOL": torch.bool}
_CODES = ("kq", "vq")
_NAMES = ("kq", "ks", "kb", "vq", "vs", "vb")


def write_safetensors(path: str, tensors: Mapping[str, torch.Tensor],
                      dtypes: Optional[Mapping[str, str]] = None,
                      metadata: Optional[Mapping[str, str]] = None) -> None:
    """Write CPU/GPU tensors to `path`. dtypes overrides the stored type name
    per tensor (int32 tensors holding uint32 bit patterns are stored "U32")."""
    header: Dict[str, dict] = {}
    blobs = []
    offset = 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        st = (dtypes or {}).get(name) or _TO_ST[t.dtype]
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": st, "shape": list(t.shape), "data_offsets": [offset, offset + len(raw)]}
        blobs.append(raw)
        offset += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str) -> Tuple[Dict[str, torch.Tensor], Dict[str, str]]:
    """Read every tensor of `path` (CPU tensors; U32 as int32 bit patterns)
    and the stored dtype names."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n).decode())
        data = f.read()
    header.pop("__metadata__", None)
    out, names = {}, {}
    for name, e in header.items():
        b0, b1 = e["data_offsets"]
        if e["dtype"] not in _FROM_ST:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {e['dtype']}")
        dt = _FROM_ST[e["dtype"]]
        buf = np.frombuffer(data[b0:b1], dtype=np.uint8).copy()
        t = torch.from_numpy(buf).view(dt) if buf.size else torch.empty(0, dtype=dt)
        out[name] = t.reshape(e["shape"])
        names[name] = e["dtype"]
    return out, names


def save_kv_cache(path: str, caches: Mapping[int, Union[KVCache, RingKVCache]],
                  cache_offset: int) -> None:
    """Save per-layer caches (batch 1) in the engine's format: the valid
    tokens only, oldest first."""
    tensors: Dict[str, torch.Tensor] = {"cache_offset": torch.tensor([cache_offset], dtype=torch.int32)}
    dtypes: Dict[str, str] = {}
    for layer, c in caches.items():
        if c.batch != 1:
            raise ValueError("the engine's cache format has batch 1")
        arrays = c.chronological() if isinstance(c, RingKVCache) else \
            tuple(t[:, :, :c.length] for t in c.tensors())
        for name, t in zip(_NAMES, arrays):
            key = f"l{layer}.{name}"
            tensors[key] = t
            if name in _CODES:
                dtypes[key] = "U32"
    write_safetensors(path, tensors, dtypes)


def load_kv_cache(path: str, device=None, capacity: Optional[int] = None,
                  windows: Optional[Mapping[int, int]] = None
                  ) -> Tuple[int, Dict[int, Union[KVCache, RingKVCache]]]:
    """Load a cache file written by the engine (or save_kv_cache). Layers in
    `windows` become RingKVCache(window) (their file holds at most the last
    window tokens); the others KVCache with room for `capacity` tokens
    (default: the stored tokens, rounded up to 4). Returns (cache_offset,
    {layer: cache})."""
    data, names = read_safetensors(path)
    offset = int(data["cache_offset"].reshape(-1)[0])
    layers = sorted({int(k[1:].split(".")[0]) for k in data if k.startswith("l") and "." in k})
    caches: Dict[int, Union[KVCache, RingKVCache]] = {}
    for layer in layers:
        arr = [data[f"l{layer}.{n}"] for n in _NAMES]
        for n, t in zip(_NAMES, arr):
            if t.dim() != 4 or t.shape[0] != 1:
                raise ValueError(f"l{layer}.{n}: expected shape (1, Hkv, T, .), got {tuple(t.shape)}")
        _, hkv, T, w8 = arr[0].shape
        D = w8 * 8
        sdt = arr[1].dtype
        if sdt == torch.bfloat16:  # an engine running in bf16; widened exactly (kernels: f16/f32)
            sdt = torch.float32
        if windows and layer in windows:
            W = windows[layer]
            if T > W:
                raise ValueError(f"layer {layer}: {T} tokens do not fit its window {W}")
            c: Union[KVCache, RingKVCache] = RingKVCache(hkv, D, W, device=device, scales_dtype=sdt)
        else:
            cap = max(capacity or 0, (T + 3) // 4 * 4, 4)
            c = KVCache(1, hkv, D, cap, device=device, scales_dtype=sdt)
        for dst, src in zip(c.tensors(), arr):
            dst[:, :, :T].copy_(src.to(dst.dtype) if src.dtype != dst.dtype else src)
        c.length = T
        if isinstance(c, RingKVCache):
            c.total = T
        caches[layer] = c
    return offset, caches

"""The engine's on-disk KV-cache format (engine/gemma4_multilayer.cpp:113-144):
safetensors read/write without a GPU -- round trip of every dtype the cache
uses, uint32 codes, empty tensors, and a file built by hand byte for byte the
way another writer lays it out (no header padding)."""
import json
import struct

import numpy as np
import torch

from gemma4metal_b200.kvstore import read_safetensors, write_safetensors


def test_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    t = {
        "cache_offset": torch.tensor([1234], dtype=torch.int32),
        "l0.kq": torch.randint(-2**31, 2**31 - 1, (1, 4, 10, 16), dtype=torch.int32, generator=g),
        "l0.ks": torch.randn(1, 4, 10, 2, generator=g).half(),
        "l0.kb": torch.randn(1, 4, 10, 2, generator=g).bfloat16(),
        "l3.vs": torch.randn(1, 2, 5, 4, generator=g),
        "empty": torch.empty(0, 3, dtype=torch.float16),
    }
    p = tmp_path / "c.safetensors"
    write_safetensors(str(p), t, {"l0.kq": "U32"})
    raw = p.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    back, names = read_safetensors(str(p))
    assert names["l0.kq"] == "U32" and names["l0.kb"] == "BF16"
    for k, v in t.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert torch.equal(back[k].view(torch.uint8), v.contiguous().view(torch.uint8))


def test_reads_unpadded_foreign_file(tmp_path):
    codes = np.arange(2 * 3 * 8, dtype=np.uint32).reshape(1, 2, 3, 8) * 0x11111111
    scales = np.linspace(-1, 1, 2 * 3 * 2).astype(np.float16).reshape(1, 2, 3, 2)
    off = np.array([7], dtype=np.int32)
    blobs = [off.tobytes(), codes.tobytes(), scales.tobytes()]
    hdr = {"cache_offset": {"dtype": "I32", "shape": [1], "data_offsets": [0, 4]},
           "l0.kq": {"dtype": "U32", "shape": [1, 2, 3, 8], "data_offsets": [4, 4 + len(blobs[1])]},
           "l0.ks": {"dtype": "F16", "shape": [1, 2, 3, 2],
                     "data_offsets": [4 + len(blobs[1]), 4 + len(blobs[1]) + len(blobs[2])]},
           "__metadata__": {"format": "mlx"}}
    h = json.dumps(hdr).encode()
    p = tmp_path / "foreign.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    back, _ = read_safetensors(str(p))
    assert int(back["cache_offset"][0]) == 7
    assert np.array_equal(back["l0.kq"].numpy().view(np.uint32), codes)
    assert np.array_equal(back["l0.ks"].numpy(), scales)

"""Sliding-window layers as a ring of `window` slots (RingKVCache): the
cache holds exactly the last W tokens, which the reference keeps by
concatenating and trimming the front (engine/gemma4_multilayer.cpp:228-249),
and decode over the ring equals decode with the window rule over the whole
sequence. The fused ring step (tq_sdpa_int4_append_at) writes the same bytes
and gives the same output as append + decode. Caches round-trip through the
engine's safetensors format."""
import os

import numpy as np
import pytest
import torch

from oracle import inputs, oracle as O
from tests.conftest import parity

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import kvstore


@pytest.fixture(params=["mma", "simt"])
def variant(request):
    old = os.environ.get("TQ_DECODE_KERNEL")
    os.environ["TQ_DECODE_KERNEL"] = request.param
    yield request.param
    if old is None:
        os.environ.pop("TQ_DECODE_KERNEL", None)
    else:
        os.environ["TQ_DECODE_KERNEL"] = old


def _stream(H, Hkv, D, N, seed):
    L = inputs.make_layer(seed, H, Hkv, D, N)
    k = torch.from_numpy(L["k"]).half().cuda()
    v = torch.from_numpy(L["v"]).half().cuda()
    q = torch.from_numpy(L["q"]).half().cuda()
    return k, v, q


@pytest.mark.parametrize("D,W", [(128, 1024), (256, 512)])
def test_ring_equals_window_over_linear_cache(D, W, variant):
    H, Hkv, N = 32, 16, 2600
    k, v, q = _stream(H, Hkv, D, N, 5)
    ring = tq.RingKVCache(Hkv, D, W)
    lin = tq.KVCache(1, Hkv, D, (N + 3) // 4 * 4)
    # chunks that wrap the ring at uneven points
    bounds = [0, 300, 1000, 1777, 1778, 2600]
    for a, b in zip(bounds, bounds[1:]):
        ring.append(k[:, :, a:b], v[:, :, a:b])
        lin.append(k[:, :, a:b], v[:, :, a:b])
        o_ring = ring.decode(q, H // Hkv, out_dtype=torch.float32)
        o_lin = tq.sdpa_int4(q, *lin.tensors(), H // Hkv, 1.0, W, n_tokens=b,
                             out_dtype=torch.float32)
        torch.cuda.synchronize()
        np.testing.assert_allclose(o_ring.cpu().numpy(), o_lin.cpu().numpy(), rtol=0, atol=2e-5)
    # the ring's chronological contents are the linear cache's last W tokens
    for a, b in zip(ring.chronological(), lin.tensors()):
        assert torch.equal(a, b[:, :, N - W:N])
    assert tq.device_error() == 0


def test_ring_fused_step_equals_append_then_decode(variant):
    H, Hkv, D, W = 32, 16, 128, 256
    N = 700
    k, v, q = _stream(H, Hkv, D, N, 6)
    a = tq.RingKVCache(Hkv, D, W)
    b = tq.RingKVCache(Hkv, D, W)
    a.append(k[:, :, :200], v[:, :, :200])
    b.append(k[:, :, :200], v[:, :, :200])
    for t in range(200, N):  # crosses the wrap twice
        oa = a.decode_step(q, k[:, :, t], v[:, :, t], H // Hkv, out_dtype=torch.float32)
        b.append(k[:, :, t:t + 1], v[:, :, t:t + 1])
        ob = b.decode(q, H // Hkv, out_dtype=torch.float32)
        if t % 97 == 0 or t == N - 1:
            torch.cuda.synchronize()
            assert torch.equal(oa, ob), t
    torch.cuda.synchronize()
    for x, y in zip(a.tensors(), b.tensors()):
        assert torch.equal(x, y)
    assert a.total == b.total == N
    # and against the oracle over the last W tokens
    kk = k[:, :, N - W:].float().cpu().numpy()
    vv = v[:, :, N - W:].float().cpu().numpy()
    ref = O.sdpa_int4(q.float().cpu().numpy(), *O.quantize(kk), *O.quantize(vv), f64=True)
    parity(oa.cpu().numpy(), ref)
    assert tq.device_error() == 0


def test_cache_file_round_trip(tmp_path):
    H, Hkv, D = 32, 16, 128
    k, v, q = _stream(H, Hkv, D, 1500, 8)
    lin = tq.KVCache(1, Hkv, D, 1600)
    lin.append(k, v)
    ring = tq.RingKVCache(Hkv, D, 1024)
    ring.append(k, v)
    p = str(tmp_path / "kv_cache.safetensors")
    kvstore.save_kv_cache(p, {0: ring, 3: lin}, cache_offset=1500)
    off, caches = kvstore.load_kv_cache(p, windows={0: 1024}, capacity=2048)
    assert off == 1500 and sorted(caches) == [0, 3]
    r2, l2 = caches[0], caches[3]
    assert isinstance(r2, tq.RingKVCache) and l2.capacity == 2048 and l2.length == 1500
    for x, y in zip(l2.tensors(), lin.tensors()):
        assert torch.equal(x[:, :, :1500], y[:, :, :1500])
    for x, y in zip(r2.chronological(), ring.chronological()):
        assert torch.equal(x, y)
    o1 = ring.decode(q, H // Hkv, out_dtype=torch.float32)
    o2 = r2.decode(q, H // Hkv, out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_allclose(o1.cpu().numpy(), o2.cpu().numpy(), rtol=0, atol=2e-5)
    # the loaded ring keeps going: its next token replaces the oldest
    r2.append(k[:, :, :1], v[:, :, :1])
    assert r2.n_valid == 1024 and r2.total == 1025

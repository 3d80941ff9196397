"""Decode steps from host memory (tq_decode_step_*, HostDecodeStep): each
run() must leave the same cache bytes and return the same output, bit for
bit, as tq_sdpa_int4_append on device copies of the same inputs (the fused
step of engine/gemma4_multilayer.cpp:222-236), over growing lengths that
cross decode-plan boundaries (graph re-capture), per-sequence lengths,
sliding windows, D = 256 and every way of handing over the host buffers; and
the first step's output must match the oracle."""
import numpy as np
import pytest

from oracle import inputs, oracle as O
from tests.conftest import parity

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gemma4metal_b200.turboquant as tq


def host(t):
    a = t.detach().cpu()
    if a.dtype == torch.bfloat16:
        a = a.float()
    a = a.numpy()
    return a.view(np.uint32) if a.dtype == np.int32 else a


def make_cache(B, Hkv, D, cap, n0, seed, sdt=torch.float16):
    """Two identical caches holding n0 (per sequence: the max) tokens."""
    L = inputs.make_layer(seed, 2 * Hkv, Hkv, D, n0, batch=B)
    a = tq.KVCache(B, Hkv, D, cap, scales_dtype=sdt)
    a.append(torch.from_numpy(L["k"]).cuda(), torch.from_numpy(L["v"]).cuda(), pos=0)
    b = tq.KVCache(B, Hkv, D, cap, scales_dtype=sdt)
    for x, y in zip(b.tensors(), a.tensors()):
        x.copy_(y)
    b.length = a.length
    return a, b


def device_step(cache, q, kn, vn, H, n, window, out_dtype, seq_lens=None):
    sl = None if seq_lens is None else torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    return tq.sdpa_int4_append(q.cuda(), kn.cuda(), vn.cuda(), *cache.tensors(),
                               H // cache.num_kv_heads, 1.0, window, n_tokens=n, seq_lens=sl,
                               out_dtype=out_dtype)


F16, F32 = torch.float16, torch.float32
CASES = [
    # B, H, Hkv, D, cap, n0, steps, window, q dtype, out dtype, scale/bias dtype
    (1, 32, 16, 128, 4096, 1700, 40, 0, F16, F16, F16),             # crosses a plan edge
    (1, 32, 16, 128, 2048, 900, 6, 512, F16, F32, F16),             # sliding window
    (3, 16, 8, 128, 1024, 600, 5, 0, torch.bfloat16, torch.bfloat16, F16),  # per-sequence lengths
    (1, 32, 8, 256, 3072, 2000, 5, 0, F16, F16, F16),               # D = 256
    (1, 32, 16, 128, 2048, 700, 4, 0, F16, F16, F32),               # f32 scales and biases
    (1, 16, 4, 512, 2048, 900, 3, 0, F16, F16, F16),                # D = 512: quantize + CUDA-core decode
]


@pytest.mark.parametrize("B,H,Hkv,D,cap,n0,steps,window,qdt,odt,sdt", CASES)
def test_host_step_matches_device_step(B, H, Hkv, D, cap, n0, steps, window, qdt, odt, sdt):
    rng = np.random.default_rng(n0 + D)
    ca, cb = make_cache(B, Hkv, D, cap, n0, seed=D + B, sdt=sdt)
    step = tq.HostDecodeStep(ca, H, 1.0, window, q_dtype=qdt, new_dtype=torch.float16,
                             out_dtype=odt)
    lens0 = [n0 - 7 * b for b in range(B)]
    for i in range(steps):
        lens = [n + 1 + i for n in lens0]
        q = torch.from_numpy(rng.standard_normal((B, H, D)).astype(np.float32)).to(qdt)
        kn = torch.from_numpy(rng.standard_normal((B, Hkv, D)).astype(np.float32)).half()
        vn = torch.from_numpy(rng.standard_normal((B, Hkv, D)).astype(np.float32)).half()
        # alternate: user host tensors, then inputs written into the staging buffers
        if i % 2 == 0:
            got = step.run(lens if B > 1 else lens[0], q, kn, vn).clone()
        else:
            step.queries.copy_(q)
            step.k_new.copy_(kn)
            step.v_new.copy_(vn)
            got = step.run(lens if B > 1 else lens[0]).clone()
        want = device_step(cb, q, kn, vn, H, max(lens), window, odt,
                           seq_lens=lens if B > 1 else None)
        torch.cuda.synchronize()
        assert torch.equal(got, want.cpu()), f"step {i}: output differs from the device step"
    for x, y in zip(ca.tensors(), cb.tensors()):
        assert torch.equal(x, y), "cache bytes differ from the device step"
    assert ca.length == max(n + steps for n in lens0)
    assert tq.device_error() == 0
    step.close()


def test_host_step_matches_oracle():
    """Config-1 shape: the first step's output against dequantize + fp64 SDPA
    over the cache the step left."""
    H, Hkv, D, N = 32, 16, 128, 3000
    L = inputs.make_layer(11, H, Hkv, D, N)
    cache = tq.KVCache(1, Hkv, D, 3004)
    cache.append(torch.from_numpy(L["k"][:, :, :N - 1]).cuda(),
                 torch.from_numpy(L["v"][:, :, :N - 1]).cuda(), pos=0)
    step = tq.HostDecodeStep(cache, H)
    q = np.ascontiguousarray(L["q"].astype(np.float16))
    kn = np.ascontiguousarray(L["k"][:, :, N - 1].astype(np.float16))
    vn = np.ascontiguousarray(L["v"][:, :, N - 1].astype(np.float16))
    out = np.empty((1, H, D), np.float16)
    step.run(N, q, kn, vn, out)
    hc = [host(t) for t in cache.tensors()]
    ref = O.sdpa_int4(q.astype(np.float32), *hc, n_tokens=[N], f64=True)
    parity(out.astype(np.float32), ref)
    # the appended row equals the quantizer's bytes for it
    kq, ks, kb = O.quantize(L["k"][:, :, N - 1:N].astype(np.float16).astype(np.float32), np.float16)
    assert np.array_equal(hc[0][:, :, N - 1:N], kq)
    assert np.array_equal(hc[1][:, :, N - 1:N], ks)
    step.close()


def test_host_step_rejects_bad_lengths():
    cache = tq.KVCache(1, 16, 128, 64)
    step = tq.HostDecodeStep(cache, 32)
    with pytest.raises(RuntimeError, match="n_tokens"):
        step.run(65)
    with pytest.raises(RuntimeError, match="n_tokens"):
        step.run(0)
    with pytest.raises(ValueError):
        step.run(3, np.zeros((1, 32, 64), np.float16))  # wrong element count
    step.close()
    step.close()  # idempotent


def test_host_step_ring_cache_matches_device_step():
    """A sliding layer's ring cache: each run() writes slot total % W and
    attends over the window; outputs and cache bytes equal
    RingKVCache.decode_step (tq_sdpa_int4_append_at) step by step, across the
    ring's wrap and the decode plans of growing windows."""
    H, Hkv, D, W, n0, steps = 32, 16, 128, 256, 200, 90
    L = inputs.make_layer(17, H, Hkv, D, n0)
    ra = tq.RingKVCache(Hkv, D, W)
    rb = tq.RingKVCache(Hkv, D, W)
    for r in (ra, rb):
        r.append(torch.from_numpy(L["k"]).cuda(), torch.from_numpy(L["v"]).cuda())
    step = tq.HostDecodeStep(ra, H)
    rng = np.random.default_rng(3)
    for i in range(steps):
        q = torch.from_numpy(rng.standard_normal((1, H, D)).astype(np.float32)).half()
        kn = torch.from_numpy(rng.standard_normal((1, Hkv, D)).astype(np.float32)).half()
        vn = torch.from_numpy(rng.standard_normal((1, Hkv, D)).astype(np.float32)).half()
        got = step.run(None, q, kn, vn).clone()
        want = rb.decode_step(q.cuda(), kn.cuda(), vn.cuda(), H // Hkv)
        torch.cuda.synchronize()
        assert torch.equal(got, want.cpu()), f"step {i}: output differs from the device ring step"
    assert ra.total == rb.total == n0 + steps and ra.n_valid == W
    for x, y in zip(ra.tensors(), rb.tensors()):
        assert torch.equal(x, y), "ring bytes differ from the device ring step"
    assert tq.device_error() == 0
    step.close()


def test_host_step_rejects_bad_slots():
    cache = tq.RingKVCache(16, 128, 64)
    step = tq.HostDecodeStep(cache, 32)
    with pytest.raises(RuntimeError, match="slots"):
        step.run(10, slots=10)  # slot must be < n_tokens
    with pytest.raises(RuntimeError, match="slots"):
        step.run(10, slots=-1)
    step.close()

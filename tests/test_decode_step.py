"""One decode step of one layer in one call (tq_sdpa_int4_append): the new
token's K/V row is quantized into slot n - 1 of the cache inside the decode
launch. The cache bytes must equal those of tq_quantize_append (the MLX
quantize + concatenate of engine/gemma4_multilayer.cpp:228-236), the output
must equal tq_sdpa_int4 over that cache bit for bit, and both must match the
oracle's dequantize + fp64 SDPA."""
import os

import numpy as np
import pytest

from oracle import inputs, oracle as O
from tests.conftest import parity

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gemma4metal_b200.turboquant as tq

TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
SBN = {"f16": np.float16, "f32": np.float32}


@pytest.fixture(params=["mma", "simt"])
def variant(request):
    old = os.environ.get("TQ_DECODE_KERNEL")
    os.environ["TQ_DECODE_KERNEL"] = request.param
    yield request.param
    if old is None:
        os.environ.pop("TQ_DECODE_KERNEL", None)
    else:
        os.environ["TQ_DECODE_KERNEL"] = old


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def host(t):
    a = t.detach().cpu()
    if a.dtype == torch.bfloat16:
        a = a.float()
    a = a.numpy()
    return a.view(np.uint32) if a.dtype == np.int32 else a


CASES = [
    # H, Hkv, D, N, window, scales, new-row dtype, batch, seq_lens
    (32, 16, 128, 4096, 0, "f16", "f16", 1, None),
    (32, 16, 128, 4096, 1024, "f16", "f16", 1, None),     # config 1, sliding window
    (32, 16, 128, 1, 0, "f16", "f16", 1, None),           # the new token alone
    (32, 16, 128, 64, 0, "f16", "f32", 1, None),          # new slot closes a 64-token chunk
    (32, 16, 128, 65, 0, "f32", "bf16", 1, None),         # new slot opens a chunk
    (32, 8, 256, 3001, 0, "f16", "f16", 1, None),         # D = 256: two writer warps
    (32, 4, 512, 1500, 1024, "f16", "f16", 1, None),      # D = 512: CUDA-core kernel, 2 launches
    (16, 8, 128, 900, 300, "f16", "f16", 3, [900, 1, 517]),  # per-sequence slots
    (32, 16, 128, 32768, 0, "f16", "f16", 1, None),       # config 1 @ 32K (split over CTAs)
]


@pytest.mark.parametrize("H,Hkv,D,N,window,sb,ndt,B,seq_lens", CASES)
def test_decode_step_matches_append_then_decode(H, Hkv, D, N, window, sb, ndt, B, seq_lens,
                                                variant):
    rng = np.random.default_rng(N + D)
    L = inputs.make_layer(N % 89, H, Hkv, D, N, batch=B)
    lens = seq_lens or [N] * B
    cap = (N + 3) // 4 * 4
    k = np.zeros((B, Hkv, cap, D), np.float32)
    v = np.zeros_like(k)
    k[:, :, :N] = L["k"]
    v[:, :, :N] = L["v"]
    cache = [*O.quantize(k, SBN[sb]), *O.quantize(v, SBN[sb])]
    # slot n - 1 of each sequence holds garbage: the step must overwrite it
    for bi, n in enumerate(lens):
        for a in cache:
            if a.dtype == np.uint32:
                a[bi, :, n - 1] = rng.integers(0, 2**32, a[bi, :, n - 1].shape, dtype=np.uint32)
            else:
                a[bi, :, n - 1] = rng.standard_normal(a[bi, :, n - 1].shape)
    fused = [dev(a) for a in cache]
    split = [dev(a) for a in cache]
    k_new = torch.from_numpy(rng.standard_normal((B, Hkv, D)).astype(np.float32)).to(TDT[ndt]).cuda()
    v_new = torch.from_numpy(rng.standard_normal((B, Hkv, D)).astype(np.float32)).to(TDT[ndt]).cuda()
    q = torch.from_numpy(L["q"]).half().cuda()
    sl = None if seq_lens is None else dev(np.asarray(seq_lens, np.int32))

    out_f = tq.sdpa_int4_append(q, k_new, v_new, *fused, H // Hkv, 1.0, window, n_tokens=N,
                                seq_lens=sl, out_dtype=torch.float32)
    pos = None if seq_lens is None else dev(np.asarray(seq_lens, np.int32) - 1)
    tq.quantize_append(k_new[:, :, None], v_new[:, :, None], *split, pos=N - 1, positions=pos)
    out_s = tq.sdpa_int4(q, *split, H // Hkv, 1.0, window, n_tokens=N, seq_lens=sl,
                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    for a, b in zip(fused, split):
        assert torch.equal(a, b), "cache bytes differ from quantize-on-append"
    assert torch.equal(out_f, out_s), "output differs from append + decode"
    hc = [host(a) for a in fused]
    ref = O.sdpa_int4(q.float().cpu().numpy(), *hc, window=window, n_tokens=lens, f64=True)
    parity(host(out_f), ref)


def test_decode_step_in_cuda_graph():
    """The fused step captured once and replayed: each replay of a fixed-n
    graph rewrites the same slot with the same bytes and gives the same
    output."""
    H, Hkv, D, N = 32, 16, 128, 2048
    L = inputs.make_layer(5, H, Hkv, D, N)
    cache = tq.KVCache(1, Hkv, D, N + 4)
    cache.append(dev(L["k"]).half(), dev(L["v"]).half(), pos=0)
    q = dev(L["q"]).half()
    kn, vn = dev(L["k_new"][:, :, 0]).half(), dev(L["v_new"][:, :, 0]).half()
    out = torch.empty(1, H, D, dtype=torch.float16, device="cuda")
    ws = tq.workspace(q.device, tq.sdpa_int4_workspace_size(1, H, Hkv, D, N + 1))
    tq.sdpa_int4_append(q, kn, vn, *cache.tensors(), H // Hkv, n_tokens=N + 1, out=out, ws=ws)
    torch.cuda.synchronize()
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            tq.sdpa_int4_append(q, kn, vn, *cache.tensors(), H // Hkv, n_tokens=N + 1, out=out,
                                ws=ws, s=s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert tq.device_error() == 0


def test_decode_step_per_sequence_slots(variant):
    """tq_sdpa_int4_append_slots: sequence b's new row goes to slots[b] (a
    device array) and attention runs over its seq_lens[b] tokens; the cache
    bytes and the output equal quantize-on-append at those positions followed
    by the decode, bit for bit."""
    H, Hkv, D, B = 16, 8, 128, 3
    lens = [700, 129, 64]
    slots = [699, 5, 63]  # the end of a sequence, a ring slot behind it, a chunk edge
    N = max(lens)
    L = inputs.make_layer(23, H, Hkv, D, N, batch=B)
    cap = (N + 3) // 4 * 4
    k = np.zeros((B, Hkv, cap, D), np.float32)
    v = np.zeros_like(k)
    k[:, :, :N] = L["k"]
    v[:, :, :N] = L["v"]
    cache = [*O.quantize(k, np.float16), *O.quantize(v, np.float16)]
    fused = [dev(a) for a in cache]
    split = [dev(a) for a in cache]
    rng = np.random.default_rng(9)
    k_new = torch.from_numpy(rng.standard_normal((B, Hkv, D)).astype(np.float32)).half().cuda()
    v_new = torch.from_numpy(rng.standard_normal((B, Hkv, D)).astype(np.float32)).half().cuda()
    q = torch.from_numpy(L["q"]).half().cuda()
    sl = dev(np.asarray(lens, np.int32))
    sp = dev(np.asarray(slots, np.int32))
    out_f = tq.sdpa_int4_append(q, k_new, v_new, *fused, H // Hkv, 1.0, 0, n_tokens=N,
                                seq_lens=sl, slots=sp, out_dtype=torch.float32)
    tq.quantize_append(k_new[:, :, None], v_new[:, :, None], *split, pos=0, positions=sp)
    out_s = tq.sdpa_int4(q, *split, H // Hkv, 1.0, 0, n_tokens=N, seq_lens=sl,
                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    for a, b in zip(fused, split):
        assert torch.equal(a, b), "cache bytes differ from quantize-on-append at the slots"
    assert torch.equal(out_f, out_s), "output differs from append + decode"
    hc = [host(a) for a in fused]
    ref = O.sdpa_int4(q.float().cpu().numpy(), *hc, n_tokens=lens, f64=True)
    parity(host(out_f), ref)

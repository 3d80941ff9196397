"""Many query rows per KV head on the tensor cores (tcgen05 + TMEM): batched
decode of many sequences over one shared int4 cache, and causal prefill
chunks, against the oracle's dequantize + fp64 SDPA with the engine's masks
(engine/gemma4_multilayer.cpp:307-308,347-367,441-464)."""
import numpy as np
import pytest
import torch

from oracle import inputs, oracle as O
from tests.conftest import parity

pytestmark = pytest.mark.gpu

TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def run(nq, H, Hkv, N, causal, pos0, window, qdt, odt, seed=7, sb=np.float16):
    import gemma4metal_b200.turboquant as tq
    L = inputs.make_layer(seed, H, Hkv, 128, N, batch=1)
    qs = inputs.make_layer(seed + 100, H * nq, H * nq, 128, 1)["q"].reshape(nq, H, 128)
    k, v = L["k"][0], L["v"][0]
    kq, ks, kb = O.quantize(k, sb)
    vq, vs, vb = O.quantize(v, sb)
    cap = (N + 3) // 4 * 4
    def dev(a):
        pad = [(0, 0)] * a.ndim
        pad[1] = (0, cap - N)
        a = np.pad(a, pad)
        if a.dtype == np.uint32:
            a = a.view(np.int32)
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q = torch.from_numpy(qs).to(TDT[qdt]).cuda()
    out = tq.sdpa_int4_multi(q, dev(kq), dev(ks), dev(kb), dev(vq), dev(vs), dev(vb), H // Hkv, 1.0,
                             window, n_tokens=N, causal=causal, pos0=pos0, out_dtype=TDT[odt])
    torch.cuda.synchronize()
    ref = O.sdpa_multi_np(q.float().cpu().numpy(), O.dequantize_np(kq, ks, kb),
                          O.dequantize_np(vq, vs, vb), 1.0, causal, pos0, window)
    return out.float().cpu().numpy(), ref


@pytest.mark.parametrize("nq,H,Hkv,N,causal,pos0,window,qdt,odt", [
    (64, 32, 16, 1000, False, 0, 0, "bf16", "f32"),      # batched decode, shared cache
    (64, 32, 16, 1000, False, 0, 300, "f16", "f32"),     # with a sliding window
    (96, 32, 16, 696, True, 600, 0, "bf16", "f32"),      # prefill chunk 600..695 (2 row tiles)
    (40, 16, 4, 777, True, 737, 128, "f16", "f32"),      # GQA 4, causal + window
    (8, 32, 16, 4096, False, 0, 0, "bf16", "f32"),       # few rows: split over the cache
    (3, 8, 8, 65, True, 62, 0, "f16", "f16"),            # GQA 1, tiny, ragged tile
    (50, 24, 8, 900, True, 850, 0, "bf16", "f32"),       # GQA 3: a query's heads straddle row tiles
    (16, 32, 4, 3000, True, 2984, 1000, "bf16", "f32"),  # GQA 8, window cuts into the splits
    (64, 32, 16, 1000, True, 936, 0, "f32", "f32"),      # f32 queries (fp16 hi + lo on the MMA)
    (4, 8, 1, 8192, False, 0, 0, "bf16", "f32"),         # one row tile: 64 splits, two-round merge
])
def test_multi_parity(nq, H, Hkv, N, causal, pos0, window, qdt, odt):
    out, ref = run(nq, H, Hkv, N, causal, pos0, window, qdt, odt)
    parity(out, ref)


def test_multi_f32_scales():
    out, ref = run(64, 32, 16, 1500, False, 0, 0, "f32", "f32", sb=np.float32)
    parity(out, ref)


def test_multi_bf16_output():
    out, ref = run(64, 32, 16, 512, True, 448, 0, "bf16", "bf16")
    parity(out, ref, max_abs=1.6e-2, min_cos=0.9999)  # bf16 output rounding alone is 2^-9


def test_multi_config2_prefill_properties():
    """Config 2's 512-query causal chunk over 8192 + 512 tokens: each query's
    output must equal the single-query decode kernel's output over the
    tokens it can see (a size-independent cross-check between two kernels)."""
    import gemma4metal_b200.turboquant as tq
    H, Hkv, N0, nq = 32, 16, 8192, 512
    N = N0 + nq
    g = torch.Generator(device="cuda").manual_seed(7)
    k = torch.randn(1, Hkv, N, 128, device="cuda", generator=g).half()
    v = torch.randn(1, Hkv, N, 128, device="cuda", generator=g).half()
    cache = tq.KVCache(1, Hkv, 128, N)
    cache.append(k, v, pos=0)
    q = (torch.randn(nq, H, 128, device="cuda", generator=g) * 0.3).bfloat16()
    out = tq.sdpa_int4_multi(q, *cache.tensors(), H // Hkv, 1.0, 0, n_tokens=N, causal=True,
                             pos0=N0, out_dtype=torch.float32)
    for i in (0, 1, 255, 511):
        ref = tq.sdpa_int4(q[i:i + 1].float(), *cache.tensors(), H // Hkv, 1.0, 0,
                           n_tokens=N0 + i + 1, out_dtype=torch.float32)
        parity(out[i].cpu().numpy(), ref[0].cpu().numpy(), max_abs=2e-3, min_cos=0.99999)

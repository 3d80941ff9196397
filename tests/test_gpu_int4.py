"""GPU parity tests of the int4 path through the C ABI (libturboquant_b200.so)
against the CPU oracle: quantize / quantize-on-append bit-exact, decode
attention within max-abs 2e-3 and cosine >= 0.99999 of the oracle's
dequantize + fp64 SDPA (the reference's baseline path,
engine/gemma4_multilayer.cpp:307-308,349)."""
import os

import numpy as np
import pytest

from oracle import inputs, oracle as O
from tests.conftest import parity

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gemma4metal_b200.turboquant as tq


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
    if a.dtype == np.int32:
        a = a.view(np.uint32)
    return a


TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
SBT = {"f16": (torch.float16, np.float16), "f32": (torch.float32, np.float32)}


# ---------------------------------------------------------------- quantize --

@pytest.mark.parametrize("xdt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("sb", ["f16", "f32"])
def test_quantize_bitexact(xdt, sb):
    L = inputs.make_layer(0, 32, 16, 128, 257)
    x = torch.from_numpy(L["k"]).to(TDT[xdt]).cuda()
    codes, s, b = tq.quantize(x, scales_dtype=SBT[sb][0])
    ref = O.quantize(x.float().cpu().numpy(), SBT[sb][1])
    torch.cuda.synchronize()
    assert np.array_equal(host(codes), ref[0])
    assert np.array_equal(host(s).view(np.uint8), ref[1].view(np.uint8))
    assert np.array_equal(host(b).view(np.uint8), ref[2].view(np.uint8))


def test_quantize_edge_rows():
    rng = np.random.default_rng(1)
    rows = [np.full(256, 2.5), np.zeros(256), np.arange(256) % 16 + 0.5, np.arange(256) * 1e4,
            rng.standard_normal(256) * 1e-6, -np.linspace(1, 9, 256), rng.standard_normal(256)]
    x = np.stack(rows).astype(np.float32)
    codes, s, b = tq.quantize(dev(x))
    ref = O.quantize(x)
    assert np.array_equal(host(codes), ref[0])
    assert np.array_equal(host(s).view(np.uint8), ref[1].view(np.uint8))
    assert np.array_equal(host(b).view(np.uint8), ref[2].view(np.uint8))


@pytest.mark.parametrize("odt", ["f32", "f16"])
def test_dequantize_matches_oracle(odt):
    L = inputs.make_layer(2, 8, 4, 256, 33)
    c = O.quantize(L["v"])
    out = tq.dequantize(*[dev(a) for a in c], dtype=TDT[odt])
    ref = O.dequantize_np(*c)
    tol = 0 if odt == "f32" else 2e-3
    np.testing.assert_allclose(host(out).astype(np.float32), ref, rtol=0, atol=tol)


def test_quantize_append_bitexact_and_in_place():
    B, Hkv, D, cap = 3, 4, 128, 64
    cache = tq.KVCache(B, Hkv, D, cap)
    rng = np.random.default_rng(5)
    ref_k = np.zeros((B, Hkv, cap, D), np.float32)
    written = np.zeros((B, cap), bool)
    # prefill 10 tokens, then single-token appends
    for n_new, pos in [(10, 0), (1, 10), (1, 11), (7, 12)]:
        kn = rng.standard_normal((B, Hkv, n_new, D)).astype(np.float32)
        vn = rng.standard_normal((B, Hkv, n_new, D)).astype(np.float32)
        cache.append(dev(kn).half(), dev(vn).half(), pos=pos)
        ref_k[:, :, pos:pos + n_new] = kn.astype(np.float16).astype(np.float32)
        written[:, pos:pos + n_new] = True
    # per-sequence positions (device array)
    posv = np.array([19, 40, 60], np.int32)
    kn = rng.standard_normal((B, Hkv, 2, D)).astype(np.float32)
    cache.append(dev(kn).half(), dev(kn).half(), positions=dev(posv))
    for bb, p in enumerate(posv):
        ref_k[bb, :, p:p + 2] = kn[bb].astype(np.float16).astype(np.float32)
        written[bb, p:p + 2] = True
    torch.cuda.synchronize()
    got = host(cache.k_quant)
    rq, rs, rb = O.quantize(ref_k)
    for bb in range(B):
        w = written[bb]
        assert np.array_equal(got[bb][:, w], rq[bb][:, w])
        assert np.array_equal(host(cache.k_scales)[bb][:, w].view(np.uint16), rs[bb][:, w].view(np.uint16))
        assert np.all(got[bb][:, ~w] == 0)  # untouched slots stay as allocated


def test_quantize_append_noncontiguous_slices():
    # token slices of a (B, Hkv, N, D) tensor are not contiguous: the host
    # wrapper copies them and must keep both copies alive until the launch
    B, Hkv, D, N = 1, 8, 256, 300
    L = inputs.make_layer(6, 16, Hkv, D, N)
    k, v = dev(L["k"]), dev(L["v"])
    cache = tq.KVCache(B, Hkv, D, 128)
    cache.append(k[:, :, 100:200], v[:, :, 100:200], pos=0)
    torch.cuda.synchronize()
    rk = O.quantize(L["k"][:, :, 100:200])
    rv = O.quantize(L["v"][:, :, 100:200])
    assert np.array_equal(host(cache.k_quant)[:, :, :100], rk[0])
    assert np.array_equal(host(cache.v_quant)[:, :, :100], rv[0])
    assert np.array_equal(host(cache.v_scales)[:, :, :100].view(np.uint16), rv[1].view(np.uint16))


# ------------------------------------------------------------------ decode --

@pytest.fixture(params=["mma", "simt"])
def variant(request):
    """Run the test against each decode kernel (tensor-core and CUDA-core)."""
    old = os.environ.get("TQ_DECODE_KERNEL")
    os.environ["TQ_DECODE_KERNEL"] = request.param
    yield request.param
    if old is None:
        os.environ.pop("TQ_DECODE_KERNEL", None)
    else:
        os.environ["TQ_DECODE_KERNEL"] = old


def run_decode(H, Hkv, D, N, seed=0, window=0, sb="f16", qdt="f16", odt="f16", batch=1,
               seq_lens=None, cap=None, scale=1.0, append_last=False):
    L = inputs.make_layer(seed, H, Hkv, D, N, batch=batch)
    sbt, sbn = SBT[sb]
    cap = cap or ((N + 3) // 4 * 4)
    k = np.zeros((batch, Hkv, cap, D), np.float32)
    v = np.zeros_like(k)
    k[:, :, :N] = L["k"]
    v[:, :, :N] = L["v"]
    if append_last:
        # tokens 0..N-2 prefilled by quantize, token N-1 through quantize-on-append
        kq, ks, kb = O.quantize(k, sbn)
        vq, vs, vb = O.quantize(v, sbn)
        dc = [dev(a) for a in (kq, ks, kb, vq, vs, vb)]
        for t in (dc[0], dc[3]):
            t[:, :, N - 1:].zero_()
        kn = torch.from_numpy(L["k"][:, :, N - 1:N]).cuda()
        vn = torch.from_numpy(L["v"][:, :, N - 1:N]).cuda()
        tq.quantize_append(kn, vn, *dc, pos=N - 1)
    else:
        kq, ks, kb = O.quantize(k, sbn)
        vq, vs, vb = O.quantize(v, sbn)
        dc = [dev(a) for a in (kq, ks, kb, vq, vs, vb)]
    q_np = L["q"]
    q = torch.from_numpy(q_np).to(TDT[qdt]).cuda()
    sl = None if seq_lens is None else dev(np.asarray(seq_lens, np.int32))
    out = tq.sdpa_int4(q, *dc, H // Hkv, scale, window, n_tokens=N, seq_lens=sl,
                       out_dtype=TDT[odt])
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    ref = O.sdpa_int4(q.float().cpu().numpy(), kq, ks, kb, vq, vs, vb, scale=scale, window=window,
                      n_tokens=seq_lens if seq_lens is not None else [N] * batch, f64=True)
    return host(out).astype(np.float32), ref


def test_config0_parity(variant):
    cfg = inputs.CONFIGS[0]
    out, ref = run_decode(cfg["H"], cfg["Hkv"], cfg["D"], cfg["N"], seed=cfg["seed"])
    parity(out, ref)


@pytest.mark.parametrize("N", [1024, 4096, 8192, 16384, 32768])
@pytest.mark.parametrize("window", [1024, 0])
def test_config1_sweep(N, window, variant):
    seed = {1024: 1, 4096: 2, 8192: 3, 16384: 4, 32768: 5}[N]
    out, ref = run_decode(32, 16, 128, N, seed=seed, window=window, append_last=True)
    parity(out, ref)


SHAPES = [
    # H, Hkv, D, N, window, sb, qdt, odt
    (8, 8, 128, 1, 0, "f16", "f16", "f16"),
    (8, 4, 128, 5, 0, "f16", "f32", "f32"),
    (16, 4, 128, 63, 0, "f32", "f16", "f16"),
    (16, 2, 128, 64, 0, "f16", "bf16", "bf16"),
    (16, 2, 128, 65, 7, "f16", "f16", "f32"),
    (8, 8, 256, 1000, 100, "f16", "f16", "f16"),
    (16, 8, 256, 777, 0, "f32", "f32", "f32"),
    (32, 8, 256, 3001, 0, "f16", "f16", "f16"),
    (32, 4, 256, 2049, 1024, "f16", "f16", "f16"),
    (4, 4, 512, 300, 0, "f16", "f16", "f16"),
    (8, 4, 512, 513, 0, "f32", "f32", "f32"),
    (16, 4, 512, 4097, 0, "f16", "f16", "f16"),
    (32, 4, 512, 1500, 1024, "f16", "bf16", "f16"),  # Gemma-4 global layer shape (G=8)
    (32, 16, 256, 1500, 1024, "f16", "f16", "f16"),  # Gemma-4 sliding layer shape
    (32, 16, 128, 20000, 30000, "f16", "f16", "f16"),  # window larger than the context
]


@pytest.mark.parametrize("H,Hkv,D,N,window,sb,qdt,odt", SHAPES)
def test_shapes(H, Hkv, D, N, window, sb, qdt, odt, variant):
    out, ref = run_decode(H, Hkv, D, N, seed=N % 97, window=window, sb=sb, qdt=qdt, odt=odt)
    if odt == "bf16":
        parity(out, ref, max_abs=1.6e-2, min_cos=0.9999)  # bf16 output rounding alone is 2^-9
    else:
        parity(out, ref)


def test_reference_test_shape_fp32(variant):
    """Mirror of tests/test_sdpa_int4.cpp:13-45: nh=16, nkv=16, N=10, hd=256,
    gqa=1, scale 1, window 0, fp32 everywhere -- with a seeded input and the
    task tolerance instead of the reference's 0.1 (tests/test_sdpa_int4.cpp:77)."""
    out, ref = run_decode(16, 16, 256, 10, seed=1, sb="f32", qdt="f32", odt="f32")
    parity(out, ref)


def test_batch_with_seq_lens(variant):
    out, ref = run_decode(16, 8, 128, 900, seed=3, batch=3, seq_lens=[900, 1, 517], window=300)
    parity(out, ref)


def test_empty_context_is_zero(variant):
    out, _ = run_decode(8, 4, 128, 8, seq_lens=[0])
    assert np.all(out == 0)


def test_scale_parameter(variant):
    out, ref = run_decode(16, 8, 128, 700, seed=8, scale=0.0884)
    parity(out, ref)


@pytest.mark.parametrize("H,Hkv,D,N,window,batch,seq_lens", [
    (4, 1, 128, 65536, 0, 1, None),          # one unit: ~444 splits, 14 groups
    (4, 1, 256, 40000, 0, 1, None),          # D = 256, ~296 splits
    (8, 2, 128, 50000, 30000, 1, None),      # window inside a long context
    (4, 1, 128, 60000, 0, 2, [60000, 13]),   # the short sequence's splits are empty
])
def test_many_splits_two_level_merge(H, Hkv, D, N, window, batch, seq_lens, variant):
    """Few (sequence, KV head) units over a long context: one wave holds
    hundreds of splits per unit, which the tensor-core kernel merges in two
    levels (groups of 32 splits, then the groups)."""
    out, ref = run_decode(H, Hkv, D, N, seed=N % 89, window=window, batch=batch, seq_lens=seq_lens)
    parity(out, ref)


def test_many_splits_partial_state():
    """The partial state of a one-unit shard with hundreds of splits (two-level
    merge into the tq_lse_merge layout) normalises to the full decode."""
    H, Hkv, D, N = 4, 1, 128, 65536
    L = inputs.make_layer(31, H, Hkv, D, N)
    c = [*O.quantize(L["k"]), *O.quantize(L["v"])]
    dc = [dev(a) for a in c]
    q = torch.from_numpy(L["q"]).half().cuda()
    part = tq.sdpa_int4_partial(q, *dc, H // Hkv, 1.0, 0, n_local=N, token_offset=0, n_total=N)
    merged = tq.lse_merge(part[None], H, D)
    full = tq.sdpa_int4(q, *dc, H // Hkv, 1.0, 0, n_tokens=N, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    np.testing.assert_allclose(host(merged), host(full), rtol=0, atol=2e-5)
    ref = O.sdpa_int4(L["q"].astype(np.float16), *c, n_tokens=[N], f64=True)
    parity(host(merged), ref)


def test_partial_shards_merge_to_full(variant):
    """Sequence split: 3 shards -> partial states -> LSE merge == unsplit."""
    H, Hkv, D, N = 16, 4, 256, 5003
    L = inputs.make_layer(21, H, Hkv, D, N)
    bounds = [(0, 1700), (1700, 3400), (3400, N)]
    q = torch.from_numpy(L["q"]).half().cuda()
    for window in (0, 2000):
        parts = []
        for (t0, t1) in bounds:
            n = t1 - t0
            cap = (n + 3) // 4 * 4
            k = np.zeros((1, Hkv, cap, D), np.float32)
            v = np.zeros_like(k)
            k[:, :, :n] = L["k"][:, :, t0:t1]
            v[:, :, :n] = L["v"][:, :, t0:t1]
            dc = [dev(a) for a in (*O.quantize(k), *O.quantize(v))]
            parts.append(tq.sdpa_int4_partial(q, *dc, H // Hkv, 1.0, window, n_local=n,
                                              token_offset=t0, n_total=N).clone())
        merged = tq.lse_merge(torch.stack(parts), H, D)
        capf = (N + 3) // 4 * 4
        kf = np.zeros((1, Hkv, capf, D), np.float32)
        vf = np.zeros_like(kf)
        kf[:, :, :N] = L["k"]
        vf[:, :, :N] = L["v"]
        c = [*O.quantize(kf), *O.quantize(vf)]
        full = tq.sdpa_int4(q, *[dev(a) for a in c], H // Hkv, 1.0, window, n_tokens=N,
                            out_dtype=torch.float32)
        ref = O.sdpa_int4(L["q"].astype(np.float16), *c, window=window, n_tokens=[N], f64=True)
        torch.cuda.synchronize()
        parity(host(merged), ref)
        np.testing.assert_allclose(host(merged), host(full), rtol=0, atol=2e-5)


def test_graph_capture_replay(variant):
    """append + decode captured in a CUDA graph replay to the same result."""
    H, Hkv, D, N = 32, 16, 128, 4096
    L = inputs.make_layer(4, H, Hkv, D, N)
    cache = tq.KVCache(1, Hkv, D, N + 4)
    cache.append(dev(L["k"]).half(), dev(L["v"]).half(), pos=0)
    q = dev(L["q"]).half()
    kn, vn = dev(L["k_new"]).half(), dev(L["v_new"]).half()
    out = torch.empty(1, H, D, dtype=torch.float16, device="cuda")
    ws = tq.workspace(q.device, tq.sdpa_int4_workspace_size(1, H, Hkv, D, N + 1))
    tq.sdpa_int4(q, *cache.tensors(), H // Hkv, n_tokens=N, out=out, ws=ws)  # eager warm-up
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            tq.quantize_append(kn, vn, *cache.tensors(), pos=N, s=s)
            tq.sdpa_int4(q, *cache.tensors(), H // Hkv, n_tokens=N + 1, out=out, ws=ws, s=s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    eager = tq.sdpa_int4(q, *cache.tensors(), H // Hkv, n_tokens=N + 1)
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    kk = np.concatenate([L["k"], L["k_new"].astype(np.float16).astype(np.float32)], 2)
    vv = np.concatenate([L["v"], L["v_new"].astype(np.float16).astype(np.float32)], 2)
    kk[:, :, :N] = kk[:, :, :N].astype(np.float16).astype(np.float32)
    vv[:, :, :N] = vv[:, :, :N].astype(np.float16).astype(np.float32)
    ref = O.sdpa_int4(L["q"].astype(np.float16), *O.quantize(kk), *O.quantize(vv), f64=True)
    parity(host(out), ref)

"""Parity at the task configs' full sizes and on caches this repo's own
quantizer never writes, all against the CPU oracle (dequantize + fp64 SDPA,
the reference's baseline path, engine/gemma4_multilayer.cpp:307-308,349):

* config 2 at its real shapes on the tcgen05 kernel: 64 sequences x 1 query
  over one 8192-token cache, and the 512-query causal chunk at positions
  8192..8703 whose keys are appended first (RMS-1 queries, scale 1.0, seed 7);
* config 4 at its real shape (262144 tokens, 8 KV heads, 32 query heads,
  head_dim 256, seed 13) on one GPU, whole and split by sequence into 2, 4
  and 8 shards merged by the log-sum-exp kernel;
* decode (both kernels), the fused append step, the ring cache and the
  tcgen05 kernel over caches with arbitrary affine parameters: negative
  scales with the bias at the group maximum (the signed, edge-anchored form
  MLX's quantizer writes, engine/gemma4_multilayer.cpp:228-229), random codes
  with random signed scales and biases unrelated to the codes, fp16 and fp32
  scales.
"""
import os

import numpy as np
import pytest

from oracle import inputs, oracle as O
from tests.conftest import parity

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SB = {"f16": np.float16, "f32": np.float32}


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def raw(t):
    """The tensor's bytes as stored (fp16 stays fp16, int32 codes as uint32)."""
    a = t.detach().cpu().numpy()
    return a.view(np.uint32) if a.dtype == np.int32 else a


def host(t):
    a = t.detach().cpu()
    if a.dtype in (torch.bfloat16, torch.float16):
        a = a.float()
    a = a.numpy()
    if a.dtype == np.int32:
        a = a.view(np.uint32)
    return a


@pytest.fixture(params=["mma", "simt"])
def variant(request):
    """Each decode kernel (tensor-core mma.sync and CUDA-core)."""
    old = os.environ.get("TQ_DECODE_KERNEL")
    os.environ["TQ_DECODE_KERNEL"] = request.param
    yield request.param
    if old is None:
        os.environ.pop("TQ_DECODE_KERNEL", None)
    else:
        os.environ["TQ_DECODE_KERNEL"] = old


def _tq():
    import gemma4metal_b200.turboquant as tq
    return tq


# ------------------------------------------------------------- config 2 --

@pytest.fixture(scope="module")
def cfg2():
    c = inputs.make_config2(seed=7)
    kq = O.quantize(np.concatenate([c["k"], c["k_chunk"]], axis=1))
    vq = O.quantize(np.concatenate([c["v"], c["v_chunk"]], axis=1))
    c["cache"] = (*kq, *vq)
    c["kd"] = O.dequantize_np(*kq)
    c["vd"] = O.dequantize_np(*vq)
    return c


def _bf16_bound(got, ref):
    """bf16 output: round-to-nearest leaves at most 2^-8 |x| (8 significant
    bits), on top of the task's 2e-3 absolute."""
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= 2e-3 + 2.0 ** -8 * np.abs(ref)), float(np.max(err - 2.0 ** -8 * np.abs(ref)))
    cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert cos >= 0.9999, cos


@pytest.mark.parametrize("odt", ["f32", "bf16"])
def test_config2_batched_decode_full(cfg2, odt):
    tq = _tq()
    H, Hkv, N0 = 32, 16, 8192
    cache = [dev(a[:, :N0]) for a in cfg2["cache"]]
    q = torch.from_numpy(cfg2["q_batched"]).bfloat16().cuda()
    od = torch.float32 if odt == "f32" else torch.bfloat16
    out = tq.sdpa_int4_multi(q, *cache, H // Hkv, 1.0, 0, n_tokens=N0, out_dtype=od)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    ref = O.sdpa_multi_f64(q.float().cpu().numpy(), cfg2["kd"][:, :N0], cfg2["vd"][:, :N0], 1.0)
    got = host(out)
    if odt == "f32":
        parity(got, ref)
    else:
        _bf16_bound(got, ref)


@pytest.mark.parametrize("odt", ["f32", "bf16"])
def test_config2_prefill_chunk_full(cfg2, odt):
    """The chunk's 512 keys/values are appended by the GPU quantizer
    (bit-exact with the oracle's), then the 512 causal queries at positions
    8192..8703 attend over 8704 tokens."""
    tq = _tq()
    H, Hkv, N0, C = 32, 16, 8192, 512
    N = N0 + C
    cache = tq.KVCache(1, Hkv, 128, N)
    cache.append(torch.from_numpy(cfg2["k"][None]).cuda(), torch.from_numpy(cfg2["v"][None]).cuda(),
                 pos=0)
    cache.append(torch.from_numpy(cfg2["k_chunk"][None]).cuda(),
                 torch.from_numpy(cfg2["v_chunk"][None]).cuda(), pos=N0)
    torch.cuda.synchronize()
    for got_t, want in zip(cache.tensors(), cfg2["cache"]):
        g = raw(got_t)[0]
        assert np.array_equal(g.view(np.uint8), np.ascontiguousarray(want).view(np.uint8))
    q = torch.from_numpy(cfg2["q_chunk"]).bfloat16().cuda()
    od = torch.float32 if odt == "f32" else torch.bfloat16
    out = tq.sdpa_int4_multi(q, *cache.tensors(), H // Hkv, 1.0, 0, n_tokens=N, causal=True,
                             pos0=N0, out_dtype=od)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    ref = O.sdpa_multi_f64(q.float().cpu().numpy(), cfg2["kd"], cfg2["vd"], 1.0, causal=True,
                           pos0=N0)
    got = host(out)
    if odt == "f32":
        parity(got, ref)
    else:
        _bf16_bound(got, ref)


# ------------------------------------------------------------- config 4 --

C4 = dict(H=32, Hkv=8, D=256, N=262144, seed=13)
NAMES = ("kq", "ks", "kb", "vq", "vs", "vb")


@pytest.fixture(scope="module")
def cfg4():
    L = inputs.make_long_layer(C4["seed"], C4["H"], C4["Hkv"], C4["D"], C4["N"], O.quantize)
    q16 = L["q"].astype(np.float16)
    G = C4["H"] // C4["Hkv"]
    refs = []
    for g0 in range(0, C4["Hkv"], 2):  # two KV heads at a time bound the oracle's scratch
        sl = slice(g0, g0 + 2)
        refs.append(O.sdpa_int4(q16[:, g0 * G:(g0 + 2) * G], *(L[n][:, sl] for n in NAMES),
                                f64=True))
    L["ref"] = np.concatenate(refs, axis=1)
    L["q16"] = q16
    return L


@pytest.mark.parametrize("parts", [1, 2, 4, 8])
def test_config4_full_sequence_split(cfg4, parts):
    """Config 4 at full size on one GPU: parts = 1 runs the whole 262144
    tokens through tq_sdpa_int4; parts > 1 runs tq_sdpa_int4_partial on each
    shard (the 64-token-aligned bounds the multi-GPU split uses) and merges
    the fp32 states with tq_lse_merge, as the ranks of the split do."""
    tq = _tq()
    from gemma4metal_b200 import seqsplit
    H, Hkv, D, N = C4["H"], C4["Hkv"], C4["D"], C4["N"]
    q = torch.from_numpy(cfg4["q16"]).cuda()
    if parts == 1:
        cache = [dev(cfg4[n]) for n in NAMES]
        out = tq.sdpa_int4(q, *cache, H // Hkv, 1.0, 0, n_tokens=N, out_dtype=torch.float32)
    else:
        states, shards = [], []  # shards stay referenced until the kernels have run
        for r in range(parts):
            t0, t1 = seqsplit.shard_bounds(N, parts, r)
            cap = (t1 - t0 + 3) // 4 * 4
            shard = []
            for n in NAMES:
                a = np.zeros((1, Hkv, cap) + cfg4[n].shape[3:], cfg4[n].dtype)
                a[:, :, :t1 - t0] = cfg4[n][:, :, t0:t1]
                shard.append(dev(a))
            states.append(tq.sdpa_int4_partial(q, *shard, H // Hkv, 1.0, 0, n_local=t1 - t0,
                                               token_offset=t0, n_total=N).reshape(1, -1))
            shards.append(shard)
        out = tq.lse_merge(torch.stack(states), H, D, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    parity(host(out).reshape(1, H, D), cfg4["ref"])


# ------------------------------------------- arbitrary affine parameters --

def _affine(kind, lead, D, sb, seed):
    """(kq, ks, kb, vq, vs, vb) over the token axis of `lead`."""
    rng = np.random.default_rng(seed)
    if kind == "signed_edge":
        L = inputs.make_layer(seed, 2, lead[1], D, lead[2], batch=lead[0])
        return (*O.quantize_signed_edge_np(L["k"], SB[sb]),
                *O.quantize_signed_edge_np(L["v"], SB[sb]))
    if kind == "random":
        return (*O.random_affine_cache(rng, lead, D, SB[sb], 0.02, 0.35, 0.5),
                *O.random_affine_cache(rng, lead, D, SB[sb], 0.02, 0.35, 1.0))
    if kind == "wide":  # fp32 parameters far from the fp16 grid and the codes' range
        return (*O.random_affine_cache(rng, lead, D, SB[sb], 1e-3, 4.0, 8.0),
                *O.random_affine_cache(rng, lead, D, SB[sb], 1e-3, 4.0, 8.0))
    raise ValueError(kind)


AFFINE_DECODE = [
    # kind, sb, H, Hkv, D, N, window
    ("signed_edge", "f16", 32, 16, 128, 4099, 0),
    ("signed_edge", "f32", 32, 16, 128, 2048, 1024),
    ("signed_edge", "f16", 32, 8, 256, 3001, 0),
    ("signed_edge", "f16", 8, 1, 128, 1500, 0),
    ("signed_edge", "f16", 16, 4, 512, 1200, 0),
    ("random", "f16", 32, 16, 128, 5000, 0),
    ("random", "f32", 32, 8, 256, 2500, 700),
    ("random", "f16", 16, 16, 128, 777, 0),
    ("wide", "f32", 32, 16, 128, 3000, 0),
]


@pytest.mark.parametrize("kind,sb,H,Hkv,D,N,window", AFFINE_DECODE)
def test_affine_cache_decode(variant, kind, sb, H, Hkv, D, N, window):
    tq = _tq()
    cap = (N + 3) // 4 * 4
    c = _affine(kind, (1, Hkv, cap), D, sb, seed=N + H)
    L = inputs.make_layer(N, H, Hkv, D, 1)
    q = torch.from_numpy(L["q"]).half().cuda()
    out = tq.sdpa_int4(q, *[dev(a) for a in c], H // Hkv, 1.0, window, n_tokens=N,
                       out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    ref = O.sdpa_int4(q.float().cpu().numpy(), *c, window=window, n_tokens=[N], f64=True)
    parity(host(out), ref)


@pytest.mark.parametrize("kind,sb,D", [("signed_edge", "f16", 128), ("random", "f32", 256),
                                       ("signed_edge", "f32", 128)])
def test_affine_cache_fused_append_step(kind, sb, D):
    """The fused step writes the new row with this repo's quantizer into a
    cache whose older rows carry arbitrary affine parameters."""
    tq = _tq()
    H, Hkv, N = 32, 16 if D == 128 else 8, 3333
    cap = (N + 3) // 4 * 4
    c = [np.ascontiguousarray(a) for a in _affine(kind, (1, Hkv, cap), D, sb, seed=77 + D)]
    L = inputs.make_layer(78, H, Hkv, D, 1)
    q = torch.from_numpy(L["q"]).half().cuda()
    dc = [dev(a) for a in c]
    out = tq.sdpa_int4_append(q, torch.from_numpy(L["k_new"][:, :, 0]).cuda(),
                              torch.from_numpy(L["v_new"][:, :, 0]).cuda(), *dc, H // Hkv, 1.0, 0,
                              n_tokens=N, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    nk = O.quantize(L["k_new"], SB[sb])
    nv = O.quantize(L["v_new"], SB[sb])
    for a, new in zip(c, (*nk, *nv)):
        a[:, :, N - 1:N] = new
    for got_t, want in zip(dc, c):
        assert np.array_equal(raw(got_t).view(np.uint8), want.view(np.uint8))
    ref = O.sdpa_int4(q.float().cpu().numpy(), *c, n_tokens=[N], f64=True)
    parity(host(out), ref)


@pytest.mark.parametrize("kind,sb", [("signed_edge", "f16"), ("random", "f32")])
def test_affine_cache_ring_step(kind, sb):
    """A sliding layer's ring (1024 slots, 5000 tokens seen) whose slots hold
    arbitrary affine rows; one fused step writes slot 5000 % 1024 and attends
    over the ring."""
    tq = _tq()
    H, Hkv, D, W = 32, 16, 128, 1024
    ring = tq.RingKVCache(Hkv, D, W, scales_dtype=torch.float16 if sb == "f16" else torch.float32)
    c = _affine(kind, (1, Hkv, W), D, sb, seed=91)
    for t, a in zip(ring.tensors(), c):
        t.copy_(dev(a))
    ring.total = 5000
    ring.length = ring.n_valid
    L = inputs.make_layer(92, H, Hkv, D, 1)
    q = torch.from_numpy(L["q"]).half().cuda()
    out = ring.decode_step(q, torch.from_numpy(L["k_new"][:, :, 0]).cuda(),
                           torch.from_numpy(L["v_new"][:, :, 0]).cuda(), H // Hkv,
                           out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    slot = 5000 % W
    cc = [np.ascontiguousarray(a) for a in c]
    for a, new in zip(cc, (*O.quantize(L["k_new"], SB[sb]), *O.quantize(L["v_new"], SB[sb]))):
        a[:, :, slot:slot + 1] = new
    for got_t, want in zip(ring.tensors(), cc):
        assert np.array_equal(raw(got_t).view(np.uint8), want.view(np.uint8))
    ref = O.sdpa_int4(q.float().cpu().numpy(), *cc, n_tokens=[W], f64=True)
    parity(host(out), ref)


@pytest.mark.parametrize("kind,sb,nq,H,Hkv,N,causal,pos0,window", [
    ("signed_edge", "f16", 64, 32, 16, 4000, False, 0, 0),
    ("signed_edge", "f32", 128, 32, 16, 2000, True, 1872, 0),
    ("random", "f16", 64, 32, 16, 3000, False, 0, 500),
    ("random", "f32", 40, 16, 4, 777, True, 737, 128),
])
def test_affine_cache_tcgen05(kind, sb, nq, H, Hkv, N, causal, pos0, window):
    tq = _tq()
    cap = (N + 3) // 4 * 4
    c = [a[0] for a in _affine(kind, (1, Hkv, cap), 128, sb, seed=nq + N)]
    qs = inputs.make_layer(nq + 5, H * nq, H * nq, 128, 1)["q"].reshape(nq, H, 128)
    q = torch.from_numpy(qs).bfloat16().cuda()
    out = tq.sdpa_int4_multi(q, *[dev(a) for a in c], H // Hkv, 1.0, window, n_tokens=N,
                             causal=causal, pos0=pos0, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    ref = O.sdpa_multi_f64(q.float().cpu().numpy(), O.dequantize_np(c[0], c[1], c[2]),
                           O.dequantize_np(c[3], c[4], c[5]), 1.0, causal, pos0, window, N)
    parity(host(out), ref)

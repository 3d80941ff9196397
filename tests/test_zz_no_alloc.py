"""tq_sdpa_int4_noalloc: the decode entry point for callers that cannot
allocate device memory (its split-KV scratch is an array built into the
library). Checked through the C ABI against the CPU oracle (dequantize +
fp64 SDPA) and against tq_sdpa_int4 with a caller workspace, on consecutive
calls that reuse the shared scratch; a call after the first one must leave
the free device memory unchanged.

This file sorts last so that a run stopping at the first failure has run
every other test first."""
import ctypes

import numpy as np
import pytest

from oracle import inputs, oracle as O
from tests.conftest import parity

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F16 = 1


def _lib():
    import gemma4metal_b200.turboquant as tq
    L = tq.load_library()
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.tq_sdpa_int4_noalloc.argtypes = [P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I, P, P, I,
                                       P]
    return tq, L


def _case(seed, H, Hkv, D, N):
    L = inputs.make_layer(seed, H, Hkv, D, N)
    cap = (N + 3) // 4 * 4
    k = np.zeros((1, Hkv, cap, D), np.float32)
    v = np.zeros_like(k)
    k[:, :, :N] = L["k"]
    v[:, :, :N] = L["v"]
    host = (*O.quantize(k), *O.quantize(v))
    dev = [torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).cuda()
           for a in host]
    q = torch.from_numpy(L["q"]).half().cuda()
    return q, dev, host, cap


def _noalloc(L, q, c, G, window, Hkv, D, N, cap, out, stream):
    return L.tq_sdpa_int4_noalloc(
        ctypes.c_void_p(q.data_ptr()), F16, *[ctypes.c_void_p(t.data_ptr()) for t in c], F16, G,
        1.0, window, 1, Hkv, D, N, cap, None, ctypes.c_void_p(out.data_ptr()), F16,
        ctypes.c_void_p(stream))


@pytest.mark.parametrize("window", [0, 1024])
def test_noalloc_matches_oracle_twice(window):
    tq, L = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row with different sizes: the second reuses the scratch
    # (and its counters) left by the first
    for seed, (H, Hkv, D, N) in [(31, (32, 16, 128, 8192)), (32, (16, 4, 256, 3001))]:
        q, c, h, cap = _case(seed, H, Hkv, D, N)
        out = torch.empty(1, H, D, dtype=torch.float16, device="cuda")
        rc = _noalloc(L, q, c, H // Hkv, window, Hkv, D, N, cap, out, stream)
        assert rc == 0, L.tq_last_error()
        torch.cuda.synchronize()
        assert tq.device_error() == 0
        got = out.float().cpu().numpy()
        ref = O.sdpa_int4(q.float().cpu().numpy(), *h, scale=1.0, window=window, n_tokens=[N],
                          f64=True)
        parity(got, ref)
        # and it agrees with the entry point that takes a caller workspace
        ws_out = tq.sdpa_int4(q, *c, H // Hkv, 1.0, window, n_tokens=N)
        parity(got, ws_out.float().cpu().numpy())


def test_noalloc_later_calls_allocate_nothing():
    """The first call on a device may make the driver place the built-in
    array there; every later call must leave the free device memory as it
    found it."""
    tq, L = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    H, Hkv, D, N = 32, 16, 128, 8192
    q, c, h, cap = _case(33, H, Hkv, D, N)
    out = torch.empty(1, H, D, dtype=torch.float16, device="cuda")
    assert _noalloc(L, q, c, H // Hkv, 0, Hkv, D, N, cap, out, stream) == 0, L.tq_last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _noalloc(L, q, c, H // Hkv, 0, Hkv, D, N, cap, out, stream) == 0, L.tq_last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    ref = O.sdpa_int4(q.float().cpu().numpy(), *h, scale=1.0, n_tokens=[N], f64=True)
    parity(out.float().cpu().numpy(), ref)


def test_noalloc_rejects_sizes_beyond_the_scratch():
    """A head_dim-512 decode over 64K tokens needs more split-KV scratch than
    the built-in area: the call must fail on the host with TQ_ERR_WORKSPACE.
    Real, correctly sized buffers are passed so that nothing invalid could
    reach the GPU even if the check were missing."""
    tq, L = _lib()
    H, Hkv, D, N = 4, 1, 512, 65536
    need = tq.sdpa_int4_workspace_size(1, H, Hkv, D, N, 0)
    assert need > 2 * 1024 * 1024
    q = torch.zeros(1, H, D, dtype=torch.float16, device="cuda")
    codes = [torch.zeros(1, Hkv, N, D // 8, dtype=torch.int32, device="cuda") for _ in range(2)]
    sb = [torch.zeros(1, Hkv, N, D // 64, dtype=torch.float16, device="cuda") for _ in range(4)]
    c = [codes[0], sb[0], sb[1], codes[1], sb[2], sb[3]]
    out = torch.empty(1, H, D, dtype=torch.float16, device="cuda")
    rc = _noalloc(L, q, c, H // Hkv, 0, Hkv, D, N, N, out, torch.cuda.current_stream().cuda_stream)
    assert rc == 4
    assert b"scratch" in L.tq_last_error()
    torch.cuda.synchronize()

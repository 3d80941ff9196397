"""The test harness's PyTorch custom operators (tests/torch_ops.py) drive the
same kernels: append + decode through torch.ops.tq.* match the oracle, and
torch.library.opcheck accepts the decode operator's schema and fake kernel."""
import numpy as np
import pytest
import torch

from oracle import inputs, oracle as O
from tests.conftest import parity

pytestmark = pytest.mark.gpu


def test_ops_append_and_decode():
    import gemma4metal_b200.turboquant as tq
    from tests import torch_ops  # noqa: F401  (registers torch.ops.tq.*)
    H, Hkv, D, N = 32, 16, 128, 700
    L = inputs.make_layer(2, H, Hkv, D, N)
    cache = tq.KVCache(1, Hkv, D, 704)
    k = torch.from_numpy(L["k"]).half().cuda()
    v = torch.from_numpy(L["v"]).half().cuda()
    torch.ops.tq.quantize_append(k, v, *cache.tensors(), 0)
    q = torch.from_numpy(L["q"]).half().cuda()
    out = torch.ops.tq.sdpa_int4(q, *cache.tensors(), H // Hkv, 1.0, 0, N)
    torch.cuda.synchronize()
    kq, ks, kb = O.quantize(L["k"].astype(np.float16).astype(np.float32))
    vq, vs, vb = O.quantize(L["v"].astype(np.float16).astype(np.float32))
    ref = O.sdpa_int4(L["q"].astype(np.float16), kq, ks, kb, vq, vs, vb, f64=True)
    parity(out.float().cpu().numpy(), ref)
    torch.library.opcheck(torch.ops.tq.sdpa_int4.default,
                          (q, *cache.tensors(), H // Hkv, 1.0, 0, N),
                          test_utils=("test_schema", "test_faketensor"))

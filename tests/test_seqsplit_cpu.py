"""Host logic of the multi-GPU sequence split, on CPU: world_size 2 and 4
gloo process groups, each rank computing its shard's partial softmax state
with the CPU oracle, all-gathering the states and merging them must reproduce
the unsplit attention; shard and head bounds must partition their ranges."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gemma4metal_b200 import seqsplit
from oracle import inputs, oracle as O


def test_shard_bounds_partition():
    for n in (1, 63, 64, 65, 1000, 262144, 262145):
        for world in (1, 2, 3, 4, 8):
            got = [seqsplit.shard_bounds(n, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            for (a0, a1), (b0, b1) in zip(got, got[1:]):
                assert a1 == b0
            sizes = [t1 - t0 for t0, t1 in got]
            assert min(sizes) >= 0
            # balanced to within one 64-token chunk, boundaries chunk-aligned
            assert max(sizes) - min(sizes) <= 64
            assert all(t0 % 64 == 0 or t0 == n for t0, _ in got)


def test_head_bounds():
    assert [seqsplit.head_bounds(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        seqsplit.head_bounds(8, 3, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, Hkv, D, N, window = case
        L = inputs.make_layer(3, H, Hkv, D, N)
        kq, ks, kb = O.quantize(L["k"][0])
        vq, vs, vb = O.quantize(L["v"][0])
        kd = O.dequantize_np(kq, ks, kb)
        vd = O.dequantize_np(vq, vs, vb)
        qh = L["q"][0]
        t0, t1 = seqsplit.shard_bounds(N, world, rank)

        def partial(queries, cache, n_local, token_offset, n_total, gqa, scale, win):
            k, v = cache
            assert n_local == t1 - t0 and token_offset == t0 and n_total == N
            lo = max(0, n_total - win) if win > 0 else 0  # the window of the whole sequence
            a, b = max(t0, lo), t1
            part = O.split_partials_np(queries[0].numpy(), k, v, [(a, b)] if b > a else [(0, 0)],
                                       scale)
            return torch.from_numpy(part)

        def merge(parts, Hh, Dd, out_dtype):
            return torch.from_numpy(O.lse_merge_np(parts[:, 0].numpy(), Hh, Dd))[None]

        out = seqsplit.seqsplit_decode(torch.from_numpy(qh)[None], (kd, vd), t1 - t0, t0, N,
                                       H // Hkv, 1.0, window, partial_fn=partial, merge_fn=merge)
        ref = O.sdpa_np(qh[None], kd[None], vd[None], 1.0, window)[0]
        err = float(np.max(np.abs(out[0].numpy() - ref)))
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,case", [
    (2, (32, 16, 128, 1000, 0)),
    (2, (8, 2, 256, 700, 300)),     # sliding window cuts into rank 0's shard
    (4, (32, 8, 256, 900, 0)),
    (4, (16, 4, 128, 130, 0)),       # shards of 64, 64, 2, 0 tokens: an empty rank
])
def test_seqsplit_gloo_matches_unsplit(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=10) for _ in range(world))
    assert len(errs) == world
    assert max(errs.values()) < 1e-5, errs

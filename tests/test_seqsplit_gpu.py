"""Sequence split over 2 GPUs through NCCL (skipped with fewer GPUs): each
rank quantizes its shard, runs the partial decode kernel, the states are
all-gathered and merged on every GPU, and the result must match the CPU
oracle's unsplit dequantize + SDPA within the task tolerance."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    from datetime import timedelta

    import torch.distributed as dist

    from gemma4metal_b200 import seqsplit
    from oracle import inputs, oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        results = []
        for (H, Hkv, D, N, win) in [(32, 8, 256, 3000, 0), (32, 16, 128, 2049, 700)]:
            L = inputs.make_layer(13, H, Hkv, D, N)
            sc = seqsplit.SeqSplitCache(N, Hkv, D, device=f"cuda:{rank}")
            sc.load_prefix(torch.from_numpy(L["k"]).cuda(), torch.from_numpy(L["v"]).cuda())
            sc.append(torch.from_numpy(L["k_new"]).cuda(), torch.from_numpy(L["v_new"]).cuda())
            out = sc.decode(torch.from_numpy(L["q"]).half().cuda(), H // Hkv, 1.0, win,
                            out_dtype=torch.float32)
            torch.cuda.synchronize()
            k = np.concatenate([L["k"], L["k_new"]], 2)
            v = np.concatenate([L["v"], L["v_new"]], 2)
            kq, ks, kb = O.quantize(k)
            vq, vs, vb = O.quantize(v)
            ref = O.sdpa_int4(L["q"].astype(np.float16), kq, ks, kb, vq, vs, vb, window=win, f64=True)
            got = out.cpu().numpy()
            err = float(np.max(np.abs(got - ref)))
            cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
            results.append((err, cos))
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_seqsplit_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    for rank, rr in res.items():
        for err, cos in rr:
            assert err <= 2e-3 and cos >= 0.99999, (rank, err, cos)


def _peer_worker(rank, world, port, q, mode):
    from datetime import timedelta

    import torch.distributed as dist

    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit
    from oracle import inputs, oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        H, Hkv, D, N = 32, 8, 256, 3000
        L = inputs.make_layer(17, H, Hkv, D, N)
        sc = seqsplit.SeqSplitCache(N, Hkv, D, device=f"cuda:{rank}")
        sc.load_prefix(torch.from_numpy(L["k"]).cuda(), torch.from_numpy(L["v"]).cuda())
        q16 = torch.from_numpy(L["q"]).half().cuda()
        # kernels load on first launch; a warm-up step keeps the ranks' first
        # peer step within the wait bound
        sc.decode(q16, H // Hkv, 1.0, 0, out_dtype=torch.float32)
        torch.cuda.synchronize()
        pub = mode.endswith("published")
        ex = seqsplit.PeerExchange(1, H, D, device=f"cuda:{rank}",
                                   timeout_us=5_000_000 if mode == "parity" else 200_000)
        if mode == "parity":
            # a second exchange for the published path (decode kernel stores
            # the states, merge-only launch)
            ex_pub = seqsplit.PeerExchange(1, H, D, device=f"cuda:{rank}")
            res, codes = [], []
            # several steps: the exchange alternates its two slots and step flags
            for step in range(5):
                kn = torch.from_numpy(L["k_new"]).cuda() * (1 + 0.1 * step)
                vn = torch.from_numpy(L["v_new"]).cuda() * (1 - 0.1 * step)
                sc.append(kn, vn)
                peer = sc.decode(q16, H // Hkv, 1.0, 0, out_dtype=torch.float32, exchange=ex)
                publ = sc.decode(q16, H // Hkv, 1.0, 0, out_dtype=torch.float32, exchange=ex_pub,
                                 published=True)
                nccl = sc.decode(q16, H // Hkv, 1.0, 0, out_dtype=torch.float32)
                torch.cuda.synchronize()
                res.append(max(float((peer - nccl).abs().max()), float((publ - nccl).abs().max())))
                codes.append(tq.device_error())
            ex_pub.close()
            assert codes == [0] * 5, codes
            # the last step against the oracle's unsplit dequantize + SDPA
            ks = [L["k"]] + [L["k_new"] * (1 + 0.1 * s) for s in range(5)]
            vs = [L["v"]] + [L["v_new"] * (1 - 0.1 * s) for s in range(5)]
            kq, kss, kb = O.quantize(np.concatenate(ks, 2))
            vq, vss, vb = O.quantize(np.concatenate(vs, 2))
            ref = O.sdpa_int4(L["q"].astype(np.float16), kq, kss, kb, vq, vss, vb, f64=True)
            got = peer.cpu().numpy()
            err = float(np.max(np.abs(got - ref)))
            cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
            q.put((rank, (max(res), err, cos)))
        else:  # rank 1 misses one step: rank 0's merge must time out, record it, return
            part_q = q16
            if rank == 0:
                out = sc.decode(part_q, H // Hkv, 1.0, 0, out_dtype=torch.float32, exchange=ex,
                                published=pub)
                torch.cuda.synchronize()
                code = tq.device_error()
                # never a merge of stale slots: the outputs are NaN
                assert bool(torch.isnan(out).all()), "timed-out merge must write NaN"
                # the exchange stays failed: the next merge gives up at once
                out2 = sc.decode(part_q, H // Hkv, 1.0, 0, out_dtype=torch.float32, exchange=ex,
                                 published=pub)
                torch.cuda.synchronize()
                assert bool(torch.isnan(out2).all())
                try:
                    ex.check()
                    raise AssertionError("check() must raise after a timeout")
                except RuntimeError:
                    pass
                try:
                    ex.merge(torch.zeros(1, H * (D + 2), device="cuda"))
                    raise AssertionError("merge() must raise on a failed exchange")
                except RuntimeError:
                    pass
            else:
                code = -1
            dist.barrier()
            q.put((rank, code))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


def _run_two(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    return dict(q.get(timeout=10) for _ in range(2))


def test_peer_exchange_two_gpus():
    """State exchange + merge over NVLink P2P stores (one kernel) equals the
    NCCL all-gather + merge path step after step, and the oracle."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    for rank, (diff, err, cos) in _run_two("parity").items():
        assert diff <= 1e-5, (rank, diff)
        assert err <= 2e-3 and cos >= 0.99999, (rank, err, cos)


@pytest.mark.parametrize("mode", ["timeout", "timeout_published"])
def test_peer_exchange_missing_rank_times_out(mode):
    """A rank that skips a step (host-side failure, no GPU fault): the other
    rank's merge gives up after its bound and reports the peer timeout in the
    device error word instead of hanging -- with whole states pushed by the
    merge kernel, and with states published per unit by the decode kernel."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_two(mode)
    assert res[0] == 2  # TQ_DEVICE_ERR_PEER_TIMEOUT


def test_peer_exchange_single_gpu_equals_merge():
    """World of one (no process group): the exchange kernel pushes to its own
    buffer and merges one state -- the same as lse_merge of that state."""
    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit
    torch.manual_seed(3)
    B, H, D = 2, 16, 128
    part = torch.randn(B, H * (D + 2), device="cuda")
    part.view(B, H * (D + 2))[:, H * D:].view(B, H, 2)[..., 1].abs_()  # l >= 0
    ex = seqsplit.PeerExchange(B, H, D)
    try:
        for _ in range(3):  # several steps (slot parity, step counter)
            got = ex.merge(part)
        ref = tq.lse_merge(part[None], H, D)
        torch.cuda.synchronize()
        assert tq.device_error() == 0
        assert torch.allclose(got, ref, rtol=1e-6, atol=1e-6)
    finally:
        ex.close()


@pytest.mark.parametrize("H,Hkv,D,N,win", [(16, 8, 128, 2049, 0), (32, 8, 256, 3001, 700),
                                           (8, 8, 128, 100, 0)])
def test_published_single_gpu_equals_partial_merge(H, Hkv, D, N, win):
    """World of one: the decode kernel stores its state into its own exchange
    buffer (split-KV merge path and, at N = 100, the one-split direct path),
    the merge-only launch merges it -- the same as lse_merge of
    tq_sdpa_int4_partial's state, over several steps."""
    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit
    from oracle import inputs
    B = 2
    L = inputs.make_layer(23, H, Hkv, D, N, batch=B)
    cache = tq.KVCache(B, Hkv, D, (N + 3) // 4 * 4)
    cache.append(torch.from_numpy(L["k"]).cuda(), torch.from_numpy(L["v"]).cuda())
    q = torch.from_numpy(L["q"]).half().cuda()
    ex = seqsplit.PeerExchange(B, H, D)
    try:
        for step in range(3):  # slot parity and step counter
            qs = q * (1 + 0.25 * step)
            got = ex.decode(qs, cache.tensors(), N, 0, N, H // Hkv, 0.125, win,
                            out_dtype=torch.float32)
            part = tq.sdpa_int4_partial(qs, *cache.tensors(), H // Hkv, 0.125, win, n_local=N)
            ref = tq.lse_merge(part[None], H, D)
            torch.cuda.synchronize()
            assert tq.device_error() == 0
            assert torch.allclose(got, ref, rtol=1e-6, atol=1e-6), float((got - ref).abs().max())
    finally:
        ex.close()


def test_published_fused_append_single_gpu():
    """World of one: the publishing decode launch also quantizes the new
    token into slot n_local - 1 (the rank holding the sequence's end) -- the
    cache bytes equal quantize_append's and the merged output equals
    quantize_append + partial + lse_merge."""
    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit
    from oracle import inputs
    H, Hkv, D, N = 32, 8, 256, 3000
    L = inputs.make_layer(29, H, Hkv, D, N)
    a = tq.KVCache(1, Hkv, D, N)
    b = tq.KVCache(1, Hkv, D, N)
    for c in (a, b):
        c.append(torch.from_numpy(L["k"][:, :, :N - 1]).cuda().half(),
                 torch.from_numpy(L["v"][:, :, :N - 1]).cuda().half())
    kn = torch.from_numpy(L["k"][:, :, N - 1]).cuda().half()  # (1, Hkv, D)
    vn = torch.from_numpy(L["v"][:, :, N - 1]).cuda().half()
    q = torch.from_numpy(L["q"]).half().cuda()
    ex = seqsplit.PeerExchange(1, H, D)
    try:
        got = ex.decode(q, a.tensors(), N, 0, N, H // Hkv, 0.0625, 0, out_dtype=torch.float32,
                        k_new=kn, v_new=vn)
        tq.quantize_append(kn[:, :, None], vn[:, :, None], *b.tensors(), pos=N - 1)
        part = tq.sdpa_int4_partial(q, *b.tensors(), H // Hkv, 0.0625, 0, n_local=N)
        ref = tq.lse_merge(part[None], H, D)
        torch.cuda.synchronize()
        assert tq.device_error() == 0
        for x, y in zip(a.tensors(), b.tensors()):
            assert torch.equal(x, y)
        assert torch.allclose(got, ref, rtol=1e-6, atol=1e-6), float((got - ref).abs().max())
    finally:
        ex.close()


def test_head_split_gather_single_gpu():
    """World of one: decode_heads (publishing decode with the append fused +
    gather kernel) equals the fused append + decode of the same cache, over
    several steps (slot parity, step counter)."""
    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit
    from oracle import inputs
    H, Hkv, D, N = 16, 4, 256, 5000
    L = inputs.make_layer(37, H, Hkv, D, N)
    a = tq.KVCache(1, Hkv, D, N)
    b = tq.KVCache(1, Hkv, D, N)
    for c in (a, b):
        c.append(torch.from_numpy(L["k"][:, :, :N - 1]).cuda().half(),
                 torch.from_numpy(L["v"][:, :, :N - 1]).cuda().half())
    kn = torch.from_numpy(L["k"][:, :, N - 1]).cuda().half()
    vn = torch.from_numpy(L["v"][:, :, N - 1]).cuda().half()
    q = torch.from_numpy(L["q"]).half().cuda()
    ex = seqsplit.PeerExchange(1, H, D)
    try:
        for step in range(3):
            qs = q * (1 + 0.25 * step)
            got = ex.decode_heads(qs, a.tensors(), N, H // Hkv, 0.0625, 0, out_dtype=torch.float32,
                                  k_new=kn, v_new=vn)
            ref = tq.sdpa_int4_append(qs, kn, vn, *b.tensors(), H // Hkv, 0.0625, 0, n_tokens=N,
                                      out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert tq.device_error() == 0
            assert torch.allclose(got, ref, rtol=1e-5, atol=1e-5), float((got - ref).abs().max())
        for x, y in zip(a.tensors(), b.tensors()):
            assert torch.equal(x, y)
    finally:
        ex.close()


def _heads_worker(rank, world, port, q):
    from datetime import timedelta

    import torch.distributed as dist

    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit
    from oracle import inputs, oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        H, Hkv, D, N = 32, 8, 256, 3001
        G = H // Hkv
        L = inputs.make_layer(41, H, Hkv, D, N)
        h0, h1 = seqsplit.head_bounds(Hkv, world, rank)
        cap = (N + 3) // 4 * 4
        c = tq.KVCache(1, h1 - h0, D, cap)
        # fp32 K/V on both sides: the oracle quantizes the same values
        c.append(torch.from_numpy(np.ascontiguousarray(L["k"][:, h0:h1, :N - 1])).cuda(),
                 torch.from_numpy(np.ascontiguousarray(L["v"][:, h0:h1, :N - 1])).cuda())
        kn = torch.from_numpy(np.ascontiguousarray(L["k"][:, h0:h1, N - 1])).cuda()
        vn = torch.from_numpy(np.ascontiguousarray(L["v"][:, h0:h1, N - 1])).cuda()
        qh = torch.from_numpy(np.ascontiguousarray(L["q"][:, h0 * G:h1 * G])).half().cuda()
        ex = seqsplit.PeerExchange(1, (h1 - h0) * G, D, device=f"cuda:{rank}")
        dist.barrier()
        for _ in range(3):  # several steps: slot parity and step counter
            out = ex.decode_heads(qh, c.tensors(), N, G, 1.0, 0, out_dtype=torch.float32,
                                  k_new=kn, v_new=vn)
        torch.cuda.synchronize()
        code = tq.device_error()
        kq, ks, kb = O.quantize(L["k"])
        vq, vs, vb = O.quantize(L["v"])
        ref = O.sdpa_int4(L["q"].astype(np.float16), kq, ks, kb, vq, vs, vb, f64=True)
        got = out.cpu().numpy()
        err = float(np.max(np.abs(got - ref)))
        cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
        q.put((rank, (code, err, cos)))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


def test_head_split_gather_two_gpus():
    """Head split over 2 GPUs: each rank decodes its KV heads over the whole
    sequence (new token appended in the same launch) and the peer gather
    assembles every head's output on every rank -- equal to the oracle's
    unsplit dequantize + SDPA."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_heads_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for rank, (code, err, cos) in dict(q.get(timeout=10) for _ in range(2)).items():
        assert code == 0, (rank, code)
        assert err <= 2e-3 and cos >= 0.99999, (rank, err, cos)

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

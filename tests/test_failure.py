"""Failure handling, in the forms that fault no GPU:

* on the host (gloo ranks on CPU, world 2 and 4): a rank that exits or
  raises between steps is named by every other rank's StepGuard.begin within
  the bound; a step that overruns its host bound aborts the communicators and
  raises StepTimeout; empty shard states (m = -inf, l = 0) and NaN states fed
  to the merge: empty ones weigh nothing, a NaN state makes its head NaN (the
  reference's normalisation, lib/turboquant.metal:886, keeps NaN: sum == 0
  gives 0, anything else divides);
* on one GPU: the bounded shared-memory barrier wait that every pipeline uses
  runs out on purpose (a barrier that expects two arrivals and gets one) and
  reports TQ_DEVICE_ERR_BARRIER_TIMEOUT with the context still usable; the
  merge kernel's handling of empty and NaN states matches the oracle's.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gemma4metal_b200 import seqsplit
from oracle import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _guard_worker(rank, world, port, mode, lost, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        guard = seqsplit.StepGuard(world, rank, timeout_s=3.0, abort=lambda: None)
        for step in range(5):
            if rank == lost and step == 3:
                if mode == "raise":
                    raise RuntimeError("rank failure planted by the test")
                q.put((rank, "left"))
                return  # leaves between steps, nothing in flight
            t0 = time.monotonic()
            try:
                guard.begin(step)
            except seqsplit.RankLost as e:
                q.put((rank, ("lost", e.step, e.missing, time.monotonic() - t0)))
                return
        q.put((rank, "done"))
    except RuntimeError as e:
        if "planted" in str(e):
            q.put((rank, "raised"))
            return
        raise
    finally:
        # no collective here: the survivors must not wait for the lost rank
        if rank != 0:
            dist.destroy_process_group()
        else:
            time.sleep(0.5)  # rank 0 hosts the store the others still read
            dist.destroy_process_group()


def _run(world, mode, lost):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_guard_worker, args=(r, world, port, mode, lost, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(world))
    for p in procs:
        p.join(60)
    return res, [p.exitcode for p in procs]


def test_step_guard_all_ranks_alive():
    res, codes = _run(2, "none", lost=-1)
    assert res == {0: "done", 1: "done"} and codes == [0, 0]


@pytest.mark.parametrize("world,lost,mode", [(2, 1, "exit"), (4, 2, "exit"), (4, 3, "raise")])
def test_step_guard_names_a_lost_rank(world, lost, mode):
    """The lost rank leaves before step 3; every other rank raises RankLost
    for step 3 naming exactly that rank, within the 3 s bound."""
    res, codes = _run(world, mode, lost)
    assert res[lost] == ("left" if mode == "exit" else "raised")
    for r in range(world):
        if r == lost:
            continue
        kind, step, missing, waited = res[r]
        assert kind == "lost" and step == 3 and missing == [lost], res[r]
        assert waited < 6.0
    assert all(c == 0 for c in codes), codes


def test_step_timeout_aborts_the_group():
    """A step whose completion the host never sees: past the bound the guard
    calls the abort (ncclCommAbort through the process group in production)
    and raises StepTimeout instead of waiting for good."""
    class Never:
        def query(self):
            return False

    aborted = []
    guard = seqsplit.StepGuard(1, 0, timeout_s=0.2, store=dist.HashStore(),
                               abort=lambda: aborted.append(True))
    t0 = time.monotonic()
    with pytest.raises(seqsplit.StepTimeout):
        guard.wait(Never())
    assert aborted == [True] and time.monotonic() - t0 < 2.0


def _states(P, H, D, seed=0):
    rng = np.random.default_rng(seed)
    parts = rng.standard_normal((P, H * (D + 2))).astype(np.float32)
    ml = parts[:, H * D:].reshape(P, H, 2)
    ml[..., 1] = np.abs(ml[..., 1]) + 0.1
    return parts


def test_merge_oracles_empty_and_nan_states():
    H, D = 8, 16
    parts = _states(4, H, D)
    empty = parts.copy()
    ml = empty[:, H * D:].reshape(4, H, 2)
    ml[2, :, 0], ml[2, :, 1] = -np.inf, 0.0
    empty[2, :H * D] = np.nan  # an empty state's o is never read
    want = O.lse_merge_np(parts[[0, 1, 3]], H, D)
    for f in (O.lse_merge_np, O.lse_merge):
        np.testing.assert_allclose(f(empty, H, D), want, rtol=1e-6, atol=1e-6)
    allempty = empty.copy()
    allempty[:, H * D:].reshape(4, H, 2)[..., 0] = -np.inf
    allempty[:, H * D:].reshape(4, H, 2)[..., 1] = 0.0
    for f in (O.lse_merge_np, O.lse_merge):
        assert np.all(f(allempty, H, D) == 0.0)
    nan = parts.copy()
    nan[1, H * D + 2 * 5] = np.nan  # m of head 5 in part 1
    for f in (O.lse_merge_np, O.lse_merge):
        got = f(nan, H, D)
        assert np.isnan(got[5]).all() and np.isfinite(np.delete(got, 5, axis=0)).all()


# ------------------------------------------------------------------ GPU --

@pytest.mark.gpu
def test_bounded_wait_runs_out_and_reports():
    import gemma4metal_b200.turboquant as tq
    L = tq.load_library()
    assert tq.device_error() == 0
    gave_up = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.monotonic()
    rc = L.tq_wait_selftest(2000, tq._ptr(gave_up), tq._stream(None))
    assert rc == 0, L.tq_last_error()
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 5.0
    assert tq.device_error() == 1  # TQ_DEVICE_ERR_BARRIER_TIMEOUT
    assert int(gave_up.item()) == 32
    # the context is still usable: a decode after it matches the oracle
    from oracle import inputs
    from tests.conftest import parity
    H, Hkv, D, N = 32, 16, 128, 2000
    Ly = inputs.make_layer(4, H, Hkv, D, N)
    c = [torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).cuda()
         for a in (*O.quantize(Ly["k"]), *O.quantize(Ly["v"]))]
    q = torch.from_numpy(Ly["q"]).half().cuda()
    out = tq.sdpa_int4(q, *c, H // Hkv, 1.0, 0, n_tokens=N, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert tq.device_error() == 0
    ref = O.sdpa_int4(q.float().cpu().numpy(), *[a for a in (*O.quantize(Ly["k"]), *O.quantize(Ly["v"]))],
                      f64=True)
    parity(out.cpu().numpy(), ref)


@pytest.mark.gpu
def test_merge_kernel_empty_and_nan_states():
    import gemma4metal_b200.turboquant as tq
    H, D = 8, 128
    parts = _states(4, H, D, seed=3)
    empty = parts.copy()
    ml = empty[:, H * D:].reshape(4, H, 2)
    ml[2, :, 0], ml[2, :, 1] = -np.inf, 0.0
    empty[2, :H * D] = np.nan
    nan = parts.copy()
    nan[1, H * D + 2 * 5] = np.nan
    for case in (empty, nan):
        got = tq.lse_merge(torch.from_numpy(case).cuda()[:, None], H, D).cpu().numpy()[0]
        want = O.lse_merge_np(case, H, D)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        ok = ~np.isnan(want)
        np.testing.assert_allclose(got[ok], want[ok], rtol=1e-5, atol=1e-6)

"""Multi-GPU decode attention over one int4 KV cache: one process per GPU with
torch.distributed (NCCL over NVLink/NVSwitch) for the plumbing.

Two ways the path shards (the reference is single-device; its engine calls
turboquant::sdpa_int4 once per layer, engine/gemma4_multilayer.cpp:280-282):

* sequence split -- rank r holds the contiguous token shard
  [t0_r, t1_r) of every KV head (`shard_bounds`), computes the partial softmax
  state (o, m, l) of its shard with `tq_sdpa_int4_partial`, the H*(D+2) fp32
  states of all ranks are all-gathered (33 KB per rank at H=32, D=256), and
  every rank merges them with the `tq_lse_merge` kernel (the same log-sum-exp
  merge the reference does across simdgroups, lib/turboquant.metal:838-888).
  New tokens are appended to the shard of the last rank.
* head split -- rank r holds KV heads [h0_r, h1_r) (`head_bounds`) and their
  query heads; no exchange is needed unless the caller wants the full output,
  which one all-gather of (H/P, D) per rank provides.

Two exchanges of the partial states: NCCL (`all_gather_into_tensor` into this
GPU's memory, then the merge kernel) or `PeerExchange`, which does the
exchange and the merge in one kernel of this library: every rank stores its
state into every rank's exchange buffer over NVLink (CUDA IPC mappings, plain
P2P stores), raises a step flag there and merges what it received once all
flags of the step are up (waits bounded; a missing rank shows up as
TQ_DEVICE_ERR_PEER_TIMEOUT in tq_device_error). Kernels only ever read their
own GPU's memory.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import turboquant as tq

CHUNK = 64  # shard boundaries on the decode kernel's 64-token chunks


def shard_bounds(n_total: int, world: int, rank: int, align: int = CHUNK) -> Tuple[int, int]:
    """Contiguous token shard [t0, t1) of `rank`: `align`-token chunks split as
    evenly as possible. The last n_chunks % world ranks get one chunk more,
    since the final chunk may be partial; shard sizes then differ by less than
    one chunk."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    chunks = (n_total + align - 1) // align
    per, extra = divmod(chunks, world)
    first_big = world - extra
    c0 = rank * per + max(0, rank - first_big)
    c1 = c0 + per + (1 if rank >= first_big else 0)
    return min(c0 * align, n_total), min(c1 * align, n_total)


def head_bounds(num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads [h0, h1) of `rank` for the head-parallel split."""
    if num_kv_heads % world:
        raise ValueError("num_kv_heads must be a multiple of the world size")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def _world_rank(group) -> Tuple[int, int]:
    """(world size, rank) of `group`; a process without a process group is a
    world of one."""
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _all_gather(part: torch.Tensor, world: int, group) -> torch.Tensor:
    parts = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
    if world == 1:
        parts[0].copy_(part)
    elif dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(parts, part.contiguous(), group=group)
    else:
        dist.all_gather(list(parts.unbind(0)), part.contiguous(), group=group)
    return parts


class PeerExchange:
    """Exchange buffers of one sequence-split group for `tq_peer_merge`.

    Collective: every rank of `group` constructs it (it allocates this rank's
    buffer, all-gathers the CUDA IPC handles as objects and maps the others'
    buffers) and calls `merge` once per step in the same order; `close` is
    collective too. State layout: that of `tq_sdpa_int4_partial`."""

    def __init__(self, batch: int, num_heads: int, head_dim: int, group=None, device=None,
                 timeout_us: int = 5_000_000):
        import ctypes
        self.group = group
        self.world, self.rank = _world_rank(group)
        self.B, self.H, self.D = batch, num_heads, head_dim
        self.timeout_us = int(timeout_us)
        self.failed = False
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = tq.load_library()
        nbytes = int(lib.tq_peer_buffer_bytes(self.world, batch, num_heads, head_dim))
        if nbytes == 0:
            raise ValueError("bad peer exchange sizes")
        buf = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            tq._check(lib.tq_peer_buffer_alloc(nbytes, ctypes.byref(buf)))
            self._own = buf.value
            handle = (ctypes.c_ubyte * 64)()
            tq._check(lib.tq_ipc_handle(self._own, handle))
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, bytes(handle), group=group)
            else:
                handles[0] = bytes(handle)
            self._opened = []
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r])
                tq._check(lib.tq_ipc_open(h, ctypes.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value)
            self.bufs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        if self.world > 1:
            dist.barrier(group=group)  # every buffer is mapped before any rank pushes

    def merge(self, part: torch.Tensor, out: Optional[torch.Tensor] = None,
              out_dtype: torch.dtype = torch.float32, s=None) -> torch.Tensor:
        """Push this rank's state (B, H*(D+2)) fp32, wait for the others',
        return the merged (B, H, D). Raises once `check` has seen a timeout:
        the exchange is then out of step with the other ranks for good."""
        if self.failed:
            raise RuntimeError("PeerExchange: a merge timed out on this exchange; close it and "
                               "build a new one on every rank")
        if out is None:
            out = torch.empty(self.B, self.H, self.D, dtype=out_dtype, device=self.device)
        pc = part.contiguous()
        tq._check(tq.load_library().tq_peer_merge(
            tq._ptr(pc), self.bufs.data_ptr(), self.world, self.rank, self.B, self.H, self.D,
            tq._ptr(out), tq._dt(out), self.timeout_us, tq._stream(s)))
        return out

    def decode(self, queries: torch.Tensor, cache, n_local: int, token_offset: int, n_total: int,
               gqa_factor: int, scale: float = 1.0, sliding_window: int = 0,
               out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
               ws: Optional[torch.Tensor] = None, k_new: Optional[torch.Tensor] = None,
               v_new: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
        """One sequence-split decode step with the exchange inside the decode
        kernel: each (sequence, KV head) slice of the partial state is stored
        into every rank's buffer as {value, step} pairs as soon as it is
        complete (`tq_sdpa_int4_partial_publish`), then a merge-only launch
        (`tq_peer_merge_published`) waits for the pairs of the step and
        merges. Same lockstep and failure rules as `merge`; use one exchange
        with either `merge` or `decode`. k_new / v_new ((B, Hkv, D), on the
        rank holding the sequence's end): the new token is quantized into
        slot n_local - 1 in the same launch."""
        if self.failed:
            raise RuntimeError("PeerExchange: a merge timed out on this exchange; close it and "
                               "build a new one on every rank")
        B, H, D = queries.shape
        if (B, H, D) != (self.B, self.H, self.D):
            raise ValueError(f"queries {tuple(queries.shape)} do not match the exchange "
                             f"({self.B}, {self.H}, {self.D})")
        if out is None:
            out = torch.empty(B, H, D, dtype=out_dtype or queries.dtype, device=self.device)
        tq.sdpa_int4_partial_publish(queries, cache, gqa_factor, scale, sliding_window, self.bufs,
                                     self.world, self.rank, n_local=n_local,
                                     token_offset=token_offset, n_total=n_total, ws=ws,
                                     k_new=k_new, v_new=v_new, s=s)
        tq._check(tq.load_library().tq_peer_merge_published(
            self.bufs.data_ptr(), self.world, self.rank, B, H, D, tq._ptr(out), tq._dt(out),
            self.timeout_us, tq._stream(s)))
        return out

    def decode_heads(self, queries: torch.Tensor, cache, n_tokens: int, gqa_factor: int,
                     scale: float = 1.0, sliding_window: int = 0,
                     out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                     ws: Optional[torch.Tensor] = None, k_new: Optional[torch.Tensor] = None,
                     v_new: Optional[torch.Tensor] = None, s=None) -> torch.Tensor:
        """One decode step of a head split: this rank's queries (B, H/world, D)
        against its KV heads' cache over the whole sequence (n_tokens), the
        state published into every rank's buffer, then every rank's heads
        gathered into the full output (B, H, D) (`tq_peer_gather_published`),
        rank k's heads at k * H/world. k_new / v_new: the new token of this
        rank's KV heads, appended in the same launch. The exchange is built
        with num_heads = H/world."""
        if self.failed:
            raise RuntimeError("PeerExchange: a merge timed out on this exchange; close it and "
                               "build a new one on every rank")
        B, Hl, D = queries.shape
        if (B, Hl, D) != (self.B, self.H, self.D):
            raise ValueError(f"queries {tuple(queries.shape)} do not match the exchange "
                             f"({self.B}, {self.H}, {self.D})")
        if out is None:
            out = torch.empty(B, Hl * self.world, D, dtype=out_dtype or queries.dtype,
                              device=self.device)
        tq.sdpa_int4_partial_publish(queries, cache, gqa_factor, scale, sliding_window, self.bufs,
                                     self.world, self.rank, n_local=n_tokens, token_offset=0,
                                     n_total=n_tokens, ws=ws, k_new=k_new, v_new=v_new, s=s)
        tq._check(tq.load_library().tq_peer_gather_published(
            self.bufs.data_ptr(), self.world, self.rank, B, Hl, D, tq._ptr(out), tq._dt(out),
            self.timeout_us, tq._stream(s)))
        return out

    def check(self, s=None) -> None:
        """Read (and clear) the device error word after the merges enqueued so
        far (synchronises the stream); raise if one of them timed out waiting
        for a rank. After that every merge raises: a timed-out exchange is
        marked failed on the device, writes NaN and never advances again."""
        code = tq.device_error(s)
        if code & 2:  # TQ_DEVICE_ERR_PEER_TIMEOUT
            self.failed = True
            raise RuntimeError("PeerExchange: a rank did not deliver its state within "
                               f"{self.timeout_us} us (device error {code})")

    def close(self) -> None:
        lib = tq.load_library()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank still stores into a buffer being released
        for p in self._opened:
            tq._check(lib.tq_ipc_close(p))
        self._opened = []
        if self._own:
            tq._check(lib.tq_peer_buffer_free(self._own))
            self._own = None


def _cuda_partial(queries, cache, n_local, token_offset, n_total, gqa, scale, window):
    return tq.sdpa_int4_partial(queries, *cache, gqa, scale, window, n_local=n_local,
                                token_offset=token_offset, n_total=n_total)


def _cuda_merge(parts, num_heads, head_dim, out_dtype):
    return tq.lse_merge(parts, num_heads, head_dim, out_dtype=out_dtype)


def seqsplit_decode(queries: torch.Tensor, cache, n_local: int, token_offset: int, n_total: int,
                    gqa_factor: int, scale: float = 1.0, sliding_window: int = 0, *,
                    group=None, out_dtype: Optional[torch.dtype] = None,
                    partial_fn: Optional[Callable] = None,
                    merge_fn: Optional[Callable] = None,
                    exchange: Optional[PeerExchange] = None,
                    published: bool = False) -> torch.Tensor:
    """Decode attention of a sequence split across the ranks of `group`.

    queries (B, H, D) (the same on every rank); cache = this rank's shard
    (k_quant, k_scales, k_biases, v_quant, v_scales, v_biases) holding global
    tokens [token_offset, token_offset + n_local) of a sequence of n_total.
    Returns (B, H, D) on every rank. partial_fn / merge_fn default to the CUDA
    kernels; tests substitute CPU implementations to check the host logic.
    With `exchange` the states move over peer memory and the merge happens in
    the same kernel (`PeerExchange.merge`) instead of all-gather + merge; with
    `published` as well, the decode kernel stores each unit's state into the
    buffers itself and a merge-only launch follows (`PeerExchange.decode`)."""
    world, _ = _world_rank(group)
    B, H, D = queries.shape
    if exchange is not None and published:
        if partial_fn is not None:
            raise ValueError("published states come from the CUDA decode kernel")
        return exchange.decode(queries, cache, n_local, token_offset, n_total, gqa_factor, scale,
                               sliding_window, out_dtype=out_dtype or queries.dtype)
    part = (partial_fn or _cuda_partial)(queries, cache, n_local, token_offset, n_total,
                                         gqa_factor, scale, sliding_window)
    part = part.reshape(B, H * (D + 2))
    if exchange is not None:
        return exchange.merge(part, out_dtype=out_dtype or queries.dtype)
    parts = _all_gather(part, world, group)
    return (merge_fn or _cuda_merge)(parts, H, D, out_dtype or queries.dtype)


class SeqSplitCache:
    """This rank's shard of a sequence-split int4 KV cache (one layer).

    Rank r owns global tokens [t0_r, t1_r) of the prefix it was built with;
    tokens appended later go to the last rank (its capacity must leave room)."""

    def __init__(self, n_prefix: int, num_kv_heads: int, head_dim: int, capacity_extra: int = 256,
                 batch: int = 1, group=None, device=None):
        self.group = group
        self.world, self.rank = _world_rank(group)
        self.t0, self.t1 = shard_bounds(n_prefix, self.world, self.rank)
        self.n_total = n_prefix
        last = self.rank == self.world - 1
        cap = (self.t1 - self.t0) + (capacity_extra if last else 0)
        cap = max(4, (cap + 3) // 4 * 4)
        self.cache = tq.KVCache(batch, num_kv_heads, head_dim, cap, device=device)

    @property
    def n_local(self) -> int:
        return self.cache.length

    def load_prefix(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantize this rank's slice [t0, t1) of the full prefix (B, Hkv, n, D)."""
        self.cache.append(k[:, :, self.t0:self.t1], v[:, :, self.t0:self.t1], pos=0)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Append new tokens (B, Hkv, n_new, D) on the last rank; every rank
        advances the global length."""
        if self.rank == self.world - 1:
            self.cache.append(k_new, v_new)
        self.n_total += k_new.shape[2]

    def decode(self, queries: torch.Tensor, gqa_factor: int, scale: float = 1.0,
               sliding_window: int = 0, out_dtype: Optional[torch.dtype] = None,
               exchange: Optional[PeerExchange] = None, published: bool = False) -> torch.Tensor:
        return seqsplit_decode(queries, self.cache.tensors(), self.n_local, self.t0, self.n_total,
                               gqa_factor, scale, sliding_window, group=self.group,
                               out_dtype=out_dtype, exchange=exchange, published=published)


# ------------------------------------------------------------- failures --
# A sequence split needs every rank at every step: one missing shard makes
# every rank's merge wrong or stuck. Failures are caught on the host, between
# steps (a rank leaves only between steps, with nothing of its own in flight):
#   * StepGuard.begin(step): every rank posts a heartbeat for `step` to the
#     process group's key-value store and waits, bounded, for the others'
#     heartbeats of the same step before it launches anything; a rank that
#     exited, crashed or hangs on the host is named in RankLost.
#   * StepGuard.wait(event): the host waits, bounded, for an enqueued step to
#     complete on the GPU; past the bound the communicator is aborted (NCCL:
#     ncclCommAbort through the process group) and StepTimeout is raised, so
#     no rank waits for good on a collective a lost rank will never join.
#   * init_split_group(): NCCL communicators are created non-blocking
#     (config.blocking = 0); the process group polls the communicator's
#     asynchronous error state (ncclCommGetAsyncError) while it waits, so an
#     init or a collective that fails is reported instead of hanging, within
#     the group's timeout.
# The peer-memory exchange has its own bound (PeerExchange: NaN outputs,
# TQ_DEVICE_ERR_PEER_TIMEOUT, check()).


class RankLost(RuntimeError):
    """Ranks of the split that did not reach a step within the bound."""

    def __init__(self, step: int, missing):
        self.step, self.missing = step, sorted(missing)
        super().__init__(f"sequence split: rank(s) {self.missing} did not reach step {step}")


class StepTimeout(RuntimeError):
    """An enqueued step did not complete within the host's bound."""


def init_split_group(backend: str = "nccl", timeout_s: float = 60.0, device=None):
    """init_process_group for a sequence split with a short timeout and, for
    NCCL, non-blocking communicator creation."""
    from datetime import timedelta
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if backend == "nccl":
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.blocking = 0
        kw["pg_options"] = opts
        if device is not None:
            kw["device_id"] = torch.device(device)
    dist.init_process_group(backend, **kw)


def abort_group(group=None) -> None:
    """Abort the group's communicators (pending collectives return with an
    error on every rank that is still there)."""
    from torch.distributed import distributed_c10d as c10d
    if hasattr(c10d, "_abort_process_group"):
        c10d._abort_process_group(group)
        return
    pg = group if group is not None else c10d._get_default_group()
    pg.abort()


class StepGuard:
    """Host-side liveness checks of a sequence split between steps (see the
    section comment above). `store` defaults to the default process group's
    store; `timeout_s` bounds each wait; `abort` is what runs when a step
    overruns (abort_group by default)."""

    def __init__(self, world: int, rank: int, timeout_s: float = 10.0, store=None,
                 prefix: str = "tq/split", abort: Optional[Callable] = None, group=None):
        from torch.distributed import distributed_c10d as c10d
        self.world, self.rank = world, rank
        self.timeout_s = float(timeout_s)
        self.store = store if store is not None else c10d._get_default_store()
        self.prefix = prefix
        self.group = group
        self.abort = abort if abort is not None else (lambda: abort_group(group))

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def begin(self, step: int) -> None:
        """Post this rank's heartbeat for `step`, then wait (bounded) until
        every rank has posted it; raise RankLost naming the missing ranks."""
        import time
        self.store.set(self._key(step, self.rank), "1")
        if step >= 2:  # keys two steps back are read by nobody any more
            try:
                self.store.delete_key(self._key(step - 2, self.rank))
            except Exception:
                pass
        deadline = time.monotonic() + self.timeout_s
        missing = {r for r in range(self.world) if r != self.rank}
        while True:
            for r in sorted(missing):
                if self.store.check([self._key(step, r)]):
                    missing.discard(r)
            if not missing:
                return
            if time.monotonic() >= deadline:
                raise RankLost(step, missing)
            time.sleep(0.0002)

    def wait(self, event, what: str = "step") -> None:
        """Wait (bounded) for `event` (anything with .query(), e.g. a
        torch.cuda.Event recorded after the step); past the bound abort the
        communicators and raise StepTimeout."""
        import time
        deadline = time.monotonic() + self.timeout_s
        while not event.query():
            if time.monotonic() > deadline:
                self.abort()
                raise StepTimeout(f"sequence split: {what} did not complete within "
                                  f"{self.timeout_s} s; communicators aborted")
            time.sleep(0.0005)

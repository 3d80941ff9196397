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

Remote partials land in this GPU's memory (the all-gather's output buffer)
before the merge kernel reads them; no kernel reads peer memory.
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


def _cuda_partial(queries, cache, n_local, token_offset, n_total, gqa, scale, window):
    return tq.sdpa_int4_partial(queries, *cache, gqa, scale, window, n_local=n_local,
                                token_offset=token_offset, n_total=n_total)


def _cuda_merge(parts, num_heads, head_dim, out_dtype):
    return tq.lse_merge(parts, num_heads, head_dim, out_dtype=out_dtype)


def seqsplit_decode(queries: torch.Tensor, cache, n_local: int, token_offset: int, n_total: int,
                    gqa_factor: int, scale: float = 1.0, sliding_window: int = 0, *,
                    group=None, out_dtype: Optional[torch.dtype] = None,
                    partial_fn: Optional[Callable] = None,
                    merge_fn: Optional[Callable] = None) -> torch.Tensor:
    """Decode attention of a sequence split across the ranks of `group`.

    queries (B, H, D) (the same on every rank); cache = this rank's shard
    (k_quant, k_scales, k_biases, v_quant, v_scales, v_biases) holding global
    tokens [token_offset, token_offset + n_local) of a sequence of n_total.
    Returns (B, H, D) on every rank. partial_fn / merge_fn default to the CUDA
    kernels; tests substitute CPU implementations to check the host logic."""
    world, _ = _world_rank(group)
    B, H, D = queries.shape
    part = (partial_fn or _cuda_partial)(queries, cache, n_local, token_offset, n_total,
                                         gqa_factor, scale, sliding_window)
    part = part.reshape(B, H * (D + 2))
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
               sliding_window: int = 0, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        return seqsplit_decode(queries, self.cache.tensors(), self.n_local, self.t0, self.n_total,
                               gqa_factor, scale, sliding_window, group=self.group,
                               out_dtype=out_dtype)

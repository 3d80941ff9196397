"""Benchmark of the int4 KV-cache decode-attention path (task configs 0-4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload all|cfg0|cfg1|cfg2|cfg3|cfg4|probe]
                    [--context 32768] [--window 0] [--exchange published|peer|nccl]

Headline (top-level keys): config 1 at 32K tokens. One step = one decode step
of one attention layer: quantize-on-append of the new token's K/V into the
preallocated int4 cache, then fused decode attention over the whole context,
in one launch (`tq_sdpa_int4_append`; `--split-step` runs them as two
launches) (H=32, Hkv=16, D=128, batch 1, fp16 Q/out, fp16 scales/biases).
Steps rotate over 8 independent layer caches (8 x 75.5 MB, larger than the
126 MB L2), so every step streams its cache from HBM; the appended slot is
rewritten on each rotation, so every step attends over exactly `--context`
tokens. The timed region is one CUDA graph of exactly `--steps` steps.
With N GPUs (torchrun, one process per GPU) every rank serves its own layer
caches (weak scaling: independent KV heads / sequences per GPU, no data-path
collective); value = total steps / max-over-ranks time.

Nested under "configs" (default `--workload all`): config 0 (one layer, 1024
tokens), config 2 (tcgen05: 64 x 1 batched decode over a shared 8K cache and
the 512-query prefill chunk), config 3 (PolarQuant + QJL compressed keys) and
a read-only HBM probe on one GPU; config 4 (one 262144-token sequence split
over all N GPUs, the decode kernel storing its partial state into every
rank's exchange buffer over NVLink + a merge-only kernel, strong scaling) at
every N, and at N > 1 the same layer split by KV heads (append + decode of a
rank's heads, NCCL all-gather of the outputs),
with its time split and its merged output checked against the C oracle.

`--impl reference` times the reference's algorithm on the host CPU instead
(the CPU oracle in oracle/: quantize the new token, concatenate it onto the
packed cache as engine/gemma4_multilayer.cpp:228-236 does, dequantize to fp32
and run SDPA, engine/gemma4_multilayer.cpp:307-308,349), OpenMP over all host
threads; MLX itself is not installable here.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, HKV, D = 32, 16, 128
LAYERS = 8


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--window", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="published", choices=["published", "peer", "nccl"],
                    help="cfg4 with N>1: partial states stored into every rank's buffer by the "
                         "decode kernel itself as {value, step} pairs and merged by a merge-only "
                         "kernel (published), exchanged and merged by one kernel over NVLink "
                         "peer memory (peer), or NCCL all-gather + merge kernel (nccl)")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="cfg4_heads (config 4 split by KV heads): the outputs gathered over "
                         "NVLink peer memory by the publishing decode + a gather kernel (peer) "
                         "or by an NCCL all-gather (nccl)")
    ap.add_argument("--split-step", action="store_true",
                    help="cfg1: run the step as two launches (quantize_append, then sdpa_int4) "
                         "instead of the fused sdpa_int4_append")
    ap.add_argument("--workload", default="all",
                    choices=["all", "cfg0", "cfg1", "cfg2", "cfg3", "cfg4", "cfg4_heads", "probe"],
                    help="all (default): the config-1 headline line with the other configs "
                         "nested (configs 0, 2, 3 and the HBM probe on one GPU; config 4's "
                         "sequence split at every GPU count, and its KV-head split at N > 1); "
                         "cfg1: the headline alone; cfg0/cfg2/cfg3/cfg4/cfg4_heads/probe: that "
                         "config's line alone")
    ap.add_argument("--no-check", action="store_true",
                    help="skip config 4's check of the merged output against the C oracle")
    return ap.parse_args()


def bytes_per_step(n_ctx: int, window: int) -> dict:
    vis = min(n_ctx, window) if window > 0 else n_ctx
    per_tok = 2 * (D // 2 + 2 * (D // 64) * 2) * HKV  # K+V codes, fp16 scale+bias, all KV heads
    attn = per_tok * vis + H * D * 2 * 2             # cache + Q + O (fp16)
    append = 2 * HKV * D * 2 + per_tok               # read new K/V fp16, write one token
    return {"attn": attn, "append": append, "step": attn + append, "per_token": per_tok}


# ------------------------------------------------------------------ clocks --

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        load = [r for r in rows if r["power"] > 250.0] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load),
                "sm_max_mhz": max(r["smax"] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows), "samples_under_load": len(load)}


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def ncu_traffic(n_ctx: int, window: int):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary,
    scaled to this context when it was captured at another size."""
    path = os.path.join(ROOT, "profiles", "sdpa_decode_int4_cfg1_global.md")
    if not os.path.exists(path) or window > 0:
        return None
    txt = open(path).read()
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)\s*@\s*context\s*(\d+)", txt)
    if not m:
        return None
    return float(m.group(1)) * n_ctx / float(m.group(2))


# -------------------------------------------------------------- ours (GPU) --

def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist
    import gemma4metal_b200.turboquant as tq

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    n_ctx, window = args.context, args.window
    cap = (n_ctx + 3) // 4 * 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)

    def rms_norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True)) * w

    wq = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    wk = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    layers = []
    for _ in range(LAYERS):
        cache = tq.KVCache(1, HKV, D, cap, device=dev)
        k = rms_norm(torch.randn(1, HKV, n_ctx - 1, D, device=dev, generator=gen), wk).half()
        v = torch.randn(1, HKV, n_ctx - 1, D, device=dev, generator=gen).half()
        cache.append(k, v, pos=0)
        del k, v
        q = rms_norm(torch.randn(1, H, D, device=dev, generator=gen), wq).half()
        kn = rms_norm(torch.randn(1, HKV, 1, D, device=dev, generator=gen), wk).half()
        vn = torch.randn(1, HKV, 1, D, device=dev, generator=gen).half()
        out = torch.empty(1, H, D, dtype=torch.float16, device=dev)
        layers.append(dict(cache=cache, q=q, kn=kn, vn=vn, out=out))
    nbytes = tq.sdpa_int4_workspace_size(1, H, HKV, D, n_ctx, window)
    wss = [tq.workspace(dev, nbytes) if i == 0 else None for i in range(1)]
    ws = wss[0]
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device=dev)

    def step(Lr, s, with_append=True):
        c = Lr["cache"]
        if with_append and not args.split_step:
            # one launch: the decode kernel quantizes the new token into slot n - 1
            tq.sdpa_int4_append(Lr["q"], Lr["kn"], Lr["vn"], *c.tensors(), H // HKV, 1.0, window,
                                s=s, n_tokens=n_ctx, out=Lr["out"], ws=ws)
            return
        if with_append:
            tq.quantize_append(Lr["kn"], Lr["vn"], *c.tensors(), pos=n_ctx - 1, s=s)
        tq.sdpa_int4(Lr["q"], *c.tensors(), H // HKV, 1.0, window, s=s, n_tokens=n_ctx,
                     out=Lr["out"], ws=ws)

    # eager warm-up (plans, occupancy, attributes), then CUDA graphs: the
    # warm-up steps and the timed steps are one graph each, of exactly
    # `--warmup` and `--steps` steps over the layer rotation, so the timed
    # region is one graph launch whatever the step count.
    with torch.cuda.stream(stream):
        for Lr in layers:
            step(Lr, stream)
    torch.cuda.synchronize()

    def capture(steps, with_append=True):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i in steps:
                    step(layers[i % LAYERS], stream, with_append)
        return g

    CHUNK = 8 * LAYERS
    warm = capture(range(args.warmup)) if args.warmup > 0 else None
    timed = capture(range(args.steps))
    kchunk = capture(range(CHUNK), with_append=False)
    torch.cuda.synchronize()

    clocks = Clocks(local_rank)
    clocks.start()
    with torch.cuda.stream(stream):
        if warm is not None:
            warm.replay()
        timed.replay()  # a graph's first launch uploads it: kept out of the timed region
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        timed.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)

    # decode kernel alone (same rotation, CHUNK launches per graph) for the
    # roofline; runs >= 1.5 s so the clock sampler sees it
    with torch.cuda.stream(stream):
        kchunk.replay()
    torch.cuda.synchronize()
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    reps, t_start = 0, time.perf_counter()
    k0.record(stream)
    with torch.cuda.stream(stream):
        while time.perf_counter() - t_start < 1.5 or reps < 8:
            for _ in range(8):
                kchunk.replay()
            reps += 8
            torch.cuda.current_stream().synchronize() if reps % 64 == 0 else None
    k1.record(stream)
    torch.cuda.synchronize()
    kern_us = k0.elapsed_time(k1) * 1000.0 / (reps * CHUNK)
    clk = clocks.stop()

    # end to end through the public API with host buffers every step: one
    # HostDecodeStep per layer cache (tq_decode_step_run: the host's q, k_new
    # and v_new go up, the fused step runs, the output comes back, all in one
    # graph launch + synchronisation). Every run() returns with the output on
    # the host, so this leg is timed by the host clock.
    nq, nkv = H * D, HKV * D
    hq = layers[0]["q"].cpu().contiguous()
    hkn = layers[0]["kn"].reshape(1, HKV, D).cpu().contiguous()
    hvn = layers[0]["vn"].reshape(1, HKV, D).cpu().contiguous()
    hout = torch.empty(1, H, D, dtype=torch.float16)
    e2e_steps = max(LAYERS, min(args.steps, 2000))
    e2e_ms = None
    if not args.split_step:  # the step object runs the fused step only
        hsteps = [tq.HostDecodeStep(Lr["cache"], H, 1.0, window) for Lr in layers]

        def e2e_loop(n):
            for i in range(n):
                hsteps[i % LAYERS].run(n_ctx, hq, hkn, hvn, hout)

        e2e_loop(2 * LAYERS)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e2e_loop(e2e_steps)
        e2e_ms = (time.perf_counter() - t0) * 1000.0
        assert tq.device_error() == 0, "a kernel reported a device error"
        for hs in hsteps:
            hs.close()

    # the same step through the asynchronous device-pointer API: one pinned
    # H2D copy of q|k_new|v_new, tq_sdpa_int4_append, one D2H copy, sync
    hin = torch.empty(nq + 2 * nkv, dtype=torch.float16, pin_memory=True)
    hin[:nq].copy_(hq.reshape(-1))
    hin[nq:nq + nkv].copy_(hkn.reshape(-1))
    hin[nq + nkv:].copy_(hvn.reshape(-1))
    hpin = torch.empty(1, H, D, dtype=torch.float16, pin_memory=True)
    e2e_in = [torch.empty(nq + 2 * nkv, dtype=torch.float16, device=dev) for _ in range(LAYERS)]
    e2e_layers = [dict(Lr, q=buf[:nq].view(1, H, D), kn=buf[nq:nq + nkv].view(1, HKV, 1, D),
                       vn=buf[nq + nkv:].view(1, HKV, 1, D))
                  for Lr, buf in zip(layers, e2e_in)]

    def async_loop(n):
        with torch.cuda.stream(stream):
            for i in range(n):
                Lr = e2e_layers[i % LAYERS]
                e2e_in[i % LAYERS].copy_(hin, non_blocking=True)
                step(Lr, stream)
                hpin.copy_(Lr["out"], non_blocking=True)
                stream.synchronize()

    async_loop(2 * LAYERS)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    async_loop(e2e_steps)
    async_ms = (time.perf_counter() - t0) * 1000.0
    assert tq.device_error() == 0, "a kernel reported a device error"
    if e2e_ms is None:
        e2e_ms = async_ms

    # max over ranks
    tt = torch.tensor([t_ms, e2e_ms, async_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, async_ms = float(tt[0]), float(tt[1]), float(tt[2])

    # release graphs before the process group goes away
    del warm, timed, kchunk
    torch.cuda.synchronize()
    return dict(t_ms=t_ms, kern_us=kern_us, e2e_ms=e2e_ms, async_ms=async_ms, e2e_steps=e2e_steps,
                clocks=clk, layer0=layers[0])


# ------------------------------------------------- config 4: sequence split --

C4_H, C4_HKV, C4_D, C4_N = 32, 8, 256, 262144


def _graph_time(stream, graph, reps: int) -> float:
    """Milliseconds of `reps` replays of `graph` on `stream` (CUDA events)."""
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def run_cfg4(args, rank: int, world: int, local_rank: int, steps: int = 256, check: bool = True):
    """Config 4: one decode step of a 262144-token global-attention layer
    (H=32, Hkv=8, D=256) whose int4 cache is split by sequence over the GPUs
    (strong scaling). Step = append the new token on the last rank + partial
    decode on every rank + exchange of the fp32 (o, m, l) states + LSE merge
    (by default the decode kernel stores its state into every rank's buffer
    and a merge-only kernel follows; --exchange peer: one peer-memory
    exchange + merge kernel; --exchange nccl: NCCL all-gather + merge kernel),
    captured in CUDA graphs; layers rotate so every step streams its shard
    from HBM. Also timed on their own: the append + partial decode, and the
    exchange + merge (for the default exchange: the step's time less that of
    the plain partial decode). `check`: rank 0 rebuilds layer 0's whole
    cache on the host with the C oracle's quantizer and compares the merged
    output with the oracle's dequantize + fp64 SDPA."""
    import math

    import torch
    import torch.distributed as dist

    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    t0, t1 = seqsplit.shard_bounds(C4_N - 1, world, rank)
    per_tok = C4_HKV * 2 * (C4_D // 2 + 4 * (C4_D // 64))
    shard_bytes = (t1 - t0) * per_tok
    layers_n = max(2, math.ceil(400e6 / max(shard_bytes, 1)))
    host_cache = None
    if check and rank == 0:
        from oracle import oracle as O
        O.set_num_threads(os.cpu_count() or 1)
        host_cache = {"k": [], "v": []}  # per chunk: (codes, scales, biases)

    def rms_norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True)) * w

    wq = 1 + 0.1 * torch.randn(C4_D, device=dev, generator=gen)
    wk = 1 + 0.1 * torch.randn(C4_D, device=dev, generator=gen)
    layers = []
    for li in range(layers_n):
        sc = seqsplit.SeqSplitCache(C4_N - 1, C4_HKV, C4_D, capacity_extra=4, device=dev)
        # every rank draws the same full-sequence chunks, quantizes its own slice
        step_tok = 16384
        for c0 in range(0, C4_N - 1, step_tok):
            c1 = min(C4_N - 1, c0 + step_tok)
            k = rms_norm(torch.randn(1, C4_HKV, c1 - c0, C4_D, device=dev, generator=gen), wk).half()
            v = torch.randn(1, C4_HKV, c1 - c0, C4_D, device=dev, generator=gen).half()
            a, b = max(c0, sc.t0), min(c1, sc.t1)
            if b > a:
                sc.cache.append(k[:, :, a - c0:b - c0], v[:, :, a - c0:b - c0], pos=a - sc.t0)
            if host_cache is not None and li == 0:  # the oracle quantizes the same values itself
                host_cache["k"].append(O.quantize(k.float().cpu().numpy()))
                host_cache["v"].append(O.quantize(v.float().cpu().numpy()))
        q = rms_norm(torch.randn(1, C4_H, C4_D, device=dev, generator=gen), wq).half()
        kn = rms_norm(torch.randn(1, C4_HKV, 1, C4_D, device=dev, generator=gen), wk).half()
        vn = torch.randn(1, C4_HKV, 1, C4_D, device=dev, generator=gen).half()
        out = torch.empty(1, C4_H, C4_D, dtype=torch.float16, device=dev)
        part = torch.empty(1, C4_H * (C4_D + 2), dtype=torch.float32, device=dev)
        parts = torch.empty(world, 1, C4_H * (C4_D + 2), dtype=torch.float32, device=dev)
        layers.append(dict(sc=sc, q=q, kn=kn, vn=vn, out=out, part=part, parts=parts))
    n_local = layers[0]["sc"].n_local
    last = rank == world - 1
    ws = tq.workspace(dev, tq.sdpa_int4_workspace_size(1, C4_H, C4_HKV, C4_D, n_local + 1, 0))
    peer = (seqsplit.PeerExchange(1, C4_H, C4_D, device=dev)
            if world > 1 and args.exchange in ("peer", "published") else None)
    published = peer is not None and args.exchange == "published"
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)

    def partial(Lr):
        sc = Lr["sc"]
        if last:  # the appended token rewrites the same slot every rotation
            tq.quantize_append(Lr["kn"], Lr["vn"], *sc.cache.tensors(), pos=n_local, s=stream)
        nl = n_local + (1 if last else 0)
        tq.sdpa_int4_partial(Lr["q"], *sc.cache.tensors(), C4_H // C4_HKV, 1.0, 0, n_local=nl,
                             token_offset=sc.t0, n_total=C4_N, part_out=Lr["part"], ws=ws, s=stream)

    def exchange(Lr):
        if peer is not None:
            peer.merge(Lr["part"], out=Lr["out"], s=stream)
            return
        if world > 1:
            dist.all_gather_into_tensor(Lr["parts"], Lr["part"])
            tq.lse_merge(Lr["parts"], C4_H, C4_D, out=Lr["out"], s=stream)
        else:  # one GPU: the merge normalises the one state in place
            tq.lse_merge(Lr["part"].view(1, 1, -1), C4_H, C4_D, out=Lr["out"], s=stream)

    def step(Lr):
        if published:  # the decode kernel stores the states; a merge-only launch follows
            sc = Lr["sc"]
            # the last rank's decode launch quantizes the new token in as well
            kn = Lr["kn"].reshape(1, C4_HKV, C4_D) if last else None
            vn = Lr["vn"].reshape(1, C4_HKV, C4_D) if last else None
            peer.decode(Lr["q"], sc.cache.tensors(), n_local + (1 if last else 0), sc.t0, C4_N,
                        C4_H // C4_HKV, 1.0, 0, out=Lr["out"], ws=ws, k_new=kn, v_new=vn, s=stream)
            return
        partial(Lr)
        exchange(Lr)

    with torch.cuda.stream(stream):
        for Lr in layers:
            step(Lr)
    torch.cuda.synchronize()
    CH = 4 * layers_n

    def capture(fn, n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    fn(layers[i % layers_n])
        return g

    # (published: a merge-only graph would wait for states nobody publishes;
    # its time is the step's minus the plain partial decode's)
    graphs = {"step": capture(step, CH), "partial": capture(partial, CH)}
    if not published:
        graphs["exchange"] = capture(exchange, CH)
    singles = [capture(step, 1) for _ in range(1)]  # the host-buffer leg re-targets layer 0 only
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # every rank has its graphs before any rank's first peer merge
    reps = max(1, steps // CH)
    clocks = Clocks(local_rank)
    clocks.start()
    times = {}
    for name in graphs:
        with torch.cuda.stream(stream):
            graphs[name].replay()  # warm-up
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        times[name] = _graph_time(stream, graphs[name], reps)
        if world > 1:
            dist.barrier()
    clk = clocks.stop()
    n_timed = reps * CH

    # end to end from host buffers on every rank: the step's q | k_new | v_new
    # go up from pinned memory, the step graph runs, the merged output comes
    # back and the host synchronises; host clock, max over ranks
    L0 = layers[0]
    nq, nkv = C4_H * C4_D, C4_HKV * C4_D
    hin = torch.empty(nq + 2 * nkv, dtype=torch.float16, pin_memory=True)
    hin[:nq].copy_(L0["q"].reshape(-1).cpu())
    hin[nq:nq + nkv].copy_(L0["kn"].reshape(-1).cpu())
    hin[nq + nkv:].copy_(L0["vn"].reshape(-1).cpu())
    hout = torch.empty(1, C4_H, C4_D, dtype=torch.float16, pin_memory=True)
    din = torch.empty(nq + 2 * nkv, dtype=torch.float16, device=dev)

    def host_step():
        with torch.cuda.stream(stream):
            din.copy_(hin, non_blocking=True)
            L0["q"].view(-1).copy_(din[:nq], non_blocking=True)
            L0["kn"].view(-1).copy_(din[nq:nq + nkv], non_blocking=True)
            L0["vn"].view(-1).copy_(din[nq + nkv:], non_blocking=True)
            singles[0].replay()
            hout.copy_(L0["out"], non_blocking=True)
        stream.synchronize()

    for _ in range(4):
        host_step()
    e2e_steps = 64
    if world > 1:
        dist.barrier()
    th0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_step()
    e2e_ms = (time.perf_counter() - th0) * 1000.0
    assert tq.device_error() == 0, "a kernel reported a device error"

    if published:
        times["exchange"] = times["step"] - times["partial"]
    tt = torch.tensor([times["step"], times["partial"], times["exchange"], e2e_ms], device=dev,
                      dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_step, t_part, t_exch, e2e_ms = (float(x) for x in tt)

    acc = None
    if host_cache is not None:
        O.set_num_threads(os.cpu_count() or 1)  # torch.distributed.run exports OMP_NUM_THREADS=1
        # the appended token sits at global position C4_N - 1 on the last rank
        host_cache["k"].append(O.quantize(L0["kn"].float().cpu().numpy()))
        host_cache["v"].append(O.quantize(L0["vn"].float().cpu().numpy()))
        full = [np.concatenate([c[f] for c in host_cache[kv]], axis=2)
                for kv in ("k", "v") for f in range(3)]
        G = C4_H // C4_HKV
        qh = L0["q"].float().cpu().numpy()
        refs = []
        for g0 in range(0, C4_HKV, 2):
            sl = slice(g0, g0 + 2)
            refs.append(O.sdpa_int4(qh[:, g0 * G:(g0 + 2) * G], *(a[:, sl] for a in full), f64=True))
        ref = np.concatenate(refs, axis=1).astype(np.float64)
        got = hout.float().numpy().astype(np.float64)
        acc = {"max_abs": float(np.max(np.abs(got - ref))),
               "cosine": float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref))),
               "oracle": "C oracle: quantize of the same values, dequantize + fp64 SDPA over all "
                         "262144 tokens (layer 0, after the timed steps)"}
        del full, host_cache
    if world > 1:
        dist.barrier()

    cpu = None
    if rank == 0 and world == 1 and check and not args.no_cpu_baseline:
        cpu = cpu_reference_cfg4(L0)
    del graphs, singles
    torch.cuda.synchronize()
    if peer is not None:
        peer.close()
    us_step = t_step * 1000.0 / n_timed
    us_part = t_part * 1000.0 / n_timed
    us_exch = t_exch * 1000.0 / n_timed
    total_bytes = C4_N * per_tok
    peaks = measured_peaks()
    # HBM roofline of the partial decode on the largest shard: algorithmic
    # bytes of that shard (+ q and the fp32 state) over its time
    shard_max = (seqsplit.shard_bounds(C4_N - 1, world, world - 1)[1]
                 - seqsplit.shard_bounds(C4_N - 1, world, world - 1)[0] + 1)
    part_bytes = shard_max * per_tok + C4_H * C4_D * 2 + C4_H * (C4_D + 2) * 4
    ach = part_bytes / (us_part * 1e-6) / 1e9
    return {
        "workload": "cfg4 decode step: 262144-token global layer (H=32, Hkv=8, D=256) split by "
                    "sequence, append + partial decode + " +
                    ("decode kernel stores its states into the peers' buffers + merge-only "
                     "kernel" if published else
                     "peer-memory exchange + merge (one kernel)" if peer is not None else
                     "NCCL all-gather + LSE merge" if world > 1 else
                     "LSE normalisation of the one state (no exchange on one GPU)"),
        "metric": "int4-KV decode-attention tokens/s", "unit": "tokens/s", "scaling": "strong",
        "n_gpus": world, "steps": n_timed,
        "value": n_timed / (t_step / 1000.0), "ms_per_step": t_step / n_timed,
        "time_split_us": {"step": us_step, "append_plus_partial_decode": us_part,
                          "exchange_plus_merge": us_exch,
                          "limiter": ("partial decode (HBM stream of the shard)"
                                      if us_part >= 0.6 * us_step else "exchange + merge")},
        "hbm_gbs_per_gpu": shard_bytes / (us_step * 1e-6) / 1e9,
        "hbm_gbs_total": total_bytes / (us_step * 1e-6) / 1e9,
        "roofline": {"bound": "hbm", "kernel": "tq::decode_mma_kernel<256,4,__half> (partial)",
                     "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / peaks["hbm_gbs"], "frac_of_8tbs_nominal": ach / 8000.0,
                     "kernel_us": us_part, "algorithmic_bytes_per_launch": part_bytes,
                     "traffic": None, "peak_source": peaks["source"]},
        "accuracy_vs_oracle": acc,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_steps / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": (nq + 2 * nkv) * 2, "d2h_bytes_per_step": nq * 2,
                "path": "pinned q|k_new|v_new -> device on every rank, step graph (append + " +
                        ("tq_sdpa_int4_partial_publish + tq_peer_merge_published" if published else
                         "tq_sdpa_int4_partial + tq_peer_merge" if peer is not None else
                         "tq_sdpa_int4_partial + " + ("NCCL all-gather + " if world > 1 else "") +
                         "tq_lse_merge") +
                        "), merged output -> pinned host, stream sync; host clock, max over ranks"},
        "layers_rotated": layers_n,
        "l2": f"inputs larger than L2: {layers_n} rotating shards of {shard_bytes / 1e6:.0f} MB",
        "gpu_launches_per_step": ("decode_mma_kernel (partial; the new token's append fused on the "
                                  "last rank), " if published else
                                  "quantize_rows_kernel (last rank), decode_mma_kernel (partial), ") + (
                                  ("peer_merge_published_kernel" if published else
                                   "peer_merge_kernel" if peer is not None else
                                   "lse_merge_kernel" + (" + NCCL all-gather" if world > 1 else ""))),
        "clocks": clk,
    }


def run_cfg4_heads(args, rank: int, world: int, local_rank: int, steps: int = 256,
                   check: bool = True):
    """Config 4 split by KV heads (N > 1, Hkv % N == 0): rank r holds the
    whole 262144-token int4 cache of KV heads seqsplit.head_bounds(8, N, r)
    and their query heads; one step = quantize-on-append of the new token +
    decode of those heads in one launch (tq_sdpa_int4_append), then an NCCL
    all-gather of the (H/N, D) outputs so every rank holds the full (H, D)
    output -- the exchange of the head-parallel form. Captured in CUDA graphs
    over rotating layers (inputs larger than L2); max over ranks. `check`:
    rank 0 compares its heads' output with the C oracle's dequantize + fp64
    SDPA over all tokens (the oracle quantizes the same values itself)."""
    import math

    import torch
    import torch.distributed as dist

    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import seqsplit

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    h0, h1 = seqsplit.head_bounds(C4_HKV, world, rank)
    hk = h1 - h0
    G = C4_H // C4_HKV
    hq = hk * G
    n_ctx = C4_N  # the new token is the last of the 262144
    per_tok = hk * 2 * (C4_D // 2 + 4 * (C4_D // 64))
    shard_bytes = (n_ctx - 1) * per_tok
    layers_n = max(2, math.ceil(400e6 / max(shard_bytes, 1)))
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    host = None
    if check and rank == 0:
        from oracle import oracle as O
        O.set_num_threads(os.cpu_count() or 1)
        host = {"k": [], "v": []}

    def rms_norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True)) * w

    wq = 1 + 0.1 * torch.randn(C4_D, device=dev, generator=gen)
    wk = 1 + 0.1 * torch.randn(C4_D, device=dev, generator=gen)
    cap = (n_ctx + 3) // 4 * 4
    layers = []
    for li in range(layers_n):
        cache = tq.KVCache(1, hk, C4_D, cap, device=dev)
        step_tok = 16384
        for c0 in range(0, n_ctx - 1, step_tok):
            c1 = min(n_ctx - 1, c0 + step_tok)
            # every rank draws the same full chunk and keeps its heads
            k = rms_norm(torch.randn(1, C4_HKV, c1 - c0, C4_D, device=dev, generator=gen), wk).half()
            v = torch.randn(1, C4_HKV, c1 - c0, C4_D, device=dev, generator=gen).half()
            cache.append(k[:, h0:h1].contiguous(), v[:, h0:h1].contiguous(), pos=c0)
            if host is not None and li == 0:
                host["k"].append(O.quantize(k[:, h0:h1].float().cpu().numpy()))
                host["v"].append(O.quantize(v[:, h0:h1].float().cpu().numpy()))
            del k, v
        q = rms_norm(torch.randn(1, C4_H, C4_D, device=dev, generator=gen), wq).half()
        kn = rms_norm(torch.randn(1, C4_HKV, 1, C4_D, device=dev, generator=gen), wk).half()
        vn = torch.randn(1, C4_HKV, 1, C4_D, device=dev, generator=gen).half()
        layers.append(dict(cache=cache, q=q[:, h0 * G:h1 * G].contiguous(),
                           kn=kn[:, h0:h1, 0].contiguous(), vn=vn[:, h0:h1, 0].contiguous(),
                           kn_full=kn, vn_full=vn,
                           out=torch.empty(1, hq, C4_D, dtype=torch.float16, device=dev),
                           full=torch.empty(world, 1, hq, C4_D, dtype=torch.float16, device=dev)))
    ws = tq.workspace(dev, tq.sdpa_int4_workspace_size(1, hq, hk, C4_D, n_ctx, 0))
    stream = torch.cuda.Stream(device=dev)
    peer = args.gather == "peer"
    ex = seqsplit.PeerExchange(1, hq, C4_D, device=dev) if peer else None
    for Lr in layers:
        Lr["gathered"] = torch.empty(1, C4_H, C4_D, dtype=torch.float16, device=dev)

    def decode(Lr):
        tq.sdpa_int4_append(Lr["q"], Lr["kn"], Lr["vn"], *Lr["cache"].tensors(), G, 1.0, 0, stream,
                            n_tokens=n_ctx, out=Lr["out"], ws=ws)

    def step(Lr):
        if peer:  # the decode publishes its heads' state; a gather kernel assembles the output
            ex.decode_heads(Lr["q"], Lr["cache"].tensors(), n_ctx, G, 1.0, 0, out=Lr["gathered"],
                            ws=ws, k_new=Lr["kn"], v_new=Lr["vn"], s=stream)
            return
        decode(Lr)
        dist.all_gather_into_tensor(Lr["full"], Lr["out"])

    with torch.cuda.stream(stream):
        for Lr in layers:
            step(Lr)
    torch.cuda.synchronize()
    CH = 4 * layers_n

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i in range(CH):
                    fn(layers[i % layers_n])
        return g

    graphs = {"step": capture(step), "decode": capture(decode)}
    torch.cuda.synchronize()
    dist.barrier()
    reps = max(1, steps // CH)
    times = {}
    for name, g in graphs.items():
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        times[name] = _graph_time(stream, g, reps)
        dist.barrier()
    n_timed = reps * CH
    tt = torch.tensor([times["step"], times["decode"]], device=dev, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_step, t_dec = (float(x) for x in tt)
    assert tq.device_error() == 0, "a kernel reported a device error"

    acc = None
    if host is not None:
        L0 = layers[0]
        O.set_num_threads(os.cpu_count() or 1)
        host["k"].append(O.quantize(L0["kn"][:, :, None].float().cpu().numpy()))
        host["v"].append(O.quantize(L0["vn"][:, :, None].float().cpu().numpy()))
        full = [np.concatenate([c[f] for c in host[kv]], axis=2) for kv in ("k", "v") for f in range(3)]
        qh = L0["q"].float().cpu().numpy()
        refs = []
        for g0 in range(0, hk, 2):
            sl = slice(g0, min(hk, g0 + 2))
            refs.append(O.sdpa_int4(qh[:, g0 * G:min(hk, g0 + 2) * G], *(a[:, sl] for a in full), f64=True))
        ref = np.concatenate(refs, axis=1).astype(np.float64)
        # the gathered output: rank 0's block holds its heads
        got = (L0["gathered"][:, :hq] if peer else L0["full"][0]).float().cpu().numpy().astype(np.float64)
        acc = {"max_abs": float(np.max(np.abs(got - ref))),
               "cosine": float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref))),
               "oracle": f"C oracle: quantize of the same values, dequantize + fp64 SDPA over all "
                         f"{n_ctx} tokens of rank 0's {hk} KV heads (layer 0, after the timed steps)"}
        del full, host
    dist.barrier()
    del graphs
    torch.cuda.synchronize()
    if ex is not None:
        ex.close()
    us_step = t_step * 1000.0 / n_timed
    us_dec = t_dec * 1000.0 / n_timed
    dec_bytes = n_ctx * per_tok + hq * C4_D * 4
    peaks = measured_peaks()
    ach = dec_bytes / (us_dec * 1e-6) / 1e9
    return {
        "workload": f"cfg4 decode step: 262144-token global layer (H=32, Hkv=8, D=256) split by KV "
                    f"heads ({hk} per GPU): append + decode of the rank's heads in one launch, " +
                    ("its state stored into every rank's buffer over NVLink + a gather kernel"
                     if peer else "NCCL all-gather of the outputs"),
        "metric": "int4-KV decode-attention tokens/s", "unit": "tokens/s", "scaling": "strong",
        "n_gpus": world, "steps": n_timed,
        "value": n_timed / (t_step / 1000.0), "ms_per_step": t_step / n_timed,
        "time_split_us": {"step": us_step, "append_plus_decode": us_dec,
                          "gather": us_step - us_dec},
        "roofline": {"bound": "hbm", "kernel": f"tq::decode_mma_kernel<256,4,__half> ({hk} KV heads)",
                     "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / peaks["hbm_gbs"], "kernel_us": us_dec,
                     "algorithmic_bytes_per_launch": dec_bytes, "traffic": None,
                     "peak_source": peaks["source"]},
        "accuracy_vs_oracle": acc,
        "layers_rotated": layers_n,
        "l2": f"inputs larger than L2: {layers_n} rotating caches of {shard_bytes / 1e6:.0f} MB",
        "gpu_launches_per_step": ("decode_mma_kernel (append fused, state published) + "
                                  "peer_gather_published_kernel" if peer else
                                  "decode_mma_kernel (append fused) + NCCL all-gather"),
    }


def cpu_reference_cfg4(L0) -> dict:
    """The reference's algorithm for config 4 on the host (dequantize + fp32
    SDPA, the C oracle with OpenMP over all host threads) on a bounded
    sample: 2 of the 8 KV heads (8 of the 32 query heads) over all 262144
    tokens, scaled to a whole step (x4)."""
    from oracle import oracle as O
    O.set_num_threads(os.cpu_count() or 1)
    sc = L0["sc"]
    n = sc.n_local
    arrs = [t[:, 0:2, :n].cpu().numpy() for t in sc.cache.tensors()]
    arrs = [a.view(np.uint32) if a.dtype == np.int32 else a for a in arrs]
    q = L0["q"][:, 0:8].float().cpu().numpy()
    base = O.Int4Baseline(q, *arrs)
    base()
    t0 = time.perf_counter()
    reps = 0
    while reps < 2 or time.perf_counter() - t0 < 4.0:
        base()
        reps += 1
    dt = (time.perf_counter() - t0) / reps * 4.0
    return {"value": 1.0 / dt, "unit": "tokens/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{reps} runs of 2 of 8 KV heads over {n} tokens (dequantize + fp32 SDPA, "
                      f"the shard of this GPU), scaled x4 to the whole step"}


# ----------------------------------------- config 2: tcgen05 multi-query --

C2_N0, C2_B, C2_CHUNK, C2_LAYERS = 8192, 64, 512, 12


def cfg2_flops() -> dict:
    """Algorithmic FLOPs of one launch (QK^T and PV, 2 flops per MAC each):
    batched: every query sees all N0 tokens; prefill: query i sees N0 + i + 1."""
    vis_pre = sum(C2_N0 + i + 1 for i in range(C2_CHUNK))
    return {"batched": 4.0 * H * D * C2_N0 * C2_B, "prefill": 4.0 * H * D * vis_pre}


def run_cfg2(args, rank: int, world: int, local_rank: int):
    """Config 2 on the tcgen05 kernel, two workloads over C2_LAYERS rotating
    layer caches (each 8.7K tokens x 16 KV heads, 20 MB; 250 MB in all):
    batched decode = 64 sequences x 1 query attending over one shared 8K-token
    int4 cache; prefill chunk = quantize-append of 512 new tokens' K/V, then
    the 512 causal queries at positions 8192..8703 over 8704 tokens.
    Q and outputs bf16. Each rank runs its own layers (weak scaling)."""
    import torch
    import torch.distributed as dist
    import gemma4metal_b200.turboquant as tq

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    N = C2_N0 + C2_CHUNK

    def rms_norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True)) * w

    wq = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    wk = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    layers = []
    for _ in range(C2_LAYERS):
        cache = tq.KVCache(1, HKV, D, N, device=dev)
        k = rms_norm(torch.randn(1, HKV, C2_N0, D, device=dev, generator=gen), wk).half()
        v = torch.randn(1, HKV, C2_N0, D, device=dev, generator=gen).half()
        cache.append(k, v, pos=0)
        kc = rms_norm(torch.randn(1, HKV, C2_CHUNK, D, device=dev, generator=gen), wk).half()
        vc = torch.randn(1, HKV, C2_CHUNK, D, device=dev, generator=gen).half()
        qb = rms_norm(torch.randn(C2_B, H, D, device=dev, generator=gen), wq).bfloat16()
        qp = rms_norm(torch.randn(C2_CHUNK, H, D, device=dev, generator=gen), wq).bfloat16()
        layers.append(dict(cache=cache, kc=kc, vc=vc, qb=qb, qp=qp,
                           ob=torch.empty(C2_B, H, D, dtype=torch.bfloat16, device=dev),
                           op=torch.empty(C2_CHUNK, H, D, dtype=torch.bfloat16, device=dev)))
    lib = tq.load_library()
    ws = tq.workspace(dev, max(int(lib.tq_sdpa_int4_multi_workspace_size(C2_B, H, HKV, D, C2_N0)),
                               int(lib.tq_sdpa_int4_multi_workspace_size(C2_CHUNK, H, HKV, D, N))))
    stream = torch.cuda.Stream(device=dev)

    def batched(Lr):
        tq.sdpa_int4_multi(Lr["qb"], *Lr["cache"].tensors(), H // HKV, 1.0, 0, n_tokens=C2_N0,
                           out=Lr["ob"], ws=ws, s=stream)

    def prefill(Lr, with_append=True):
        c = Lr["cache"]
        if with_append:  # rewrites the same 512 slots every rotation
            tq.quantize_append(Lr["kc"], Lr["vc"], *c.tensors(), pos=C2_N0, s=stream)
        tq.sdpa_int4_multi(Lr["qp"], *c.tensors(), H // HKV, 1.0, 0, n_tokens=N, causal=True,
                           pos0=C2_N0, out=Lr["op"], ws=ws, s=stream)

    with torch.cuda.stream(stream):
        for Lr in layers:
            prefill(Lr)
            batched(Lr)
    torch.cuda.synchronize()
    CH = 2 * C2_LAYERS

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i in range(CH):
                    fn(layers[i % C2_LAYERS])
        return g

    graphs = {"batched": capture(batched), "prefill": capture(prefill),
              "prefill_attn": capture(lambda Lr: prefill(Lr, False))}
    torch.cuda.synchronize()

    def timed(name, steps, warmup):
        g = graphs[name]
        reps = max(1, steps // CH)
        with torch.cuda.stream(stream):
            for _ in range(max(1, warmup // CH)):
                g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return reps * CH, e0.elapsed_time(e1)

    clocks = Clocks(local_rank)
    clocks.start()
    nb, tb = timed("batched", args.steps, max(args.warmup, CH))
    npf, tpf = timed("prefill", max(CH, args.steps // 4), max(args.warmup, CH))
    # kernel times for the roofline: >= 1.5 s of replays each, so the clock
    # sampler sees the kernels under load
    soak = {}
    for name in ("batched", "prefill_attn"):
        g = graphs[name]
        k0 = torch.cuda.Event(enable_timing=True)
        k1 = torch.cuda.Event(enable_timing=True)
        reps, t_start = 0, time.perf_counter()
        k0.record(stream)
        with torch.cuda.stream(stream):
            while time.perf_counter() - t_start < 1.5 or reps < 8:
                for _ in range(8):
                    g.replay()
                reps += 8
                if reps % 64 == 0:
                    stream.synchronize()
        k1.record(stream)
        torch.cuda.synchronize()
        soak[name] = (reps * CH, k0.elapsed_time(k1))
    clk = clocks.stop()
    (nkb, tkb), (npa, tpa) = soak["batched"], soak["prefill_attn"]

    # end to end through the public API: queries from pinned host memory in,
    # outputs back to pinned host memory, every step
    hq = torch.empty(C2_B, H, D, dtype=torch.bfloat16, pin_memory=True)
    ho = torch.empty(C2_B, H, D, dtype=torch.bfloat16, pin_memory=True)
    hq.copy_(layers[0]["qb"].cpu())
    e2e_steps = max(10, min(args.steps, 1000))

    def e2e_loop(n):
        with torch.cuda.stream(stream):
            for i in range(n):
                Lr = layers[i % C2_LAYERS]
                Lr["qb"].copy_(hq, non_blocking=True)
                batched(Lr)
                ho.copy_(Lr["ob"], non_blocking=True)
                stream.synchronize()

    e2e_loop(10)
    torch.cuda.synchronize()
    ee0 = torch.cuda.Event(enable_timing=True)
    ee1 = torch.cuda.Event(enable_timing=True)
    ee0.record(stream)
    e2e_loop(e2e_steps)
    ee1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ee0.elapsed_time(ee1)
    assert tq.device_error() == 0, "a kernel reported a device error"
    tt = torch.tensor([tb, tpf, tpa, tkb, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    tb, tpf, tpa, tkb, e2e_ms = (float(x) for x in tt)
    del graphs
    torch.cuda.synchronize()
    return dict(nb=nb, tb=tb, npf=npf, tpf=tpf, npa=npa, tpa=tpa, nkb=nkb, tkb=tkb, e2e_ms=e2e_ms,
                e2e_steps=e2e_steps, clocks=clk)


def cpu_reference_cfg2(budget_s: float = 15.0, seed: int = 7):
    """The reference's algorithm for config 2 on the host: MLX-style
    dequantize of the int4 cache to fp32, then SDPA in fp32 with the causal
    mask the engine builds (engine/gemma4_multilayer.cpp:307-308,347-367) —
    numpy matmuls over all host threads. Times one batched-decode step
    (64 queries x 8K tokens) and the prefill chunk on a bounded sample of
    its queries; returns queries/s for each."""
    from oracle import inputs, oracle as O
    L = inputs.make_layer(seed, H, HKV, D, C2_N0 + C2_CHUNK)
    kq, ks, kb = O.quantize(L["k"][0])
    vq, vs, vb = O.quantize(L["v"][0])
    del L
    rng = np.random.default_rng(seed)
    G = H // HKV

    def attend(q, n_tokens, pos):
        kd = O.dequantize_np(kq, ks, kb)[:, :n_tokens].astype(np.float32)
        vd = O.dequantize_np(vq, vs, vb)[:, :n_tokens].astype(np.float32)
        nq = q.shape[0]
        out = np.empty((nq, H, D), np.float32)
        t = np.arange(n_tokens)
        vis = t[None, :] <= pos[:, None]
        for hk in range(HKV):
            qh = q[:, hk * G:(hk + 1) * G].reshape(nq * G, D)
            s = qh @ kd[hk].T
            s = np.where(np.repeat(vis, G, axis=0), s, -np.inf)
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            o = (p @ vd[hk]) / p.sum(axis=1, keepdims=True)
            out[:, hk * G:(hk + 1) * G] = o.reshape(nq, G, D)
        return out

    qb = rng.standard_normal((C2_B, H, D)).astype(np.float32)
    attend(qb[:4], C2_N0, np.full(4, C2_N0 - 1))  # untimed warm-up
    t0 = time.perf_counter()
    nb = 0
    while nb == 0 or time.perf_counter() - t0 < budget_s / 2:
        attend(qb, C2_N0, np.full(C2_B, C2_N0 - 1))
        nb += 1
    tb = time.perf_counter() - t0
    sample = 64  # queries of the 512-query chunk per timed call (positions spread over the chunk)
    qp = rng.standard_normal((sample, H, D)).astype(np.float32)
    pos = C2_N0 + np.linspace(0, C2_CHUNK - 1, sample).astype(np.int64)
    t0 = time.perf_counter()
    npf = 0
    while npf == 0 or time.perf_counter() - t0 < budget_s / 2:
        attend(qp, C2_N0 + C2_CHUNK, pos)
        npf += 1
    tp = time.perf_counter() - t0
    return {"batched_tokens_s": nb * C2_B / tb, "prefill_tokens_s": npf * sample / tp,
            "cores": os.cpu_count(), "seconds": tb + tp,
            "sample": f"{nb} batched steps (64 queries x 8192 tokens) and {npf} x {sample} of the "
                      f"512 prefill queries (positions spread over the chunk), dequantize + fp32 SDPA"}


def cfg2_line(args, world, res, cpu):
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    src = "measured (MEASURED_PEAKS.json bf16_tflops, burst)" if peaks else "fallback"
    fl = cfg2_flops()
    us_b = res["tkb"] * 1000.0 / res["nkb"]
    us_pa = res["tpa"] * 1000.0 / res["npa"]
    ach_b = fl["batched"] / (us_b * 1e-6) / 1e12
    ach_p = fl["prefill"] / (us_pa * 1e-6) / 1e12
    traffic = None
    path = os.path.join(ROOT, "profiles", "attn_tc_cfg2.md")
    if os.path.exists(path):
        m = re.search(r"traffic_bytes_per_launch_batched:\s*([0-9.eE+]+)", open(path).read())
        traffic = float(m.group(1)) if m else None
    value = res["nb"] * C2_B * world / (res["tb"] / 1000.0)
    line = {"metric": "int4-KV decode-attention tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": res["nb"], "warmup": args.warmup,
            "ms_per_step": res["tb"] / res["nb"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 (exact int4 codes and bf16-exact Q on the tensor cores), f32 softmax",
            "data": "synthetic (seeded torch.randn, RMS-normalised Q/K as task configs[0])",
            "config": {"workload": "cfg2 batched decode: 64 sequences x 1 query over one shared "
                                   "8192-token int4 cache (tcgen05)",
                       "batch": C2_B, "heads": H, "kv_heads": HKV, "head_dim": D, "context": C2_N0,
                       "q_out": "bf16", "layers_rotated": C2_LAYERS,
                       "l2": f"inputs larger than L2: {C2_LAYERS} rotating 20 MB layer caches",
                       "parallelism": f"dp{world} (independent layers per GPU)"},
            "roofline": {"bound": "tensor", "achieved": ach_b, "peak": peak, "unit": "TFLOP/s",
                         "frac": ach_b / peak, "traffic": traffic,
                         "kernel": "tq::attn_tc_kernel (tcgen05.mma kind::f16, TMEM) + attn_tc_merge_kernel",
                         "kernel_us": us_b, "algorithmic_flops_per_launch": fl["batched"],
                         "peak_source": src},
            "prefill_chunk": {"workload": "cfg2 prefill: append 512 tokens + 512 causal queries at "
                                          "8192..8703 (tcgen05)",
                              "tokens_per_s": res["npf"] * C2_CHUNK * world / (res["tpf"] / 1000.0),
                              "ms_per_step": res["tpf"] / res["npf"],
                              "attn_us": us_pa, "attn_tflops": ach_p, "attn_frac": ach_p / peak},
            "cpu_baseline": None if cpu is None else {
                "value": cpu["batched_tokens_s"], "unit": "tokens/s", "cores": cpu["cores"],
                "kind": "port", "sample": cpu["sample"],
                "prefill_tokens_s": cpu["prefill_tokens_s"]},
            "e2e": {"value": res["e2e_steps"] * C2_B * world / (res["e2e_ms"] / 1000.0),
                    "unit": "tokens/s", "h2d_bytes_per_step": C2_B * H * D * 2,
                    "d2h_bytes_per_step": C2_B * H * D * 2,
                    "path": "gemma4metal_b200.turboquant.sdpa_int4_multi (ctypes C ABI), batched"},
            "gpu_launches": 2 * res["nb"],
            "launches_per_step": "2 (attn_tc_kernel, attn_tc_merge_kernel)",
            "clocks": res["clocks"]}
    return line


# ------------------------------------------------- config 0: one layer --

C0_N, C0_LAYERS, C0_STEPS = 1024, 128, 1024


def run_cfg0(args, local_rank: int) -> dict:
    """Config 0: one decode step of one attention layer over 1024 cached
    tokens (H=32, Hkv=16, D=128, fp16 Q/out, scale 1.0), no append: the
    reference test's single-layer case. 128 rotating layer caches (302 MB,
    larger than L2); one graph of C0_STEPS steps. Latency-bound: 2.4 MB per
    step."""
    import torch

    import gemma4metal_b200.turboquant as tq
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)

    def rms_norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True)) * w

    wq = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    wk = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    layers = []
    for _ in range(C0_LAYERS):
        cache = tq.KVCache(1, HKV, D, C0_N, device=dev)
        cache.append(rms_norm(torch.randn(1, HKV, C0_N, D, device=dev, generator=gen), wk).half(),
                     torch.randn(1, HKV, C0_N, D, device=dev, generator=gen).half(), pos=0)
        q = rms_norm(torch.randn(1, H, D, device=dev, generator=gen), wq).half()
        layers.append(dict(cache=cache, q=q, out=torch.empty(1, H, D, dtype=torch.float16, device=dev)))
    ws = tq.workspace(dev, tq.sdpa_int4_workspace_size(1, H, HKV, D, C0_N, 0))
    stream = torch.cuda.Stream(device=dev)

    def step(Lr):
        tq.sdpa_int4(Lr["q"], *Lr["cache"].tensors(), H // HKV, 1.0, 0, s=stream, n_tokens=C0_N,
                     out=Lr["out"], ws=ws)

    with torch.cuda.stream(stream):
        for Lr in layers:
            step(Lr)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for i in range(C0_STEPS):
                step(layers[i % C0_LAYERS])
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    reps = 4
    t_ms = _graph_time(stream, g, reps)
    n = reps * C0_STEPS
    us = t_ms * 1000.0 / n

    # end to end: pinned q up, the decode, the output back, synchronise
    Lr0 = layers[0]
    hq = torch.empty(1, H, D, dtype=torch.float16, pin_memory=True)
    hq.copy_(Lr0["q"].cpu())
    ho = torch.empty(1, H, D, dtype=torch.float16, pin_memory=True)

    def host_step():
        with torch.cuda.stream(stream):
            Lr0["q"].copy_(hq, non_blocking=True)
            step(Lr0)
            ho.copy_(Lr0["out"], non_blocking=True)
        stream.synchronize()

    for _ in range(20):
        host_step()
    e2e_n = 500
    th = time.perf_counter()
    for _ in range(e2e_n):
        host_step()
    e2e_ms = (time.perf_counter() - th) * 1000.0
    assert tq.device_error() == 0, "a kernel reported a device error"
    del g
    torch.cuda.synchronize()

    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as O
        O.set_num_threads(os.cpu_count() or 1)
        arrs = [t.cpu().numpy() for t in Lr0["cache"].tensors()]
        arrs = [a.view(np.uint32) if a.dtype == np.int32 else a for a in arrs]
        base = O.Int4Baseline(Lr0["q"].cpu().numpy(), *arrs)
        base()
        t0 = time.perf_counter()
        k = 0
        while k < 5 or time.perf_counter() - t0 < 2.0:
            base()
            k += 1
        dt = (time.perf_counter() - t0) / k
        cpu = {"value": 1.0 / dt, "unit": "tokens/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{k} decode steps of the same layer (dequantize + fp32 SDPA, C oracle)"}
    bytes_step = 2304 * C0_N + 2 * H * D * 2
    peaks = measured_peaks()
    ach = bytes_step / (us * 1e-6) / 1e9
    return {"workload": "cfg0 decode step: one layer, 1024 tokens, no append (sdpa_int4)",
            "metric": "int4-KV decode-attention tokens/s", "unit": "tokens/s", "steps": n,
            "value": n / (t_ms / 1000.0), "ms_per_step": t_ms / n, "latency_us": us,
            "roofline": {"bound": "hbm (latency in practice: 2.4 MB per launch)",
                         "kernel": "tq::decode_mma_kernel<128,2,__half,false>", "achieved": ach,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": ach / peaks["hbm_gbs"],
                         "kernel_us": us, "algorithmic_bytes_per_launch": bytes_step,
                         "traffic": None, "peak_source": peaks["source"]},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_n / (e2e_ms / 1000.0), "unit": "tokens/s",
                    "h2d_bytes_per_step": H * D * 2, "d2h_bytes_per_step": H * D * 2,
                    "path": "pinned q -> device, tq_sdpa_int4, output -> pinned host, stream sync "
                            "(host clock)"},
            "layers_rotated": C0_LAYERS, "l2": "inputs larger than L2: 128 rotating 2.4 MB layers",
            "gpu_launches": n}


# ------------------------------------- config 3: PolarQuant + QJL keys --

C3_N, C3_BLOCK, C3_M, C3_LAYERS, C3_STEPS = 4096, 128, 256, 24, 192


def run_cfg3(args, local_rank: int) -> dict:
    """Config 3: compressed-key attention. Keys of 16 KV heads x 4096 tokens
    (D=128) as PolarQuant (one 128-value block: 7 levels of 4-bit angles +
    fp16 radius) + QJL (256 sign bits of the residual through a seeded
    Gaussian 256x128 matrix + fp16 residual norm), int4 V; 32 query heads
    (GQA 2), scale 1.0. A step is one compressed attention (scores with the
    QJL correction, softmax, . int4 V) over one layer; 24 rotating layers
    (270 MB). Encode throughput (polar_quantize + qjl_encode of all 65536
    keys) is timed on its own."""
    import torch

    import gemma4metal_b200.turboquant as tq
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)

    def rms_norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True)) * w

    levels = 7
    cb = tq.uniform_codebooks(levels, device="cpu")
    S = tq.qjl_matrix(C3_M, D, 11, device=dev)
    wq = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    wk = 1 + 0.1 * torch.randn(D, device=dev, generator=gen)
    layers = []
    for _ in range(C3_LAYERS):
        k = rms_norm(torch.randn(HKV, C3_N, D, device=dev, generator=gen), wk)
        v = torch.randn(HKV, C3_N, D, device=dev, generator=gen)
        _, pk, rad = tq.polar_quantize(k, C3_BLOCK, cb)
        kh = tq.polar_dequantize(pk, rad, D, C3_BLOCK, cb)
        sg, rn = tq.qjl_encode(k, kh, S)
        vq, vs, vb = tq.quantize(v.half())
        q = rms_norm(torch.randn(H, D, device=dev, generator=gen), wq).half()
        layers.append(dict(k=k if not layers else None, pk=pk, rad=rad, sg=sg, rn=rn, vq=vq, vs=vs,
                           vb=vb, q=q, out=torch.empty(H, D, dtype=torch.float16, device=dev)))
        del kh, v
    lib = tq.load_library()
    ws = tq.workspace(dev, int(lib.tq_compressed_sdpa_workspace_size(H, HKV, D, C3_N)))
    stream = torch.cuda.Stream(device=dev)

    def step(Lr):
        tq.compressed_sdpa(Lr["q"], Lr["pk"], Lr["rad"], cb, Lr["vq"], Lr["vs"], Lr["vb"], C3_BLOCK,
                           1.0, Lr["sg"], Lr["rn"], S, out=Lr["out"], ws=ws, s=stream)

    with torch.cuda.stream(stream):
        for Lr in layers:
            step(Lr)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for i in range(C3_STEPS):
                step(layers[i % C3_LAYERS])
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    reps = 8
    t_ms = _graph_time(stream, g, reps)
    n = reps * C3_STEPS
    us = t_ms * 1000.0 / n

    # encode of all keys of one layer (polar + its decode for the residual + QJL)
    k0 = layers[0]["k"]
    ek = 10
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        tq.polar_quantize(k0, C3_BLOCK, cb, s=stream)
        e0.record(stream)
        for _ in range(ek):
            _, pk0, rad0 = tq.polar_quantize(k0, C3_BLOCK, cb, s=stream)
            kh0 = tq.polar_dequantize(pk0, rad0, D, C3_BLOCK, cb, s=stream)
            tq.qjl_encode(k0, kh0, S, s=stream)
        e1.record(stream)
    torch.cuda.synchronize()
    enc_us = e0.elapsed_time(e1) * 1000.0 / ek

    # end to end: pinned q up, the compressed attention, the output back, sync
    Lr0 = layers[0]
    hq = torch.empty(H, D, dtype=torch.float16, pin_memory=True)
    hq.copy_(Lr0["q"].cpu())
    ho = torch.empty(H, D, dtype=torch.float16, pin_memory=True)

    def host_step():
        with torch.cuda.stream(stream):
            Lr0["q"].copy_(hq, non_blocking=True)
            step(Lr0)
            ho.copy_(Lr0["out"], non_blocking=True)
        stream.synchronize()

    for _ in range(10):
        host_step()
    e2e_n = 300
    th = time.perf_counter()
    for _ in range(e2e_n):
        host_step()
    e2e_ms = (time.perf_counter() - th) * 1000.0
    assert tq.device_error() == 0, "a kernel reported a device error"
    del g
    torch.cuda.synchronize()

    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as O
        O.set_num_threads(os.cpu_count() or 1)
        hn = lambda t: t.cpu().numpy()
        a = dict(q=hn(Lr0["q"]).astype(np.float32), pk=hn(Lr0["pk"]), rad=hn(Lr0["rad"]),
                 sg=hn(Lr0["sg"]).view(np.uint32), rn=hn(Lr0["rn"]), vq=hn(Lr0["vq"]).view(np.uint32),
                 vs=hn(Lr0["vs"]), vb=hn(Lr0["vb"]), S=hn(S), cb=cb.numpy())

        def one():
            return O.compressed_sdpa(a["q"], a["pk"], a["rad"], a["cb"], C3_BLOCK, a["vq"], a["vs"],
                                     a["vb"], 1.0, a["sg"], a["rn"], a["S"])
        ref = one()
        err = float(np.max(np.abs(ho.float().numpy() - ref)))
        t0 = time.perf_counter()
        kk = 0
        while kk < 3 or time.perf_counter() - t0 < 2.0:
            one()
            kk += 1
        dt = (time.perf_counter() - t0) / kk
        cpu = {"value": 1.0 / dt, "unit": "tokens/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{kk} compressed attention steps of the same layer (C oracle: polar "
                         f"decode + QJL correction + softmax . int4 V)",
               "max_abs_vs_gpu_fp16_out": err}
    per_key = D // 2 + 2 + C3_M // 8 + 2 + (D // 2 + 4 * (D // 64))
    bytes_step = HKV * C3_N * per_key + 2 * H * D * 2
    peaks = measured_peaks()
    ach = bytes_step / (us * 1e-6) / 1e9
    return {"workload": "cfg3 compressed-key attention: PolarQuant (7 levels x 4 bit + fp16 radius) "
                        "+ QJL (256 bits + fp16 norm) keys, int4 V, 16 KV heads x 4096 keys",
            "metric": "int4-KV decode-attention tokens/s", "unit": "tokens/s", "steps": n,
            "value": n / (t_ms / 1000.0), "ms_per_step": t_ms / n,
            "roofline": {"bound": "hbm (latency in practice: 11.3 MB per launch)",
                         "kernel": "tq::compressed_attn_kernel", "achieved": ach,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": ach / peaks["hbm_gbs"],
                         "kernel_us": us, "algorithmic_bytes_per_launch": bytes_step,
                         "traffic": None, "peak_source": peaks["source"]},
            "encode": {"keys": HKV * C3_N, "us": enc_us, "keys_per_s": HKV * C3_N / (enc_us * 1e-6),
                       "kernels": "polar_encode_kernel + polar_decode_kernel (residual) + qjl_encode_kernel"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_n / (e2e_ms / 1000.0), "unit": "tokens/s",
                    "h2d_bytes_per_step": H * D * 2, "d2h_bytes_per_step": H * D * 2,
                    "path": "pinned q -> device, tq_compressed_sdpa, output -> pinned host, stream "
                            "sync (host clock)"},
            "layers_rotated": C3_LAYERS, "l2": "inputs larger than L2: 24 rotating 11.3 MB layers",
            "gpu_launches": n}


# ------------------------------------------------ read-only HBM probe --

def run_probe(local_rank: int) -> dict:
    """tq_read_probe: the read-only ceiling. (a) decode-shaped: one launch
    reads one config-1 layer's cache bytes (75.5 MB) with the decode grid's
    CTA count (432, 3 per SM) through bulk copies into shared memory, 8
    rotating buffers; (b) a 2 GiB stream, bulk copies with 3 CTAs per SM;
    (c) the same with 16-byte non-caching loads, 4 CTAs of 512 threads per SM."""
    import torch

    import gemma4metal_b200.turboquant as tq
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    lib = tq.load_library()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    stream = torch.cuda.Stream(device=dev)
    res = {}
    layer = bytes_per_step(32768, 0)["attn"] - H * D * 4  # cache bytes of one layer
    layer = layer // 16 * 16
    cases = [("decode_shaped", layer, 8, 432, 0), ("stream_bulk", 2 << 30, 1, 3 * sms, 0),
             ("stream_ldg", 2 << 30, 1, 4 * sms, 1)]
    for name, nbytes, nbuf, ctas, mode in cases:
        bufs = [torch.empty(nbytes, dtype=torch.uint8, device=dev).fill_(i + 1) for i in range(nbuf)]
        sink = torch.zeros(ctas, dtype=torch.int32, device=dev)
        launches = 64 if nbuf > 1 else 8

        def go(n):
            for i in range(n):
                b = bufs[i % nbuf]
                tq._check(lib.tq_read_probe(tq._ptr(b), nbytes, ctas, mode, tq._ptr(sink),
                                            tq._stream(stream)))

        go(nbuf)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                go(launches)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        t_ms = _graph_time(stream, g, 4)
        us = t_ms * 1000.0 / (4 * launches)
        res[name] = {"bytes_per_launch": nbytes, "ctas": ctas, "us_per_launch": us,
                     "gbs": nbytes / (us * 1e-6) / 1e9,
                     "mode": "bulk copies into smem" if mode == 0 else "16-byte ld.global.nc"}
        del g, bufs
        torch.cuda.synchronize()
    assert tq.device_error() == 0, "a kernel reported a device error"
    torch.cuda.empty_cache()
    return res


# ----------------------------------------------------------- CPU reference --

def cpu_reference(n_ctx: int, window: int, steps: int, warmup: int, seed: int = 5):
    """Reference algorithm on the host: quantize the new token, concatenate it
    onto the packed cache (the reference's append copies the whole cache,
    engine/gemma4_multilayer.cpp:230-236), dequantize K/V to fp32 and run
    SDPA (engine/gemma4_multilayer.cpp:307-308,349)."""
    from oracle import inputs, oracle as O
    L = inputs.make_layer(seed, H, HKV, D, n_ctx - 1)
    kq, ks, kb = O.quantize(L["k"])
    vq, vs, vb = O.quantize(L["v"])
    q = L["q"].astype(np.float16)
    kn, vn = L["k_new"], L["v_new"]
    del L

    def one():
        nk = O.quantize(kn)
        nv = O.quantize(vn)
        ck = [np.concatenate([a, b], axis=2) for a, b in zip((kq, ks, kb), nk)]
        cv = [np.concatenate([a, b], axis=2) for a, b in zip((vq, vs, vb), nv)]
        return O.sdpa_int4(q, *ck, *cv, window=window)

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = time.perf_counter() - t0
    return steps / dt, O.num_threads(), dt


# --------------------------------------------------------------------- main --

def reference_line(args, config: dict) -> dict:
    """The reference arm: the reference's algorithm for config 1 on the host
    cores (the oracle port: quantize the new token, concatenate it onto the
    packed cache, dequantize, fp32 SDPA), OpenMP over every host thread --
    set explicitly, since torch.distributed.run exports OMP_NUM_THREADS=1."""
    from oracle import oracle as O
    O.set_num_threads(os.cpu_count() or 1)
    steps = max(1, min(args.steps, 20))
    warm = max(0, min(args.warmup, 2))
    value, cores, dt = cpu_reference(args.context, args.window, steps, warm)
    return {"metric": "int4-KV decode-attention tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": warm,
            "ms_per_step": 1000.0 / value, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy)",
            "config": config, "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{steps} full decode steps (quantize+concatenate "
                                       f"append, dequantize, fp32 SDPA) of the same layer"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def _nested(line: dict) -> dict:
    """A standalone line as a nested object of the headline line."""
    drop = ("n_gpus", "warmup", "higher_is_better", "vs_baseline", "data")
    return {k: v for k, v in line.items() if k not in drop}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n_ctx, window = args.context, args.window
    bps = bytes_per_step(n_ctx, window)
    workload = f"cfg1 decode step: append 1 token + sdpa_int4, ctx {n_ctx}, " + \
               (f"sliding window {window}" if window > 0 else "global")
    config = {"workload": workload, "batch": 1, "heads": H, "kv_heads": HKV, "head_dim": D,
              "context": n_ctx, "window": window, "codes": "int4 (group 64)", "scales": "fp16", "q_out": "fp16",
              "layers_rotated": LAYERS,
              "l2": f"inputs larger than L2: {LAYERS} rotating layer caches "
                    f"({LAYERS * bps['attn'] / 1e6:.0f} MB > 126 MB L2)",
              "parallelism": f"dp{args.gpus} (independent KV heads/sequences per GPU)"}

    if args.impl == "reference" and args.workload == "cfg2":
        if rank != 0:
            return
        from oracle import oracle as O
        O.set_num_threads(os.cpu_count() or 1)
        cpu = cpu_reference_cfg2()
        v = cpu["batched_tokens_s"]
        line = {"metric": "int4-KV decode-attention tokens/s", "value": v, "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": C2_B * 1000.0 / v,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded numpy)", "impl": "reference",
                "config": {"workload": "cfg2 batched decode: 64 sequences x 1 query over one shared "
                                       "8192-token int4 cache", "batch": C2_B, "heads": H,
                           "kv_heads": HKV, "head_dim": D, "context": C2_N0},
                "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cpu["cores"], "kind": "port",
                                 "sample": cpu["sample"], "prefill_tokens_s": cpu["prefill_tokens_s"]},
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(reference_line(args, config)), flush=True)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))

    def finish(line):
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()

    if args.workload in ("cfg4", "cfg4_heads"):
        if args.workload == "cfg4_heads" and (world < 2 or C4_HKV % world):
            raise SystemExit("cfg4_heads needs 2, 4 or 8 GPUs (8 KV heads split evenly)")
        fn = run_cfg4 if args.workload == "cfg4" else run_cfg4_heads
        line = fn(args, rank, world, local_rank, steps=max(64, args.steps), check=not args.no_check)
        line.update({"n_gpus": world, "warmup": args.warmup, "higher_is_better": True,
                     "vs_baseline": None, "dtype": "f32",
                     "data": "synthetic (seeded torch.randn, RMS-normalised Q/K as task configs[0])"})
        return finish(line)
    if args.workload == "cfg2":
        res = run_cfg2(args, rank, world, local_rank)
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            cpu = cpu_reference_cfg2()
        return finish(cfg2_line(args, world, res, cpu))
    if args.workload in ("cfg0", "cfg3", "probe"):
        fn = {"cfg0": lambda: run_cfg0(args, local_rank), "cfg3": lambda: run_cfg3(args, local_rank),
              "probe": lambda: run_probe(local_rank)}[args.workload]
        return finish(fn())

    res = run_ours(args, rank, world, local_rank)
    steps_total = args.steps * world
    value = steps_total / (res["t_ms"] / 1000.0)
    peaks = measured_peaks()
    achieved = bps["attn"] / (res["kern_us"] * 1e-6) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": ncu_traffic(n_ctx, window),
                "kernel": ("tq::decode_kernel<128,2,__half> (CUDA cores)"
                           if os.environ.get("TQ_DECODE_KERNEL") == "simt" else
                           "tq::decode_mma_kernel<128,2,__half,false> (mma.sync)"),
                "kernel_us": res["kern_us"], "algorithmic_bytes_per_launch": bps["attn"],
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, copy read+write)",
                "frac_of_8tbs_nominal": achieved / 8000.0}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        O.set_num_threads(os.cpu_count() or 1)
        cv, cores, dt = cpu_reference(n_ctx, window, steps=10, warmup=1)
        cpu = {"value": cv, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"10 decode steps of one layer at ctx {n_ctx} ({dt:.1f} s): "
                         "quantize+concatenate append, dequantize, fp32 SDPA"}
    e2e_value = res["e2e_steps"] * world / (res["e2e_ms"] / 1000.0)
    async_value = res["e2e_steps"] * world / (res["async_ms"] / 1000.0)
    line = {"metric": "int4-KV decode-attention tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["t_ms"] / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded torch.randn, RMS-normalised Q/K as task configs[0])",
            "config": config, "roofline": roofline, "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    "h2d_bytes_per_step": (H * D + 2 * HKV * D) * 2 + (0 if args.split_step else 4),
                    "d2h_bytes_per_step": H * D * 2,
                    "path": ("gemma4metal_b200.turboquant.quantize_append + sdpa_int4 (ctypes C ABI)"
                             if args.split_step else
                             "gemma4metal_b200.turboquant.HostDecodeStep.run (tq_decode_step_run: "
                             "pageable host q/k_new/v_new/out, one graph launch + sync per step)"),
                    "timer": "host clock (every step returns with its output on the host)",
                    "async_api": {"value": async_value, "unit": "tokens/s",
                                  "path": "pinned H2D copy, tq_sdpa_int4_append, D2H copy, "
                                          "stream sync (three enqueues per step)"}},
            "gpu_launches": (2 if args.split_step else 1) * args.steps,
            "launches_per_step": ("2 (quantize_rows_kernel for K+V, decode_mma_kernel)" if args.split_step
                                  else "1 (decode_mma_kernel with the new token's quantize-on-append fused)"),
            "timed_region": f"one CUDA graph of exactly {args.steps} steps",
            "clocks": res["clocks"],
            "hbm_gbs_step": bps["step"] * value / world / 1e9}
    del res
    torch.cuda.empty_cache()

    if args.workload == "all":
        # the other configs, nested; the sequence split (config 4) at every N,
        # the single-GPU configs on one GPU only
        nested = {}
        if world == 1:
            nested["cfg0"] = run_cfg0(args, local_rank)
            torch.cuda.empty_cache()
            r2 = run_cfg2(args, rank, world, local_rank)
            cpu2 = None if args.no_cpu_baseline else cpu_reference_cfg2(budget_s=8.0)
            nested["cfg2"] = _nested(cfg2_line(args, world, r2, cpu2))
            torch.cuda.empty_cache()
            nested["cfg3"] = run_cfg3(args, local_rank)
            torch.cuda.empty_cache()
            nested["hbm_probe"] = run_probe(local_rank)
            if nested["hbm_probe"]:
                best = max(v["gbs"] for v in nested["hbm_probe"].values())
                line["roofline"]["frac_of_read_probe"] = achieved / best
                line["roofline"]["read_probe_gbs"] = best
        nested["cfg4"] = run_cfg4(args, rank, world, local_rank, steps=256, check=not args.no_check)
        torch.cuda.empty_cache()
        if world > 1 and C4_HKV % world == 0:
            # the same layer split by KV heads instead of by sequence
            nested["cfg4_heads"] = run_cfg4_heads(args, rank, world, local_rank, steps=256,
                                                  check=not args.no_check)
            torch.cuda.empty_cache()
        line["configs"] = nested
    finish(line)


if __name__ == "__main__":
    main()

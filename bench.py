"""Benchmark: packed KIVI decode attention (BASELINE configs 2 and 3) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload config2|config3|config3split]
    python bench.py --leg long_query|config1|config5    (one secondary leg alone, for profiling)

Headline (default, config 2) per GPU: 16 sequences, 28 query / 4 KV heads,
head_dim 128, 8192 KIVI 2-bit (group 32) packed tokens + 128 bf16 residual
tokens, K,V ~ N(0,1) with 4 key outlier channels x10 (seeded synthetic data:
no dataset is involved).  One step = one decode token for every sequence = one
launch of the decode kernel plus one launch of the state-merge kernel.  A
replica of the packed caches is 55 MB, below the 126 MB L2, so steps rotate
over 8 independent replicas (438 MB) and no step finds its cache in L2.  The
device-timed region is one replay of a CUDA graph holding exactly K steps
(captured once, warmed by W eager steps and one untimed replay), max over
ranks.

Multi-GPU (torchrun): requests are batch-partitioned -- every rank decodes its
own sequences, no collective in the timed loop (weak scaling).

The same JSON line carries, at every N:
* ``config3``: BASELINE config 3's batch half, 8 sequences per GPU of 32768 +
  128 tokens, 4-bit, group 64 (weak scaling; 64 sequences at N = 8);
* ``config3split``: its long-context half, ONE 131072 + 128-token sequence
  split over the ranks (strong scaling), each step ending with the exchange of
  every rank's (out, LSE) over NVLink peer memory and the LSE merge (the NCCL
  all-gather variant timed beside it);
* ``config5``: the Qwen2-7B-shaped decoder (28 layers, random bf16 weights)
  decoding 32 sequences per GPU over H2O 20% + 2-bit KIVI prompt caches with
  a growing dense suffix, one CUDA-graph replay per step (weak scaling);
and at N = 1: ``long_query`` (config 4: the tcgen05 kernel alone and the whole
``long_query_attention_summary`` call over the real segment mix), ``config1``
(the GPU pipeline and its CPU port), ``pack`` and the CPU baseline.

``e2e`` = the headline metric through the public API (DecodeStepGraph) with
the query read from pinned host memory and the output and LSE written back
every step.  ``--impl reference`` times the reference's own CPU path (a torch
restatement in oracle/reference_cpu.py, all host cores) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from dataclasses import dataclass

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q_HEADS = 28
KV_HEADS = 4
HEAD_DIM = 128
METRIC = "packed-KV attention HBM GB/s & decode tokens/s/GPU at 1/2/4/8 B200"


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int      # sequences per GPU (1 for the split: one sequence over all GPUs)
    tokens: int     # packed tokens per sequence
    residual: int   # bf16 residual tokens per sequence
    bits: int
    group: int
    replicas: int   # cache replicas the steps rotate over (beyond L2)

    def pair_bytes(self, tokens: int | None = None, residual: int | None = None) -> int:
        """Bytes one decode step must move per (sequence, KV head)."""

        t = self.tokens if tokens is None else tokens
        r = self.residual if residual is None else residual
        codes = 2 * t * HEAD_DIM * self.bits // 8
        key_stats = (t // self.group) * HEAD_DIM * 2 * 2
        value_stats = t * (HEAD_DIM // self.group) * 2 * 2
        return codes + key_stats + value_stats + r * HEAD_DIM * 2 * 2 + (Q_HEADS // KV_HEADS) * HEAD_DIM * 2 * 2

    def step_bytes(self) -> int:
        return self.pair_bytes() * self.batch * KV_HEADS

    def describe(self) -> str:
        if self.name == "config3split":
            return (f"config3split: one sequence of {self.tokens} packed KIVI {self.bits}-bit G{self.group} + "
                    f"{self.residual} bf16 tokens split over the GPUs, 28/4 heads, D=128")
        return (f"{self.name}: packed KIVI {self.bits}-bit G{self.group} decode, {self.batch} seqs/GPU, "
                f"T={self.tokens}+{self.residual} bf16 residual, 28/4 heads, D=128")


WORKLOADS = {
    # 16 sequences per GPU, 8192 + 128 tokens, 2-bit, group 32
    "config2": Workload("config2", 16, 8192, 128, 2, 32, 8),
    # BASELINE config 3 per GPU (batch 64 over 8 GPUs): 8 sequences, 32768 + 128 tokens, 4-bit, group 64
    "config3": Workload("config3", 8, 32768, 128, 4, 64, 2),
    # BASELINE config 3, long-context half: one 131072 + 128-token sequence split over the GPUs
    "config3split": Workload("config3split", 1, 131072, 128, 4, 64, 0),
}


def measured_peak(key: str, fallback: float) -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as handle:
            return float(json.load(handle)[key]), "measured"
    except (OSError, KeyError, ValueError):
        return fallback, "fallback"


def hbm_roofline(step_bytes: float, seconds: float) -> dict:
    peak, kind = measured_peak("hbm_gbs", 6650.0)
    achieved = step_bytes / seconds / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": kind}


def ncu_traffic() -> float | None:
    """Per-launch DRAM bytes of the config-2 decode kernel from the committed ncu summary."""

    try:
        with open(os.path.join(ROOT, "profiles", "decode_config2_traffic.json")) as handle:
            return float(json.load(handle)["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML while running (reads only)."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int):
        self.index = index
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)

            def loop():
                while not self._stop.is_set():
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                    mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                    for name, bit in self.REASONS.items():
                        if mask & bit:
                            self.reasons.add(name)
                    time.sleep(0.0005)  # the timed replay lasts milliseconds: sample densely

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception:  # NVML missing: report no clocks rather than fail the run
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ run context
class Run:
    """Process-group plumbing shared by the legs: every rank runs the same legs
    in the same order, so every collective below is matched."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local_rank)
        self.device = torch.device("cuda", self.local_rank)
        self.dist = dist
        if self.world > 1:
            import datetime

            dist.init_process_group("nccl", device_id=self.device, timeout=datetime.timedelta(seconds=120))

    def barrier(self) -> None:
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, values: list[float]) -> list[float]:
        if self.world == 1:
            return values
        import torch

        t = torch.tensor(values, device=self.device, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t]

    def graph_seconds(self, step_fn, steps: int, sampler: bool = False):
        """Device time of ``steps`` calls of step_fn(i) captured in one CUDA graph
        (barrier + synchronize on both sides of the replay)."""

        import torch

        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                for i in range(steps):
                    step_fn(i)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph.replay()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        clocks = ClockSampler(self.local_rank) if sampler else None
        if clocks:
            clocks.__enter__()
        t0.record()
        graph.replay()
        t1.record()
        torch.cuda.synchronize()
        if clocks:
            clocks.__exit__(None, None, None)
        self.barrier()
        del graph  # released before the process group is destroyed
        return t0.elapsed_time(t1) / 1000.0, clocks

    def eager_seconds(self, step_fn, steps: int, warmup: int) -> float:
        import torch

        for i in range(warmup):
            step_fn(i)
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(steps):
            step_fn(i)
        t1.record()
        torch.cuda.synchronize()
        self.barrier()
        return t0.elapsed_time(t1) / 1000.0

    def close(self) -> None:
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ------------------------------------------------------------------ batch-partitioned decode
def build_batches(run: Run, wl: Workload, seed: int):
    """``wl.replicas`` decode batches of ``wl.batch`` packed sequences each
    (generated on the GPU, seeded per rank); returns (batches, pack seconds per
    replica, the first replica's dense K/V)."""

    import torch

    from unicache_b200 import PackedKIVICache, PhysicalDecodeBatch

    dev = run.device
    gen = torch.Generator(device=dev).manual_seed(seed + 7919 * run.rank)
    outlier = torch.randperm(HEAD_DIM, generator=torch.Generator().manual_seed(0))[:4].to(dev)
    batches, pack_times, first_dense = [], [], None
    n = wl.tokens + wl.residual
    for r in range(wl.replicas):
        dense = []
        for _ in range(wl.batch):
            k = torch.randn(n, KV_HEADS, HEAD_DIM, generator=gen, device=dev)
            k[:, :, outlier] *= 10.0
            v = torch.randn(n, KV_HEADS, HEAD_DIM, generator=gen, device=dev)
            dense.append((k.to(torch.bfloat16), v.to(torch.bfloat16)))
            del k, v
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record()
        seqs = [[PackedKIVICache.from_dense(k, v, logical_token_ids=torch.arange(n, device=dev), token_type_id=3,
                                            k_bits=wl.bits, v_bits=wl.bits, group_size=wl.group,
                                            residual_length=wl.residual)] for k, v in dense]
        stop.record()
        torch.cuda.synchronize()
        pack_times.append(start.elapsed_time(stop) / 1000.0)
        if r == 0:
            first_dense = dense
        del dense
        batches.append(PhysicalDecodeBatch(seqs, num_kv_heads=KV_HEADS, head_dim=HEAD_DIM))
    torch.cuda.empty_cache()
    return batches, pack_times, first_dense


def decode_leg(run: Run, wl: Workload, *, headline: bool) -> dict:
    """Batch-partitioned decode of ``wl``: device-timed graph of K steps, and
    for the headline also the end-to-end legs through the public API."""

    import torch

    from unicache_b200 import DecodeStepGraph, kernels

    args = run.args
    batches, pack_times, first_dense = build_batches(run, wl, seed=1234 if wl.name == "config2" else 4321)
    dev = run.device
    gen = torch.Generator(device=dev).manual_seed(77 + run.rank)
    query = torch.randn(wl.batch, Q_HEADS, HEAD_DIM, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty_like(query)
    lse = torch.empty(wl.batch, Q_HEADS, device=dev, dtype=torch.float32)
    for i in range(args.warmup):
        batches[i % wl.replicas](query, out=out, lse=lse)
    elapsed, clocks = run.graph_seconds(lambda i: batches[i % wl.replicas](query, out=out, lse=lse), args.steps,
                                        sampler=headline)
    result = {}
    e2e_elapsed = eager_elapsed = 0.0
    if headline:
        # end to end through the public API with host buffers: DecodeStepGraph
        # (query read from pinned host memory, decode, merge storing out + LSE
        # to pinned host memory, as one graph per step), and
        # the eager per-call path with copy_ calls
        host_q = torch.empty_like(query, device="cpu").pin_memory()
        host_q.copy_(query.cpu())
        host_o = torch.empty_like(out, device="cpu").pin_memory()
        host_l = torch.empty_like(lse, device="cpu").pin_memory()
        steps = [DecodeStepGraph(b, host_q, host_o, host_l) for b in batches]
        for step in steps:  # first replays upload each graph
            step()
            step()
        e2e_elapsed = run.eager_seconds(lambda i: steps[i % wl.replicas](), args.steps, args.warmup)
        del steps
        dev_q = torch.empty_like(query)

        def eager_step(i):
            dev_q.copy_(host_q, non_blocking=True)
            o, l = batches[i % wl.replicas](dev_q)
            host_o.copy_(o, non_blocking=True)
            host_l.copy_(l, non_blocking=True)

        eager_elapsed = run.eager_seconds(eager_step, args.steps, args.warmup)
        result["h2d"] = query.numel() * query.element_size()
        result["d2h"] = out.numel() * out.element_size() + lse.numel() * lse.element_size()
    status = kernels.device_status()
    elapsed, e2e_elapsed, eager_elapsed, status = run.max_over_ranks(
        [elapsed, e2e_elapsed, eager_elapsed, float(status)])
    tokens = wl.batch * run.world * args.steps
    step_s = elapsed / args.steps
    result.update({
        "value": tokens / elapsed,
        "ms_per_step": 1000.0 * step_s,
        "roofline": dict(hbm_roofline(wl.step_bytes(), step_s), algorithmic_bytes_per_launch=wl.step_bytes(),
                         kernel_ms=1000.0 * step_s,
                         kernel="decode step = decode_kernel + state_merge_kernel, timed over a graph replay"),
        "device_status": int(status),
        "clocks": clocks.summary() if clocks else None,
        "pack_seconds": statistics.median(pack_times),
        "first_dense": first_dense,
    })
    if headline:
        result["e2e_value"] = tokens / e2e_elapsed
        result["eager_value"] = tokens / eager_elapsed
    return result


# ------------------------------------------------------------------ sequence split
def shard_bytes(wl: Workload, tokens: int, residual: int) -> int:
    return KV_HEADS * wl.pair_bytes(tokens, residual)


def split_leg(run: Run) -> dict:
    """BASELINE config 3, long-context half: one sequence split over the ranks
    in contiguous group-aligned shards (the last rank also holds the residual).
    A step = every rank decodes its shard, then the peer-memory exchange of
    every rank's (out, LSE) and the LSE merge in one kernel (NCCL all-gather +
    merge kernel timed the same way); strong scaling, max over ranks."""

    import torch

    from unicache_b200 import PackedKIVICache, kernels
    from unicache_b200.distributed import PeerExchange, SequenceSplitDecode, split_tokens

    wl = WORKLOADS["config3split"]
    args, dev, world, rank = run.args, run.device, run.world, run.rank
    start, stop = split_tokens(wl.tokens + wl.residual, world, wl.group, wl.residual)[rank]
    n_local = stop - start
    residual = wl.residual if rank == world - 1 else 0
    local_bytes = shard_bytes(wl, n_local - residual, residual)
    replicas = max(2, math.ceil(256e6 / local_bytes))
    gen = torch.Generator(device=dev).manual_seed(4321 + 7919 * rank)
    outlier = torch.randperm(HEAD_DIM, generator=torch.Generator().manual_seed(0))[:4].to(dev)
    peer = PeerExchange(Q_HEADS, dev) if world > 1 else None
    decoders, nccl_decoders = [], []
    for _ in range(replicas):
        k = torch.randn(n_local, KV_HEADS, HEAD_DIM, generator=gen, device=dev)
        k[:, :, outlier] *= 10.0
        v = torch.randn(n_local, KV_HEADS, HEAD_DIM, generator=gen, device=dev)
        cache = PackedKIVICache.from_dense(k.to(torch.bfloat16), v.to(torch.bfloat16),
                                           logical_token_ids=torch.arange(start, stop, device=dev), token_type_id=3,
                                           k_bits=wl.bits, v_bits=wl.bits, group_size=wl.group,
                                           residual_length=residual)
        del k, v
        decoders.append(SequenceSplitDecode([[cache]], num_kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                                            exchange="peer" if world > 1 else "nccl", peer_exchange=peer))
        nccl_decoders.append(SequenceSplitDecode([[cache]], num_kv_heads=KV_HEADS, head_dim=HEAD_DIM))
    torch.cuda.empty_cache()
    qgen = torch.Generator(device=dev).manual_seed(99)  # every rank decodes the same query
    query = torch.randn(1, Q_HEADS, HEAD_DIM, generator=qgen, device=dev).to(torch.bfloat16)
    # eager per-call steps (they also warm the NCCL communicator before capture)
    eager = run.eager_seconds(lambda i: decoders[i % replicas](query), args.steps, args.warmup)
    run.eager_seconds(lambda i: nccl_decoders[i % replicas](query), args.steps, args.warmup)
    local = run.eager_seconds(lambda i: decoders[i % replicas].plan.run(query), args.steps, args.warmup)
    elapsed, _ = run.graph_seconds(lambda i: decoders[i % replicas](query), args.steps)
    nccl, _ = run.graph_seconds(lambda i: nccl_decoders[i % replicas](query), args.steps)
    status = kernels.device_status()
    elapsed, nccl, eager, local, status = run.max_over_ranks([elapsed, nccl, eager, local, float(status)])
    if peer is not None:
        torch.cuda.synchronize()
        peer.close()
    step_s = elapsed / args.steps
    total = shard_bytes(wl, wl.tokens, wl.residual)
    return {
        "workload": wl.describe(),
        "n_gpus": world,
        "scaling": "strong",
        "value": args.steps / elapsed,
        "unit": "tokens/s",
        "ms_per_step": 1000.0 * step_s,
        "exchange": "peer-memory kernel (epoch-tagged NVLink peer stores + LSE merge)" if world > 1 else "none",
        "nccl_exchange_ms_per_step": 1000.0 * nccl / args.steps,
        "local_decode_ms_per_step_eager": 1000.0 * local / args.steps,
        "eager_ms_per_step": 1000.0 * eager / args.steps,
        "roofline_per_gpu": dict(hbm_roofline(total / world, step_s), algorithmic_bytes_per_gpu=total // world),
        "l2": f"steps rotate over {replicas} shard replicas ({replicas * local_bytes / 1e6:.0f} MB per GPU)",
        "device_status": int(status),
    }


# ------------------------------------------------------------------ N = 1 legs
def pack_leg(run: Run, wl: Workload, dense_kv) -> dict:
    """Quantize + pack of the batch's quantized tokens: every sequence's key
    and value halves in ONE launch over a device job table
    (``KiviPackBatch``, what ``PackedKIVICache.from_dense_batch`` runs),
    captured in a CUDA graph.  Algorithmic bytes = bf16 K and V read + codes
    and statistics written."""

    from unicache_b200 import kernels

    pairs = [(k[:wl.tokens], v[:wl.tokens]) for k, v in dense_kv]
    batch = kernels.KiviPackBatch(pairs, k_bits=wl.bits, v_bits=wl.bits, group_size=wl.group)
    batch.run()
    reps = 5
    elapsed, _ = run.graph_seconds(lambda _i: batch.run(), reps)
    seconds = elapsed / reps / len(pairs)
    per_seq = (2 * wl.tokens * KV_HEADS * HEAD_DIM * 2
               + 2 * wl.tokens * KV_HEADS * HEAD_DIM * wl.bits // 8
               + 2 * 2 * wl.tokens * KV_HEADS * HEAD_DIM // wl.group * 2)
    return {"us_per_sequence": seconds * 1e6, "algorithmic_bytes_per_sequence": per_seq,
            "sequences_per_launch": len(pairs) if batch.fused else 1, "roofline": hbm_roofline(per_seq, seconds)}


def long_query_leg(run: Run) -> dict:
    """BASELINE config 4, one layer: the 1024-token latent block (28 query / 4
    KV heads) over 3095 cached tokens per KV head (H2O instruction and ViT
    rows, packed VAE tokens, residual, boundary and latent rows), non-causal.
    ``us_per_layer``: the product path's launches on that segment mix with
    its span tables built (the staged form: one staging kernel, then the
    tcgen05 kernel by TMA), device time of a CUDA-graph replay;
    ``in_place_us``: the same call reading the spans in place;
    ``dense_operand_us``: the tcgen05 kernel alone on resident dense bf16
    operands of the same size (eager); ``e2e``: the whole
    ``long_query_attention_summary`` call, eager (host work included).
    FLOPs = 4 * Lq * Hq * D * N."""

    import torch

    from unicache_b200 import kernels
    from unicache_b200.adapters.attention import long_query_attention_summary
    from unicache_b200.workloads import config4_layer

    dev = run.device
    heads, grp, lq, n = KV_HEADS, Q_HEADS // KV_HEADS, 1024, 3095
    n_pad = (n + 7) // 8 * 8
    gen = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(heads, lq * grp, HEAD_DIM, generator=gen, device=dev).to(torch.bfloat16)
    k = torch.zeros(heads, n_pad, HEAD_DIM, device=dev, dtype=torch.bfloat16)
    vt = torch.zeros(heads, HEAD_DIM, n_pad, device=dev, dtype=torch.bfloat16)
    k[:, :n] = torch.randn(heads, n, HEAD_DIM, generator=gen, device=dev).to(torch.bfloat16)
    vt[:, :, :n] = torch.randn(heads, HEAD_DIM, n, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    lse = torch.empty(heads, lq * grp, device=dev, dtype=torch.float32)
    reps = 20
    dense_s = run.eager_seconds(lambda i: kernels.prefill_attention(q, k, vt, n, out=out, lse=lse), reps, 3) / reps
    layer = config4_layer(dev, seed=1)
    assert layer.key_tokens == n
    segs = [(layer.dense_key, layer.dense_value), *layer.segments]
    tables = kernels.long_query_tables([segs], heads, [0], [lq * grp], dev)
    lq_out = torch.empty_like(layer.query)
    lq_lse = torch.empty(Q_HEADS, lq, device=dev, dtype=torch.float32)

    def product(staged):
        return lambda i: kernels.long_query_attention(layer.query, tables, num_kv_heads=heads, out=lq_out,
                                                      lse=lq_lse, staged=staged)

    def graphed(fn):  # device time of `reps` calls in one CUDA graph, after eager warm-up calls
        run.eager_seconds(fn, 1, 3)
        return run.graph_seconds(fn, reps)[0] / reps

    kernel_s = graphed(product(True))
    in_place_s = graphed(product(False))
    e2e_s = run.eager_seconds(lambda i: long_query_attention_summary(layer.query, layer.segments,
                                                                     dense_key=layer.dense_key,
                                                                     dense_value=layer.dense_value), reps, 3) / reps
    flops = 4.0 * lq * Q_HEADS * HEAD_DIM * n
    peak, kind = measured_peak("bf16_tflops", 1590.0)

    def roof(seconds):
        achieved = flops / seconds / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": kind}

    return {"workload": "config4 layer: Lq=1024 x 28/4 heads over 3095 keys (51+980 H2O, 992 packed 2-bit G32 + "
                        "32 residual, 16 boundary, 1024 latent), D=128, bf16, non-causal",
            "us_per_layer": kernel_s * 1e6, "tflops": flops / kernel_s / 1e12, "roofline": roof(kernel_s),
            "kernel": "staged long-query call: stage_kernel (key spaces gathered once) + prefill_kernel (TMA)",
            "in_place_us_per_layer": in_place_s * 1e6, "in_place_roofline": roof(in_place_s),
            "dense_operand_us_per_layer": dense_s * 1e6, "dense_operand_roofline": roof(dense_s),
            "e2e_us_per_layer": e2e_s * 1e6, "e2e_roofline": roof(e2e_s),
            "e2e_api": "long_query_attention_summary over the segment list"}


def config1_leg(run: Run) -> dict:
    """BASELINE config 1 (one fp32 layer, 2048 tokens): KIVI fake quantization
    of the first 1920 tokens (2-bit, group 32), H2O scores of 64 decode queries
    (LSE pass + scoring kernel), top-k selection and compaction to 410 tokens
    per KV head, then one decode step; timed on the GPU (CUDA events) and as
    the CPU port of the reference algorithm (numpy oracle, one core)."""

    import numpy as np
    import torch

    from oracle import attention, h2o, kivi
    from unicache_b200 import GQAH2OCache, kernels
    from unicache_b200.adapters.attention import fused_h2o_decode
    from unicache_b200.operators.physical import kivi_fake_quant_key, kivi_fake_quant_value
    from unicache_b200.synthetic import make_kv, make_query

    dev = run.device
    key, value = make_kv(2048, KV_HEADS, HEAD_DIM, seed=0, dtype=torch.float32, device=dev)
    queries = make_query(64, Q_HEADS, HEAD_DIM, seed=100, dtype=torch.float32, device=dev)
    query = make_query(1, Q_HEADS, HEAD_DIM, seed=0, device=dev)
    ids = torch.arange(2048, device=dev)
    scale = 1.0 / math.sqrt(HEAD_DIM)

    def pipeline(_i):
        fk = kivi_fake_quant_key(key[:1920], bits=2, group_size=32)
        fv = kivi_fake_quant_value(value[:1920], bits=2, group_size=32)
        k_all = torch.cat([fk, key[1920:]])
        v_all = torch.cat([fv, value[1920:]])
        scores = kernels.h2o_scores(queries, k_all, None, kv_heads=KV_HEADS, softmax_scale=scale)
        cache = GQAH2OCache.from_dense(k_all.to(torch.bfloat16), v_all.to(torch.bfloat16), logical_token_ids=ids,
                                       token_type_id=1, per_kv_head_scores=scores, target_tokens=410,
                                       recent_tokens=102, selection_frozen=True)
        return fused_h2o_decode(query, None, None, [cache])

    reps = 10
    gpu_s = run.eager_seconds(pipeline, reps, 3) / reps
    hk, hv, hq, hq1 = (t.float().cpu().numpy() for t in (key, value, queries, query))
    cpu_times = []
    for _ in range(2):
        t0 = time.perf_counter()
        ek = kivi.fake_quant_key(hk[:1920], "float32", bits=2, group_size=32)
        ev = kivi.fake_quant_value(hv[:1920], "float32", bits=2, group_size=32)
        ok, ov = np.concatenate([ek, hk[1920:]]), np.concatenate([ev, hv[1920:]])
        sc = h2o.reduce_probabilities(attention.attention_probabilities(hq, ok), KV_HEADS)
        kept = h2o.h2o_from_dense(ok, ov, np.arange(2048), sc, 410, 102)
        attention.attention_summary(hq1, kept["key"].transpose(1, 0, 2), kept["value"].transpose(1, 0, 2))
        cpu_times.append(time.perf_counter() - t0)
    return {"workload": "config1: fp32 layer, 2048 tokens (1920 fake-quantized 2-bit G32 + 128 fp32), H2O scores "
                        "of 64 queries, keep 410/KV head (308 heavy + 102 recent), one decode step",
            "gpu_ms_per_layer": gpu_s * 1e3,
            "cpu_port_ms_per_layer": min(cpu_times) * 1e3, "cpu_cores": 1,
            "cpu_kind": "port (numpy restatement of the reference algorithm, float64 attention)"}


def config5_leg(run: Run) -> dict:
    """the Qwen2-7B-shaped decoder (random bf16 weights, 28
    layers) decoding 32 sequences per GPU over a 16384-token prompt cache per
    layer compressed by H2O to 20% (3277 tokens per KV head) and packed in
    2-bit KIVI (group 32, 32-token residual), new tokens in a dense bf16
    suffix.  One step (every layer and the LM head, greedy) is one CUDA-graph
    replay.  The suffix is pre-filled so that the timed steps sit around the
    middle of the 512-token decode (its mean length).  Bytes per step: every
    weight matrix once, every layer's packed prompt and the live suffix."""

    import torch

    from unicache_b200 import kernels
    from unicache_b200.workloads import Qwen2PackedDecode

    args = run.args
    steps = min(args.steps, 256)
    mean_len = 256
    prefilled = max(0, mean_len - (args.warmup + 1 + steps) // 2)
    build0 = time.perf_counter()
    model = Qwen2PackedDecode(run.device, batch=32, prompt=16384, new_tokens=512, prefilled=prefilled,
                              seed=5 + run.rank)
    build_s = time.perf_counter() - build0
    model.step()  # first-call set-up
    torch.cuda.synchronize()
    model.capture()
    for _ in range(args.warmup):
        model.replay()
    torch.cuda.synchronize()
    run.barrier()
    torch.cuda.synchronize()
    len0 = int(model.length)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        model.replay()
    t1.record()
    torch.cuda.synchronize()
    run.barrier()
    elapsed = t0.elapsed_time(t1) / 1000.0
    # end to end: each step's next-token ids read back to pinned host memory
    host_ids = torch.empty(model.batch, dtype=torch.int64).pin_memory()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e_steps = min(steps, 512 - int(model.length))
    e0.record()
    for _ in range(e_steps):
        model.replay()
        host_ids.copy_(model.ids, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e = e0.elapsed_time(e1) / 1000.0
    status = kernels.device_status()
    elapsed, e2e, status = run.max_over_ranks([elapsed, e2e, float(status)])
    mean_suffix = len0 + (steps + 1) / 2
    step_bytes = model.weight_bytes() + model.cache_bytes(int(round(mean_suffix)))
    step_s = elapsed / steps
    per_gpu = model.batch * steps / elapsed
    result = {
        "workload": "config5: Qwen2-7B-shaped decoder (hidden 3584, 28 layers, 28/4 heads, FFN 18944, vocab "
                    "151936, random bf16 weights), 32 seqs/GPU, 16384-token prompt per layer -> H2O 20% "
                    "(3277/KV head) -> KIVI 2-bit G32 (R=32), dense bf16 suffix, greedy decode",
        "n_gpus": run.world, "scaling": "weak", "global_batch": model.batch * run.world,
        "value": per_gpu * run.world, "unit": "tokens/s", "tokens_per_s_per_gpu": per_gpu,
        "ms_per_step": 1000.0 * step_s, "steps": steps, "suffix_tokens_timed": [len0 + 1, len0 + steps],
        "roofline": dict(hbm_roofline(step_bytes, step_s), algorithmic_bytes_per_step=step_bytes,
                         weight_bytes=model.weight_bytes()),
        "e2e": {"value": model.batch * e_steps * run.world / e2e, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": model.batch * 8,
                "api": "Qwen2PackedDecode.replay + next-token ids copied to pinned host memory per step"},
        # per layer: decode + state merge, two RMSNorms, rope + suffix append, SwiGLU gate; the final RMSNorm
        "gpu_launches_ours_per_step": 6 * model.layers + 1,
        "build_seconds": build_s,
        "device_status": int(status),
    }
    del model
    torch.cuda.empty_cache()
    return result


# ------------------------------------------------------------------ CPU reference path
_CPU_CACHES: dict = {}


def cpu_reference_steps(wl: Workload, steps: int, warmup: int, seqs_per_step: int) -> tuple[float, str, int]:
    """Times the reference's own CPU decode path (oracle/reference_cpu.py: its
    unpack, grouped dequantization, fp32 logits, softmax and bf16 AV product,
    every KV head) with torch using every host core.  A step decodes one token
    of ``seqs_per_step`` sequences of the workload, one after the other;
    returns (tokens/s, sample description, cores)."""

    import torch

    from oracle import kivi, reference_cpu
    from unicache_b200.synthetic import make_kv, make_query

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    seeds = [10_000 + i for i in range(seqs_per_step)]
    for s in seeds:
        if (wl.name, s) not in _CPU_CACHES:
            key, value = make_kv(wl.tokens + wl.residual, KV_HEADS, HEAD_DIM, seed=s)
            ref = kivi.packed_from_dense(key.float().numpy(), value.float().numpy(), "bfloat16", k_bits=wl.bits,
                                         v_bits=wl.bits, group_size=wl.group, residual_length=wl.residual)
            layout = {}
            for name in ("key_code", "value_code"):
                layout[name] = torch.from_numpy(np.ascontiguousarray(ref[name]).astype(np.int32))
            for name in ("key_scale", "key_minimum", "value_scale", "value_minimum", "residual_key",
                         "residual_value"):
                layout[name] = torch.from_numpy(np.ascontiguousarray(ref[name], dtype=np.float32)).to(torch.bfloat16)
            cache = reference_cpu.cache_from_layout(layout, k_bits=wl.bits, v_bits=wl.bits, group_size=wl.group,
                                                    quantized_tokens=wl.tokens, head_dim=HEAD_DIM)
            _CPU_CACHES[(wl.name, s)] = (cache, make_query(1, Q_HEADS, HEAD_DIM, seed=s))
    for _ in range(warmup):
        for s in seeds:
            reference_cpu.decode(*_CPU_CACHES[(wl.name, s)])
    t0 = time.perf_counter()
    for _ in range(steps):
        for s in seeds:
            reference_cpu.decode(*_CPU_CACHES[(wl.name, s)])
    elapsed = time.perf_counter() - t0
    sample = (f"{seqs_per_step} of the workload's sequences per step ({wl.tokens}+{wl.residual} tokens, all "
              f"{KV_HEADS} KV heads), one decode token each, through the reference's CPU path (unpack, grouped "
              f"dequantization, fp32 logits, softmax, bf16 AV) in torch with {cores} threads")
    return seqs_per_step * steps / elapsed, sample, cores


def run_reference(args) -> None:
    """``--impl reference``: the reference's CPU path on the host cores, rank 0 only."""

    if int(os.environ.get("RANK", "0")) != 0:
        return
    wl = WORKLOADS[args.workload]
    per_step = 4 if wl.tokens <= 8192 else 1
    value, sample, cores = cpu_reference_steps(wl, args.steps, args.warmup, per_step)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * per_step / value,
        "higher_is_better": True,
        "scaling": "strong" if wl.name == "config3split" else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": headline_config(wl, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def headline_config(wl: Workload, world: int) -> dict:
    step_bytes = wl.step_bytes()
    return {
        "workload": wl.describe(),
        "global_batch": wl.batch * world,
        "seq_len": wl.tokens + wl.residual,
        "parallelism": f"batch-partitioned x{world}",
        "l2": f"steps rotate over {wl.replicas} cache replicas ({wl.replicas * step_bytes / 1e6:.0f} MB > 126 MB L2)",
    }


def run_b200(args) -> None:
    run = Run(args)
    wl = WORKLOADS[args.workload]
    head = decode_leg(run, wl, headline=True)
    pack = pack_leg(run, wl, head.pop("first_dense")) if run.world == 1 else None
    sub3 = None
    if wl.name != "config3":
        r3 = decode_leg(run, WORKLOADS["config3"], headline=False)
        r3.pop("first_dense")
        c3 = WORKLOADS["config3"]
        sub3 = {"workload": c3.describe(), "n_gpus": run.world, "scaling": "weak", "global_batch": c3.batch * run.world,
                "value": r3["value"], "unit": "tokens/s", "ms_per_step": r3["ms_per_step"],
                "roofline": r3["roofline"], "device_status": r3["device_status"]}
    split = split_leg(run)
    cfg5 = config5_leg(run)
    extra = {}
    if run.world == 1:
        extra["long_query"] = long_query_leg(run)
        extra["config1"] = config1_leg(run)
    if run.rank == 0:
        line = {
            "metric": METRIC,
            "value": head["value"],
            "unit": "tokens/s",
            "n_gpus": run.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": headline_config(wl, run.world),
            "hbm_gbs": head["roofline"]["achieved"],
            "roofline": dict(head["roofline"], traffic=ncu_traffic() if wl.name == "config2" else None),
            "e2e": {"value": head["e2e_value"], "unit": "tokens/s", "h2d_bytes_per_step": head["h2d"],
                    "d2h_bytes_per_step": head["d2h"],
                    "api": "DecodeStepGraph (per step, one graph launch: copy kernel reads the query from pinned host memory, decode, merge stores out + LSE to pinned host memory)"},
            "e2e_eager": {"value": head["eager_value"], "unit": "tokens/s",
                          "api": "PhysicalDecodeBatch.__call__ with per-step copy_ calls"},
            "gpu_launches": 2 * args.steps,
            "clocks": head["clocks"],
            "device_status": head["device_status"],
            "config3": sub3,
            "config3split": split,
            "config5": cfg5,
        }
        if pack is not None:
            line["pack"] = dict(pack, from_dense_seconds_per_batch=head["pack_seconds"])
        line.update(extra)
        if run.world == 1:
            value, sample, cores = cpu_reference_steps(wl, 3, 1, 4)
            line["cpu_baseline"] = {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                                    "sample": sample}
        print(json.dumps(line))
    run.close()


def run_split_headline(args) -> None:
    """--workload config3split: the split leg as the headline line."""

    run = Run(args)
    split = split_leg(run)
    if run.rank == 0:
        wl = WORKLOADS["config3split"]
        line = {
            "metric": METRIC, "value": split["value"], "unit": "tokens/s", "n_gpus": run.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": split["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": wl.describe(), "global_batch": 1, "seq_len": wl.tokens + wl.residual,
                       "parallelism": f"sequence-split x{run.world}", "l2": split["l2"]},
            "roofline": dict(split["roofline_per_gpu"], traffic=None),
            "gpu_launches": (3 if run.world > 1 else 2) * args.steps,
            "config3split": split,
        }
        print(json.dumps(line))
    run.close()


LEGS = {"long_query": lambda run: long_query_leg(run), "config1": lambda run: config1_leg(run),
        "config5": lambda run: config5_leg(run)}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=256)
    parser.add_argument("--warmup", type=int, default=16)
    parser.add_argument("--impl", default="b200", choices=["b200", "reference"])
    parser.add_argument("--workload", default="config2", choices=sorted(WORKLOADS))
    parser.add_argument("--leg", default=None, choices=sorted(LEGS),
                        help="run one secondary leg alone on one GPU and print its JSON object (for profiling)")
    args = parser.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.leg:
        run = Run(args)
        print(json.dumps({args.leg: LEGS[args.leg](run)}))
        run.close()
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "config3split":
        run_split_headline(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()

"""Benchmark: packed 2-bit KIVI decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload per GPU (config 2): 16 sequences, 28 query / 4 KV heads, head_dim 128,
8192 KIVI 2-bit (group 32) packed tokens + 128 bf16 residual tokens, K,V ~ N(0,1)
with 4 key outlier channels x10 (seeded synthetic data).  One step = one decode
token for every sequence = one launch of the decode kernel plus one launch of
the state-merge kernel.  Inputs (the packed caches) are 55 MB per replica, below
the 126 MB L2, so steps rotate over 8 independent cache replicas (438 MB) and no
step finds its cache in L2.  The device-timed region is one replay of a CUDA
graph holding exactly K steps (captured once, warmed by W eager steps and one
untimed replay); the e2e leg calls the public API eagerly every step.

Multi-GPU (torchrun): requests are batch-partitioned -- every rank decodes its
own 16 sequences, no collective in the timed loop (weak scaling); the step time
is the max over ranks.

--workload config3 is config 3's per-GPU batch (8 sequences of 32768 + 128
tokens, 4-bit, group 64); --workload config3split is its long-context half:
ONE 131072 + 128-token sequence split over the ranks (strong scaling), each
step ending with the exchange of every rank's (out, LSE) over NVLink peer
memory and the LSE merge (the NCCL all-gather variant is timed beside it).

Reported: value = decode tokens/s (whole job); e2e = the same through the
public API (DecodeStepGraph) with the query copied from pinned host memory and
the output and LSE read back every step (e2e_eager: the same through per-call
PhysicalDecodeBatch and copy_ calls); the roofline of the decode step against
the measured HBM copy bandwidth; and the CPU baseline (the oracle port of the
reference algorithm).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BATCH = 16
TOKENS = 8192
RESIDUAL = 128
WORKLOAD = "config2"

Q_HEADS = 28
KV_HEADS = 4
HEAD_DIM = 128
BITS = 2
GROUP = 32
REPLICAS = 8
METRIC = "packed-KV attention HBM GB/s & decode tokens/s/GPU at 1/2/4/8 B200"


def algorithmic_bytes_per_pair() -> int:
    """Bytes one decode step must move per (sequence, KV head)."""

    codes = 2 * TOKENS * HEAD_DIM * BITS // 8
    key_stats = (TOKENS // GROUP) * HEAD_DIM * 2 * 2
    value_stats = TOKENS * (HEAD_DIM // GROUP) * 2 * 2
    residual = RESIDUAL * HEAD_DIM * 2 * 2
    q_and_o = (Q_HEADS // KV_HEADS) * HEAD_DIM * 2 * 2
    return codes + key_stats + value_stats + residual + q_and_o


def measured_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def measured_bf16_peak() -> tuple[float, str]:
    """Dense bf16 tensor throughput (TFLOP/s, burst) of this pool's B200s."""

    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def pack_leg(device, dense_kv) -> dict:
    """Quantize + pack (KIVI, the workload's bits and group) of the sequences' quantized
    tokens: one fused key+value pack launch per sequence (group 32; the key
    and value kernels separately for other groups), captured in a CUDA graph
    and timed with CUDA events.  Algorithmic bytes = bf16 K and V read +
    codes and statistics written."""

    import torch

    from unicache_b200 import kernels

    keys = [k[:TOKENS] for k, _ in dense_kv]
    vals = [v[:TOKENS] for _, v in dense_kv]
    def run():
        for k, v in zip(keys, vals):
            kernels.kivi_pack_kv(k, v, k_bits=BITS, v_bits=BITS, group_size=GROUP)
    run()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=device)
    stream.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            run()
    torch.cuda.current_stream(device).wait_stream(stream)
    graph.replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    reps = 5
    t0.record()
    for _ in range(reps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    seconds = t0.elapsed_time(t1) / 1000.0 / reps / len(keys)
    per_seq = (2 * TOKENS * KV_HEADS * HEAD_DIM * 2                       # bf16 K and V read
               + 2 * TOKENS * KV_HEADS * HEAD_DIM * BITS // 8               # codes written
               + 2 * 2 * TOKENS * KV_HEADS * HEAD_DIM // GROUP * 2)         # scale + min, K and V
    peak, kind = measured_peaks()
    gbs = per_seq / seconds / 1e9
    del graph
    return {"us_per_sequence": seconds * 1e6, "algorithmic_bytes_per_sequence": per_seq,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "peak_source": kind}}


def long_query_leg(device) -> dict:
    """BASELINE config 4, one layer: a 1024-token query block (28 query / 4 KV
    heads) against 3095 cached tokens per KV head (51 + 980 H2O, 992 packed +
    32 residual, 16 boundary, 1024 current-latent), non-causal, on the tcgen05
    kernel with the operands resident; FLOPs = 4 * Lq * Hq * D * N."""

    import torch

    from unicache_b200 import kernels

    heads, grp, lq, n = KV_HEADS, Q_HEADS // KV_HEADS, 1024, 3095
    n_pad = (n + 7) // 8 * 8
    gen = torch.Generator(device=device).manual_seed(1)
    q = torch.randn(heads, lq * grp, HEAD_DIM, generator=gen, device=device).to(torch.bfloat16)
    k = torch.zeros(heads, n_pad, HEAD_DIM, device=device, dtype=torch.bfloat16)
    vt = torch.zeros(heads, HEAD_DIM, n_pad, device=device, dtype=torch.bfloat16)
    k[:, :n] = torch.randn(heads, n, HEAD_DIM, generator=gen, device=device).to(torch.bfloat16)
    vt[:, :, :n] = torch.randn(heads, HEAD_DIM, n, generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    lse = torch.empty(heads, lq * grp, device=device, dtype=torch.float32)
    for _ in range(3):
        kernels.prefill_attention(q, k, vt, n, out=out, lse=lse)
    torch.cuda.synchronize()
    reps = 20
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        kernels.prefill_attention(q, k, vt, n, out=out, lse=lse)
    t1.record()
    torch.cuda.synchronize()
    seconds = t0.elapsed_time(t1) / 1000.0 / reps
    flops = 4.0 * lq * Q_HEADS * HEAD_DIM * n
    peak, kind = measured_bf16_peak()
    achieved = flops / seconds / 1e12
    return {"workload": "config4 layer: Lq=1024 x 28/4 heads over 3095 keys, D=128, bf16, non-causal",
            "us_per_layer": seconds * 1e6, "tflops": achieved,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": kind}}


def ncu_traffic() -> float | None:
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""

    path = os.path.join(ROOT, "profiles", "decode_config2_traffic.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML while running."""

    REASONS = {
        "sw_power_cap": 0x4,
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

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
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


_ORACLE_CACHES: dict = {}


SAMPLE_KV_HEADS = 1  # the CPU sample decodes one of the KV_HEADS heads of a sequence


def cpu_oracle_sample(seq_seed: int) -> tuple[float, int]:
    """Decode one token of one sequence with the oracle port of the reference
    algorithm (dequantize the packed cache, float64 attention) on one core,
    on a bounded sample: one KV head with its 7 query heads, a quarter of the
    sequence's work.  Returns (seconds scaled to the whole sequence, tokens
    decoded).  The packed cache of a seed is built once per process and
    reused, as a decode loop reuses its cache; only the decode is timed."""

    from oracle import attention, kivi
    from unicache_b200.synthetic import make_kv, make_query

    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    if seq_seed not in _ORACLE_CACHES:
        key, value = make_kv(TOKENS + RESIDUAL, SAMPLE_KV_HEADS, HEAD_DIM, seed=seq_seed)
        query = make_query(1, Q_HEADS // KV_HEADS * SAMPLE_KV_HEADS, HEAD_DIM, seed=seq_seed)
        cache = kivi.packed_from_dense(key.float().numpy(), value.float().numpy(), "bfloat16", k_bits=BITS,
                                       v_bits=BITS, group_size=GROUP, residual_length=RESIDUAL)
        _ORACLE_CACHES[seq_seed] = (cache, query.float().numpy())
    cache, q = _ORACLE_CACHES[seq_seed]
    ctx = threadpool_limits(limits=1) if threadpool_limits else None
    if ctx:
        ctx.__enter__()
    try:
        start = time.perf_counter()
        rk, rv = kivi.packed_dequantize(cache)
        attention.attention_summary(q, rk, rv)
        elapsed = (time.perf_counter() - start) * (KV_HEADS / SAMPLE_KV_HEADS)
    finally:
        if ctx:
            ctx.__exit__(None, None, None)
    return elapsed, 1


def _set_workload(name: str) -> None:
    """Pool workers start fresh (spawn): give them the parent's workload and
    one thread each."""

    global WORKLOAD
    WORKLOAD = name
    globals().update(WORKLOADS[name])
    import torch

    torch.set_num_threads(1)


def run_reference(args) -> None:
    """The reference algorithm's CPU path (the oracle port) on the host cores."""

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    per_step = cores
    seeds = [10_000 + i for i in range(per_step)]
    ctx = mp.get_context("spawn")
    times = []
    with ctx.Pool(processes=cores, initializer=_set_workload, initargs=(WORKLOAD,)) as pool:
        for _ in range(args.warmup):
            pool.map(cpu_oracle_sample, seeds)
        for _ in range(args.steps):
            # the step's sequences decode in parallel: the step takes as long as its slowest
            results = pool.map(cpu_oracle_sample, seeds)
            times.append(max(r[0] for r in results))
    total = sum(times)
    value = per_step * args.steps / total
    sample = (f"{per_step} {WORKLOAD} sequences per step ({TOKENS}+{RESIDUAL} tokens), one decode token each, timed on "
              f"one of the {KV_HEADS} KV heads (7 query heads) and scaled x{KV_HEADS}")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if WORKLOAD == "config3split" else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": workload_name(),
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from unicache_b200 import PackedKIVICache, PhysicalDecodeBatch, kernels

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))

    # ---- build REPLICAS x BATCH packed caches (generated on the GPU, seeded per rank)
    gen = torch.Generator(device=device).manual_seed(1234 + 7919 * rank)
    outlier = torch.randperm(HEAD_DIM, generator=torch.Generator().manual_seed(0))[:4].to(device)
    replicas = []
    pack_times = []
    for r in range(REPLICAS):
        seqs = []
        dense = []
        for _ in range(BATCH):
            k = torch.randn(TOKENS + RESIDUAL, KV_HEADS, HEAD_DIM, generator=gen, device=device)
            k[:, :, outlier] *= 10.0
            v = torch.randn(TOKENS + RESIDUAL, KV_HEADS, HEAD_DIM, generator=gen, device=device)
            dense.append((k.to(torch.bfloat16), v.to(torch.bfloat16)))
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record()
        for k, v in dense:
            seqs.append([PackedKIVICache.from_dense(k, v, logical_token_ids=torch.arange(TOKENS + RESIDUAL, device=device),
                                                    token_type_id=3, k_bits=BITS, v_bits=BITS, group_size=GROUP,
                                                    residual_length=RESIDUAL)])
        stop.record()
        torch.cuda.synchronize()
        pack_times.append(start.elapsed_time(stop) / 1000.0)
        if r == 0:
            pack_inputs = dense
        del dense
        replicas.append(PhysicalDecodeBatch(seqs, num_kv_heads=KV_HEADS, head_dim=HEAD_DIM))
    torch.cuda.empty_cache()
    query = (torch.randn(BATCH, Q_HEADS, HEAD_DIM, generator=gen, device=device)).to(torch.bfloat16)
    out = torch.empty_like(query)
    lse = torch.empty(BATCH, Q_HEADS, device=device, dtype=torch.float32)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timed loop: the K decode steps (one decode kernel and
    # one state-merge kernel each, rotating over the replicas) are captured
    # once in a CUDA graph; W eager steps and one untimed replay warm it up.
    for i in range(args.warmup):
        replicas[i % REPLICAS](query, out=out, lse=lse)
    torch.cuda.synchronize()
    capture_stream = torch.cuda.Stream(device=device)
    capture_stream.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(capture_stream):
        with torch.cuda.graph(graph, stream=capture_stream):
            for i in range(args.steps):
                replicas[i % REPLICAS](query, out=out, lse=lse)
    torch.cuda.current_stream(device).wait_stream(capture_stream)
    graph.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        t0.record()
        graph.replay()
        t1.record()
        torch.cuda.synchronize()
    barrier()
    elapsed = t0.elapsed_time(t1) / 1000.0
    kernel_s = [elapsed / args.steps]
    status = kernels.device_status()
    del graph

    # ---- end-to-end through the public API with host buffers.  Each step
    # copies the query from pinned host memory, decodes and copies the output
    # and LSE back to pinned host memory; DecodeStepGraph replays those five
    # operations as one graph (the eager per-call path is timed as well).
    from unicache_b200 import DecodeStepGraph

    host_q = torch.empty_like(query, device="cpu").pin_memory()
    host_q.copy_(query.cpu())
    host_o = torch.empty_like(out, device="cpu").pin_memory()
    host_l = torch.empty_like(lse, device="cpu").pin_memory()
    steps = [DecodeStepGraph(rep, host_q, host_o, host_l) for rep in replicas]
    for step in steps:  # first replays upload each graph
        step()
        step()
    for i in range(args.warmup):
        steps[i % REPLICAS]()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        steps[i % REPLICAS]()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_elapsed = e0.elapsed_time(e1) / 1000.0
    del steps

    dev_q = torch.empty_like(query)
    for i in range(args.warmup):
        dev_q.copy_(host_q, non_blocking=True)
        o, l = replicas[i % REPLICAS](dev_q)
        host_o.copy_(o, non_blocking=True)
        host_l.copy_(l, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        dev_q.copy_(host_q, non_blocking=True)
        o, l = replicas[i % REPLICAS](dev_q)
        host_o.copy_(o, non_blocking=True)
        host_l.copy_(l, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    eager_elapsed = e0.elapsed_time(e1) / 1000.0

    if world > 1:
        t = torch.tensor([elapsed, e2e_elapsed, eager_elapsed, float(status)], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_elapsed, eager_elapsed, status = float(t[0]), float(t[1]), float(t[2]), int(t[3])

    if rank == 0:
        tokens = BATCH * world * args.steps
        value = tokens / elapsed
        step_bytes = algorithmic_bytes_per_pair() * BATCH * KV_HEADS
        mean_kernel = statistics.mean(kernel_s)
        achieved = step_bytes / mean_kernel / 1e9
        peak, peak_kind = measured_peaks()
        cpu_s, cpu_tokens = cpu_oracle_sample(4242)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": 1000.0 * elapsed / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": workload_name(),
                "global_batch": BATCH * world,
                "seq_len": TOKENS + RESIDUAL,
                "parallelism": f"batch-partitioned x{world}",
                "l2": f"steps rotate over {REPLICAS} cache replicas ({REPLICAS * step_bytes / 1e6:.0f} MB > 126 MB L2)",
            },
            "hbm_gbs": achieved,
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "peak_source": peak_kind,
                "traffic": ncu_traffic() if WORKLOAD == "config2" else None,
                "algorithmic_bytes_per_launch": step_bytes,
                "kernel_ms": 1000.0 * mean_kernel,
                "kernel": "decode step = decode_kernel + state_merge_kernel, timed over a graph replay",
            },
            "pack": dict(pack_leg(device, pack_inputs),
                         from_dense_seconds_per_16_seqs=statistics.median(pack_times)),
            "e2e": {"value": tokens / e2e_elapsed, "unit": "tokens/s",
                    "h2d_bytes_per_step": query.numel() * query.element_size(),
                    "d2h_bytes_per_step": out.numel() * out.element_size() + lse.numel() * lse.element_size(),
                    "api": "DecodeStepGraph (per step: H2D query, decode, merge, D2H out + LSE, one graph launch)"},
            "e2e_eager": {"value": tokens / eager_elapsed, "unit": "tokens/s",
                          "api": "PhysicalDecodeBatch.__call__ with per-step copy_ calls"},
            "gpu_launches": 2 * args.steps,
            "long_query": long_query_leg(device) if world == 1 else None,
            "clocks": clocks.summary(),
            "device_status": status,
            "cpu_baseline": {"value": cpu_tokens / cpu_s, "unit": "tokens/s", "cores": 1, "kind": "port",
                             "sample": f"one {WORKLOAD} sequence, one decode token (dequantize + float64 attention), "
                                       f"timed on one of the {KV_HEADS} KV heads and scaled x{KV_HEADS}"},
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def shard_bytes(tokens: int, residual: int) -> int:
    """Bytes one decode step moves for one sequence shard of ``tokens`` packed
    + ``residual`` bf16 tokens, over all KV heads (query and output included)."""

    codes = 2 * tokens * HEAD_DIM * BITS // 8
    key_stats = (tokens // GROUP) * HEAD_DIM * 2 * 2
    value_stats = tokens * (HEAD_DIM // GROUP) * 2 * 2
    res = residual * HEAD_DIM * 2 * 2
    q_and_o = (Q_HEADS // KV_HEADS) * HEAD_DIM * 2 * 2
    return KV_HEADS * (codes + key_stats + value_stats + res + q_and_o)


def run_split(args) -> None:
    """BASELINE config 3, long-context half: ONE sequence of TOKENS packed
    (4-bit, group 64) + RESIDUAL bf16 tokens split over the ranks in
    contiguous group-aligned shards (the last rank also holds the residual).
    A step = every rank decodes its shard (decode + state merge), one NCCL
    all-gather of every rank's (out, LSE), and the LSE merge; the step time is
    the max over ranks (strong scaling: the sequence is fixed).  Steps rotate
    over enough shard replicas to exceed the 126 MB L2."""

    import torch
    import torch.distributed as dist

    from unicache_b200 import PackedKIVICache, kernels
    from unicache_b200.distributed import PeerExchange, SequenceSplitDecode, split_tokens

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    start, stop = split_tokens(TOKENS + RESIDUAL, world, GROUP, RESIDUAL)[rank]
    n_local = stop - start
    residual = RESIDUAL if rank == world - 1 else 0
    local_bytes = shard_bytes(n_local - residual, residual)
    replicas_n = max(2, math.ceil(256e6 / local_bytes))
    gen = torch.Generator(device=device).manual_seed(4321 + 7919 * rank)
    outlier = torch.randperm(HEAD_DIM, generator=torch.Generator().manual_seed(0))[:4].to(device)
    decoders, nccl_decoders = [], []
    peer = PeerExchange(Q_HEADS, device) if world > 1 else None
    for _ in range(replicas_n):
        k = torch.randn(n_local, KV_HEADS, HEAD_DIM, generator=gen, device=device)
        k[:, :, outlier] *= 10.0
        v = torch.randn(n_local, KV_HEADS, HEAD_DIM, generator=gen, device=device)
        cache = PackedKIVICache.from_dense(k.to(torch.bfloat16), v.to(torch.bfloat16),
                                           logical_token_ids=torch.arange(start, stop, device=device),
                                           token_type_id=3, k_bits=BITS, v_bits=BITS, group_size=GROUP,
                                           residual_length=residual)
        del k, v
        decoders.append(SequenceSplitDecode([[cache]], num_kv_heads=KV_HEADS, head_dim=HEAD_DIM, group=group,
                                            exchange="peer", peer_exchange=peer))
        nccl_decoders.append(SequenceSplitDecode([[cache]], num_kv_heads=KV_HEADS, head_dim=HEAD_DIM, group=group))
    torch.cuda.empty_cache()
    qgen = torch.Generator(device=device).manual_seed(99)  # every rank decodes the same query
    query = torch.randn(1, Q_HEADS, HEAD_DIM, generator=qgen, device=device).to(torch.bfloat16)

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(step_fn) -> float:
        for i in range(args.warmup):
            step_fn(i)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            step_fn(i)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / 1000.0

    # eager per-call steps (also warm the NCCL communicator before capture)
    eager_elapsed = timed(lambda i: decoders[i % replicas_n](query))
    timed(lambda i: nccl_decoders[i % replicas_n](query))
    local_elapsed = timed(lambda i: decoders[i % replicas_n].plan.run(query))

    def graph_timed(decs):
        # the K steps captured once in a CUDA graph (the exchange included)
        capture_stream = torch.cuda.Stream(device=device)
        capture_stream.wait_stream(torch.cuda.current_stream(device))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(capture_stream):
            with torch.cuda.graph(graph, stream=capture_stream):
                for i in range(args.steps):
                    decs[i % replicas_n](query)
        torch.cuda.current_stream(device).wait_stream(capture_stream)
        graph.replay()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as sampler:
            g0.record()
            graph.replay()
            g1.record()
            torch.cuda.synchronize()
        barrier()
        del graph  # released before the process group is destroyed
        return g0.elapsed_time(g1) / 1000.0, sampler

    # device-timed region: decode, state merge and the peer-memory exchange +
    # merge kernel per step; the NCCL exchange is timed the same way for
    # comparison
    elapsed, clocks = graph_timed(decoders)
    nccl_elapsed, _ = graph_timed(nccl_decoders)
    host_q = query.cpu().pin_memory()
    host_o = torch.empty(query.shape, dtype=query.dtype).pin_memory()
    host_l = torch.empty((1, Q_HEADS), dtype=torch.float32).pin_memory()
    dev_q = torch.empty_like(query)

    def e2e_step(i):
        dev_q.copy_(host_q, non_blocking=True)
        o, l = decoders[i % replicas_n](dev_q)
        host_o.copy_(o, non_blocking=True)
        host_l.copy_(l, non_blocking=True)

    e2e_elapsed = timed(e2e_step)
    status = kernels.device_status()
    if world > 1:
        t = torch.tensor([elapsed, local_elapsed, e2e_elapsed, eager_elapsed, nccl_elapsed, float(status)],
                         device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, local_elapsed, e2e_elapsed, eager_elapsed, nccl_elapsed, status = (
            float(t[0]), float(t[1]), float(t[2]), float(t[3]), float(t[4]), int(t[5]))
    total_bytes = shard_bytes(TOKENS, RESIDUAL)
    if rank == 0:
        step_s = elapsed / args.steps
        peak, peak_kind = measured_peaks()
        achieved = total_bytes / world / step_s / 1e9  # per GPU
        cpu_s, cpu_tokens = cpu_oracle_sample(4242)
        line = {
            "metric": METRIC,
            "value": args.steps / elapsed,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": 1000.0 * step_s,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": (f"config3split: one sequence of {TOKENS} packed KIVI {BITS}-bit G{GROUP} + {RESIDUAL} bf16 "
                             f"tokens split over {world} GPU(s), 28/4 heads, D=128"),
                "global_batch": 1,
                "seq_len": TOKENS + RESIDUAL,
                "parallelism": (f"sequence-split x{world} + one kernel: epoch-tagged peer stores of (out, LSE) "
                                f"over NVLink + LSE merge" if world > 1 else "one GPU"),
                "l2": f"steps rotate over {replicas_n} shard replicas ({replicas_n * local_bytes / 1e6:.0f} MB per GPU > 126 MB L2)",
            },
            "hbm_gbs": achieved,
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "peak_source": peak_kind,
                "traffic": None,
                "algorithmic_bytes_per_launch": total_bytes // world,
                "kernel_ms": 1000.0 * step_s,
                "kernel": "per GPU: shard decode + state merge + peer exchange/merge, one graph replay of K steps",
            },
            "local_decode_ms_per_step": 1000.0 * local_elapsed / args.steps,
            "eager_ms_per_step": 1000.0 * eager_elapsed / args.steps,
            "nccl_exchange_ms_per_step": 1000.0 * nccl_elapsed / args.steps,
            "e2e": {"value": args.steps / e2e_elapsed, "unit": "tokens/s",
                    "h2d_bytes_per_step": query.numel() * query.element_size(),
                    "d2h_bytes_per_step": host_o.numel() * host_o.element_size() + host_l.numel() * 4,
                    "api": "SequenceSplitDecode.__call__ with the query copied from and the result copied to pinned host memory"},
            "gpu_launches": (3 if world > 1 else 2) * args.steps,
            "clocks": clocks.summary(),
            "device_status": status,
            "cpu_baseline": {"value": cpu_tokens / cpu_s, "unit": "tokens/s", "cores": 1, "kind": "port",
                             "sample": f"the whole {TOKENS}+{RESIDUAL}-token sequence, one decode token (dequantize + "
                                       f"float64 attention), timed on one of the {KV_HEADS} KV heads and scaled x{KV_HEADS}"},
        }
        print(json.dumps(line))
    if peer is not None:
        torch.cuda.synchronize()
        peer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


WORKLOADS = {
    # 16 sequences per GPU, 8192 + 128 tokens, 2-bit, group 32
    "config2": dict(BATCH=16, TOKENS=8192, RESIDUAL=128, BITS=2, GROUP=32, REPLICAS=8),
    # BASELINE config 3 per GPU (batch 64 over 8 GPUs): 8 sequences, 32768 + 128
    # tokens, 4-bit, group 64
    "config3": dict(BATCH=8, TOKENS=32768, RESIDUAL=128, BITS=4, GROUP=64, REPLICAS=2),
    # BASELINE config 3, long-context half: one 131072 + 128 token sequence,
    # 4-bit, group 64, split over the GPUs (strong scaling)
    "config3split": dict(BATCH=1, TOKENS=131072, RESIDUAL=128, BITS=4, GROUP=64, REPLICAS=0),
}


def workload_name() -> str:
    if WORKLOAD == "config3split":
        return (f"{WORKLOAD}: one sequence of {TOKENS} packed KIVI {BITS}-bit G{GROUP} + {RESIDUAL} bf16 tokens "
                f"split over the GPUs, 28/4 heads, D=128")
    return (f"{WORKLOAD}: packed KIVI {BITS}-bit G{GROUP} decode, {BATCH} seqs/GPU, T={TOKENS}+{RESIDUAL} "
            f"bf16 residual, 28/4 heads, D=128")


def main() -> None:
    global WORKLOAD
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=256)
    parser.add_argument("--warmup", type=int, default=16)
    parser.add_argument("--impl", default="b200", choices=["b200", "reference"])
    parser.add_argument("--workload", default="config2", choices=sorted(WORKLOADS))
    args = parser.parse_args()
    WORKLOAD = args.workload
    globals().update(WORKLOADS[args.workload])
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif WORKLOAD == "config3split":
        run_split(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()

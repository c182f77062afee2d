"""Attention fast paths over physical segments: the counterparts of the
reference adapter's physical attention helpers (Superone77/UniCache,
unicache/adapters/bagel.py):

* ``merge_attention_summaries``   bagel.py:57-72 (LSE merge kernel)
* ``fused_h2o_decode``            bagel.py:1860-1901 without the per-step
                                  ``torch.cat`` of every retained H2O row
* ``fused_mixed_decode``          bagel.py:1598-1858 for q_len == 1: dense,
                                  H2O, KIVI residual and packed KIVI tokens in
                                  one decode launch, no bf16 workspace
* ``PhysicalDecodeBatch``         batched decode over many sequences (the
                                  shape of ``apply_static_physical_attention_batch``,
                                  bagel.py:773-980, for decoding)
* ``DecodeStepGraph``             one such decode step with its host transfers
                                  captured as a CUDA graph
* ``long_query_attention_summary`` multi-query attention over the same
                                  segments (bagel.py:1598-1858 with q_len > 1)
* ``batched_long_query_attention`` several samples' query blocks in one
                                  launch (bagel.py:773-980, varlen)
"""

from __future__ import annotations

import math

import torch

from .. import kernels
from ..storage.physical import GQAH2OCache, PackedKIVICache


def merge_attention_summaries(
    summaries: list[tuple[torch.Tensor, torch.Tensor]],
) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge normalised segment outputs using their per-row log-sum-exp."""

    return kernels.lse_merge(summaries)


def _segments_for(dense_key, dense_value, physical_segments) -> list:
    segments: list = []
    if dense_key is not None and int(dense_key.shape[0]):
        segments.append((dense_key, dense_value))
    segments.extend(physical_segments)
    return segments


class PhysicalDecodeBatch:
    """Decode attention for a batch of sequences whose physical caches are
    frozen.  The device tables are built once; ``__call__`` launches one
    kernel per decode step."""

    def __init__(self, sequences: list[list], *, num_kv_heads: int, head_dim: int = 128,
                 target_ctas: int | None = None):
        self.plan = kernels.build_decode_plan(sequences, num_kv_heads=num_kv_heads, head_dim=head_dim,
                                              target_ctas=target_ctas)

    @property
    def bytes_per_step(self) -> int:
        return self.plan.bytes_per_step

    def __call__(self, query: torch.Tensor, *, out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
        """query [B, Hq, D] bf16 -> (out [B, Hq, D] bf16, lse [B, Hq] fp32 natural log)."""

        return self.plan.run(query, out=out, lse=lse)


class DecodeStepGraph:
    """One decode step of a ``PhysicalDecodeBatch`` with its host transfers,
    captured as a CUDA graph: every replay reads the query from
    ``host_query``, decodes, and writes the output and LSE to ``host_out`` /
    ``host_lse`` (all three pinned host tensors).  The transfers run in
    kernels over the mapped pinned buffers, not as DMA copies: a copy kernel
    reads the query across PCIe once into a device buffer (the decode
    kernel's CTAs then read it from there; several CTAs share a sequence's
    query rows under split-KV, so reading the host rows from the decode
    kernel itself moved several times the query's bytes across PCIe), and
    the state merge stores the results across PCIe.  So one step is one
    graph of three kernels.  Capture once, then call it every step after
    writing the next query into ``host_query``.  The call is asynchronous on
    the current stream: synchronize before reading the host outputs."""

    def __init__(self, batch: PhysicalDecodeBatch, host_query: torch.Tensor, host_out: torch.Tensor,
                 host_lse: torch.Tensor):
        for name, t in (("host_query", host_query), ("host_out", host_out), ("host_lse", host_lse)):
            if t.is_cuda or not t.is_pinned() or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous pinned host tensor")
        plan = batch.plan
        b, hq, d = map(int, host_query.shape)
        if host_query.dtype != torch.bfloat16 or host_out.dtype != torch.bfloat16 or host_lse.dtype != torch.float32:
            raise ValueError("host_query/host_out must be bfloat16 and host_lse float32")
        if (b, d) != (plan.num_seqs, plan.head_dim) or tuple(host_out.shape) != (b, hq, d) or \
                tuple(host_lse.shape) != (b, hq):
            raise ValueError("host buffers must be [B, Hq, D], [B, Hq, D] and [B, Hq] for this batch")
        self.host_query, self.host_out, self.host_lse = host_query, host_out, host_lse
        q_ptr = kernels.host_device_pointer(host_query)
        o_ptr = kernels.host_device_pointer(host_out)
        l_ptr = kernels.host_device_pointer(host_lse)
        device = plan.device
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream(device))
        self._query = torch.empty(b, hq, d, dtype=torch.bfloat16, device=device)
        dq_ptr, q_bytes = self._query.data_ptr(), host_query.numel() * host_query.element_size()

        def launch():
            kernels.copy_ranges([(dq_ptr, q_ptr, q_bytes)], stream.cuda_stream)
            plan.launch(dq_ptr, hq * d, hq, o_ptr, hq * d, l_ptr, stream.cuda_stream)

        launch()  # first-call set-up outside the capture
        stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(self.graph, stream=stream):
                launch()
        torch.cuda.current_stream(device).wait_stream(stream)
        self.h2d_bytes = host_query.numel() * host_query.element_size()
        self.d2h_bytes = host_out.numel() * host_out.element_size() + host_lse.numel() * host_lse.element_size()

    def __call__(self) -> None:
        self.graph.replay()


_PLANS_PER_OWNER = 8


def _single_sequence_decode(query, segments, num_kv_heads, head_dim, owner=None, key=None):
    """Decode of one query token over ``segments``.  The decode plan (device
    tables) is cached on the first physical segment, keyed by every segment's
    signature (identity, addresses, strides and lengths), so a decode loop
    over the same segments plans once; a segment that changes (an append, a
    trim, a repack) has a new signature and gets a new plan."""

    if int(query.shape[0]) != 1:
        raise ValueError("decode attention takes a single query token")
    if owner is None:
        owner = next((s for s in segments if isinstance(s, (PackedKIVICache, GQAH2OCache))), None)
        key = (num_kv_heads, head_dim, tuple(kernels._segment_signature(s) for s in segments))
    plan = None
    if owner is not None:
        plans = owner.__dict__.setdefault("_decode_plans", {})
        plan = plans.get(key)
    if plan is None:
        plan = kernels.build_decode_plan([segments], num_kv_heads=num_kv_heads, head_dim=head_dim)
        if owner is not None:
            # the owner keeps itself alive; the plan keeps the other segments
            plan.keepalive = [k for k in plan.keepalive if k is not owner]
            plans = owner.__dict__["_decode_plans"]
            if len(plans) >= _PLANS_PER_OWNER:
                plans.pop(next(iter(plans)))
            plans[key] = plan
    out, lse = plan.run(query.to(torch.bfloat16))
    return out.to(query.dtype), lse


def fused_h2o_decode(query: torch.Tensor, dense_key: torch.Tensor, dense_value: torch.Tensor,
                     physical_segments: list[GQAH2OCache]) -> torch.Tensor:
    """Decode over [dense ‖ H2O segments] reading the compacted rows in place."""

    if not all(isinstance(s, GQAH2OCache) for s in physical_segments):
        raise ValueError("fused H2O decode takes GQAH2OCache segments")
    kv_heads = int(dense_key.shape[1]) if dense_key is not None else physical_segments[0].num_kv_heads
    out, _ = _single_sequence_decode(query, _segments_for(dense_key, dense_value, physical_segments), kv_heads,
                                     int(query.shape[-1]))
    return out


def fused_mixed_decode(query: torch.Tensor, dense_key: torch.Tensor | None, dense_value: torch.Tensor | None,
                       physical_segments: list) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode over [dense ‖ H2O ‖ packed KIVI (+ residual)] in one launch;
    returns (out [1, Hq, D], lse [1, Hq])."""

    if not physical_segments and dense_key is None:
        raise ValueError("mixed decode needs at least one segment")
    first = physical_segments[0] if physical_segments else None
    kv_heads = int(dense_key.shape[1]) if dense_key is not None else first.num_kv_heads
    return _single_sequence_decode(query, _segments_for(dense_key, dense_value, physical_segments), kv_heads,
                                   int(query.shape[-1]))


def _kv_heads_of(segs) -> int:
    first = segs[0]
    if isinstance(first, (PackedKIVICache, GQAH2OCache)):
        return first.num_kv_heads
    return int(first[0].shape[1])


def batched_long_query_attention(queries: list, segments_by_sample: list, *, dense_by_sample: list | None = None,
                                 include_residual: bool = True, staged: bool | None = None) -> list:
    """Non-causal attention of several samples' query blocks over their own
    physical segments in one tcgen05 launch, the counterpart of the varlen
    launch of apply_static_physical_attention_batch (bagel.py:773-980).  The
    segments are described by a span table: either read in place (dense and
    H2O rows by cp.async, packed KIVI tiles restored in shared memory by
    every row block) or, when several row blocks read each key space
    (``staged`` None picks; see ``kernels.long_query_attention``), gathered
    once per launch into a bf16 workspace that the kernel streams by TMA.

    queries[i] [Lq_i, Hq, D]; segments_by_sample[i] the sample's segments;
    dense_by_sample[i] an optional (key, value) [N, Hkv, D] pair of the
    sample's own current tokens.  Returns [(out_i [Lq_i, Hq, D],
    lse_i [Hq, Lq_i] natural log)]."""

    if not queries or len(queries) != len(segments_by_sample):
        raise ValueError("one segment list per query block is required")
    dense_by_sample = dense_by_sample or [None] * len(queries)
    samples = []
    for query, segs, dense in zip(queries, segments_by_sample, dense_by_sample):
        kernels.require_cuda(query, "query")
        all_segs = _segments_for(dense[0] if dense else None, dense[1] if dense else None, segs)
        if not all_segs:
            raise ValueError("every sample needs at least one segment")
        samples.append((query, all_segs))
    hkv = _kv_heads_of(samples[0][1])
    hq, d = int(samples[0][0].shape[1]), int(samples[0][0].shape[-1])
    pos0, rows = [], []
    start = 0
    for query, segs in samples:
        if _kv_heads_of(segs) != hkv or int(query.shape[-1]) != d or int(query.shape[1]) != hq:
            raise ValueError("all samples must share query heads, KV heads and head_dim")
        if hq % hkv:
            raise ValueError("Query heads must be divisible by KV heads")
        pos0.append(start)
        rows.append(int(query.shape[0]) * (hq // hkv))
        start += int(query.shape[0])
    q = torch.cat([query.to(torch.bfloat16) for query, _ in samples]).contiguous()
    tables = kernels.long_query_tables([segs for _, segs in samples], hkv, pos0, rows, q.device, include_residual)
    out, lse = kernels.long_query_attention(q, tables, num_kv_heads=hkv, staged=staged)
    results = []
    for (query, _), p0 in zip(samples, pos0):
        lq = int(query.shape[0])
        results.append((out[p0:p0 + lq].to(query.dtype), lse[:, p0:p0 + lq]))
    return results


def long_query_attention_summary(query: torch.Tensor, segments: list, *, dense_key=None, dense_value=None,
                                 include_residual: bool = True,
                                 staged: bool | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Multi-query (non-causal) attention over physical segments on the tcgen05
    tensor cores: (out [Lq, Hq, D], lse [Hq, Lq] natural log).

    The query rows of each KV head ((position, head-in-group) pairs) form one
    M x N attention problem; the kernel reads the query and writes the
    outputs in the caller's layout.  Keys and values are read in place (dense
    and H2O rows copied, packed KIVI tiles restored in shared memory) or,
    when several row blocks read them, staged once per call into a bf16
    workspace streamed by TMA (``staged``: see
    ``kernels.long_query_attention``)."""

    kernels.require_cuda(query, "query")
    segs = _segments_for(dense_key, dense_value, segments)
    if not segs:
        raise ValueError("long-query attention needs at least one segment")
    hkv = _kv_heads_of(segs)
    lq, hq, d = map(int, query.shape)
    if hq % hkv:
        raise ValueError("Query heads must be divisible by KV heads")
    q = query if (query.dtype == torch.bfloat16 and query.is_contiguous()) else query.to(torch.bfloat16).contiguous()
    tables = kernels.long_query_tables([segs], hkv, [0], [lq * (hq // hkv)], query.device, include_residual)
    out, lse = kernels.long_query_attention(q, tables, num_kv_heads=hkv, staged=staged)
    return out.to(query.dtype), lse

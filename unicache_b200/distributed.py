"""Multi-GPU decode over packed physical caches, one process per GPU.

* Batch-partitioned decode (independent requests): ``partition_requests``
  gives each rank a contiguous block of requests.  Ranks never communicate on
  the data path; only timing or metrics are reduced, off the hot path.
* Sequence split of one long context: ``split_tokens`` cuts a sequence into
  contiguous group-aligned shards, one per rank.  Each rank packs and decodes
  its shard locally.  ``SequenceSplitDecode`` then gathers every rank's
  normalised output and log-sum-exp with one all-gather (NCCL over NVLink on
  GPUs, gloo on CPU) and merges them with the LSE merge kernel.  That merge is
  the reference's merge_attention_summaries (unicache/adapters/bagel.py:57-72)
  applied across ranks instead of across segments.  Each rank exchanges
  its output rows (bf16) and their LSE (fp32) as one buffer in one
  all-gather.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import kernels


def partition_requests(num_requests: int, world: int, rank: int) -> range:
    """Contiguous block of request indices owned by ``rank`` (sizes differ by
    at most one)."""

    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if num_requests < 0:
        raise ValueError("num_requests must be non-negative")
    base, extra = divmod(num_requests, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def split_tokens(tokens: int, world: int, group_size: int, residual_length: int = 0) -> list[tuple[int, int]]:
    """Contiguous shards [start, stop) of a ``tokens``-long sequence, one per
    rank.  Every boundary is a multiple of ``group_size``, so each shard packs
    whole KIVI groups.  The last shard also holds the final ``residual_length``
    full-precision tokens.  Raises ValueError when a rank would get no whole
    group."""

    if world <= 0 or group_size <= 0:
        raise ValueError("world and group_size must be positive")
    quantized = max(0, (tokens - residual_length) // group_size * group_size)
    groups = quantized // group_size
    if groups < world:
        raise ValueError(f"{tokens} tokens give {groups} groups of {group_size}; need at least one per rank")
    shards = []
    for r in range(world):
        g = partition_requests(groups, world, r)
        shards.append((g.start * group_size, g.stop * group_size))
    shards[-1] = (shards[-1][0], tokens)
    return shards


def exchange_summaries(out: torch.Tensor, lse: torch.Tensor, group=None) -> tuple[list, list]:
    """All-gather every rank's (out [B, Hq, D], lse [B, Hq]) in ONE collective:
    both travel as the bytes of one buffer (out first; its byte size is a
    multiple of 4, so the fp32 LSE stays aligned).  Without an initialised
    process group the local pair is returned alone."""

    if not dist.is_available() or not dist.is_initialized():
        return [out], [lse]
    world = dist.get_world_size(group)
    ob = out.contiguous().view(torch.uint8).reshape(-1)
    lb = lse.contiguous().view(torch.uint8).reshape(-1)
    if ob.numel() % 4:
        raise ValueError("out must span a multiple of 4 bytes")
    send = torch.cat([ob, lb])
    parts = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(parts, send, group=group)
    outs = [p[:ob.numel()].view(out.dtype).view(out.shape) for p in parts]
    lses = [p[ob.numel():].view(lse.dtype).view(lse.shape) for p in parts]
    return outs, lses


def merge_rank_summaries(outs: list, lses: list) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge per-rank decode results (out [B, Hq, D], lse [B, Hq]) on the GPU."""

    if len(outs) == 1:
        return outs[0], lses[0]
    merged, total = kernels.lse_merge([(o, l.t()) for o, l in zip(outs, lses)])
    return merged, total.t().contiguous()


class PeerExchange:
    """This rank's exchange buffer for ``ucb_split_merge_peer``, mapped on
    every rank of ``group`` through CUDA IPC handles.

    Construction and ``close`` are collective (every rank calls them in the
    same order).  ``merge(out, lse)`` exchanges and merges one decode step's
    summaries (out [B, Hq, 128] bf16, lse [B, Hq] fp32) in one kernel on the
    current stream: epoch-tagged peer stores over NVLink, a bounded wait and
    the LSE merge."""

    def __init__(self, rows: int, device: torch.device, group=None):
        from . import _capi

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the peer exchange serves at most 8 ranks")
        self.rows = int(rows)
        nbytes = int(_capi.load().ucb_peer_buffer_bytes(self.rows))
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(device):
            kernels.call("ucb_peer_buffer_alloc", nbytes, ctypes.byref(own), handle)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self._own = own.value
            self._opened = []
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                kernels.call("ucb_peer_buffer_open", ctypes.create_string_buffer(h, 64), ctypes.byref(peer))
                self._opened.append(peer.value)
                ptrs.append(peer.value)
            dist.barrier(group=group)  # every mapping exists before the first exchange
        self._bufs = (ctypes.c_void_p * self.world)(*ptrs)

    def merge(self, out: torch.Tensor, lse: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        b, hq, d = map(int, out.shape)
        if b * hq != self.rows or d != 128 or out.dtype != torch.bfloat16 or lse.dtype != torch.float32:
            raise ValueError("summary shape differs from the exchange buffer's")
        out = out.contiguous()
        lse = lse.contiguous()
        merged = torch.empty_like(out)
        total = torch.empty_like(lse)
        kernels.call("ucb_split_merge_peer", self.rank, self.world, self._bufs, out.data_ptr(), lse.data_ptr(),
                     self.rows, d, merged.data_ptr(), total.data_ptr(), kernels.stream_of(out))
        return merged, total

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers, then frees its own."""

        if self._bufs is None:
            return
        torch.cuda.synchronize()
        for p in self._opened:
            kernels.call("ucb_peer_buffer_close", ctypes.c_void_p(p))
        dist.barrier(group=self.group)
        kernels.call("ucb_peer_buffer_free", ctypes.c_void_p(self._own))
        self._bufs = None


class SequenceSplitDecode:
    """Decode of sequences whose tokens are split across ranks.

    ``local_sequences`` holds, for each sequence of the batch, this rank's
    segments (its shard of the packed cache, plus dense or H2O segments it
    owns).  Every rank calls it with the same query; every rank gets the
    merged result.

    One step is three operations on the current stream: the local decode
    writes its output rows (bf16) and LSE (fp32) straight into a preallocated
    send buffer, ONE ``all_gather_into_tensor`` fills a preallocated receive
    buffer with every rank's buffer, and the LSE merge kernel folds the
    ranks' summaries in place (out viewed as [1, B*Hq, D] and LSE as
    [B*Hq, 1], so no transposes are needed).  A second call reuses the
    buffers: steps are ordered on the stream, so a step's merge has read the
    receive buffer before the next step's all-gather overwrites it."""

    def __init__(self, local_sequences: list[list], *, num_kv_heads: int, head_dim: int = 128, group=None,
                 exchange: str = "nccl", peer_exchange: "PeerExchange | None" = None):
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'")
        self.plan = kernels.build_decode_plan(local_sequences, num_kv_heads=num_kv_heads, head_dim=head_dim)
        self.group = group
        self.exchange = exchange
        self._buffers = None  # (q_heads, send, recv, out view, lse view, out pointers, lse pointers, world)
        self._peer = peer_exchange  # may be shared by decoders that run in order on one stream
        self._owns_peer = peer_exchange is None

    def _setup(self, query: torch.Tensor):
        b, hq, d = map(int, query.shape)
        world = dist.get_world_size(self.group)
        ob, lb = b * hq * d * 2, b * hq * 4
        send = torch.empty(ob + lb, dtype=torch.uint8, device=query.device)
        recv = torch.empty(world * (ob + lb), dtype=torch.uint8, device=query.device)
        out_view = send[:ob].view(torch.bfloat16).view(b, hq, d)
        lse_view = send[ob:].view(torch.float32).view(b, hq)
        base = recv.data_ptr()
        optrs = (ctypes.c_void_p * world)(*[base + r * (ob + lb) for r in range(world)])
        lptrs = (ctypes.c_void_p * world)(*[base + r * (ob + lb) + ob for r in range(world)])
        self._buffers = (hq, send, recv, out_view, lse_view, optrs, lptrs, world)

    def __call__(self, query: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """query [B, Hq, D] bf16 -> (out [B, Hq, D] bf16, lse [B, Hq] fp32)."""

        if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return self.plan.run(query)
        if query.dtype != torch.bfloat16 or query.dim() != 3:
            raise ValueError("query must be bfloat16 [B, Hq, D]")
        if self.exchange == "peer":
            # one kernel: epoch-tagged peer stores of this rank's summary + merge
            if self._peer is None:
                self._peer = PeerExchange(int(query.shape[0]) * int(query.shape[1]), query.device, self.group)
            out, lse = self.plan.run(query)
            return self._peer.merge(out, lse)
        if self._buffers is None or self._buffers[0] != int(query.shape[1]) or \
                self._buffers[1].device != query.device:
            self._setup(query)
        hq, send, recv, out_view, lse_view, optrs, lptrs, world = self._buffers
        b, _, d = map(int, query.shape)
        self.plan.run(query, out=out_view, lse=lse_view)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        merged = torch.empty_like(out_view)
        total = torch.empty_like(lse_view)
        kernels.call("ucb_lse_merge", world, optrs, lptrs, kernels.dtype_code(torch.bfloat16), 1, b * hq, d,
                     merged.data_ptr(), total.data_ptr(), kernels.stream_of(query))
        return merged, total

    def close(self) -> None:
        """Collective when this decoder created a peer exchange: releases it."""

        if self._peer is not None and self._owns_peer:
            self._peer.close()
        self._peer = None

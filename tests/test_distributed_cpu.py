"""Host-side logic of multi-GPU decode, run as world_size-2 gloo process
groups on CPU: request partitioning, group-aligned sequence shards, the
(out, lse) all-gather, and a sequence split whose per-rank attention (float64
oracle) merged across ranks equals attention over the whole sequence."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention
from unicache_b200.distributed import exchange_summaries, partition_requests, split_tokens


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_requests_covers_every_request_once():
    for n in (0, 1, 7, 16, 64, 129):
        for world in (1, 2, 3, 8):
            blocks = [partition_requests(n, world, r) for r in range(world)]
            assert [i for b in blocks for i in b] == list(range(n))
            assert max(len(b) for b in blocks) - min(len(b) for b in blocks) <= 1
    with pytest.raises(ValueError):
        partition_requests(4, 2, 2)


def test_split_tokens_is_group_aligned_and_contiguous():
    shards = split_tokens(131072 + 128, 8, 64, residual_length=128)
    assert shards[0][0] == 0 and shards[-1][1] == 131072 + 128
    assert all(a[1] == b[0] for a, b in zip(shards, shards[1:]))
    assert all(start % 64 == 0 for start, _ in shards)
    assert all(stop % 64 == 0 for _, stop in shards[:-1])
    assert [stop - start for start, stop in shards[:-1]] == [16384] * 7
    with pytest.raises(ValueError):
        split_tokens(100, 4, 32)


def _worker(rank: int, world: int, port: int, result_dir: str) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        # exchange: every rank sees every rank's pair, in rank order
        out = torch.full((2, 3, 4), float(rank))
        lse = torch.full((2, 3), 10.0 + rank)
        outs, lses = exchange_summaries(out, lse)
        assert [float(o[0, 0, 0]) for o in outs] == [float(r) for r in range(world)]
        assert [float(l[0, 0]) for l in lses] == [10.0 + r for r in range(world)]

        # sequence split with the float64 oracle as each rank's local attention
        rng = np.random.default_rng(7)
        tokens, heads, d = 320, 2, 16
        key = rng.standard_normal((tokens, heads, d))
        value = rng.standard_normal((tokens, heads, d))
        query = rng.standard_normal((1, 6, d))
        start, stop = split_tokens(tokens, world, 32, residual_length=16)[rank]
        o, l = attention.attention_summary(query, key[start:stop], value[start:stop])
        outs, lses = exchange_summaries(torch.from_numpy(np.ascontiguousarray(o, np.float64)),
                                        torch.from_numpy(np.ascontiguousarray(l, np.float64)))
        merged, merged_lse = attention.merge_attention_summaries([(x.numpy(), y.numpy()) for x, y in zip(outs, lses)])
        whole, whole_lse = attention.attention_summary(query, key, value)
        assert np.abs(merged - whole).max() < 1e-9
        assert np.abs(merged_lse - whole_lse).max() < 1e-9
        open(os.path.join(result_dir, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


def test_sequence_split_exchange_and_merge_on_two_gloo_ranks(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]

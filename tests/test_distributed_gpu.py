"""Sequence-split decode on the GPU: a long packed sequence cut into
group-aligned shards, each decoded on its own plan, merged by the LSE merge
kernel; checked against the float64 oracle of the whole sequence (north-star
tolerance).  With two or more GPUs the same split runs as NCCL ranks."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import attention, kivi
from unicache_b200 import PackedKIVICache
from unicache_b200.distributed import SequenceSplitDecode, merge_rank_summaries, split_tokens
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import MAX_ABS, MEAN_ABS, host, need_gpu

pytestmark = pytest.mark.gpu

TOKENS, HEADS, GROUP, RESIDUAL = 4096 + 64, 4, 64, 64


def _shard_cache(key, value, start, stop, last):
    return PackedKIVICache.from_dense(key[start:stop], value[start:stop],
                                      logical_token_ids=torch.arange(start, stop, device=key.device), token_type_id=3,
                                      k_bits=4, v_bits=4, group_size=GROUP, residual_length=RESIDUAL if last else 0)


def _oracle(key, value, query, world):
    keys, vals = [], []
    for r, (start, stop) in enumerate(split_tokens(TOKENS, world, GROUP, RESIDUAL)):
        ref = kivi.packed_from_dense(host(key[start:stop]), host(value[start:stop]), "bfloat16", k_bits=4, v_bits=4,
                                     group_size=GROUP, residual_length=RESIDUAL if r == world - 1 else 0)
        k, v = kivi.packed_dequantize(ref)
        keys.append(k)
        vals.append(v)
    return attention.mixed_attention(host(query), keys, vals)


def _check(out, lse, expected):
    e_out, e_lse = expected
    diff = np.abs(host(out).astype(np.float64) - e_out)
    assert diff.max() <= MAX_ABS and diff.mean() <= MEAN_ABS, (diff.max(), diff.mean())
    assert np.abs(host(lse).T - e_lse).max() <= 2e-2


def test_sequence_split_shards_merge_to_the_whole_sequence():
    need_gpu()
    world = 4
    key, value = make_kv(TOKENS, HEADS, 128, seed=91, device="cuda")
    query = make_query(1, 28, 128, seed=92, device="cuda")
    outs, lses = [], []
    shards = split_tokens(TOKENS, world, GROUP, RESIDUAL)
    for r, (start, stop) in enumerate(shards):
        local = SequenceSplitDecode([[_shard_cache(key, value, start, stop, r == world - 1)]], num_kv_heads=HEADS)
        o, l = local.plan.run(query)
        outs.append(o)
        lses.append(l)
    out, lse = merge_rank_summaries(outs, lses)
    torch.cuda.synchronize()
    _check(out, lse, _oracle(key, value, query, world))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        # two sequences split the same way; two calls reuse the step buffers
        kvs = [make_kv(TOKENS, HEADS, 128, seed=91 + 10 * b, device="cuda") for b in range(2)]
        query = make_query(2, 28, 128, seed=92, device="cuda")
        start, stop = split_tokens(TOKENS, world, GROUP, RESIDUAL)[rank]
        decode = SequenceSplitDecode([[_shard_cache(k, v, start, stop, rank == world - 1)] for k, v in kvs],
                                     num_kv_heads=HEADS)
        out, lse = decode(query)
        out2, lse2 = decode(query)
        torch.cuda.synchronize()
        assert torch.equal(out, out2) and torch.equal(lse, lse2)
        for b, (k, v) in enumerate(kvs):
            _check(out[b:b + 1], lse[b:b + 1], _oracle(k, v, query[b:b + 1], world))
        # the same step through the peer-memory exchange (one kernel:
        # epoch-tagged peer stores, then the merge) equals the NCCL exchange
        # bit for bit, call after call (epochs advance, slot parities alternate)
        peer = SequenceSplitDecode([[_shard_cache(k, v, start, stop, rank == world - 1)] for k, v in kvs],
                                   num_kv_heads=HEADS, exchange="peer")
        for _ in range(4):
            po, pl = peer(query)
            torch.cuda.synchronize()
            assert torch.equal(po, out) and torch.equal(pl, lse)
        from unicache_b200 import kernels

        assert kernels.device_status() == 0
        peer.close()
        open(os.path.join(result_dir, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


def test_sequence_split_over_nccl_ranks(tmp_path):
    need_gpu()
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    assert sorted(os.listdir(tmp_path)) == [f"ok{r}" for r in range(world)]

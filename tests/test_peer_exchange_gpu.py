"""The sequence-split merge over peer memory (ucb_split_merge_peer) on one
GPU: with one rank it returns the local summary; with a second "rank" that
never sends, its bounded wait runs out, the device error word reports it and
the GPU stays usable.  The multi-GPU exchange is checked against the NCCL
path in tests/test_distributed_gpu.py."""

from __future__ import annotations

import ctypes

import pytest
import torch

from unicache_b200 import _capi, kernels

from .gpu_util import need_gpu

pytestmark = pytest.mark.gpu

TIMEOUT_BIT = 1  # DEVERR_MBAR_TIMEOUT


def _alloc(rows):
    nbytes = int(_capi.load().ucb_peer_buffer_bytes(rows))
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_char * 64)()
    kernels.call("ucb_peer_buffer_alloc", nbytes, ctypes.byref(ptr), handle)
    return ptr.value


def _summary(rows, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    out = torch.randn(rows, 128, generator=gen, device="cuda").to(torch.bfloat16)
    lse = torch.randn(rows, generator=gen, device="cuda") * 3
    return out, lse


def test_single_rank_returns_the_local_summary_every_call():
    need_gpu()
    rows = 28
    buf = _alloc(rows)
    try:
        bufs = (ctypes.c_void_p * 1)(buf)
        for step in range(3):  # epochs advance, parities alternate
            out, lse = _summary(rows, seed=step)
            merged = torch.empty_like(out)
            total = torch.empty_like(lse)
            kernels.call("ucb_split_merge_peer", 0, 1, bufs, out.data_ptr(), lse.data_ptr(), rows, 128,
                         merged.data_ptr(), total.data_ptr(), kernels.stream_of(out))
            torch.cuda.synchronize()
            assert torch.equal(merged, out)
            assert torch.allclose(total, lse, atol=1e-5, rtol=0)
        assert kernels.device_status() == 0
    finally:
        kernels.call("ucb_peer_buffer_free", ctypes.c_void_p(buf))


def test_missing_peer_times_out_and_reports():
    """Rank 0 of a two-rank exchange whose second rank never runs: its wait
    for rank 1's words ends after the 1 s budget, the kernel returns without
    writing the output and the error word carries the timeout bit."""
    need_gpu()
    rows = 28
    own, other = _alloc(rows), _alloc(rows)
    try:
        bufs = (ctypes.c_void_p * 2)(own, other)
        out, lse = _summary(rows, seed=7)
        merged = torch.full_like(out, 5.0)
        total = torch.full_like(lse, 5.0)
        assert kernels.device_status() == 0
        kernels.call("ucb_split_merge_peer", 0, 2, bufs, out.data_ptr(), lse.data_ptr(), rows, 128,
                     merged.data_ptr(), total.data_ptr(), kernels.stream_of(out))
        torch.cuda.synchronize()
        assert kernels.device_status() & TIMEOUT_BIT
        assert bool((merged == 5.0).all()) and bool((total == 5.0).all())
        x = torch.ones(1024, device="cuda")  # the context is still usable
        assert float(x.sum()) == 1024.0
    finally:
        kernels.call("ucb_peer_buffer_free", ctypes.c_void_p(own))
        kernels.call("ucb_peer_buffer_free", ctypes.c_void_p(other))


def test_peer_entry_rejects_bad_arguments():
    need_gpu()
    out, lse = _summary(4, seed=1)
    bufs = (ctypes.c_void_p * 1)(None)
    with pytest.raises(ValueError):
        kernels.call("ucb_split_merge_peer", 0, 9, bufs, out.data_ptr(), lse.data_ptr(), 4, 128, out.data_ptr(),
                     lse.data_ptr(), kernels.stream_of(out))
    with pytest.raises(ValueError):
        kernels.call("ucb_split_merge_peer", 0, 1, bufs, out.data_ptr(), lse.data_ptr(), 4, 128, out.data_ptr(),
                     lse.data_ptr(), kernels.stream_of(out))

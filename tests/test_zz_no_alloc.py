"""The allocation-free decode entry point (ucb_decode_attention_noalloc) against
the regular one (ucb_decode_attention) on the same plan, through the C ABI.

It keeps its warp-state slots in a static device array shared by every call,
so two calls in a row must both match; the file is named to be collected
last and also passes alone in a fresh process.  Tolerance: the north-star
attention bound (max-abs 2e-2, mean-abs 1e-3) and 2e-2 on the LSE."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from unicache_b200 import PackedKIVICache, PhysicalDecodeBatch, _capi, kernels
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import MAX_ABS, MEAN_ABS, need_gpu

pytestmark = pytest.mark.gpu


def _plan(seqs=2, tokens=576, heads=4):
    caches = []
    for s in range(seqs):
        key, value = make_kv(tokens, heads, 128, seed=70 + s, device="cuda")
        caches.append([PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(tokens, device="cuda"),
                                                  token_type_id=3, k_bits=2, v_bits=2, group_size=32,
                                                  residual_length=64)])
    return PhysicalDecodeBatch(caches, num_kv_heads=heads).plan


def _noalloc(plan, query, num_partials=None):
    out = torch.full_like(query, float("nan"))
    lse = torch.full((plan.num_seqs, int(query.shape[1])), float("nan"), device=query.device, dtype=torch.float32)
    _capi.call("ucb_decode_attention_noalloc", query.data_ptr(), query.stride(0), int(query.shape[1]),
               plan.num_kv_heads, plan.head_dim, plan.spans.data_ptr(), plan.num_spans, plan.ctas.data_ptr(),
               plan.num_ctas, plan.warp_bounds.data_ptr(), plan.pairs.data_ptr(), plan.num_pairs,
               plan.warp_slots.data_ptr(), plan.num_partials if num_partials is None else num_partials,
               plan.k_bits, plan.v_bits,
               plan.group_size, _capi.UCB_BF16, 1.0 / np.sqrt(plan.head_dim), out.data_ptr(), out.stride(0),
               lse.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out, lse


def _close(actual, expected, what):
    diff = (actual.float() - expected.float()).abs()
    assert torch.isfinite(actual.float()).all(), what
    assert float(diff.max()) <= MAX_ABS, f"{what}: max abs {float(diff.max()):.3e}"
    assert float(diff.mean()) <= MEAN_ABS, f"{what}: mean abs {float(diff.mean()):.3e}"


def test_noalloc_decode_matches_the_allocating_entry_on_two_calls_in_a_row():
    need_gpu()
    plan = _plan()
    assert plan.num_partials <= 512, plan.num_partials
    queries = [make_query(plan.num_seqs, 28, 128, seed=s, device="cuda") for s in (5, 6)]
    results = [_noalloc(plan, q) for q in queries]  # two calls in a row, different queries
    torch.cuda.synchronize()
    for q, (out, lse) in zip(queries, results):
        ref_out, ref_lse = plan.run(q)
        torch.cuda.synchronize()
        _close(out, ref_out, "noalloc output")
        assert float((lse - ref_lse).abs().max()) <= 2e-2
    assert kernels.device_status() == 0


def test_noalloc_decode_rejects_plans_beyond_the_static_scratch():
    need_gpu()
    plan = _plan(seqs=1)
    query = make_query(1, 28, 128, seed=9, device="cuda")
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(plan, query, num_partials=513)

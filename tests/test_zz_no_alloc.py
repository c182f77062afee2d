"""The allocation-free decode entry point (ucb_decode_attention_noalloc) against
the regular one (ucb_decode_attention) on the same plan, through the C ABI.

It keeps its warp-state slots in a static device array shared by every call,
so two calls in a row must both match; the file is named to be collected
last and also passes alone in a fresh process.  Both entry points run the same
kernels on the same plan, so the outputs and LSE must be bit-identical."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from unicache_b200 import PackedKIVICache, PhysicalDecodeBatch, _capi, kernels
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import need_gpu

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
        assert torch.isfinite(out.float()).all()
        assert torch.equal(out, ref_out), "noalloc output differs from the allocating entry point"
        assert torch.equal(lse, ref_lse), "noalloc LSE differs from the allocating entry point"
    assert kernels.device_status() == 0


def test_noalloc_decode_rejects_plans_beyond_the_static_scratch():
    need_gpu()
    plan = _plan(seqs=1)
    query = make_query(1, 28, 128, seed=9, device="cuda")
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(plan, query, num_partials=513)


def test_noalloc_decode_flags_slot_indices_beyond_the_declared_count():
    """A caller that declares fewer slots than its plan uses gets the invalid-
    descriptor flag (2) from the kernels, which skip the out-of-range slots
    instead of writing past the static array; a correct call afterwards is
    unaffected."""

    need_gpu()
    plan = _plan(seqs=1)
    assert plan.num_partials >= 2
    query = make_query(1, 28, 128, seed=11, device="cuda")
    _noalloc(plan, query, num_partials=plan.num_partials - 1)
    assert kernels.device_status() & 2
    out, lse = _noalloc(plan, query)
    ref_out, ref_lse = plan.run(query)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
    assert kernels.device_status() == 0

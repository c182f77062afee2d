"""Long-query attention over span tables, both launch forms: reading the
segments in place (ucb_long_query_attention: dense and H2O rows copied into
the tensor-core operand tiles, packed KIVI tiles restored in shared memory)
and staged (ucb_long_query_attention_staged: every key space gathered once
into a bf16 workspace by ucb_long_query_stage, then streamed by TMA).  The
staged workspace is checked bit for bit against a numpy restore of the same
codes (code * scale + minimum, one rounding to bf16), and both launch forms
against each other.

Checked against (a) the workspace path it replaces: the bit-exact dequant
kernel restores every packed span into a bf16 workspace, then the TMA-fed
kernel runs over it (same operand values, keys in another order, so the
outputs agree to about one bf16 ulp), and (b) the float64 oracle within the north-star bound (max-abs 2e-2,
mean-abs 1e-3; LSE 2e-2).  Span layouts cover packed spans that start
mid-tile and mid-word, spans straddling tile boundaries, 4-bit codes, group
64/128, head-major H2O rows, and ragged last tiles."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, kivi
from unicache_b200 import GQAH2OCache, PackedKIVICache, kernels
from unicache_b200.adapters.attention import batched_long_query_attention, long_query_attention_summary
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import assert_attention_close, host, need_gpu

pytestmark = pytest.mark.gpu


def _segments(seed, layout, bits, group):
    segs, keys, vals = [], [], []
    for i, (kind, n) in enumerate(layout):
        k, v = make_kv(n, 4, 128, seed=seed * 10 + i, device="cuda")
        if kind == "packed":
            seg = PackedKIVICache.from_dense(k, v, logical_token_ids=torch.arange(n, device="cuda"), token_type_id=3,
                                             k_bits=bits, v_bits=bits, group_size=group, residual_length=group // 2)
            ref = kivi.packed_from_dense(host(k), host(v), "bfloat16", k_bits=bits, v_bits=bits, group_size=group,
                                         residual_length=group // 2)
            rk, rv = kivi.packed_dequantize(ref)
        elif kind == "h2o":
            sc = torch.rand(4, n, generator=torch.Generator().manual_seed(seed + i)).to("cuda")
            seg = GQAH2OCache.from_dense(k, v, logical_token_ids=torch.arange(n, device="cuda"), token_type_id=1,
                                         per_kv_head_scores=sc, target_tokens=max(1, n // 3), recent_tokens=n // 12)
            rk, rv = host(seg.key).transpose(1, 0, 2), host(seg.value).transpose(1, 0, 2)
        else:
            seg = (k, v)
            rk, rv = host(k), host(v)
        segs.append(seg)
        keys.append(rk)
        vals.append(rv)
    return segs, keys, vals


def _workspace_path(query, segs):
    """The replaced path: every segment restored into [H, Np, D] / [H, D, Np] bf16 workspaces."""

    hkv = 4
    parts_k, parts_v = [], []
    for seg in segs:
        if isinstance(seg, PackedKIVICache):
            k, v = seg.dequantize(dtype=torch.bfloat16)
            parts_k.append(k.transpose(0, 1))
            parts_v.append(v.transpose(0, 1))
        elif isinstance(seg, GQAH2OCache):
            parts_k.append(seg.key)
            parts_v.append(seg.value)
        else:
            parts_k.append(seg[0].transpose(0, 1))
            parts_v.append(seg[1].transpose(0, 1))
    kw = torch.cat(parts_k, dim=1)
    vw = torch.cat(parts_v, dim=1)
    n = int(kw.shape[1])
    pad = (n + 7) // 8 * 8
    k = torch.zeros(hkv, pad, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    k[:, :n] = kw
    v[:, :n] = vw
    lq, hq, d = map(int, query.shape)
    grp = hq // hkv
    q = query.reshape(lq, hkv, grp, d).permute(1, 0, 2, 3).reshape(hkv, lq * grp, d).contiguous()
    out, lse = kernels.prefill_attention(q, k, v.transpose(1, 2).contiguous(), n)
    out = out.view(hkv, lq, grp, d).permute(1, 0, 2, 3).reshape(lq, hq, d)
    return out, lse.view(hkv, lq, grp).permute(0, 2, 1).reshape(hq, lq)


LAYOUTS = [
    # (bits, group, [(kind, tokens)], query length)
    (2, 32, [("dense", 16), ("h2o", 150), ("packed", 1024), ("dense", 100)], 1024),
    (2, 32, [("h2o", 7), ("packed", 333), ("packed", 200), ("dense", 1)], 96),
    (4, 64, [("packed", 700), ("dense", 129)], 300),
    (4, 128, [("dense", 40), ("packed", 1000)], 37),
    (2, 64, [("packed", 64)], 512),
]


@pytest.mark.parametrize("staged", [False, True])
@pytest.mark.parametrize("case", range(len(LAYOUTS)))
def test_long_query_spans_match_workspace_path_and_oracle(case, staged):
    need_gpu()
    bits, group, layout, lq = LAYOUTS[case]
    segs, keys, vals = _segments(50 + case, layout, bits, group)
    query = make_query(lq, 28, 128, seed=60 + case, device="cuda")
    out, lse = long_query_attention_summary(query, segs, staged=staged)
    w_out, w_lse = _workspace_path(query, segs)
    torch.cuda.synchronize()
    diff = (out.float() - w_out.float()).abs()
    # same operands, keys in another order (packed spans first): bf16 rounding only
    assert float(diff.max()) <= 2e-2 and float(diff.mean()) <= 5e-4, (float(diff.max()), float(diff.mean()))
    assert float((lse - w_lse).abs().max()) <= 1e-3
    e_out, e_lse = attention.mixed_attention(host(query), keys, vals)
    assert_attention_close(out, e_out, what=f"long-query spans case {case}")
    assert np.abs(host(lse) - e_lse).max() <= 2e-2
    # a second call reuses the cached span tables and is bitwise identical
    out2, lse2 = long_query_attention_summary(query, segs, staged=staged)
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
    # the other launch form: the same operand values in the same key order,
    # key ranges split differently (merges round differently: bf16 ulps)
    o_out, o_lse = long_query_attention_summary(query, segs, staged=not staged)
    torch.cuda.synchronize()
    cross = (out.float() - o_out.float()).abs()
    assert float(cross.max()) <= 2e-2 and float(cross.mean()) <= 5e-4, (float(cross.max()), float(cross.mean()))
    assert float((lse - o_lse).abs().max()) <= 1e-3
    assert kernels.device_status() == 0


@pytest.mark.parametrize("staged", [False, True])
def test_batched_long_query_spans_three_samples(staged):
    need_gpu()
    samples, queries, expects = [], [], []
    for i, (layout, lq) in enumerate([([("h2o", 90), ("packed", 500)], 40),
                                      ([("packed", 1088)], 300), ([("dense", 70), ("h2o", 150)], 7)]):
        segs, keys, vals = _segments(80 + i, layout, 2, 32)
        q = make_query(lq, 28, 128, seed=90 + i, device="cuda")
        samples.append(segs)
        queries.append(q)
        expects.append(attention.mixed_attention(host(q), keys, vals))
    results = batched_long_query_attention(queries, samples, staged=staged)
    torch.cuda.synchronize()
    for (out, lse), (e_out, e_lse) in zip(results, expects):
        assert_attention_close(out, e_out, what="batched spans")
        assert np.abs(host(lse) - e_lse).max() <= 2e-2
    assert kernels.device_status() == 0


def _bf16_single_round(x: np.ndarray) -> np.ndarray:
    """Round float64 values (exact here: code * scale + minimum of bf16
    operands) to bf16 once, round-half-even."""

    mant, exp = np.frexp(x)
    return np.ldexp(np.rint(mant * 256.0), exp - 8)


def _unpack(code: np.ndarray, bits: int, count: int, axis: int) -> np.ndarray:
    f, mask = 32 // bits, (1 << bits) - 1
    w = code.astype(np.int64) & 0xFFFFFFFF
    idx = np.arange(count)
    if axis == 0:  # packed along tokens: [T/f, D] -> [T, D]
        return (w[idx // f] >> (bits * (idx % f))[:, None]) & mask
    return (w[:, idx // f] >> (bits * (idx % f))[None, :]) & mask  # along channels: [T, D/f] -> [T, D]


def _restored(seg: PackedKIVICache, h: int):
    n, g = seg.quantized_tokens, seg.group_size
    kc = _unpack(host(seg.key_code[h]), seg.k_bits, n, 0)
    ks = np.repeat(host(seg.key_scale[h]).astype(np.float64), g, axis=0)[:n]
    km = np.repeat(host(seg.key_minimum[h]).astype(np.float64), g, axis=0)[:n]
    vc = _unpack(host(seg.value_code[h]), seg.v_bits, 128, 1)
    vs = np.repeat(host(seg.value_scale[h]).astype(np.float64), g, axis=1)
    vm = np.repeat(host(seg.value_minimum[h]).astype(np.float64), g, axis=1)
    return _bf16_single_round(kc * ks + km), _bf16_single_round(vc * vs + vm)


def _expected_key_space(segs, h):
    """Keys and values of KV head h in span order: packed spans first, then
    the dense, H2O and residual rows in segment order."""

    pk, pv, dk, dv = [], [], [], []
    for seg in segs:
        if isinstance(seg, PackedKIVICache):
            if seg.quantized_tokens:
                k, v = _restored(seg, h)
                pk.append(k)
                pv.append(v)
            dk.append(host(seg.residual_key[:, h]))
            dv.append(host(seg.residual_value[:, h]))
        elif isinstance(seg, GQAH2OCache):
            dk.append(host(seg.key[h]))
            dv.append(host(seg.value[h]))
        else:
            dk.append(host(seg[0][:, h]))
            dv.append(host(seg[1][:, h]))
    return np.concatenate(pk + dk), np.concatenate(pv + dv)


@pytest.mark.parametrize("bits,group", [(2, 32), (4, 64), (2, 128)])
def test_stage_workspace_is_the_single_rounding_restore(bits, group):
    need_gpu()
    samples = [_segments(120, [("dense", 40), ("packed", 333), ("h2o", 150)], bits, group)[0],
               _segments(121, [("packed", 700), ("dense", 9)], bits, group)[0]]
    tables = kernels.long_query_tables(samples, 4, [0, 5], [35, 21], "cuda")
    k_ws, vt_ws = kernels.long_query_stage(tables, 4, "cuda")
    torch.cuda.synchronize()
    kh, vth = host(k_ws), host(vt_ws)
    base = 0
    for segs in samples:
        extent = 0
        for h in range(4):
            ek, ev = _expected_key_space(segs, h)
            n = int(ek.shape[0])
            padded = -(-n // 128) * 128
            extent = max(extent, padded)
            assert np.array_equal(kh[h, base:base + n], ek.astype(np.float32)), (h, base)
            assert np.array_equal(vth[h, :, base:base + n], ev.T.astype(np.float32)), (h, base)
            assert not kh[h, base + n:base + padded].any() and not vth[h, :, base + n:base + padded].any()
        base += extent
    assert tables.ws_rows == base
    assert kernels.device_status() == 0


@pytest.mark.parametrize("case", range(len(LAYOUTS)))
def test_persistent_staged_launch_matches_one_cta_per_item(case):
    """The persistent staged launch (at most one CTA per SM, each running an
    equal share of (row block, key tile) units, cut row blocks merged from
    several partials) against the one-CTA-per-item staged launch and the
    oracle; a repeated call is bitwise identical."""

    need_gpu()
    bits, group, layout, lq = LAYOUTS[case]
    segs, keys, vals = _segments(50 + case, layout, bits, group)
    query = make_query(lq, 28, 128, seed=60 + case, device="cuda")
    tables = kernels.long_query_tables([segs], 4, [0], [lq * 7], "cuda")
    assert tables.num_ctas <= torch.cuda.get_device_properties(0).multi_processor_count
    out, lse = kernels.long_query_attention(query, tables, num_kv_heads=4, staged=True, persistent=True)
    ref_out, ref_lse = kernels.long_query_attention(query, tables, num_kv_heads=4, staged=True, persistent=False)
    out2, lse2 = kernels.long_query_attention(query, tables, num_kv_heads=4, staged=True, persistent=True)
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
    diff = (out.float() - ref_out.float()).abs()
    assert float(diff.max()) <= 2e-2 and float(diff.mean()) <= 5e-4, (float(diff.max()), float(diff.mean()))
    assert float((lse - ref_lse).abs().max()) <= 1e-3
    e_out, e_lse = attention.mixed_attention(host(query), keys, vals)
    assert_attention_close(out, e_out, what=f"persistent staged case {case}")
    assert np.abs(host(lse) - e_lse).max() <= 2e-2
    assert kernels.device_status() == 0


@pytest.mark.parametrize("min_tiles", [2, 6])
def test_persistent_staged_short_query_many_pieces(min_tiles, monkeypatch):
    """8 query positions over a 3095-key segment mix: every row block is cut
    into pieces of ``min_tiles`` tiles (about a dozen at 2), so each merge
    item folds in several partials."""

    need_gpu()
    monkeypatch.setattr(kernels, "PERSIST_MIN_TILES", min_tiles)
    segs, keys, vals = _segments(140 + min_tiles, [("h2o", 150), ("packed", 1024), ("dense", 1921)], 2, 32)
    query = make_query(8, 28, 128, seed=141, device="cuda")
    tables = kernels.long_query_tables([segs], 4, [0], [8 * 7], "cuda")
    assert tables.p_slots >= 4 * (24 // min_tiles - 1)
    out, lse = kernels.long_query_attention(query, tables, num_kv_heads=4, staged=True, persistent=True)
    torch.cuda.synchronize()
    e_out, e_lse = attention.mixed_attention(host(query), keys, vals)
    assert_attention_close(out, e_out, what="persistent staged, 8 positions")
    assert np.abs(host(lse) - e_lse).max() <= 2e-2
    assert kernels.device_status() == 0

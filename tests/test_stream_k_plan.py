"""Invariants of the persistent long-query plan (kernels.plan_stream_k), on
the CPU: every (row block, key tile) unit is covered exactly once; CTA ranges
are contiguous and within one tile of each other; a row block cut into
pieces runs its first piece as the merge item, which is the last item of its
CTA, and its other pieces as partial items, each the first item of its CTA
(so a merge item waits only on items that never wait before them); partial
slots of a row block are consecutive and start at the merge item's slot."""

from __future__ import annotations

import pytest

from unicache_b200.kernels import PREFILL_KEY_TILE, plan_stream_k


def _blocks(spec):
    rows = []
    for head, (tokens, nblocks) in enumerate(spec):
        for r in range(nblocks):
            rows.append([head, 256 * r, 256, 0, tokens, 0, 0, 5 * head, 3, 0, 1024 * head, 0])
    return rows


CASES = [
    ([(3095, 28)] * 4, 148),      # the configuration-4 layer
    ([(3095, 1)] * 4, 148),       # 8 query positions: pieces of ~2 tiles
    ([(129, 3), (5000, 2), (64, 1)], 148),
    ([(1000, 7)] * 2, 16),
    ([(128, 1)], 148),            # one tile in total
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_stream_k_plan_invariants(case):
    spec, sms = CASES[case]
    blocks = _blocks(spec)
    rows, offsets, slots = plan_stream_k(blocks, sms)
    ctas = len(offsets) - 1
    assert 1 <= ctas <= sms and offsets[0] == 0 and offsets[-1] == len(rows)
    assert all(a <= b for a, b in zip(offsets, offsets[1:]))
    # coverage: each block's tiles exactly once, keys in order
    covered = {}
    for r in rows:
        key = (r[0], r[1])
        covered.setdefault(key, []).append((r[3], r[3] + r[4], r))
    for b in blocks:
        pieces = sorted(covered[(b[0], b[1])], key=lambda p: p[0])
        assert pieces[0][0] == 0 and pieces[-1][1] == b[4]
        assert all(p[1] == q[0] for p, q in zip(pieces, pieces[1:]))
        assert all(p[0] % PREFILL_KEY_TILE == 0 for p in pieces)
        for _, _, r in pieces:
            assert r[7:11] == b[7:11] and r[2] == b[2]
        if len(pieces) == 1:
            assert pieces[0][2][5] == 0
        else:
            merge = pieces[0][2]
            assert merge[5] == 2 and merge[11] == len(pieces) - 1
            assert [p[2][5] for p in pieces[1:]] == [1] * (len(pieces) - 1)
            assert [p[2][6] for p in pieces[1:]] == list(range(merge[6], merge[6] + len(pieces) - 1))
    # ordering: merge items last in their CTA, partial items first
    for c in range(ctas):
        items = rows[offsets[c]:offsets[c + 1]]
        assert items, "every CTA has work"
        for i, r in enumerate(items):
            if r[5] == 2:
                assert i == len(items) - 1
            if r[5] == 1:
                assert i == 0
    # balance: tile counts per CTA differ by at most one
    per = [sum(-(-r[4] // PREFILL_KEY_TILE) for r in rows[offsets[c]:offsets[c + 1]]) for c in range(ctas)]
    assert max(per) - min(per) <= 1
    assert slots == sum(1 for r in rows if r[5] == 1)

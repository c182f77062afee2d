"""CPU tests of host-side logic: decode work partitioning, operator parameter
validation and the budget arithmetic of the physical requests."""

from __future__ import annotations

import random

import pytest

from unicache_b200 import H2OPhysicalGQAOperator, KIVIPackedQuantizationOperator
from unicache_b200.kernels import MAX_PAIRS_PER_CTA, _assign_ctas, _split_warps
from unicache_b200.storage.physical import normalize_backend


def _units(pairs, packed_units, dense_units, packed_w=6144.0, dense_w=4096.0):
    weights, unit_pair, seg = [], [], []
    sid = -1
    for p in range(pairs):
        for kind, n, w in ((0, packed_units, packed_w), (1, dense_units, dense_w)):
            if n == 0:
                continue
            sid += 1
            weights += [w] * n
            unit_pair += [p] * n
            seg += [sid] * n
    return weights, unit_pair, seg


def _check(bounds_list, weights, unit_pair, seg, warps):
    covered = []
    for bounds in bounds_list:
        assert len(bounds) == warps + 1
        assert all(a <= b for a, b in zip(bounds, bounds[1:]))
        covered.append((bounds[0], bounds[-1]))
        assert len({unit_pair[u] for u in range(bounds[0], bounds[-1])}) <= MAX_PAIRS_PER_CTA
        for w in range(warps):
            a, b = bounds[w], bounds[w + 1]
            crossings = sum(1 for u in range(a + 1, b) if seg[u] != seg[u - 1])
            assert crossings <= 1
    # ranges tile the unit space in order
    assert covered[0][0] == 0 and covered[-1][1] == len(weights)
    assert all(x[1] == y[0] for x, y in zip(covered, covered[1:]))


@pytest.mark.parametrize("pairs,packed,dense", [(64, 128, 16), (4, 128, 16), (32, 512, 16), (200, 3, 2),
                                                (1, 2048, 0), (7, 0, 40)])
def test_decode_partition_invariants(pairs, packed, dense):
    weights, unit_pair, seg = _units(pairs, packed, dense)
    bounds = _assign_ctas(weights, unit_pair, seg, 148, 12)
    _check(bounds, weights, unit_pair, seg, 12)


def test_decode_partition_is_balanced_for_config2():
    weights, unit_pair, seg = _units(64, 128, 16)
    bounds = _assign_ctas(weights, unit_pair, seg, 148, 12)
    assert len(bounds) == 148
    per_cta = [sum(weights[b[0]:b[-1]]) for b in bounds]
    assert max(per_cta) / (sum(per_cta) / len(per_cta)) < 1.06


def test_split_warps_rejects_two_boundaries_in_one_warp():
    weights = [1.0] * 6
    seg = [0, 0, 1, 1, 2, 2]
    assert _split_warps(weights, seg, 0, 6, 1) is None
    assert _split_warps(weights, seg, 0, 6, 3) is not None


def test_random_partitions_hold_invariants():
    rng = random.Random(3)
    for _ in range(40):
        pairs = rng.randint(1, 80)
        weights, unit_pair, seg = [], [], []
        sid = -1
        for p in range(pairs):
            for kind in range(rng.randint(1, 3)):
                n = rng.randint(1, 60)
                sid += 1
                weights += [rng.choice([6144.0, 4096.0, 2048.0])] * n
                unit_pair += [p] * n
                seg += [sid] * n
        warps = rng.choice([8, 12])
        _check(_assign_ctas(weights, unit_pair, seg, rng.randint(1, 200), warps), weights, unit_pair, seg, warps)


def test_operator_parameter_validation_matches_reference_rules():
    kivi = KIVIPackedQuantizationOperator()
    params = kivi.build_params({"bits": 2, "group_size": 32})
    assert params["k_bits"] == params["v_bits"] == 2 and params["residual_length"] == 32
    assert params["backend"] == "b200"
    assert kivi.build_params({"bits": 4, "backend": "cuda"})["backend"] == "b200"
    for bad in ({"bits": 3}, {"group_size": 0}, {"backend": "reference"}):
        with pytest.raises(ValueError):
            kivi.build_params(bad)
    h2o = H2OPhysicalGQAOperator()
    params = h2o.build_params({})
    assert params["target_budget_ratio"] == 0.2 and params["recent_budget_fraction"] == 0.25
    for bad in ({"target_budget_ratio": 0.0}, {"target_budget_ratio": 1.5}, {"recent_budget_fraction": -0.1}):
        with pytest.raises(ValueError):
            h2o.build_params(bad)


def test_backend_names():
    assert normalize_backend("b200") == normalize_backend("cuda") == "b200"
    with pytest.raises(ValueError):
        normalize_backend("reference")
    with pytest.raises(ValueError):
        normalize_backend("triton")


def test_key_split_plan():
    """plan_key_split: no split once row blocks fill the SMs or when it saves
    less than a tile time; otherwise the first part leaves room for the
    second parts on the free SMs (config 4: 112 row blocks of 25 tiles on
    148 SMs -> 23 + 2; a single 4-block problem -> 12 + 13)."""
    from unicache_b200.kernels import PREFILL_CTA_FIXED_TILES as F
    from unicache_b200.kernels import plan_key_split

    assert plan_key_split(148, 25, 148) is None
    assert plan_key_split(200, 25, 148) is None
    assert plan_key_split(10, 1, 148) is None
    assert plan_key_split(112, 25, 148) == 23
    assert plan_key_split(4, 25, 148) == 12
    for rows, tiles in [(1, 8), (8, 8), (40, 64), (112, 128), (147, 30)]:
        first = plan_key_split(rows, tiles, 148)
        if first is None:
            continue
        assert 1 <= first < tiles
        rounds = -(-rows // (148 - rows))
        cost = max(F + first + 0.5, rounds * (F + tiles - first))
        assert cost <= F + tiles - 1


def test_split_prefill_items_layout():
    """Split rows: merge parts first, then unsplit rows, then partial parts;
    each pair shares a slot and covers its row block's keys exactly once."""
    from unicache_b200.kernels import split_prefill_items

    rows = [[h, 256 * b, 256, 0, 3095, 0, 0, 0] for h in range(2) for b in range(3)] + [[0, 768, 49, 3136, 16, 0, 0, 0]]
    out, slots = split_prefill_items(rows, 148)
    assert slots == 6 and len(out) == 6 + 1 + 6
    merges, whole, parts = out[:6], out[6:7], out[7:]
    assert all(r[5] == 2 for r in merges) and all(r[5] == 1 for r in parts) and whole[0][5] == 0
    for m, p in zip(merges, parts):
        assert m[6] == p[6] and m[:3] == p[:3]
        assert p[3] == m[3] + m[4] and m[4] + p[4] == 3095 and m[4] % 128 == 0
    same, none = split_prefill_items(rows * 30, 148)
    assert none == 0 and all(r[5] == 0 for r in same)

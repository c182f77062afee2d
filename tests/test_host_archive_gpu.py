"""Packed KIVI host replicas on the GPU: restore is bit-exact (every tensor),
restored caches decode identically, files round-trip, and the archive's
transitions follow the reference's rule (unicache/storage/hierarchy.py:70-125)
while really moving the replica bytes."""

from __future__ import annotations

import pytest
import torch

from unicache_b200 import PhysicalDecodeBatch, kernels
from unicache_b200.storage import HostPackedKIVI, PackedKIVICache, QuantizedHostArchive
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import need_gpu

pytestmark = pytest.mark.gpu

FIELDS = ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum", "residual_key",
          "residual_value", "logical_token_ids")
META = ("token_type_id", "k_bits", "v_bits", "group_size", "quantized_tokens", "head_dim", "num_kv_heads",
        "residual_length")


def _cache(key, value, kb, vb, group=32, residual=64):
    t = key.shape[0]
    return PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(t, device="cuda"), token_type_id=3,
                                      k_bits=kb, v_bits=vb, group_size=group, residual_length=residual)


def _same(a, b):
    for name in FIELDS:
        x, y = getattr(a, name), getattr(b, name)
        assert (x is None) == (y is None), name
        if x is not None:
            assert x.dtype == y.dtype and x.shape == y.shape and torch.equal(x, y), name
    for name in META:
        assert getattr(a, name) == getattr(b, name), name


@pytest.mark.parametrize("kb,vb,group", [(2, 2, 32), (4, 2, 64), (2, 4, 128), (8, 4, 128)])
def test_restore_is_bit_exact_and_decodes_identically(kb, vb, group, tmp_path):
    need_gpu()
    key, value = make_kv(1500, 4, 128, seed=kb + vb, device="cuda")
    cache = _cache(key, value, kb, vb, group)
    host = cache.to_host()
    assert host.blob.is_pinned() and host.resident_bytes == cache.resident_bytes
    restored = host.to_device()
    _same(cache, restored)
    host.save(tmp_path / "seg.ucbkivi")
    from_file = HostPackedKIVI.load(tmp_path / "seg.ucbkivi").to_device()
    _same(cache, from_file)
    if max(kb, vb) == 8:
        return  # the decode kernel takes 2- and 4-bit segments
    query = make_query(1, 28, 128, seed=9, device="cuda")
    out_a, lse_a = PhysicalDecodeBatch([[cache]], num_kv_heads=4)(query)
    out_b, lse_b = PhysicalDecodeBatch([[from_file]], num_kv_heads=4)(query)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    assert kernels.device_status() == 0


def test_restored_cache_keeps_streaming():
    """A restored replica accepts appends like the original."""
    need_gpu()
    key, value = make_kv(700, 4, 128, seed=4, device="cuda")
    original = _cache(key[:600], value[:600], 2, 2)
    restored = original.to_host().to_device()
    for c in (original, restored):
        c.append(key[600:], value[600:], logical_token_ids=torch.arange(600, 700, device="cuda"))
    _same(original, restored)


def test_archive_transitions_follow_the_reference_rule():
    need_gpu()
    key, value = make_kv(2048, 4, 128, seed=11, device="cuda")
    full = 2048 * 4 * 128 * 2 * 2
    c4, c2 = _cache(key, value, 4, 4), _cache(key, value, 2, 2)
    archive = QuantizedHostArchive(full_archive_bytes=full)
    archive.store(("kivi", 4), c4)
    archive.store(("kivi", 2), c2.to_host())
    seq = [("kivi", 4), ("kivi", 4), ("kivi", 2), ("kivi", 4)]
    kinds, h2d, released = [], [], []
    for d in seq:
        tr, cache = archive.materialize(descriptor=d)
        _same(cache, c4 if d[1] == 4 else c2)
        kinds.append(tr.transition_kind)
        h2d.append(tr.h2d_bytes)
        released.append(tr.released_bytes)
    r4, r2 = c4.resident_bytes, c2.resident_bytes
    assert kinds == ["initial", "reuse", "downgrade", "upgrade"]
    assert h2d == [0, 0, r2, r4] and released == [0, 0, r4, r2]
    s = archive.summary()
    assert s["precision_transitions"] == 3 and s["materializations"] == 4
    assert s["cumulative_h2d_bytes"] == r2 + r4 and s["cumulative_released_bytes"] == r4 + r2
    assert s["cumulative_full_rebuild_h2d_bytes"] == r4 + r2 + r4
    assert s["host_replica_catalog_bytes"] == r4 + r2 and s["host_replica_variants"] == 2
    assert s["current_resident_bytes"] == r4 and s["peak_resident_ratio"] == pytest.approx(r4 / full)
    # initial, downgrade and upgrade copied a replica; reuse did not
    blobs = {d: archive._replicas[d].nbytes for d in archive._replicas}
    assert s["copied_h2d_bytes"] == 2 * blobs[("kivi", 4)] + blobs[("kivi", 2)]
    with pytest.raises(KeyError):
        archive.materialize(descriptor=("kivi", 8))

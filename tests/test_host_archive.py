"""Packed KIVI host replicas: file format round trip and validation (CPU).
The archive's transition accounting is checked on the GPU."""

from __future__ import annotations

import json
import struct

import pytest
import torch

from unicache_b200.storage import HostPackedKIVI, PackedKIVICache
from unicache_b200.storage.hierarchy import MAGIC


def _cpu_cache(tokens=96, residual=32, heads=4, d=128, kb=2, vb=4, group=32, seed=0):
    """A cache with the b200 layout's shapes, built on the CPU from random
    words (format tests only: no kernel runs)."""

    gen = torch.Generator().manual_seed(seed)
    q = tokens

    def words(*shape):
        return torch.randint(-2**31, 2**31 - 1, shape, generator=gen, dtype=torch.int64).to(torch.int32)

    def stats(*shape):
        return torch.randn(*shape, generator=gen).to(torch.bfloat16)

    return PackedKIVICache(
        key_code=words(heads, q * kb // 32, d), key_scale=stats(heads, q // group, d),
        key_minimum=stats(heads, q // group, d), value_code=words(heads, q, d * vb // 32),
        value_scale=stats(heads, q, d // group), value_minimum=stats(heads, q, d // group),
        residual_key=stats(residual, heads, d), residual_value=stats(residual, heads, d),
        logical_token_ids=torch.arange(q + residual), token_type_id=3, k_bits=kb, v_bits=vb, group_size=group,
        quantized_tokens=q, head_dim=d, num_kv_heads=heads, residual_length=residual)


FIELDS = ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum", "residual_key",
          "residual_value", "logical_token_ids")


def test_host_replica_file_round_trip(tmp_path):
    cache = _cpu_cache()
    host = HostPackedKIVI.from_cache(cache)
    assert host.resident_bytes == cache.resident_bytes
    assert all(spec["offset"] % 256 == 0 for spec in host.fields.values())
    size = host.save(tmp_path / "seg.ucbkivi")
    assert size == (tmp_path / "seg.ucbkivi").stat().st_size
    back = HostPackedKIVI.load(tmp_path / "seg.ucbkivi")
    assert back.meta == host.meta and back.fields == host.fields
    assert torch.equal(back.blob, host.blob)


def test_all_residual_cache_round_trip(tmp_path):
    cache = _cpu_cache(tokens=0, residual=20)
    for name in FIELDS[:6]:
        setattr(cache, name, None)
    host = HostPackedKIVI.from_cache(cache)
    host.save(tmp_path / "r.ucbkivi")
    back = HostPackedKIVI.load(tmp_path / "r.ucbkivi")
    assert back.fields["key_code"] is None and back.meta["quantized_tokens"] == 0


def _rewrite(path, mutate):
    data = path.read_bytes()
    (hlen,) = struct.unpack("<Q", data[8:16])
    header = json.loads(data[16:16 + hlen])
    mutate(header)
    new = json.dumps(header, sort_keys=True).encode()
    start = (16 + len(new) + 63) // 64 * 64
    old_start = (16 + hlen + 63) // 64 * 64
    path.write_bytes(MAGIC + struct.pack("<Q", len(new)) + new + b"\0" * (start - 16 - len(new)) + data[old_start:])


def test_malformed_files_are_rejected(tmp_path):
    good = tmp_path / "good.ucbkivi"
    HostPackedKIVI.from_cache(_cpu_cache()).save(good)
    data = good.read_bytes()

    bad = tmp_path / "bad"
    bad.write_bytes(b"NOTKIVI!" + data[8:])
    with pytest.raises(ValueError, match="magic"):
        HostPackedKIVI.load(bad)
    bad.write_bytes(data[:-1])
    with pytest.raises(ValueError, match="blob"):
        HostPackedKIVI.load(bad)
    bad.write_bytes(data[:20])
    with pytest.raises(ValueError):
        HostPackedKIVI.load(bad)

    cases = {
        "outside": lambda h: h["fields"]["value_code"].update(offset=h["blob_bytes"]),
        "unaligned": lambda h: h["fields"]["key_scale"].update(offset=h["fields"]["key_scale"]["offset"] + 2),
        "shape": lambda h: h["fields"]["key_code"].update(shape=[4, 7, 128]),
        "version": lambda h: h.update(version=99),
        "ids": lambda h: h["fields"]["logical_token_ids"].update(shape=[5]),
    }
    for name, mutate in cases.items():
        path = tmp_path / f"{name}.ucbkivi"
        path.write_bytes(data)
        _rewrite(path, mutate)
        with pytest.raises(ValueError):
            HostPackedKIVI.load(path)


def test_restore_needs_a_cuda_device():
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    with pytest.raises(RuntimeError):
        HostPackedKIVI.from_cache(_cpu_cache()).to_device()

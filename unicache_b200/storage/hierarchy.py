"""Host replicas of packed KIVI caches: one contiguous blob per replica.

The reference models its host archive as byte accounting only
(unicache/storage/hierarchy.py:43-157, ``LogicalQuantizedHostArchive``:
"Track full Host KV plus one all-token quantized GPU replica"; switching
precision "transfers that replica and releases the old GPU payload").  This
module moves the payload for real:

* ``HostPackedKIVI`` holds every tensor of a ``PackedKIVICache`` (codes,
  statistics, bf16 residual, logical ids) in ONE host buffer, pinned when a
  GPU is present, at 256-byte aligned offsets.  ``to_device`` restores it
  with a single host-to-device copy into one device buffer whose views are
  the cache tensors, so the decode kernels read it in place (every segment
  base stays 16-byte aligned for the bulk copies).
* ``save`` / ``load`` write the same blob to a file behind a small header
  (magic ``UCBKIVI1``, header length, JSON header, 64-byte aligned blob).
* ``QuantizedHostArchive`` keeps one host replica per precision descriptor
  and materialises the requested one on the GPU, returning the reference's
  ``QuantizedWorkingSetTransition`` with the reference's accounting rule
  (hierarchy.py:70-125) and tracking the bytes it really copied.
"""

from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

import torch

from .physical import PackedKIVICache

MAGIC = b"UCBKIVI1"
FORMAT_VERSION = 1
ALIGN = 256
_TENSOR_FIELDS = ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum",
                  "residual_key", "residual_value", "logical_token_ids")
_META_FIELDS = ("token_type_id", "k_bits", "v_bits", "group_size", "quantized_tokens", "head_dim", "num_kv_heads",
                "backend", "kernel_native_layout", "budget_shortfall_events", "residual_length")
_DTYPES = {"int32": torch.int32, "uint8": torch.uint8, "int64": torch.int64, "bfloat16": torch.bfloat16,
           "float16": torch.float16, "float32": torch.float32}
_DTYPE_NAMES = {v: k for k, v in _DTYPES.items()}


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def _pinned_empty(nbytes: int) -> torch.Tensor:
    return torch.empty(nbytes, dtype=torch.uint8, pin_memory=torch.cuda.is_available())


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def _view(buf: torch.Tensor, spec: dict) -> torch.Tensor:
    dtype = _DTYPES[spec["dtype"]]
    nb = _numel(spec["shape"]) * dtype.itemsize
    return buf[spec["offset"]: spec["offset"] + nb].view(dtype).view(spec["shape"])


@dataclass
class HostPackedKIVI:
    """One packed KIVI segment in host memory (layout ``b200``: head-major
    codes and statistics, token-major residual)."""

    blob: torch.Tensor  # uint8 [nbytes], pinned when a GPU is present
    fields: dict  # name -> {"offset", "shape", "dtype"} or None
    meta: dict

    @property
    def nbytes(self) -> int:
        return int(self.blob.numel())

    @property
    def resident_bytes(self) -> int:
        """Bytes of the tensors (as ``PackedKIVICache.resident_bytes``),
        without the blob's alignment padding."""

        return sum(_numel(spec["shape"]) * _DTYPES[spec["dtype"]].itemsize
                   for spec in self.fields.values() if spec is not None)

    # ------------------------------------------------------------ building
    @classmethod
    def from_cache(cls, cache: PackedKIVICache) -> "HostPackedKIVI":
        """Copy every tensor of ``cache`` into one host blob (device-to-host
        copies on the current stream, then a stream synchronisation)."""

        layout: dict = {}
        offset = 0
        for name in _TENSOR_FIELDS:
            t = getattr(cache, name)
            if t is None:
                layout[name] = None
                continue
            if t.dtype not in _DTYPE_NAMES:
                raise ValueError(f"{name}: unsupported dtype {t.dtype}")
            layout[name] = {"offset": offset, "shape": list(t.shape), "dtype": _DTYPE_NAMES[t.dtype]}
            offset = _round_up(offset + t.numel() * t.element_size(), ALIGN)
        blob = _pinned_empty(max(offset, ALIGN))
        for name in _TENSOR_FIELDS:
            spec = layout[name]
            if spec is not None:
                _view(blob, spec).copy_(getattr(cache, name).contiguous(), non_blocking=True)
        if any(getattr(cache, n) is not None and getattr(cache, n).is_cuda for n in _TENSOR_FIELDS):
            torch.cuda.current_stream().synchronize()
        meta = {name: getattr(cache, name) for name in _META_FIELDS}
        return cls(blob=blob, fields=layout, meta=meta)

    # ------------------------------------------------------------ restoring
    def to_device(self, device: torch.device | str | int | None = None) -> PackedKIVICache:
        """One host-to-device copy of the blob (asynchronous on the current
        stream when the blob is pinned); the cache tensors are views of it."""

        if not torch.cuda.is_available():
            raise RuntimeError("restoring a packed KIVI replica needs a CUDA device")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if device.type != "cuda":
            raise ValueError("packed KIVI replicas are restored to a CUDA device")
        dev = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        dev.copy_(self.blob, non_blocking=self.blob.is_pinned())
        tensors = {name: (None if spec is None else _view(dev, spec)) for name, spec in self.fields.items()}
        return PackedKIVICache(**tensors, **self.meta)

    # ------------------------------------------------------------ files
    def save(self, path: str | os.PathLike) -> int:
        """Write header + blob; returns the file size in bytes."""

        header = json.dumps({"version": FORMAT_VERSION, "meta": self.meta, "fields": self.fields,
                             "blob_bytes": self.nbytes}, sort_keys=True).encode()
        start = _round_up(len(MAGIC) + 8 + len(header), 64)
        with open(path, "wb") as f:
            f.write(MAGIC)
            f.write(struct.pack("<Q", len(header)))
            f.write(header)
            f.write(b"\0" * (start - len(MAGIC) - 8 - len(header)))
            f.write(self.blob.numpy().tobytes())
        return start + self.nbytes

    @classmethod
    def load(cls, path: str | os.PathLike) -> "HostPackedKIVI":
        """Read a file written by ``save``; malformed files raise ValueError."""

        with open(path, "rb") as f:
            data = f.read()
        if len(data) < len(MAGIC) + 8 or data[: len(MAGIC)] != MAGIC:
            raise ValueError(f"{path}: not a packed KIVI replica (bad magic)")
        (hlen,) = struct.unpack("<Q", data[len(MAGIC): len(MAGIC) + 8])
        if len(MAGIC) + 8 + hlen > len(data):
            raise ValueError(f"{path}: truncated header")
        try:
            header = json.loads(data[len(MAGIC) + 8: len(MAGIC) + 8 + hlen])
        except ValueError as exc:
            raise ValueError(f"{path}: unreadable header ({exc})") from None
        if header.get("version") != FORMAT_VERSION:
            raise ValueError(f"{path}: unsupported format version {header.get('version')}")
        start = _round_up(len(MAGIC) + 8 + hlen, 64)
        nbytes = int(header["blob_bytes"])
        if start + nbytes != len(data):
            raise ValueError(f"{path}: blob is {len(data) - start} bytes, header says {nbytes}")
        fields, meta = header["fields"], header["meta"]
        if set(fields) != set(_TENSOR_FIELDS) or set(meta) != set(_META_FIELDS):
            raise ValueError(f"{path}: header does not describe a packed KIVI cache")
        for name, spec in fields.items():
            if spec is None:
                continue
            if spec["dtype"] not in _DTYPES or spec["offset"] % ALIGN:
                raise ValueError(f"{path}: {name}: bad dtype or unaligned offset")
            size = _numel(spec["shape"]) * _DTYPES[spec["dtype"]].itemsize
            if spec["offset"] < 0 or spec["offset"] + size > nbytes:
                raise ValueError(f"{path}: {name} lies outside the blob")
        _check_shapes(fields, meta, path)
        blob = _pinned_empty(nbytes)
        blob.copy_(torch.frombuffer(bytearray(data[start:]), dtype=torch.uint8))
        return cls(blob=blob, fields=fields, meta=meta)


def _check_shapes(fields: dict, meta: dict, path) -> None:
    """The b200 layout invariants of PackedKIVICache (physical.py:204-227
    with the first two axes swapped)."""

    heads, d, t = int(meta["num_kv_heads"]), int(meta["head_dim"]), int(meta["quantized_tokens"])
    g, kb, vb = int(meta["group_size"]), int(meta["k_bits"]), int(meta["v_bits"])
    res = fields["residual_key"]
    if res is None or len(res["shape"]) != 3 or res["shape"][1:] != [heads, d]:
        raise ValueError(f"{path}: residual shape does not match the cache geometry")
    if fields["residual_value"] is None or fields["residual_value"]["shape"] != res["shape"]:
        raise ValueError(f"{path}: residual key/value shapes differ")
    if fields["logical_token_ids"] is None or _numel(fields["logical_token_ids"]["shape"]) != t + res["shape"][0]:
        raise ValueError(f"{path}: one logical id per token is required")
    if t == 0:
        return
    kwords = t if kb == 8 else t * kb // 32
    vwords = d if vb == 8 else d * vb // 32
    expect = {"key_code": [heads, kwords, d], "key_scale": [heads, t // g, d], "key_minimum": [heads, t // g, d],
              "value_code": [heads, t, vwords], "value_scale": [heads, t, d // g], "value_minimum": [heads, t, d // g]}
    for name, shape in expect.items():
        if fields[name] is None or fields[name]["shape"] != shape:
            raise ValueError(f"{path}: {name} shape {fields[name] and fields[name]['shape']} != {shape}")


def to_host(cache: PackedKIVICache) -> HostPackedKIVI:
    return HostPackedKIVI.from_cache(cache)


@dataclass(frozen=True)
class QuantizedWorkingSetTransition:
    """hierarchy.py:33-40 (same fields)."""

    resident_bytes: int
    h2d_bytes: int
    released_bytes: int
    resident_ratio: float
    transition_kind: str
    descriptor: tuple


@dataclass
class QuantizedHostArchive:
    """Full host KV plus packed host replicas, one GPU replica at a time.

    ``store(descriptor, replica)`` registers a host replica;
    ``materialize(descriptor=...)`` makes it the GPU-resident cache (one
    host-to-device copy when the descriptor changes, none on reuse) and
    returns ``(transition, cache)``.  The transition follows the reference's
    rule (hierarchy.py:70-125): the first materialisation is "initial" with no
    counted transfer, an unchanged descriptor is "reuse", a change is
    "upgrade"/"downgrade"/"repack" by resident bytes and counts the replica's
    bytes as H2D and the previous replica's as released.  ``summary()`` has
    the reference's keys plus ``copied_h2d_bytes`` (bytes really copied)."""

    full_archive_bytes: int
    _replicas: dict = field(default_factory=dict, init=False, repr=False)
    _current_descriptor: tuple | None = field(default=None, init=False, repr=False)
    _current_cache: PackedKIVICache | None = field(default=None, init=False, repr=False)
    _current_resident_bytes: int = field(default=0, init=False, repr=False)
    _resident_byte_invocations: int = field(default=0, init=False, repr=False)
    _archive_byte_invocations: int = field(default=0, init=False, repr=False)
    _peak_resident_ratio: float = field(default=0.0, init=False, repr=False)
    _materializations: int = field(default=0, init=False, repr=False)
    _precision_transitions: int = field(default=0, init=False, repr=False)
    _cumulative_h2d_bytes: int = field(default=0, init=False, repr=False)
    _cumulative_full_rebuild_h2d_bytes: int = field(default=0, init=False, repr=False)
    _cumulative_released_bytes: int = field(default=0, init=False, repr=False)
    _copied_h2d_bytes: int = field(default=0, init=False, repr=False)

    def __post_init__(self) -> None:
        if int(self.full_archive_bytes) <= 0:
            raise ValueError("full_archive_bytes must be positive")
        self.full_archive_bytes = int(self.full_archive_bytes)

    def store(self, descriptor: tuple, replica: HostPackedKIVI | PackedKIVICache) -> HostPackedKIVI:
        if isinstance(replica, PackedKIVICache):
            replica = HostPackedKIVI.from_cache(replica)
        self._replicas[tuple(descriptor)] = replica
        return replica

    @property
    def current_cache(self) -> PackedKIVICache | None:
        return self._current_cache

    def materialize(self, *, descriptor: tuple, device=None) -> tuple[QuantizedWorkingSetTransition, PackedKIVICache]:
        descriptor = tuple(descriptor)
        if descriptor not in self._replicas:
            raise KeyError(f"no host replica stored for descriptor {descriptor!r}")
        replica = self._replicas[descriptor]
        previous_descriptor = self._current_descriptor
        previous_bytes = self._current_resident_bytes
        changed = previous_descriptor != descriptor
        if changed or self._current_cache is None:
            cache = replica.to_device(device)
            self._copied_h2d_bytes += replica.nbytes
        else:
            cache = self._current_cache
        resident_bytes = int(cache.resident_bytes)
        if previous_descriptor is None:
            kind, h2d, released = "initial", 0, 0
        elif not changed:
            kind, h2d, released = "reuse", 0, 0
        else:
            kind = ("upgrade" if resident_bytes > previous_bytes else
                    "downgrade" if resident_bytes < previous_bytes else "repack")
            h2d, released = resident_bytes, previous_bytes
        if previous_descriptor is not None:
            self._cumulative_full_rebuild_h2d_bytes += resident_bytes
        if changed:
            self._precision_transitions += 1
        self._current_descriptor = descriptor
        self._current_cache = cache  # the previous GPU replica is released here
        self._current_resident_bytes = resident_bytes
        self._materializations += 1
        self._resident_byte_invocations += resident_bytes
        self._archive_byte_invocations += self.full_archive_bytes
        ratio = float(resident_bytes / self.full_archive_bytes)
        self._peak_resident_ratio = max(self._peak_resident_ratio, ratio)
        self._cumulative_h2d_bytes += h2d
        self._cumulative_released_bytes += released
        return QuantizedWorkingSetTransition(resident_bytes=resident_bytes, h2d_bytes=h2d, released_bytes=released,
                                             resident_ratio=ratio, transition_kind=kind, descriptor=descriptor), cache

    def summary(self) -> dict:
        """hierarchy.py:127-157 keys, plus ``copied_h2d_bytes``."""

        return {
            "archive_bytes": self.full_archive_bytes,
            "current_resident_bytes": self._current_resident_bytes,
            "resident_byte_invocations": self._resident_byte_invocations,
            "archive_byte_invocations": self._archive_byte_invocations,
            "average_resident_ratio": float(self._resident_byte_invocations / max(self._archive_byte_invocations, 1)),
            "peak_resident_ratio": self._peak_resident_ratio,
            "materializations": self._materializations,
            "precision_transitions": self._precision_transitions,
            "current_descriptor": [f"mask-bytes:{len(i)}" if isinstance(i, bytes) else i
                                   for i in (self._current_descriptor or ())],
            "host_replica_catalog_bytes": int(sum(r.resident_bytes for r in self._replicas.values())),
            "host_replica_variants": len(self._replicas),
            "cumulative_h2d_bytes": self._cumulative_h2d_bytes,
            "cumulative_full_rebuild_h2d_bytes": self._cumulative_full_rebuild_h2d_bytes,
            "cumulative_released_bytes": self._cumulative_released_bytes,
            "cumulative_logical_restored_tokens": 0,
            "cumulative_logical_evicted_tokens": 0,
            "cumulative_kv_head_restored_tokens": 0,
            "cumulative_kv_head_evicted_tokens": 0,
            "copied_h2d_bytes": self._copied_h2d_bytes,
        }

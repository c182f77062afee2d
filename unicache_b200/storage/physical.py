"""Physical cache layouts backed by the B200 kernels.

Drop-in counterparts of the reference's storage classes
(Superone77/UniCache, unicache/storage/physical.py): the same dataclass fields,
constructors, byte accounting and methods, with ``backend="b200"`` running on
the sm_100a kernels of ``libunicache_b200.so``.  ``backend="cuda"`` (the
reference's GPU default) is accepted as an alias of ``"b200"``.  The
reference's ``backend="reference"`` is its CPU torch path; this package ships
no CPU path and rejects it.

Packed KIVI layout "b200" (per layer, per sequence): the reference layout with
its first two axes swapped (head-major), int32 words identical:
    key_code  [H, T/fk, D] int32 (uint8 [H, T, D] at 8 bits)  scale/min [H, T/G, D]
    value_code [H, T, D/fv] int32 (uint8 [H, T, D] at 8 bits) scale/min [H, T, D/G]
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import torch

from .. import kernels

BACKENDS = ("b200", "cuda")
SUPPORTED_GROUPS = (32, 64, 128)
SUPPORTED_HEAD_DIMS = (64, 128)


def tensor_bytes(tensor: torch.Tensor | None) -> int:
    """physical.py:16-17."""

    return 0 if tensor is None else int(tensor.numel() * tensor.element_size())


def normalize_backend(backend: str) -> str:
    backend = str(backend)
    if backend == "reference":
        raise ValueError(
            "backend='reference' is the reference's CPU torch path; unicache_b200 runs on B200 "
            "kernels only (backend='b200')"
        )
    if backend not in BACKENDS:
        raise ValueError(f"Unknown KIVI physical backend: {backend}")
    return "b200"


def gqa_query_key_logits(query: torch.Tensor, key: torch.Tensor) -> torch.Tensor:
    """physical.py:20-39 (generic, non-fused path): [Lq, Hq, D] x [N, Hkv, D] -> [Hq, Lq, N] fp32."""

    if query.dim() != 3 or key.dim() != 3:
        raise ValueError("GQA QK expects [tokens, heads, head_dim] tensors")
    if int(query.shape[-1]) != int(key.shape[-1]):
        raise ValueError("GQA QK query/key head dimensions must match")
    hq, hkv = int(query.shape[1]), int(key.shape[1])
    if hq % hkv:
        raise ValueError("GQA query heads must be divisible by KV heads")
    groups = hq // hkv
    q = query.transpose(0, 1).reshape(hkv, groups, int(query.shape[0]), int(query.shape[-1]))
    k = key.transpose(0, 1).unsqueeze(1)
    return torch.matmul(q.float(), k.float().transpose(-1, -2)).reshape(hq, int(query.shape[0]), int(key.shape[0]))


def gqa_probability_value(probabilities: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
    """physical.py:42-63 (generic, non-fused path)."""

    if probabilities.dim() != 3 or value.dim() != 3:
        raise ValueError("GQA AV expects probabilities [heads, queries, keys] and values [keys, heads, dim]")
    hq, hkv = int(probabilities.shape[0]), int(value.shape[1])
    if hq % hkv:
        raise ValueError("GQA probability heads must be divisible by KV heads")
    if int(probabilities.shape[-1]) != int(value.shape[0]):
        raise ValueError("GQA AV probability key width must match value tokens")
    groups = hq // hkv
    p = probabilities.reshape(hkv, groups, int(probabilities.shape[1]), int(probabilities.shape[2]))
    v = value.transpose(0, 1).unsqueeze(1)
    return torch.matmul(p.to(value.dtype), v).reshape(hq, int(probabilities.shape[1]), int(value.shape[-1]))


@dataclass
class PackedKIVICache:
    """A KIVI-style packed KV segment with a full-precision residual suffix
    (physical.py:204-227)."""

    key_code: torch.Tensor | None
    key_scale: torch.Tensor | None
    key_minimum: torch.Tensor | None
    value_code: torch.Tensor | None
    value_scale: torch.Tensor | None
    value_minimum: torch.Tensor | None
    residual_key: torch.Tensor
    residual_value: torch.Tensor
    logical_token_ids: torch.Tensor
    token_type_id: int
    k_bits: int
    v_bits: int
    group_size: int
    quantized_tokens: int
    head_dim: int
    num_kv_heads: int
    backend: str = "b200"
    kernel_native_layout: bool = True
    budget_shortfall_events: int = 0
    residual_length: int = 0  # requested full-precision window (streaming append keeps it)

    @classmethod
    def from_dense(
        cls,
        key: torch.Tensor,
        value: torch.Tensor,
        *,
        logical_token_ids: torch.Tensor,
        token_type_id: int,
        k_bits: int,
        v_bits: int,
        group_size: int,
        residual_length: int,
        backend: str = "b200",
        _packed=None,
    ) -> "PackedKIVICache":
        """physical.py:228-332: split ``((T - R) // G) * G`` quantized tokens
        from a full-precision suffix and pack them on the GPU."""

        if key.shape != value.shape or key.dim() != 3:
            raise ValueError("KIVI physical cache expects matching [tokens, kv_heads, head_dim] tensors")
        if k_bits not in {2, 4, 8} or v_bits not in {2, 4, 8}:
            raise ValueError("KIVI physical cache supports 2, 4, or 8 bit payloads")
        tokens, heads, head_dim = map(int, key.shape)
        if group_size <= 0:
            raise ValueError("KIVI physical cache group_size must be positive")
        backend = normalize_backend(backend)
        kernels.require_cuda(key, "key")
        kernels.require_cuda(value, "value")
        if group_size not in SUPPORTED_GROUPS:
            raise ValueError(f"The b200 KIVI kernels support group_size {SUPPORTED_GROUPS}")
        if head_dim not in SUPPORTED_HEAD_DIMS or head_dim % group_size:
            raise ValueError("The b200 KIVI kernels require head_dim 64/128 divisible by group_size")
        requested_residual = min(tokens, max(0, int(residual_length)))
        quantized = ((tokens - requested_residual) // group_size) * group_size
        packed = None
        if quantized:
            q_key = key[:quantized]
            q_value = value[:quantized]
            if q_key.stride(2) != 1:
                q_key = q_key.contiguous()
            if q_value.stride(2) != 1:
                q_value = q_value.contiguous()
            if _packed is not None:
                packed = _packed(q_key, q_value)
            else:
                packed = kernels.kivi_pack_kv(q_key, q_value, k_bits=k_bits, v_bits=v_bits, group_size=group_size)
        return cls._assemble(key, value, packed, quantized, logical_token_ids, token_type_id, k_bits, v_bits,
                             group_size, head_dim, heads, backend, residual_length)

    @classmethod
    def from_dense_batch(cls, keys: list, values: list, *, logical_token_ids: list, token_type_id: int, k_bits: int,
                         v_bits: int, group_size: int, residual_length: int,
                         backend: str = "b200") -> list["PackedKIVICache"]:
        """``from_dense`` of several segments with one pack launch for all of
        them (group 32 and aligned rows; other shapes pack segment by segment):
        a batch prefill or all layers of one sequence at once."""

        if not (len(keys) == len(values) == len(logical_token_ids)) or not keys:
            raise ValueError("from_dense_batch needs matching, non-empty key/value/id lists")
        pending: list = []

        def defer(q_key, q_value):
            pending.append((q_key, q_value))
            return len(pending) - 1

        caches = [cls.from_dense(k, v, logical_token_ids=ids, token_type_id=token_type_id, k_bits=k_bits,
                                 v_bits=v_bits, group_size=group_size, residual_length=residual_length,
                                 backend=backend, _packed=defer)
                  for k, v, ids in zip(keys, values, logical_token_ids)]
        if pending:
            outputs = kernels.kivi_pack_kv_batch(pending, k_bits=k_bits, v_bits=v_bits, group_size=group_size)
            for cache in caches:
                if cache.quantized_tokens:
                    slot = cache.__dict__.pop("_pending_pack")
                    (cache.key_code, cache.key_scale, cache.key_minimum, cache.value_code, cache.value_scale,
                     cache.value_minimum) = outputs[slot]
        return caches

    @classmethod
    def _assemble(cls, key, value, packed, quantized, logical_token_ids, token_type_id, k_bits, v_bits, group_size,
                  head_dim, heads, backend, residual_length) -> "PackedKIVICache":
        if isinstance(packed, tuple):
            key_code, key_scale, key_minimum, value_code, value_scale, value_minimum = packed
        else:  # not packed yet (from_dense_batch fills these in) or nothing to pack
            key_code = key_scale = key_minimum = value_code = value_scale = value_minimum = None
        cache = cls(
            key_code=key_code,
            key_scale=key_scale,
            key_minimum=key_minimum,
            value_code=value_code,
            value_scale=value_scale,
            value_minimum=value_minimum,
            residual_key=key[quantized:].clone(),
            residual_value=value[quantized:].clone(),
            logical_token_ids=logical_token_ids.detach().clone(),
            token_type_id=int(token_type_id),
            k_bits=int(k_bits),
            v_bits=int(v_bits),
            group_size=int(group_size),
            quantized_tokens=quantized,
            head_dim=head_dim,
            num_kv_heads=heads,
            backend=backend,
            kernel_native_layout=True,
            residual_length=max(0, int(residual_length)),
        )
        if isinstance(packed, int):
            cache.__dict__["_pending_pack"] = packed
        return cache

    # ---------------------------------------------------------------- streaming append
    def append(self, key: torch.Tensor, value: torch.Tensor, *, logical_token_ids: torch.Tensor) -> int:
        """Append decoded tokens [n, H, D] at the end of the segment.

        The full-precision residual keeps between ``residual_length`` and
        ``residual_length + group_size - 1`` tokens; every whole group that
        leaves it is quantized and packed on the GPU and appended to the packed
        tensors, oldest first, so the cache stays equal, bit for bit, to
        ``from_dense`` over the whole sequence with the same residual length.
        Returns the number of tokens packed.  Flushed groups are written in
        place into capacity stores that double when full (the packed tensors
        are views of them), so a flush moves only the new groups.  Decode
        plans built on this cache must be rebuilt after an append (token
        counts change; the cache drops the plans it cached itself)."""

        if key.shape != value.shape or key.dim() != 3 or tuple(key.shape[1:]) != (self.num_kv_heads, self.head_dim):
            raise ValueError("appended key/value must be [tokens, kv_heads, head_dim] matching the cache")
        if key.dtype != self.residual_key.dtype or value.dtype != self.residual_value.dtype:
            raise ValueError("appended key/value must have the residual's dtype")
        n = int(key.shape[0])
        if int(logical_token_ids.numel()) != n:
            raise ValueError("one logical token id per appended token is required")
        kernels.require_cuda(key, "key")
        kernels.require_cuda(value, "value")
        total = self.token_count + n
        target = max(0, (total - self.residual_length) // self.group_size * self.group_size)
        flush = target - self.quantized_tokens
        # the residual window holds fewer than residual_length + group_size rows: small copies
        res_key = torch.cat([self.residual_key, key], dim=0)
        res_value = torch.cat([self.residual_value, value], dim=0)
        if flush > 0:
            new = kernels.kivi_pack_kv(res_key[:flush].contiguous(), res_value[:flush].contiguous(),
                                       k_bits=self.k_bits, v_bits=self.v_bits, group_size=self.group_size)
            self._write_packed(new, self.quantized_tokens, target)
            self.quantized_tokens = target
            res_key = res_key[flush:].clone()
            res_value = res_value[flush:].clone()
        self.residual_key, self.residual_value = res_key, res_value
        self._append_ids(logical_token_ids.to(self.logical_token_ids.device, self.logical_token_ids.dtype))
        self.__dict__.pop("_decode_plans", None)
        return max(0, flush)

    _PACKED = ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum")

    def _units(self, name: str, tokens: int) -> int:
        """Length along dim 1 (b200 layout) of ``name`` holding ``tokens`` tokens."""

        if name == "key_code":
            return tokens if self.k_bits == 8 else tokens // (32 // self.k_bits)
        if name in ("key_scale", "key_minimum"):
            return tokens // self.group_size
        return tokens  # value codes and statistics run per token

    def _write_packed(self, new: tuple, start: int, stop: int) -> None:
        """Store freshly packed tokens [start, stop) in place.  The packed
        tensors are views of capacity stores that grow geometrically, so a
        flush copies only the new groups (and, rarely, the store once when it
        doubles) instead of concatenating the whole cache."""

        store = self.__dict__.get("_store")
        capacity = self.__dict__.get("_capacity", 0)
        if store is None or stop > capacity:
            grown = max(stop, 2 * capacity, 4 * self.group_size)
            grown = -(-grown // self.group_size) * self.group_size
            fresh = {}
            for name, tensor in zip(self._PACKED, new):
                shape = list(tensor.shape)
                shape[1] = self._units(name, grown)
                fresh[name] = torch.empty(shape, device=tensor.device, dtype=tensor.dtype)
                old = getattr(self, name)
                if old is not None and start:
                    fresh[name][:, :self._units(name, start)].copy_(old)
            self.__dict__["_store"], self.__dict__["_capacity"] = fresh, grown
            store = fresh
        for name, tensor in zip(self._PACKED, new):
            a, b = self._units(name, start), self._units(name, stop)
            store[name][:, a:b].copy_(tensor)
            setattr(self, name, store[name][:, :b])

    def _append_ids(self, ids: torch.Tensor) -> None:
        store = self.__dict__.get("_id_store")
        used = int(self.logical_token_ids.numel())
        need = used + int(ids.numel())
        if store is None or need > int(store.numel()):
            grown = torch.empty(max(need, 2 * used, 64), device=ids.device, dtype=self.logical_token_ids.dtype)
            grown[:used].copy_(self.logical_token_ids)
            self.__dict__["_id_store"] = store = grown
        store[used:need].copy_(ids)
        self.logical_token_ids = store[:need]

    def to_host(self):
        """A contiguous host replica of this cache (``storage.hierarchy``)."""

        from .hierarchy import HostPackedKIVI

        return HostPackedKIVI.from_cache(self)

    # ---------------------------------------------------------------- accounting
    @property
    def token_count(self) -> int:
        return int(self.logical_token_ids.numel())

    @property
    def resident_bytes(self) -> int:
        tensors = (
            self.key_code, self.key_scale, self.key_minimum, self.value_code, self.value_scale,
            self.value_minimum, self.residual_key, self.residual_value, self.logical_token_ids,
        )
        return sum(tensor_bytes(item) for item in tensors)

    @property
    def byte_breakdown(self) -> dict[str, int]:
        return {
            "payload_bytes": tensor_bytes(self.key_code) + tensor_bytes(self.value_code),
            "scale_bytes": tensor_bytes(self.key_scale) + tensor_bytes(self.value_scale),
            "minimum_bytes": tensor_bytes(self.key_minimum) + tensor_bytes(self.value_minimum),
            "residual_bytes": tensor_bytes(self.residual_key) + tensor_bytes(self.residual_value),
            "indices_bytes": tensor_bytes(self.logical_token_ids),
            "score_bytes": 0,
        }

    @property
    def full_precision_bytes(self) -> int:
        element_size = int(self.residual_key.element_size())
        return self.token_count * self.num_kv_heads * self.head_dim * 2 * element_size

    def reference_layout(self) -> dict[str, torch.Tensor | None]:
        """The packed tensors in the reference's CPU layout (physical.py:291-304):
        K codes [T/f, H, D], K stats [T/G, H, D], V codes [T, H, D/f], V stats [T, H, D/G]."""

        names = ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum")
        return {
            name: (None if getattr(self, name) is None else getattr(self, name).transpose(0, 1))
            for name in names
        }

    # ---------------------------------------------------------------- dequantize
    def dequantize_range(self, start: int, stop: int, *, dtype: torch.dtype, output_key: torch.Tensor,
                         output_value: torch.Tensor) -> None:
        """Write quantized tokens [start, stop) into the given [N, H, D] views."""

        # appended caches keep their packed tensors in capacity stores: the
        # per-head extent the kernels step over is the store's capacity
        extent = self.__dict__.get("_capacity", self.quantized_tokens) if "_store" in self.__dict__ \
            else self.quantized_tokens
        if not 0 <= start <= stop <= self.quantized_tokens:
            raise ValueError("dequantize range outside the quantized tokens")
        common = dict(bits=0, group_size=self.group_size, quantized_tokens=extent,
                      heads=self.num_kv_heads, head_dim=self.head_dim, start=start, stop=stop)
        common["bits"] = self.k_bits
        kernels.kivi_dequant("key", self.key_code, self.key_scale, self.key_minimum, out=output_key, **common)
        common["bits"] = self.v_bits
        kernels.kivi_dequant("value", self.value_code, self.value_scale, self.value_minimum, out=output_value,
                             **common)

    def dequantize(self, dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """physical.py:379-423, bit-exact: round(fp32(code*scale) + minimum)."""

        dtype = dtype or self.residual_key.dtype
        total = self.quantized_tokens + int(self.residual_key.shape[0])
        device = self.residual_key.device
        key = torch.empty((total, self.num_kv_heads, self.head_dim), device=device, dtype=dtype)
        value = torch.empty_like(key)
        if self.quantized_tokens:
            self.dequantize_range(0, self.quantized_tokens, dtype=dtype, output_key=key, output_value=value)
        key[self.quantized_tokens:] = self.residual_key.to(dtype)
        value[self.quantized_tokens:] = self.residual_value.to(dtype)
        return key, value

    def repack_monotonic(self, *, bits: int, group_size: int | None = None) -> bool:
        """physical.py:425-450: lower precision; never raise it back."""

        target_bits = int(bits)
        target_group = int(group_size or self.group_size)
        if target_bits > self.k_bits or target_bits > self.v_bits or target_group < self.group_size:
            self.budget_shortfall_events += 1
            return False
        if target_bits == self.k_bits and target_bits == self.v_bits and target_group == self.group_size:
            return True
        key, value = self.dequantize(dtype=self.residual_key.dtype)
        replacement = PackedKIVICache.from_dense(
            key,
            value,
            logical_token_ids=self.logical_token_ids,
            token_type_id=self.token_type_id,
            k_bits=target_bits,
            v_bits=target_bits,
            group_size=target_group,
            residual_length=int(self.residual_key.shape[0]),
            backend=self.backend,
        )
        shortfalls = self.budget_shortfall_events
        self.__dict__.pop("_decode_plans", None)
        self.__dict__.update(replacement.__dict__)
        self.budget_shortfall_events = shortfalls
        return True

    # ---------------------------------------------------------------- attention
    def attention_parts(self, query: torch.Tensor) -> tuple[torch.Tensor, Callable[[torch.Tensor], torch.Tensor]]:
        """physical.py:452-475 / kivi_cuda.py:238-329: logits [Hq, Lq, T+R]
        scaled by 1/sqrt(D) and a closure applying probabilities to the values."""

        from .kivi_b200 import packed_kivi_attention_parts

        return packed_kivi_attention_parts(self, query)


@dataclass
class GQAH2OCache:
    """Per-KV-head physical H2O cache with fixed-width selected storage
    (physical.py:478-492)."""

    key: torch.Tensor  # [kv_heads, retained_tokens, head_dim]
    value: torch.Tensor
    logical_token_ids: torch.Tensor  # [kv_heads, retained_tokens]
    cumulative_scores: torch.Tensor
    token_type_id: int
    original_tokens: int
    heavy_tokens: int
    recent_tokens: int
    selection_frozen: bool = False
    budget_shortfall_tokens: int = 0

    @classmethod
    def from_dense(
        cls,
        key: torch.Tensor,
        value: torch.Tensor,
        *,
        logical_token_ids: torch.Tensor,
        token_type_id: int,
        per_kv_head_scores: torch.Tensor,
        target_tokens: int,
        recent_tokens: int,
        selection_frozen: bool = False,
    ) -> "GQAH2OCache":
        """physical.py:493-547 on the GPU: heavy top-k per KV head over the
        history (ties -> lower index), ascending, then the recent window."""

        if key.shape != value.shape or key.dim() != 3:
            raise ValueError("Physical H2O expects matching [tokens, kv_heads, head_dim] tensors")
        tokens, kv_heads, head_dim = map(int, key.shape)
        if tuple(per_kv_head_scores.shape) != (kv_heads, tokens):
            raise ValueError("Physical H2O scores must be [kv_heads, segment_tokens]")
        kernels.require_cuda(key, "key")
        target = min(tokens, max(1, int(target_tokens)))
        recent = min(target, max(0, int(recent_tokens)))
        heavy = target - recent
        history_end = tokens - recent
        heavy_k = min(heavy, history_end)
        scores = per_kv_head_scores.to(device=key.device, dtype=torch.float32).contiguous()
        index = kernels.h2o_select(scores, history_end=history_end, heavy_k=heavy_k, recent=recent)
        keep = heavy_k + recent
        out_key = torch.empty((kv_heads, keep, head_dim), device=key.device, dtype=key.dtype)
        out_value = torch.empty_like(out_key)
        kernels.gather_rows(key, index, head_stride=key.stride(1), token_stride=key.stride(0),
                            row_elems=head_dim, out=out_key)
        kernels.gather_rows(value, index, head_stride=value.stride(1), token_stride=value.stride(0),
                            row_elems=head_dim, out=out_value)
        ids = logical_token_ids.to(device=key.device, dtype=torch.int64).contiguous()
        out_ids = torch.empty((kv_heads, keep), device=key.device, dtype=torch.int64)
        kernels.gather_rows(ids, index, head_stride=0, token_stride=1, row_elems=1, out=out_ids)
        out_scores = torch.empty((kv_heads, keep), device=key.device, dtype=torch.float32)
        kernels.gather_rows(scores, index, head_stride=scores.stride(0), token_stride=1, row_elems=1,
                            out=out_scores)
        return cls(
            key=out_key,
            value=out_value,
            logical_token_ids=out_ids,
            cumulative_scores=out_scores,
            token_type_id=int(token_type_id),
            original_tokens=tokens,
            heavy_tokens=heavy,
            recent_tokens=recent,
            selection_frozen=bool(selection_frozen),
        )

    @property
    def num_kv_heads(self) -> int:
        return int(self.key.shape[0])

    @property
    def retained_tokens(self) -> int:
        return int(self.key.shape[1])

    @property
    def resident_bytes(self) -> int:
        return sum(
            tensor_bytes(item) for item in (self.key, self.value, self.logical_token_ids, self.cumulative_scores)
        )

    @property
    def byte_breakdown(self) -> dict[str, int]:
        return {
            "payload_bytes": tensor_bytes(self.key) + tensor_bytes(self.value),
            "scale_bytes": 0,
            "minimum_bytes": 0,
            "residual_bytes": 0,
            "indices_bytes": tensor_bytes(self.logical_token_ids),
            "score_bytes": tensor_bytes(self.cumulative_scores),
        }

    @property
    def full_precision_bytes(self) -> int:
        return self.original_tokens * self.num_kv_heads * int(self.key.shape[-1]) * 2 * self.key.element_size()

    def attention_parts(self, query: torch.Tensor) -> tuple[torch.Tensor, Callable[[torch.Tensor], torch.Tensor]]:
        """physical.py:585-596 (generic path; the fused decode path reads the
        compacted rows directly without this)."""

        key = self.key.transpose(0, 1)
        value = self.value.transpose(0, 1)
        logits = gqa_query_key_logits(query, key) / math.sqrt(query.shape[-1])

        def apply_value(probabilities: torch.Tensor) -> torch.Tensor:
            return gqa_probability_value(probabilities, value)

        return logits, apply_value

    def update_scores(self, probabilities: torch.Tensor) -> None:
        """physical.py:598-610: add per-KV-head received attention."""

        if probabilities.dim() != 3:
            raise ValueError("H2O probabilities must be [query_heads, queries, tokens]")
        if int(probabilities.shape[0]) % self.num_kv_heads != 0:
            raise ValueError("Query heads must be divisible by KV heads for GQA H2O")
        scores = self.cumulative_scores.clone()
        kernels.accumulate_probs(probabilities, self.num_kv_heads, scores)
        self.cumulative_scores = scores

    def update_scores_from_lse(self, query: torch.Tensor, lse: torch.Tensor,
                               softmax_scale: float | None = None) -> None:
        """``update_scores`` without the [Hq, Lq, T] probabilities: each
        probability of the retained rows is recomputed on the tensor cores from
        the query [Lq, Hq, D] and the attention's natural-log LSE [Hq, Lq]
        (the decode and long-query kernels return it), and the per-KV-head sums
        are added to ``cumulative_scores``."""

        scale = (1.0 / math.sqrt(int(query.shape[-1]))) if softmax_scale is None else float(softmax_scale)
        scores = self.cumulative_scores.float().contiguous().clone()
        kernels.h2o_scores(query.to(self.key.dtype), self.key, lse, kv_heads=self.num_kv_heads, softmax_scale=scale,
                           scores=scores, head_major=True)
        self.cumulative_scores = scores

    def enforce_budget(self) -> None:
        self.trim(self.heavy_tokens + self.recent_tokens, self.recent_tokens)

    def request_budget(self, target_tokens: int, recent_tokens: int) -> int:
        """physical.py:615-622."""

        requested = max(1, int(target_tokens))
        effective = min(requested, self.retained_tokens)
        self.budget_shortfall_tokens += requested - effective
        self.recent_tokens = min(effective, max(0, int(recent_tokens)))
        self.heavy_tokens = effective - self.recent_tokens
        self.enforce_budget()
        return effective

    def trim(self, target_tokens: int, recent_tokens: int) -> None:
        """physical.py:624-654, every head in one launch."""

        retained = self.retained_tokens
        target = min(retained, max(1, int(target_tokens)))
        if target >= retained:
            return
        recent = min(target, max(0, int(recent_tokens)))
        heavy = target - recent
        history_end = retained - recent
        heavy_k = min(heavy, history_end)
        scores = self.cumulative_scores.float().contiguous()
        index = kernels.h2o_select(scores, history_end=history_end, heavy_k=heavy_k, recent=recent)
        keep = heavy_k + recent
        heads, head_dim = self.num_kv_heads, int(self.key.shape[-1])
        key = torch.empty((heads, keep, head_dim), device=self.key.device, dtype=self.key.dtype)
        value = torch.empty_like(key)
        kernels.gather_rows(self.key, index, head_stride=self.key.stride(0), token_stride=self.key.stride(1),
                            row_elems=head_dim, out=key)
        kernels.gather_rows(self.value, index, head_stride=self.value.stride(0), token_stride=self.value.stride(1),
                            row_elems=head_dim, out=value)
        ids = torch.empty((heads, keep), device=self.key.device, dtype=torch.int64)
        kernels.gather_rows(self.logical_token_ids.contiguous(), index, head_stride=retained, token_stride=1,
                            row_elems=1, out=ids)
        kept = torch.empty((heads, keep), device=self.key.device, dtype=torch.float32)
        kernels.gather_rows(scores, index, head_stride=retained, token_stride=1, row_elems=1, out=kept)
        self.key, self.value, self.logical_token_ids, self.cumulative_scores = key, value, ids, kept


PhysicalSegment = PackedKIVICache | GQAH2OCache


@dataclass
class PhysicalLayerCache:
    """physical.py:660-673."""

    segments: list[PhysicalSegment]

    @property
    def resident_bytes(self) -> int:
        return sum(segment.resident_bytes for segment in self.segments)

    @property
    def full_precision_bytes(self) -> int:
        return sum(segment.full_precision_bytes for segment in self.segments)

    def add(self, segment: PhysicalSegment) -> None:
        self.segments.append(segment)

"""The two physical-cache operators of the plugin API, on the B200 path.

Same names, parameters, validation, capabilities and request contents as the
reference's operators (Superone77/UniCache, unicache/operators/physical.py),
derived from the plugin contract's ``ProcessingOperator``, so a plan that
names ``h2o_physical_gqa`` or ``kivi_packed_quantization`` runs unchanged and
the reference's ``KVRegistry`` accepts them.  Devices are ``cuda`` only: the
B200 path has no CPU implementation.  ``execute`` / ``update_after_attention`` take the reference's
``OperatorExecutionContext`` (any object with its attributes: ``params``,
``k``, ``segment_mask``, ``step.segment_id``, ``runtime.kv_metadata``,
``storage_num_kv_heads``, ``record``, ``physical_request``).
"""

from __future__ import annotations

import torch

from .. import kernels
from ..core.decisions import PhysicalCacheRequest
from ..core.plugin import CapabilityDescriptor, ProcessingOperator


class H2OPhysicalGQAOperator(ProcessingOperator):
    """H2O real-drop semantics on GQA storage (physical.py:14-101)."""

    name = "h2o_physical_gqa"
    family = "eviction"
    stages = {"attention"}
    executable = True
    uses_final_attention = True
    preserves_attention_dispatch = False
    capabilities = CapabilityDescriptor(
        stages=frozenset(stages),
        layouts=frozenset({"attention_view", "dense"}),
        devices=frozenset({"cuda"}),
        requires=frozenset({"query", "key", "value", "segment_mask", "cache_storage_view"}),
        produces_selection=True,
        stateful=True,
        mutation_scope="persistent_cache",
        physical_storage_mutation=True,
    )

    def build_params(self, params: dict) -> dict:
        out = dict(params)
        ratio = float(out.get("target_budget_ratio", 0.2))
        if not 0.0 < ratio <= 1.0:
            raise ValueError("h2o_physical_gqa target_budget_ratio must be in (0, 1]")
        recent_fraction = float(out.get("recent_budget_fraction", 0.25))
        if not 0.0 <= recent_fraction <= 1.0:
            raise ValueError("h2o_physical_gqa recent_budget_fraction must be in [0, 1]")
        out["target_budget_ratio"] = ratio
        out["recent_budget_fraction"] = recent_fraction
        out["selection_frozen"] = bool(out.get("selection_frozen", False))
        return out

    def execute(self, ctx):
        return ctx

    def update_after_attention(self, ctx, attention_probs: torch.Tensor):
        """Reduce [Hq, Lq, T] probabilities to per-KV-head scores on the GPU
        (physical.py:63-65) and queue a physical request (:66-101)."""

        if ctx.storage_num_kv_heads is None:
            raise RuntimeError("Physical H2O requires native KV-head metadata")
        kv_heads = int(ctx.storage_num_kv_heads)
        query_heads = int(attention_probs.shape[0])
        if query_heads % kv_heads != 0:
            raise ValueError("BAGEL query heads must be divisible by KV heads")
        return self._request(ctx, kernels.accumulate_probs(attention_probs, kv_heads), query_heads, kv_heads)

    def update_after_attention_lse(self, ctx, query: torch.Tensor, lse: torch.Tensor | None,
                                   softmax_scale: float | None = None):
        """``update_after_attention`` without materialised probabilities: the
        per-KV-head received attention of the dense keys ``ctx.k`` [T, Hkv, D]
        is recomputed on the tensor cores from ``query`` [Lq, Hq, D] and the
        attention's natural-log LSE [Hq, Lq] (None: the attention covered
        exactly ``ctx.k``), then the same physical request is queued."""

        if ctx.storage_num_kv_heads is None:
            raise RuntimeError("Physical H2O requires native KV-head metadata")
        kv_heads = int(ctx.storage_num_kv_heads)
        query_heads = int(query.shape[1])
        if query_heads % kv_heads != 0:
            raise ValueError("BAGEL query heads must be divisible by KV heads")
        scale = (1.0 / float(int(query.shape[-1])) ** 0.5) if softmax_scale is None else float(softmax_scale)
        scores = kernels.h2o_scores(query.to(ctx.k.dtype), ctx.k, lse, kv_heads=kv_heads, softmax_scale=scale)
        return self._request(ctx, scores, query_heads, kv_heads)

    def _request(self, ctx, per_kv_head_scores: torch.Tensor, query_heads: int, kv_heads: int):
        """Queue the physical request and record the budget (physical.py:66-101)."""

        groups = query_heads // kv_heads
        ctx.physical_request = PhysicalCacheRequest(
            operator=self.name,
            segment_id=ctx.step.segment_id,
            token_count=int(ctx.k.shape[0]),
            segment_mask=ctx.segment_mask.detach(),
            params=dict(ctx.params),
            per_kv_head_scores=per_kv_head_scores.detach(),
            metadata={
                "query_heads": query_heads,
                "kv_heads": kv_heads,
                "gqa_groups": groups,
                "observation": "full_kv_first_call",
                "token_type_id": ctx.runtime.kv_metadata.get("current_segment_type_id"),
                "token_span": ctx.runtime.kv_metadata.get("current_segment_span"),
            },
        )
        segment_tokens = ctx.runtime.kv_metadata.get("current_segment_tokens")
        if segment_tokens is None:
            segment_tokens = int(ctx.segment_mask.sum().item())
        segment_tokens = int(segment_tokens)
        requested = ctx.params.get("budget", ctx.params.get("keep_k"))
        if requested is None:
            requested = max(1, int(round(segment_tokens * float(ctx.params["target_budget_ratio"]))))
        ctx.record(
            {
                "physical_h2o_requests": 1,
                "physical_h2o_source_tokens": segment_tokens,
                "physical_h2o_target_tokens_per_kv_head": int(requested),
            }
        )
        return ctx


class KIVIPackedQuantizationOperator(ProcessingOperator):
    """Move a typed dense segment into KIVI packed physical storage
    (physical.py:104-178)."""

    name = "kivi_packed_quantization"
    family = "quantization"
    stages = {"pre_attention"}
    executable = True
    uses_final_attention = False
    preserves_attention_dispatch = False
    capabilities = CapabilityDescriptor(
        stages=frozenset(stages),
        layouts=frozenset({"attention_view", "dense"}),
        devices=frozenset({"cuda"}),
        requires=frozenset({"key", "value", "segment_mask", "cache_storage_view"}),
        mutation_scope="persistent_cache",
        physical_storage_mutation=True,
        accepts_quantized_input=False,
    )

    def build_params(self, params: dict) -> dict:
        out = dict(params)
        bits = int(out.get("bits", 4))
        k_bits = int(out.get("k_bits", bits))
        v_bits = int(out.get("v_bits", bits))
        if k_bits not in {2, 4, 8} or v_bits not in {2, 4, 8}:
            raise ValueError("kivi_packed_quantization supports 2, 4, or 8 bits")
        group_size = int(out.get("group_size", 64))
        if group_size <= 0:
            raise ValueError("kivi_packed_quantization group_size must be positive")
        backend = str(out.get("backend", "b200"))
        if backend not in {"b200", "cuda"}:
            raise ValueError("kivi_packed_quantization backend must be b200 (or its alias cuda)")
        out.update(
            {
                "bits": bits,
                "k_bits": k_bits,
                "v_bits": v_bits,
                "group_size": group_size,
                "residual_length": max(0, int(out.get("residual_length", 32))),
                "backend": "b200",
            }
        )
        return out

    def execute(self, ctx):
        if ctx.k.device.type != "cuda":
            raise RuntimeError("Physical KIVI backend=b200 cannot fall back to fake quantization or CPU")
        segment_tokens = ctx.runtime.kv_metadata.get("current_segment_tokens")
        if segment_tokens is None:
            segment_tokens = int(ctx.segment_mask.sum().item())
        segment_tokens = int(segment_tokens)
        ctx.physical_request = PhysicalCacheRequest(
            operator=self.name,
            segment_id=ctx.step.segment_id,
            token_count=int(ctx.k.shape[0]),
            segment_mask=ctx.segment_mask.detach(),
            params=dict(ctx.params),
            metadata={
                "observation": "dense_prefill_cache",
                "token_type_id": ctx.runtime.kv_metadata.get("current_segment_type_id"),
                "token_span": ctx.runtime.kv_metadata.get("current_segment_span"),
            },
        )
        quantized = max(0, segment_tokens - int(ctx.params["residual_length"]))
        ctx.record(
            {
                "physical_kivi_requests": 1,
                "physical_kivi_source_tokens": segment_tokens,
                "physical_kivi_quantized_tokens": quantized,
                "physical_kivi_bits": int(ctx.params["bits"]),
            }
        )
        return ctx


def kivi_fake_quant_key(k_segment: torch.Tensor, *, bits: int, group_size: int) -> torch.Tensor:
    """unicache/operators/builtin.py:56-59 on the GPU: keys grouped along tokens."""

    return kernels.fake_quant(k_segment, bits=bits, dim=0, group_size=group_size)


def kivi_fake_quant_value(v_segment: torch.Tensor, *, bits: int, group_size: int) -> torch.Tensor:
    """unicache/operators/builtin.py:62-65 on the GPU: values grouped along head_dim."""

    return kernels.fake_quant(v_segment, bits=bits, dim=-1, group_size=group_size)


def asymmetric_fake_quant(data: torch.Tensor, *, bits: int, dim: int, group_size: int) -> torch.Tensor:
    """unicache/operators/builtin.py:31-53 on the GPU."""

    return kernels.fake_quant(data, bits=bits, dim=dim, group_size=group_size)

"""Physical storage layouts and their B200 kernels (counterpart of unicache/storage)."""

from .hierarchy import HostPackedKIVI, QuantizedHostArchive, QuantizedWorkingSetTransition, to_host
from .kivi_b200 import (
    dequantize_kivi_chunk,
    packed_kivi_attention_parts,
    packed_kivi_quantized_attention_summary,
    quantize_kivi_b200,
)
from .physical import (
    GQAH2OCache,
    PackedKIVICache,
    PhysicalLayerCache,
    PhysicalSegment,
    gqa_probability_value,
    gqa_query_key_logits,
    tensor_bytes,
)
from .tensor_backend import CacheMutationResult, TensorCacheStorageBackend

__all__ = [
    "CacheMutationResult",
    "GQAH2OCache",
    "HostPackedKIVI",
    "QuantizedHostArchive",
    "QuantizedWorkingSetTransition",
    "PackedKIVICache",
    "PhysicalLayerCache",
    "PhysicalSegment",
    "TensorCacheStorageBackend",
    "dequantize_kivi_chunk",
    "gqa_probability_value",
    "gqa_query_key_logits",
    "packed_kivi_attention_parts",
    "packed_kivi_quantized_attention_summary",
    "quantize_kivi_b200",
    "tensor_bytes",
    "to_host",
]

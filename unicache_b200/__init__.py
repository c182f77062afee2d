"""unicache_b200: the UniCache physical-engine hot path on NVIDIA B200 (sm_100a).

KIVI quantize/pack and dequantize, packed-KV decode attention, H2O scoring,
selection and compaction, LSE merging and dense-cache compaction, as
hand-written CUDA kernels behind a C ABI (include/unicache_b200.h), with the
reference's storage / operator API on top.
"""

from .adapters import (
    DecodeStepGraph,
    PhysicalDecodeBatch,
    batched_long_query_attention,
    fused_h2o_decode,
    fused_mixed_decode,
    long_query_attention_summary,
    merge_attention_summaries,
)
from .core import PhysicalCacheRequest
from .operators import (
    H2OPhysicalGQAOperator,
    KIVIPackedQuantizationOperator,
    asymmetric_fake_quant,
    kivi_fake_quant_key,
    kivi_fake_quant_value,
)
from .storage import (
    CacheMutationResult,
    GQAH2OCache,
    HostPackedKIVI,
    PackedKIVICache,
    PhysicalLayerCache,
    PhysicalSegment,
    QuantizedHostArchive,
    TensorCacheStorageBackend,
    dequantize_kivi_chunk,
    gqa_probability_value,
    gqa_query_key_logits,
    packed_kivi_attention_parts,
    packed_kivi_quantized_attention_summary,
    quantize_kivi_b200,
    tensor_bytes,
)

__all__ = [name for name in dir() if not name.startswith("_")]

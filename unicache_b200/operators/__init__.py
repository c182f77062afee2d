"""Physical-cache operators of the plugin API (counterpart of unicache/operators)."""

from .physical import (
    H2OPhysicalGQAOperator,
    KIVIPackedQuantizationOperator,
    asymmetric_fake_quant,
    kivi_fake_quant_key,
    kivi_fake_quant_value,
)

__all__ = [
    "H2OPhysicalGQAOperator",
    "KIVIPackedQuantizationOperator",
    "asymmetric_fake_quant",
    "kivi_fake_quant_key",
    "kivi_fake_quant_value",
]

"""The operators' plugin contract, on the CPU.

The B200 operators derive from ``ProcessingOperator`` and carry a
``CapabilityDescriptor`` with the reference's fields (unicache/core/
registry.py:28-57, unicache/core/capabilities.py:12-79).  When the reference
project is present in this container, the operators are also registered in
the reference's own ``KVRegistry`` and their descriptors compared with the
reference operators' (devices differ on purpose: the B200 path is CUDA only).
"""

from __future__ import annotations

import os
import sys

import pytest

from unicache_b200 import H2OPhysicalGQAOperator, KIVIPackedQuantizationOperator
from unicache_b200.core import CapabilityDescriptor, ProcessingOperator

REFERENCE = "/root/reference"


def test_operators_carry_the_contract():
    for op in (H2OPhysicalGQAOperator(), KIVIPackedQuantizationOperator()):
        assert isinstance(op, ProcessingOperator) and op.name and op.executable
        cap = op.capability_descriptor()
        assert cap.devices == frozenset({"cuda"}) and cap.physical_storage_mutation
        cap.validate_runtime(operator=op.name, stage=next(iter(op.stages)), phase="prefill", device="cuda",
                             layout="dense", available_features=set(cap.requires))
        with pytest.raises(ValueError, match="device cpu"):
            cap.validate_runtime(operator=op.name, stage=next(iter(op.stages)), phase="prefill", device="cpu",
                                 layout="dense", available_features=set(cap.requires))
        with pytest.raises(ValueError, match="unavailable runtime features"):
            cap.validate_runtime(operator=op.name, stage=next(iter(op.stages)), phase="prefill", device="cuda",
                                 layout="dense", available_features=set())
    with pytest.raises(ValueError, match="stage"):
        KIVIPackedQuantizationOperator().capability_descriptor().validate_static(operator="k", stage="attention")
    assert CapabilityDescriptor().to_dict()["stages"] == ["*"]


def test_operator_parameter_rules():
    h2o = H2OPhysicalGQAOperator()
    assert h2o.build_params({}) == {"target_budget_ratio": 0.2, "recent_budget_fraction": 0.25,
                                    "selection_frozen": False}
    for bad in ({"target_budget_ratio": 0.0}, {"target_budget_ratio": 1.5}, {"recent_budget_fraction": -0.1}):
        with pytest.raises(ValueError):
            h2o.build_params(bad)
    kivi = KIVIPackedQuantizationOperator()
    params = kivi.build_params({"bits": 2, "group_size": 32})
    assert params["k_bits"] == params["v_bits"] == 2 and params["residual_length"] == 32
    for bad in ({"bits": 3}, {"group_size": 0}, {"backend": "reference"}):
        with pytest.raises(ValueError):
            kivi.build_params(bad)


@pytest.mark.skipif(not os.path.isdir(REFERENCE), reason="the reference project is not present")
def test_operators_register_in_the_reference_registry():
    sys.path.insert(0, REFERENCE)
    try:
        from unicache.core.registry import KVRegistry
        from unicache.operators.physical import H2OPhysicalGQAOperator as RefH2O
        from unicache.operators.physical import KIVIPackedQuantizationOperator as RefKIVI
    except Exception as exc:  # pragma: no cover - depends on the container
        pytest.skip(f"reference not importable: {exc}")
    finally:
        sys.path.remove(REFERENCE)
    registry = KVRegistry()
    ours = [H2OPhysicalGQAOperator(), KIVIPackedQuantizationOperator()]
    for op in ours:
        registry.add_processing_operator(op)
        assert registry.require_operator(op.name) is op
    for op, ref in zip(ours, (RefH2O(), RefKIVI())):
        mine, theirs = op.capability_descriptor().to_dict(), ref.capability_descriptor().to_dict()
        assert theirs.pop("devices") == ["cpu", "cuda"] and mine.pop("devices") == ["cuda"]
        assert mine == theirs, op.name
        for name in ("family", "stages", "executable", "uses_final_attention", "preserves_attention_dispatch"):
            assert getattr(op, name) == getattr(ref, name), (op.name, name)

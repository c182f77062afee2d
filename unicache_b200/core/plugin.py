"""The operator side of the reference's plugin contract.

A physical-cache operator is registered by name in the reference's
``KVRegistry`` (unicache/core/registry.py:166-241, which only reads
``operator.name``) and described to planners and adapters by a capability
record (unicache/core/capabilities.py:12-79) with the same fields and
wildcard rule.  These classes restate that contract so the B200 operators
carry it without importing the reference: an engine that runs the reference
registers them as they are.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

ANY = "*"


def _allows(values: frozenset[str], value: str) -> bool:
    return ANY in values or value in values


@dataclass(frozen=True)
class CapabilityDescriptor:
    """Where an operator runs and what it changes: stages, phases, devices and
    cache layouts it accepts (``"*"`` = any), runtime features it requires, and
    whether it selects tokens, keeps state or mutates physical storage."""

    stages: frozenset[str] = frozenset({ANY})
    phases: frozenset[str] = frozenset({ANY})
    devices: frozenset[str] = frozenset({ANY})
    layouts: frozenset[str] = frozenset({ANY})
    requires: frozenset[str] = frozenset()
    produces_selection: bool = False
    stateful: bool = False
    mutation_scope: str = "none"
    physical_storage_mutation: bool = False
    accepts_quantized_input: bool = False

    def validate_static(self, *, operator: str, stage: str) -> None:
        """Raise ValueError when ``stage`` is not one the operator runs in."""

        if not _allows(self.stages, stage):
            raise ValueError(f"Operator {operator} does not support stage {stage}; "
                             f"supported stages are {sorted(self.stages)}")

    def validate_runtime(self, *, operator: str, stage: str, phase: str, device: str, layout: str,
                         available_features: set[str]) -> None:
        """Raise ValueError when the stage, phase, device or cache layout is not
        accepted or a required runtime feature is missing."""

        self.validate_static(operator=operator, stage=stage)
        checks = (("phase", self.phases, phase), ("device", self.devices, device),
                  ("cache layout", self.layouts, layout))
        for label, accepted, value in checks:
            if not _allows(accepted, value):
                raise ValueError(f"Operator {operator} does not support {label} {value}; "
                                 f"supported values are {sorted(accepted)}")
        missing = sorted(set(self.requires) - set(available_features))
        if missing:
            raise ValueError(f"Operator {operator} requires unavailable runtime features: {missing}")

    def to_dict(self) -> dict[str, object]:
        out: dict[str, object] = {}
        for name in ("stages", "phases", "devices", "layouts", "requires"):
            out[name] = sorted(getattr(self, name))
        for name in ("produces_selection", "stateful", "mutation_scope", "physical_storage_mutation",
                     "accepts_quantized_input"):
            out[name] = getattr(self, name)
        return out


class ProcessingOperator:
    """Base of a processing operator: a registry name, the stages it runs in,
    its capabilities, parameter normalisation, and the two hooks the adapter
    calls (``execute`` before attention, ``update_after_attention`` after)."""

    name: str = ""
    family: str = "generic"
    stages: set[str] = {"attention"}
    executable: bool = False
    capabilities: CapabilityDescriptor | None = None
    uses_final_attention: bool = False
    preserves_attention_dispatch: bool = False

    def capability_descriptor(self) -> CapabilityDescriptor:
        return self.capabilities if self.capabilities is not None else \
            CapabilityDescriptor(stages=frozenset(self.stages))

    def supports(self, segment: Any, ctx: Any) -> bool:
        return True

    def build_params(self, params: dict[str, Any]) -> dict[str, Any]:
        return dict(params)

    def execute(self, ctx: Any) -> Any:
        raise NotImplementedError(f"Operator {self.name} has no executable runtime implementation")

    def update_after_attention(self, ctx: Any, attention_probs: Any) -> Any:
        return ctx

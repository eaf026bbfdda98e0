"""Hardware identity expectations, extended with the B200.

Same checks as ``src/heliostune/hardware.py:8-126``; the reference has no Blackwell entry
(its H200 entry excludes the "B200" name token), so ``B200`` is added here: compute
capability 10.0 and the 183,359 MiB (179.06 GiB) this pool's B200s report.
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass
from types import MappingProxyType

from heliostune_b200.errors import ProtocolError
from heliostune_b200.schema import HardwareProfile


@dataclass(frozen=True, slots=True)
class HardwareExpectation:
    """One allowed GPU identity and its memory envelope in GiB."""

    gpu: str
    compute_capability: tuple[int, int]
    minimum_memory_gb: float
    maximum_memory_gb: float
    required_name_tokens: tuple[str, ...] = ()
    excluded_name_tokens: tuple[str, ...] = ()

    def __post_init__(self) -> None:
        if not self.gpu or self.gpu != self.gpu.strip():
            raise ValueError("hardware expectation gpu must be nonblank without whitespace")
        capability = self.compute_capability
        if (
            type(capability) is not tuple
            or len(capability) != 2
            or any(type(part) is not int or part < 0 for part in capability)
        ):
            raise ValueError("hardware expectation capability must be a non-negative integer pair")
        low, high = self.minimum_memory_gb, self.maximum_memory_gb
        if not (math.isfinite(low) and math.isfinite(high)) or low <= 0 or high < low:
            raise ValueError("hardware expectation memory range must be finite and positive")
        for label, tokens in (
            ("required_name_tokens", self.required_name_tokens),
            ("excluded_name_tokens", self.excluded_name_tokens),
        ):
            if any(type(t) is not str or not t or t != t.strip() for t in tokens):
                raise ValueError(f"hardware expectation {label} contains an invalid token")


HARDWARE_EXPECTATIONS: Mapping[str, HardwareExpectation] = MappingProxyType(
    {
        "L4": HardwareExpectation("L4", (8, 9), 20.0, 26.0, ("L4",)),
        "A10": HardwareExpectation("A10", (8, 6), 20.0, 26.0, ("A10",), ("A100",)),
        "T4": HardwareExpectation("T4", (7, 5), 13.0, 17.0, ("T4",)),
        "H100": HardwareExpectation("H100", (9, 0), 75.0, 85.0, ("H100",), ("H200",)),
        "A100-80GB": HardwareExpectation("A100-80GB", (8, 0), 75.0, 85.0, ("A100",)),
        "H200": HardwareExpectation("H200", (9, 0), 135.0, 145.0, ("H200",), ("H100", "B200")),
        "B200": HardwareExpectation("B200", (10, 0), 175.0, 185.0, ("B200",), ("GB200",)),
    }
)


def expectation_for_gpu(gpu: str) -> HardwareExpectation:
    try:
        return HARDWARE_EXPECTATIONS[gpu]
    except KeyError as exc:
        choices = ", ".join(HARDWARE_EXPECTATIONS)
        raise ProtocolError(f"unknown hardware expectation {gpu!r}; choose from {choices}") from exc


def validate_hardware(profile: HardwareProfile, expectation: HardwareExpectation) -> None:
    """Reject a runtime profile that does not match the requested GPU identity."""
    context = f"requested {expectation.gpu}, observed {profile.device_name!r}"
    if profile.gpu != expectation.gpu:
        raise ProtocolError(
            f"hardware selector mismatch: expected {expectation.gpu!r}, got {profile.gpu!r}"
        )
    if profile.compute_capability != expectation.compute_capability:
        raise ProtocolError(
            f"hardware capability mismatch for {context}: expected "
            f"{expectation.compute_capability}, got {profile.compute_capability}"
        )
    if not expectation.minimum_memory_gb <= profile.total_memory_gb <= expectation.maximum_memory_gb:
        raise ProtocolError(
            f"hardware memory mismatch for {context}: expected "
            f"{expectation.minimum_memory_gb:g}-{expectation.maximum_memory_gb:g} GiB, "
            f"got {profile.total_memory_gb:.3f} GiB"
        )
    name = profile.device_name.upper()
    missing = [t for t in expectation.required_name_tokens if t.upper() not in name]
    forbidden = [t for t in expectation.excluded_name_tokens if t.upper() in name]
    if missing or forbidden:
        details = []
        if missing:
            details.append(f"missing name token(s) {missing!r}")
        if forbidden:
            details.append(f"contains excluded token(s) {forbidden!r}")
        raise ProtocolError(f"hardware name mismatch for {context}: {'; '.join(details)}")

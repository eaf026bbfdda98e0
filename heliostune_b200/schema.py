"""The hardware record that conditions the bandit features.

Same fields and validation as ``HardwareProfile`` at ``src/heliostune/schema.py:75-150``.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

from heliostune_b200.errors import SchemaError
from heliostune_b200.validation import exact_fields, exact_int, finite_float, nonblank_string


@dataclass(frozen=True, slots=True)
class HardwareProfile:
    """Runtime properties of one GPU."""

    gpu: str
    device_name: str
    compute_capability: tuple[int, int]
    multiprocessor_count: int
    total_memory_gb: float
    cuda_version: str | None = None
    torch_version: str | None = None
    triton_version: str | None = None

    def __post_init__(self) -> None:
        nonblank_string(self.gpu, context="hardware gpu")
        nonblank_string(self.device_name, context="hardware device_name")
        if type(self.compute_capability) is not tuple or len(self.compute_capability) != 2:
            raise SchemaError("hardware compute_capability must be a two-element integer tuple")
        for index, part in enumerate(self.compute_capability):
            exact_int(part, context=f"hardware compute_capability[{index}]", minimum=0)
        exact_int(self.multiprocessor_count, context="hardware multiprocessor_count", minimum=1)
        finite_float(self.total_memory_gb, context="hardware total_memory_gb", strictly_positive=True)
        for name in ("cuda_version", "torch_version", "triton_version"):
            value = getattr(self, name)
            if value is not None:
                nonblank_string(value, context=f"hardware {name}")

    def to_dict(self) -> dict[str, object]:
        data = asdict(self)
        data["compute_capability"] = list(self.compute_capability)
        return data

    @classmethod
    def from_dict(cls, value: object) -> HardwareProfile:
        names = (
            "gpu",
            "device_name",
            "compute_capability",
            "multiprocessor_count",
            "total_memory_gb",
            "cuda_version",
            "torch_version",
            "triton_version",
        )
        data = exact_fields(value, required=names, context="hardware")
        capability = data["compute_capability"]
        if type(capability) is not list or len(capability) != 2:
            raise SchemaError("hardware compute_capability must be a two-element integer array")
        return cls(
            gpu=nonblank_string(data["gpu"], context="hardware gpu"),
            device_name=nonblank_string(data["device_name"], context="hardware device_name"),
            compute_capability=(
                exact_int(capability[0], context="hardware compute_capability[0]", minimum=0),
                exact_int(capability[1], context="hardware compute_capability[1]", minimum=0),
            ),
            multiprocessor_count=exact_int(
                data["multiprocessor_count"], context="hardware multiprocessor_count", minimum=1
            ),
            total_memory_gb=finite_float(
                data["total_memory_gb"], context="hardware total_memory_gb", strictly_positive=True
            ),
            cuda_version=data["cuda_version"],  # type: ignore[arg-type]
            torch_version=data["torch_version"],  # type: ignore[arg-type]
            triton_version=data["triton_version"],  # type: ignore[arg-type]
        )


#: The B200 as this pool reports it (148 SMs, 183,359 MiB), used when no device is present.
B200_PROFILE = HardwareProfile("B200", "NVIDIA B200", (10, 0), 148, 179.0615234375)

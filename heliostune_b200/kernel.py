"""Drop-in for ``heliostune.kernel``: the tile-family FP16 matmul on the B200.

``matmul(a, b, config)`` keeps the reference's signature, validation order, error messages and
ownership (``src/heliostune/kernel.py:83-118``): it validates, allocates the FP16 output (and any
workspace) with ``torch.empty`` on the inputs' device, and launches asynchronously on the current
stream. The launch goes through ``hst_matmul_tile`` of the C-ABI library to the tcgen05 tile
kernel; there is no other implementation to fall back to.
"""

from __future__ import annotations

import contextlib
import ctypes
from typing import Any

import torch

from heliostune_b200 import _native
from heliostune_b200.configs import KernelConfig
from heliostune_b200.schema import HardwareProfile


def _validate(a: torch.Tensor, b: torch.Tensor) -> tuple[int, int, int]:
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("matmul inputs must be two-dimensional")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"incompatible matmul shapes: {tuple(a.shape)} and {tuple(b.shape)}")
    if a.device.type != "cuda" or b.device.type != "cuda" or a.device != b.device:
        raise ValueError("matmul inputs must be on the same CUDA device")
    if a.dtype != torch.float16 or b.dtype != torch.float16:
        raise ValueError("matmul inputs must have dtype torch.float16")
    return int(a.shape[0]), int(b.shape[1]), int(a.shape[1])


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The device's current CUDA stream as a raw handle."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if _RAW_STREAM is not None:
        return _RAW_STREAM(index)
    return torch.cuda.current_stream(index).cuda_stream


def _device_guard(device: torch.device) -> contextlib.AbstractContextManager[Any]:
    """Make ``device`` current for a launch; nothing to do when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


#: Workspace sizes by everything the native planner reads: the config, the operands' strides and
#: 16-byte alignment, the shape and the device. Bounded; cleared when full.
_WORKSPACE_SIZES: dict[tuple[Any, ...], int] = {}
_WORKSPACE_CACHE_LIMIT = 4096


def _workspace(
    config: _native.GemmConfig, a: torch.Tensor, b: torch.Tensor, m: int, n: int, k: int
) -> tuple[torch.Tensor | None, int, int]:
    """Allocate (per call, as the reference) the workspace the native planner asks for."""
    device = a.device.index if a.device.index is not None else torch.cuda.current_device()
    a_ptr, b_ptr = a.data_ptr(), b.data_ptr()
    key = (
        config.family, config.block_m, config.block_n, config.block_k, config.num_warps,
        config.num_stages, config.group_m, config.split_k, a_ptr & 15, a.stride(0), a.stride(1),
        b_ptr & 15, b.stride(0), b.stride(1), m, n, k, device,
    )  # fmt: skip
    nbytes = _WORKSPACE_SIZES.get(key)
    if nbytes is None:
        size = ctypes.c_size_t(0)
        _native.check(
            _native.library().hst_gemm_workspace_size(
                ctypes.byref(config), a_ptr, a.stride(0), a.stride(1), b_ptr, b.stride(0), b.stride(1),
                m, n, k, device, ctypes.byref(size),
            )  # fmt: skip
        )
        nbytes = size.value
        if len(_WORKSPACE_SIZES) >= _WORKSPACE_CACHE_LIMIT:
            _WORKSPACE_SIZES.clear()
        _WORKSPACE_SIZES[key] = nbytes
    if nbytes == 0:
        return None, 0, 0
    buffer = torch.empty(nbytes, device=a.device, dtype=torch.uint8)
    return buffer, buffer.data_ptr(), nbytes


def matmul(a: torch.Tensor, b: torch.Tensor, config: KernelConfig) -> torch.Tensor:
    """Multiply two CUDA FP16 matrices with one tile-family launch configuration."""
    m, n, k = _validate(a, b)
    output = torch.empty((m, n), device=a.device, dtype=torch.float16)
    native = _native.GemmConfig(
        _native.FAMILY_TILE,
        config.block_m,
        config.block_n,
        config.block_k,
        config.num_warps,
        config.num_stages,
        config.group_m,
        0,
    )
    workspace, ws_ptr, ws_bytes = _workspace(native, a, b, m, n, k)
    with _device_guard(a.device):
        _native.check(
            _native.library().hst_matmul_tile(
                config.block_m,
                config.block_n,
                config.block_k,
                config.num_warps,
                config.num_stages,
                config.group_m,
                a.data_ptr(),
                a.stride(0),
                a.stride(1),
                b.data_ptr(),
                b.stride(0),
                b.stride(1),
                output.data_ptr(),
                n,
                m,
                n,
                k,
                ws_ptr,
                ws_bytes,
                _stream(a.device),
            )
        )
    del workspace  # stream-ordered reuse by the caching allocator is safe on this stream
    return output


def get_hardware_profile(gpu: str | None = None, device: torch.device | None = None) -> HardwareProfile:
    """Read the active CUDA device into the portable schema (``kernel.py:121-138``)."""
    selected = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    props = torch.cuda.get_device_properties(selected)
    return HardwareProfile(
        gpu=gpu or props.name,
        device_name=props.name,
        compute_capability=(props.major, props.minor),
        multiprocessor_count=props.multi_processor_count,
        total_memory_gb=props.total_memory / (1024**3),
        cuda_version=None if torch.version.cuda is None else str(torch.version.cuda),
        torch_version=str(torch.__version__),
        triton_version=None,
    )


#: Compute capability of the only GPU this library is built for (sm_100a code only).
B200_COMPUTE_CAPABILITY = (10, 0)


def require_b200(profile: HardwareProfile) -> None:
    """Raise ``ProtocolError`` unless ``profile`` describes a GPU this library's kernels run on.

    The kernels are compiled for sm_100a alone, so the check is the compute capability (10.0);
    the device name must also carry "B200", since a profile is part of a run's identity and other
    10.0 parts have other memory systems and SM counts than the ones the tuner pool assumes.
    """
    from heliostune_b200.errors import ProtocolError

    if tuple(profile.compute_capability) != B200_COMPUTE_CAPABILITY:
        raise ProtocolError(
            f"{profile.device_name} has compute capability {profile.compute_capability}; "
            f"the kernels are built for {B200_COMPUTE_CAPABILITY} (sm_100a) only"
        )
    if "B200" not in profile.device_name.upper():
        raise ProtocolError(f"{profile.device_name!r} is not a B200")


def _within_tolerance(difference: Any, expected: Any, *, atol: float, rtol: float) -> bool:
    """Elementwise ``|out - ref| <= atol + rtol * |ref|`` (``kernel.py:161-168``)."""
    return bool(torch.all(difference <= (atol + rtol * torch.abs(expected))).item())

"""Loader of the C-ABI library ``libheliostune_b200.so`` and its build recipe.

The library is built in-tree (``build_library``) by nvcc for sm_100a and loaded with ctypes.
There is no fallback: when the library is missing or fails to load, every GPU entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

from heliostune_b200.errors import KernelError

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "libheliostune_b200.so"
HEADER_PATH = PACKAGE_DIR.parent / "include" / "heliostune_b200.h"
SOURCES = (PACKAGE_DIR / "csrc" / "capi.cu",)
NVCC_FLAGS = (
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
)

HST_OK = 0
HST_ERR_INVALID = 1
HST_ERR_UNSUPPORTED = 2
HST_ERR_WORKSPACE = 3
HST_ERR_CUDA = 4
HST_ERR_TIMEOUT = 5

HST_PEER_STORES = 0
HST_PEER_BULK = 1

FAMILY_TILE = 0
FAMILY_PERSISTENT = 1
FAMILY_SPLIT_K = 2
FAMILY_STREAM = 3
FAMILY_PAIR = 4

#: Every symbol include/heliostune_b200.h declares.
EXPORTED_SYMBOLS = (
    "hst_abi_version",
    "hst_last_error",
    "hst_device_sm_count",
    "hst_gemm_workspace_size",
    "hst_gemm",
    "hst_matmul_tile",
    "hst_matmul_persistent",
    "hst_matmul_split_k",
    "hst_matmul_stream",
    "hst_matmul_pair",
    "hst_rmsnorm",
    "hst_residual_rmsnorm",
    "hst_gated_mlp_stream",
    "hst_status",
    "hst_probe_wait_timeout",
    "hst_matmul_split_k_noalloc",
    "hst_column_assemble",
    "hst_matmul_pair_fanout",
    "hst_peer_barrier",
    "hst_ipc_export",
    "hst_ipc_import",
    "hst_ipc_close",
    "hst_pair_stream_k_tiles",
    "hst_rmsnorm_matmul_stream",
)


class GemmConfig(ctypes.Structure):
    """``hst_gemm_config`` of the header."""

    _fields_ = [
        ("family", ctypes.c_int32),
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("num_warps", ctypes.c_int32),
        ("num_stages", ctypes.c_int32),
        ("group_m", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
    ]


def build_library(*, force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA sources into ``libheliostune_b200.so`` next to this file."""
    newest = max(p.stat().st_mtime for p in (PACKAGE_DIR / "csrc").iterdir())
    newest = max(newest, HEADER_PATH.stat().st_mtime)
    if not force and LIBRARY_PATH.exists() and LIBRARY_PATH.stat().st_mtime >= newest:
        return LIBRARY_PATH
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = LIBRARY_PATH.with_suffix(f".so.tmp{os.getpid()}")
    command = [nvcc, *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr[-4000:]}")
    if verbose and result.stderr:
        print(result.stderr)
    os.replace(tmp, LIBRARY_PATH)
    return LIBRARY_PATH


_lock = threading.Lock()
_library: ctypes.CDLL | None = None

_i32, _i64, _u64, _size = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_size_t
_ptr = ctypes.c_void_p


def _declare(lib: ctypes.CDLL) -> None:
    sig = {
        "hst_abi_version": ([], ctypes.c_int),
        "hst_last_error": ([], ctypes.c_char_p),
        "hst_device_sm_count": ([ctypes.c_int, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
        "hst_gemm_workspace_size": (
            [ctypes.POINTER(GemmConfig), _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64, _i64,
             ctypes.c_int, ctypes.POINTER(_size)],
            ctypes.c_int,
        ),
        "hst_gemm": (
            [ctypes.POINTER(GemmConfig), _ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64,
             _i64, _i64, _ptr, _size, _ptr],
            ctypes.c_int,
        ),
        "hst_matmul_tile": (
            [_i32] * 6 + [_ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64,
                          _ptr, _size, _ptr],
            ctypes.c_int,
        ),
        "hst_matmul_persistent": ([_i32] * 6 + [_ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr], ctypes.c_int),
        "hst_matmul_split_k": (
            [_i32] * 6 + [_ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64,
                          _ptr, _size, _ptr],
            ctypes.c_int,
        ),
        "hst_matmul_stream": (
            [_i32] * 5 + [_ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64,
                          _ptr, _size, _ptr],
            ctypes.c_int,
        ),
        "hst_pair_stream_k_tiles": ([_i64, _i64, _i64, ctypes.POINTER(_i64)], ctypes.c_int),
        "hst_rmsnorm_matmul_stream": (
            [_i32] * 5 + [_ptr, _i64, _ptr, ctypes.c_float, _ptr, _i64, _ptr, _i64, _i64, _i64, _i64, _ptr],
            ctypes.c_int,
        ),
        "hst_matmul_pair": (
            [_i32] * 5 + [_ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64,
                          _ptr, _size, _ptr],
            ctypes.c_int,
        ),
        "hst_rmsnorm": (
            [_ptr, _i64, _ptr, _ptr, _i64, _i64, _i64, ctypes.c_float, _ptr],
            ctypes.c_int,
        ),
        "hst_residual_rmsnorm": (
            [_ptr, _i64, _ptr, _i64, _ptr, _ptr, _i64, _i64, _i64, ctypes.c_float, _i32, _ptr],
            ctypes.c_int,
        ),
        "hst_gated_mlp_stream": (
            [_i32] * 4 + [_ptr, _i64, _ptr, _i64, _ptr, _i64, _ptr, _i64, _i64, _i64, _i64, _ptr],
            ctypes.c_int,
        ),
        "hst_status": ([ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int], ctypes.c_int),
        "hst_probe_wait_timeout": ([_u64, _ptr], ctypes.c_int),
        "hst_column_assemble": ([_ptr, _ptr, _i64, _i64, _i64, _i64, _ptr], ctypes.c_int),
        "hst_ipc_export": ([_ptr, _ptr, ctypes.POINTER(_u64)], ctypes.c_int),
        "hst_ipc_import": ([_ptr, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
        "hst_ipc_close": ([_ptr], ctypes.c_int),
        "hst_matmul_pair_fanout": (
            [_i32] * 4 + [_ptr, _ptr, ctypes.POINTER(ctypes.c_void_p), _i32, _i32, _i64, _i64, _i64, _i32, _ptr],
            ctypes.c_int,
        ),
        "hst_peer_barrier": (
            [ctypes.POINTER(ctypes.c_void_p), _i32, _i32, _i32, ctypes.c_uint64, ctypes.c_uint64, _ptr],
            ctypes.c_int,
        ),
        "hst_matmul_split_k_noalloc": (
            [_i32] * 6 + [_ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64, _ptr],
            ctypes.c_int,
        ),
    }
    for name, (args, result) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = result


def library() -> ctypes.CDLL:
    """The loaded C-ABI library; raises ``KernelError`` if it is missing or unloadable."""
    global _library
    if _library is None:
        with _lock:
            if _library is None:
                if not LIBRARY_PATH.exists():
                    raise KernelError(
                        f"{LIBRARY_PATH.name} is not built; run heliostune_b200._native.build_library()"
                    )
                try:
                    lib = ctypes.CDLL(str(LIBRARY_PATH))
                except OSError as exc:
                    raise KernelError(f"cannot load {LIBRARY_PATH}: {exc}") from exc
                _declare(lib)
                if lib.hst_abi_version() != 1:
                    raise KernelError("libheliostune_b200 ABI version mismatch")
                _library = lib
    return _library


def check(rc: int) -> None:
    """Map a C-ABI return code onto the reference's exception types."""
    if rc == HST_OK:
        return
    message = library().hst_last_error().decode(errors="replace")
    if rc in (HST_ERR_INVALID, HST_ERR_UNSUPPORTED, HST_ERR_WORKSPACE):
        raise ValueError(message)
    raise KernelError(message)


def status(device: int, *, clear: bool = False) -> int:
    """Status bits of a device (synchronises it)."""
    bits = ctypes.c_int(0)
    check(library().hst_status(device, ctypes.byref(bits), int(clear)))
    return bits.value

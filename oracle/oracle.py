"""CPU oracle of the FP16 matmul path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module, and only as the checker or the timed CPU baseline; the product never does.

Each function restates one piece of the reference (mottopanikeiku/heliostune):

* :func:`gemm_fp32_reference` -- the check value ``torch.mm(a, b, out_dtype=torch.float32)``
  with TF32 off (``src/heliostune/action_expansion.py:206-211``,
  ``tests/test_action_expansion.py:29-40``): FP16 operands, exact products, FP64 sum, one
  rounding to FP32.
* :func:`gemm_fp32_blas` -- the same value as an FP32 BLAS product.
* :func:`gemm_fp16_torch_cpu` -- ``torch.matmul`` of the FP16 operands on the host cores, the
  path the reference's decode shape runs on without a GPU (the reference times ``torch.matmul``
  as its baseline, ``src/heliostune/kernel.py:141-168``); the timed CPU baseline.
* :func:`gemm_split_k` -- the split-K algorithm (``action_expansion.py:56-121``) in the C
  restatement ``oracle.c``.
* :func:`rmsnorm_reference` -- ``local_executor.py:1982-1985``, with or without the residual.
* :func:`within_tolerance` -- ``kernel.py:161-168``.

Pinned against ``tests/golden/`` (made by ``tests/golden/make_golden.py`` from the reference's
own code and known-answer tests) by ``tests/test_oracle.py``.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = ORACLE_DIR / "liboracle.so"

_lib: ctypes.CDLL | None = None


def build() -> Path:
    """Compile ``oracle.c`` with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIBRARY_PATH


def _library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            build()
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        p, i64 = ctypes.c_void_p, ctypes.c_int64
        lib.hst_oracle_gemm.argtypes = [p, i64, i64, p, i64, i64, p, i64, i64, i64]
        lib.hst_oracle_gemm.restype = None
        lib.hst_oracle_gemm_splitk.argtypes = [p, i64, i64, p, i64, i64, p, i64, i64, i64, i64, i64]
        lib.hst_oracle_gemm_splitk.restype = None
        lib.hst_oracle_rmsnorm.argtypes = [p, p, p, p, i64, i64, ctypes.c_double, ctypes.c_int, ctypes.c_int]
        lib.hst_oracle_rmsnorm.restype = None
        lib.hst_oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.hst_oracle_f32_to_f16.restype = ctypes.c_uint16
        _lib = lib
    return _lib


def _bits(x: np.ndarray) -> tuple[np.ndarray, int, int]:
    """A uint16 view of an FP16/BF16-bit array, with element strides."""
    if x.dtype == np.float16:
        x = x.view(np.uint16)
    if x.dtype != np.uint16:
        raise TypeError("expected float16 or uint16 bit patterns")
    return x, x.strides[0] // 2, x.strides[1] // 2 if x.ndim > 1 else 1


def gemm_fp32_reference(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """FP32 value of ``A @ B`` for FP16 ``A [M, K]``, ``B [K, N]`` (FP64 accumulation)."""
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)


def gemm_fp32_reference_c(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The same value from the C restatement (scalar loops; small shapes only)."""
    a_bits, sa0, sa1 = _bits(a)
    b_bits, sb0, sb1 = _bits(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    _library().hst_oracle_gemm(
        a_bits.ctypes.data, sa0, sa1, b_bits.ctypes.data, sb0, sb1, c.ctypes.data, m, n, k
    )
    return c


def gemm_fp32_blas(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``fp32(A) @ fp32(B)`` with FP32 accumulation through the host BLAS (all host threads)."""
    return a.astype(np.float32) @ b.astype(np.float32)


def gemm_fp16_torch_cpu(a, b):  # type: ignore[no-untyped-def]
    """``torch.matmul`` of FP16 CPU tensors on the host cores (the caller sets the thread count)."""
    import torch

    return torch.matmul(a, b)


def gemm_split_k(a: np.ndarray, b: np.ndarray, block_k: int, splits: int) -> np.ndarray:
    """FP16 result of the reference's split-K algorithm (C restatement)."""
    a_bits, sa0, sa1 = _bits(a)
    b_bits, sb0, sb1 = _bits(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.uint16)
    _library().hst_oracle_gemm_splitk(
        a_bits.ctypes.data, sa0, sa1, b_bits.ctypes.data, sb0, sb1, c.ctypes.data, m, n, k,
        block_k, splits,
    )
    return c.view(np.float16)


def rmsnorm_reference(
    x: np.ndarray, gamma: np.ndarray, eps: float, *, bf16: bool = False, residual: np.ndarray | None = None
) -> np.ndarray:
    """``cast((z * rsqrt(mean(z^2) + eps)) * gamma)`` per row with ``z = x`` or, given
    ``residual``, ``z = fp32(x) + fp32(residual)``; FP64 row sum.

    With ``bf16`` the inputs are BF16 bit patterns (uint16) and the output is BF16 bits.
    """
    x = np.ascontiguousarray(x)
    gamma = np.ascontiguousarray(gamma)
    x_bits = x.view(np.uint16)
    g_bits = gamma.view(np.uint16)
    rows, hidden = x.shape
    r_ptr = None
    if residual is not None:
        residual = np.ascontiguousarray(residual)
        if residual.shape != x.shape:
            raise ValueError("residual must have the shape of x")
        r_ptr = residual.view(np.uint16).ctypes.data
    y = np.empty((rows, hidden), dtype=np.uint16)
    _library().hst_oracle_rmsnorm(
        x_bits.ctypes.data, r_ptr, g_bits.ctypes.data, y.ctypes.data, rows, hidden, eps, int(bf16), int(bf16)
    )
    return y if bf16 else y.view(np.float16)


def f32_to_f16(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even FP16 conversion of the C restatement (checked against numpy)."""
    lib = _library()
    flat = np.asarray(values, dtype=np.float32).ravel()
    out = np.fromiter((lib.hst_oracle_f32_to_f16(float(v)) for v in flat), dtype=np.uint16, count=flat.size)
    return out.reshape(np.shape(values)).view(np.float16)


def within_tolerance(output: np.ndarray, expected: np.ndarray, *, atol: float, rtol: float) -> bool:
    """``|out - ref| <= atol + rtol * |ref|`` elementwise in FP32 (``kernel.py:161-168``)."""
    difference = np.abs(output.astype(np.float32) - expected.astype(np.float32))
    return bool(np.all(difference <= atol + rtol * np.abs(expected.astype(np.float32))))


def normwise_error(output: np.ndarray, expected: np.ndarray) -> float:
    """``max |out - ref| / max |ref|``: the build's size-independent parity measure."""
    expected = expected.astype(np.float64)
    scale = float(np.max(np.abs(expected))) if expected.size else 0.0
    if scale == 0.0:
        return float(np.max(np.abs(output.astype(np.float64)))) if output.size else 0.0
    return float(np.max(np.abs(output.astype(np.float64) - expected)) / scale)

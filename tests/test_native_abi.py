"""The C-ABI boundary without a GPU: the header and the built library agree, the library loads,
and the Python layer rejects bad calls before any CUDA work."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest
import torch

from heliostune_b200 import _native
from heliostune_b200.action_configs import NON_SPLIT_CANDIDATES, SPLIT_K_CANDIDATES, SplitKConfig
from heliostune_b200.configs import HopperGemmConfig, KernelConfig


def _declared_symbols() -> set[str]:
    text = _native.HEADER_PATH.read_text()
    return set(re.findall(r"^\s*(?:int|const char\*)\s+(hst_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    _native.build_library()
    return _native.library()


def test_header_declares_exactly_the_exported_entry_points() -> None:
    assert _declared_symbols() == set(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib: ctypes.CDLL) -> None:
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIBRARY_PATH)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\sT\s(hst_\w+)$", out.stdout, flags=re.M))
    assert _declared_symbols() <= exported
    for name in _declared_symbols():
        assert hasattr(lib, name)


def test_library_is_built_for_sm_100a(lib: ctypes.CDLL) -> None:
    # The build recipe compiles for sm_100a alone: one -gencode, real code, no PTX for other targets.
    flags = list(_native.NVCC_FLAGS)
    gencodes = [flags[i + 1] for i, f in enumerate(flags) if f == "-gencode"]
    assert gencodes == ["arch=compute_100a,code=sm_100a"]
    assert lib.hst_abi_version() == 1
    assert lib.hst_last_error() == b""


def test_inputs_are_validated_before_any_cuda_work() -> None:
    from heliostune_b200.action_expansion import _split_k_matmul, launch
    from heliostune_b200.hopper_kernel import hopper_matmul
    from heliostune_b200.kernel import matmul

    a = torch.zeros((4, 8), dtype=torch.float16)
    b = torch.zeros((8, 8), dtype=torch.float16)
    with pytest.raises(ValueError, match="same CUDA device"):
        matmul(a, b, KernelConfig(128, 128, 64, 4, 5))
    with pytest.raises(ValueError, match="two-dimensional"):
        matmul(a[0], b, KernelConfig(128, 128, 64, 4, 5))
    with pytest.raises(ValueError, match="incompatible matmul shapes"):
        hopper_matmul(a, b[:4], HopperGemmConfig(128, 128, 64, 4, 4))
    # The device is checked before the dtype, in the reference's order (kernel.py:85-92).
    with pytest.raises(ValueError, match="same CUDA device"):
        _split_k_matmul(a.float(), b, SplitKConfig(16, 64, 64, 4, 3, 4))
    with pytest.raises(TypeError, match="unknown action configuration"):
        launch(a, b, type("Fake", (), {"config": object()})())  # type: ignore[arg-type]


@pytest.mark.parametrize(
    ("family", "entrypoint"),
    (("tile", "matmul"), ("persistent", "hopper_matmul"), ("split_k", "_split_k_matmul")),
)
def test_launch_propagates_failures_without_another_implementation(
    monkeypatch: pytest.MonkeyPatch, family: str, entrypoint: str
) -> None:
    """Port of tests/test_action_expansion.py:85-109 of the reference."""
    from heliostune_b200 import action_expansion

    candidate = next(c for c in (*NON_SPLIT_CANDIDATES, *SPLIT_K_CANDIDATES) if c.family == family)
    failure = RuntimeError("requested kernel failed")

    def fail(*args: object) -> None:
        raise failure

    def forbidden(*args: object) -> None:
        raise AssertionError("another implementation must not run")

    for name in ("matmul", "hopper_matmul", "_split_k_matmul", "_stream_matmul"):
        monkeypatch.setattr(action_expansion, name, fail if name == entrypoint else forbidden)
    with pytest.raises(RuntimeError) as raised:
        action_expansion.launch(None, None, candidate)  # type: ignore[arg-type]
    assert raised.value is failure


def test_missing_library_fails_loudly(monkeypatch: pytest.MonkeyPatch, tmp_path) -> None:  # type: ignore[no-untyped-def]
    monkeypatch.setattr(_native, "_library", None)
    monkeypatch.setattr(_native, "LIBRARY_PATH", tmp_path / "absent.so")
    with pytest.raises(_native.KernelError, match="not built"):
        _native.library()


def test_stream_k_planning_matches_the_python_rule(lib: ctypes.CDLL) -> None:
    from heliostune_b200.action_configs import pair_stream_k_tiles

    out = ctypes.c_int64(-1)
    for tiles in (0, 1, 3, 28, 32, 73, 74, 75, 112, 128, 148, 149, 448, 512, 576, 896, 1184):
        for k_blocks in (1, 2, 5, 56, 64, 296):
            for pairs in (1, 37, 74):
                assert lib.hst_pair_stream_k_tiles(tiles, k_blocks, pairs, ctypes.byref(out)) == 0
                assert out.value == pair_stream_k_tiles(tiles, k_blocks, pairs)
    assert lib.hst_pair_stream_k_tiles(4, 4, 0, ctypes.byref(out)) == _native.HST_ERR_INVALID


def test_fanout_entry_rejects_an_unknown_peer_write_form(lib: ctypes.CDLL) -> None:
    outputs = (ctypes.c_void_p * 2)(None, None)
    rc = lib.hst_matmul_pair_fanout(256, 64, 6, 8, 1, 1, outputs, 2, 0, 512, 1024, 512, 7, None)
    assert rc == _native.HST_ERR_INVALID
    assert b"peer_writes" in lib.hst_last_error()


def test_peer_barrier_rejects_bad_arguments_before_any_cuda_work(lib: ctypes.CDLL) -> None:
    words = (ctypes.c_void_p * 2)(8, 16)
    assert lib.hst_peer_barrier(words, 0, 0, 0, 1, 0, None) == _native.HST_ERR_INVALID
    assert lib.hst_peer_barrier(words, 2, 2, 0, 1, 0, None) == _native.HST_ERR_INVALID
    assert lib.hst_peer_barrier(words, 2, 0, 2, 1, 0, None) == _native.HST_ERR_INVALID
    assert b"slot" in lib.hst_last_error()
    assert lib.hst_peer_barrier(words, 2, 0, 1, 0, 0, None) == _native.HST_ERR_INVALID
    assert b"epoch" in lib.hst_last_error()
    unaligned = (ctypes.c_void_p * 2)(8, 12)
    assert lib.hst_peer_barrier(unaligned, 2, 0, 1, 1, 0, None) == _native.HST_ERR_INVALID
    assert b"aligned" in lib.hst_last_error()
    assert lib.hst_peer_barrier(words, 2, 0, 1, 1, 61_000_000_000, None) == _native.HST_ERR_INVALID
    # One rank: nothing to wait for, nothing launched.
    assert lib.hst_peer_barrier(words, 1, 0, 0, 1, 0, None) == _native.HST_OK


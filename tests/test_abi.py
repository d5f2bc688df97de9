"""The C-ABI library loads and exports exactly what include/tropnn_b200.h declares (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from tropnn_b200 import _native as nat
from tropnn_b200 import build as b200_build

HEADER = Path(__file__).resolve().parent.parent / "include" / "tropnn_b200.h"


def _declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TROPNN_B200_API\s+[\w\s\*]+?\b(tropnn_b200_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    b200_build.build()
    return nat.load()


def test_header_declares_the_bound_symbols() -> None:
    assert _declared_symbols() == sorted(nat.SIGNATURES)


def test_library_exports_every_declared_symbol(lib: ctypes.CDLL) -> None:
    out = subprocess.run(["nm", "-D", "--defined-only", str(nat.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tropnn_b200_\w+)$", out, flags=re.M))
    assert set(_declared_symbols()) <= exported
    for name in _declared_symbols():
        assert getattr(lib, name) is not None


def test_library_is_built_for_sm100a_only() -> None:
    # The build compiles and links every source for one target, sm_100a, and nothing else.
    assert b200_build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert not any("arch" in flag or "code=" in flag for flag in b200_build.NVCC_FLAGS)


def test_abi_version_and_error_plumbing(lib: ctypes.CDLL) -> None:
    assert lib.tropnn_b200_abi_version() == nat.ABI_VERSION
    assert isinstance(nat.last_error(), str)


def test_workspace_queries_are_host_only(lib: ctypes.CDLL) -> None:
    # Pairwise: perm [T,N] + seg [T,2^C+1] + anchor map + gu + r*; 256-byte aligned slots.
    size = lib.tropnn_b200_pairwise_backward_workspace_size(4096, 16, 6, 256, 1)
    assert size >= 4096 * 16 * 4 + 16 * 65 * 4 + 257 * 4 + 192 * 4 + 4096 * 16 * 4 + 4096 * 16
    assert size % 256 == 0
    assert lib.tropnn_b200_pairwise_backward_workspace_size(4096, 16, 13, 256, 1) == 0  # comparisons > 12
    size_t = lib.tropnn_b200_trop_backward_workspace_size(512, 256, 16, 1)
    assert size_t >= 512 * 256 * 4 * 5
    assert lib.tropnn_b200_trop_backward_workspace_size(512, 256, 16, 0) < size_t
    # The half-precision route (tcgen05 scores, bias in the epilogue) takes no scratch; the f32 one
    # keeps its split operands in the workspace.
    assert lib.tropnn_b200_trop_route_workspace_size(512, 64, 256, 16, nat.F16, nat.F16) == 0
    assert lib.tropnn_b200_trop_route_workspace_size(512, 64, 256, 16, nat.F32, nat.F32) > 0

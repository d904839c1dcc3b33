"""The C-ABI library builds, loads and exports every entry point that
include/nkv.h declares. CPU only: no compute calls."""

import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _header_functions() -> list[str]:
    text = (REPO / "include" / "nkv.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nkv_[a-z_0-9]+)\s*\(", text)))


def test_library_builds_and_exports_every_symbol():
    from nanokv_b200 import _lib, build

    build.build()
    lib = _lib.load()
    declared = _header_functions()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in nkv.h but not exported"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes bindings out of sync with nkv.h"
    assert lib.nkv_abi_version() == 100
    assert lib.nkv_status_string(3) == b"NKV_ERR_WORKSPACE"


def test_workspace_query_is_pure_host():
    from nanokv_b200 import _lib

    lib = _lib.load()
    n = lib.nkv_paged_decode_workspace_size(256, 32, 8, 128, 32, 256)
    assert n > 0 and n % 256 == 0
    assert lib.nkv_paged_decode_workspace_size(256, 30, 8, 128, 32, 256) == 0  # Hq % Hk != 0


def test_argument_errors_need_no_gpu():
    """Validation happens before any CUDA call, so it is testable on CPU."""
    from nanokv_b200 import _lib

    lib = _lib.load()
    # unsupported head_dim
    assert lib.nkv_paged_decode(16, 0, 0, 16, 16, 1, 16, 1, 16, 16, 4096, 1, 32, 8, 64, 256,
                                0.1, 16, 1 << 20, None) == 2
    # workspace too small
    assert lib.nkv_paged_decode(16, 4096, 128, 16, 16, 1, 16, 1, 16, 16, 4096, 1, 32, 8, 128, 256,
                                0.1, 16, 8, None) == 3
    # misaligned q
    assert lib.nkv_paged_decode(18, 4096, 128, 16, 16, 1, 16, 1, 16, 16, 4096, 1, 32, 8, 128, 256,
                                0.1, 16, 1 << 30, None) == 4
    # zero tokens is a no-op for the store
    assert lib.nkv_store_kvcache(16, 1024, 16, 1024, 16, 16, 100, 16, 0, 8, 128, None) == 0
    # obs_window other than 1 is not the reference's periodic path
    assert lib.nkv_window_compress(16, 4096, 16, 16, 10, 16, 8, 16, 16, 16, 1, 4, 513, 2, 32, 8,
                                   128, 256, 0.1, None, None, None) == 2

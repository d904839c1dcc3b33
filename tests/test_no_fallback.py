"""The product path has no fallback: a missing library, a library without an
entry point of include/nkv.h, or host (CPU) tensors all fail loudly instead
of computing anything on the host. CPU only."""

import subprocess

import pytest
import torch


def test_missing_library_raises(tmp_path):
    from nanokv_b200 import _lib

    with pytest.raises(ImportError, match="no fallback"):
        _lib.load(tmp_path / "libnkv.so")


def test_library_without_an_entry_point_fails_to_load(tmp_path):
    from nanokv_b200 import _lib

    src = tmp_path / "stub.c"
    src.write_text("int nkv_abi_version(void) { return 100; }\n")
    so = tmp_path / "libstub.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(so), str(src)], check=True)
    with pytest.raises(AttributeError):
        _lib.load(so)


def test_ops_reject_host_tensors():
    from nanokv_b200 import ops

    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    kc = torch.zeros(4, 256, 2, 128, dtype=torch.bfloat16)
    bt = torch.zeros(2, 2, dtype=torch.int32)
    cl = torch.ones(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        ops.paged_decode(q, kc, kc, bt, cl, 128 ** -0.5)
    k = torch.zeros(2, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        ops.store_kvcache(k, k, kc, kc, torch.zeros(2, dtype=torch.int32))
    qkv = torch.zeros(2, 12 * 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        ops.qk_norm_rope_store(qkv, torch.zeros(2, dtype=torch.int64), torch.zeros(16, 128),
                               torch.ones(128, dtype=torch.bfloat16),
                               torch.ones(128, dtype=torch.bfloat16), 1e-6, 8, 2)

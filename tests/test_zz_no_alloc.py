"""The paged-decode entry point that allocates nothing.

Some callers of this attention path cannot allocate device memory: code that
runs while a CUDA graph is being captured, serving runtimes whose memory pool
is sealed after start-up, and plugin hosts that pass a kernel its inputs and
outputs but no scratch buffer. nkv_paged_decode_static_scratch serves them
with a fixed scratch array inside the library. This file checks, through the
C ABI, that two calls in a row give what the workspace-taking
nkv_paged_decode gives and what the CPU oracle of flash_attn_with_kvcache
gives (the decode tests' tolerances: max-abs 2e-2, relative 1e-2), and that a
problem too large for the array is refused before anything is launched.
Pytest collects this file last, so a failure here leaves every other test
already run.
"""

import pytest
import torch

from oracle.attention import paged_decode_ref
from oracle.inputs import make_paged_batch

pytestmark = pytest.mark.gpu

DEV = "cuda"
ATOL = 2e-2
RTOL = 1e-2


def _static_call(lib, q, kc, vc, bt, cl, out, Hq, Hk, scale):
    return lib.nkv_paged_decode_static_scratch(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.shape[0],
        bt.data_ptr(), bt.size(1), cl.data_ptr(), out.data_ptr(), out.stride(0), q.shape[0],
        Hq, Hk, 128, kc.shape[1], scale, torch.cuda.current_stream().cuda_stream)


def test_static_scratch_decode_matches_workspace_decode(cuda_lib):
    from nanokv_b200 import _lib, ops

    lib = cuda_lib
    Hq, Hk, scale = 32, 8, 128 ** -0.5
    # ragged lengths: single- and multi-split items, partial tiles, one empty row
    pb = make_paged_batch(seed=90, lens=[3000, 1, 257, 0, 6000, 1024, 130, 2500], Hq=Hq, Hk=Hk)
    q, kc, vc = pb.q.to(DEV), pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    bt, cl = pb.block_tables.to(DEV), pb.context_lens.to(DEV)
    need = lib.nkv_paged_decode_workspace_size(q.shape[0], Hq, Hk, 128, bt.size(1), kc.shape[1])
    assert 0 < need <= _lib.STATIC_SCRATCH_BYTES
    expected = ops.paged_decode(q, kc, vc, bt, cl, scale).float()
    ref = paged_decode_ref(pb.q, pb.k_cache, pb.v_cache, pb.block_tables, pb.context_lens, scale)
    for _ in range(2):  # the second call sees the first call's leftover scratch
        out = torch.full((q.shape[0], Hq, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        assert _static_call(lib, q, kc, vc, bt, cl, out, Hq, Hk, scale) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert (out.float() - expected).abs().max().item() <= ATOL
        got = out.float().cpu()
        assert (got - ref).abs().max().item() <= ATOL
        assert ((got - ref).norm() / ref.norm()).item() <= RTOL
    assert _lib.read_device_error(clear=True) == 0


def test_static_scratch_refuses_oversized_problem(cuda_lib):
    from nanokv_b200 import _lib

    lib = cuda_lib
    B, Hq, Hk, max_blocks = 2048, 32, 8, 32  # 2048 rows of 8k-token contexts: ~35 MB of scratch
    assert lib.nkv_paged_decode_workspace_size(B, Hq, Hk, 128, max_blocks, 256) > _lib.STATIC_SCRATCH_BYTES
    q = torch.zeros(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    kc = torch.zeros(4, 256, Hk, 128, dtype=torch.bfloat16, device=DEV)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32, device=DEV)
    cl = torch.ones(B, dtype=torch.int32, device=DEV)
    out = torch.full((B, Hq, 128), 7.0, dtype=torch.bfloat16, device=DEV)
    assert _static_call(lib, q, kc, kc, bt, cl, out, Hq, Hk, 0.1) == 3  # NKV_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing ran

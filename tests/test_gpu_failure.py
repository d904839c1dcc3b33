"""Failure detection without a GPU fault: a device-side wait that runs out.

The o_proj + all-reduce kernel (nkv_oproj_allreduce_p2p, replacing
nanokvllm/layers/linear.py:151-155) waits at an in-kernel barrier for every
rank's arrivals. Here one GPU calls it declaring TWO ranks, and the second
rank's arrival counter is a word that nothing reads, so this rank's counter
never reaches its target: every wait must give up after its limit (1 ms),
raise NKV_DEVERR_WAIT_TIMEOUT, record the barrier bit in the call's status
word, write NaN (not a plausible partial sum) to y, leave the call's counter
targets and epoch where they were, and let the kernel finish -- no hang, no
trap -- and the context must stay usable (a following single-rank call gives
the right result). All pointers are this GPU's own memory.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _call(lib, x, w, y, recv, recv_ptrs, sig_ptrs, sig_local, flags, ws, world, timeout_ns):
    from nanokv_b200 import ops
    T, K = x.shape
    N = w.shape[0]
    return lib.nkv_oproj_allreduce_p2p(
        x.data_ptr(), K, w.data_ptr(), K, T, K, N, recv_ptrs.data_ptr(), T * N,
        sig_ptrs.data_ptr(), sig_local.data_ptr(), flags.data_ptr(), 0, world, timeout_ns,
        ws.data_ptr(), ws.numel() * 4, y.data_ptr(), N, ops._stream(x.device))


def test_oproj_barrier_wait_gives_up_with_status(cuda_lib):
    from nanokv_b200 import _lib
    lib = _lib.load()
    _lib.read_device_error(clear=True)
    T, K, N = 64, 512, 1024
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    ws = torch.empty(4 * 128 * N, dtype=torch.float32, device=DEV)
    ref = F.linear(x.float(), w.float())

    # declared world 2: both ranks' receive buffers are this buffer, rank 1's
    # arrival counter is `absent` (nothing waits on it, nothing else adds to
    # this rank's counter), so the barrier cannot complete
    world = 2
    recv = torch.zeros(2 * world * T * N, dtype=torch.bfloat16, device=DEV)
    sig = torch.zeros(4, dtype=torch.int32, device=DEV)
    absent = torch.zeros(4, dtype=torch.int32, device=DEV)
    recv_ptrs = torch.tensor([recv.data_ptr()] * world, dtype=torch.int64, device=DEV)
    sig_ptrs = torch.tensor([sig.data_ptr(), absent.data_ptr()], dtype=torch.int64, device=DEV)
    flags = torch.zeros(5, dtype=torch.int32, device=DEV)
    y = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    assert _call(lib, x, w, y, recv, recv_ptrs, sig_ptrs, sig, flags, ws, world, 1_000_000) == 0
    torch.cuda.synchronize()
    assert _lib.read_device_error(clear=True) & _lib.DEVERR_WAIT_TIMEOUT
    # this rank arrived once per CTA at both counters; the target needed twice
    arrivals = int(sig[0].item())
    assert arrivals > 0 and int(absent[0].item()) == arrivals
    # the barrier never passed: y is NaN everywhere, the status word names
    # the barrier, and the targets / epoch were not advanced
    from nanokv_b200.layers.linear import oproj_status_text
    assert bool(torch.isnan(y.float()).all())
    status = int(flags[3].item())
    assert status == 8, oproj_status_text(status)
    assert int(flags[0].item()) == 0 and int(flags[4].item()) == 0

    # the context is usable: a single-rank call completes without error
    sig1 = torch.zeros(4, dtype=torch.int32, device=DEV)
    flags1 = torch.zeros(5, dtype=torch.int32, device=DEV)
    recv1 = torch.zeros(2 * T * N, dtype=torch.bfloat16, device=DEV)
    y1 = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    assert _call(lib, x, w, y1, recv1,
                 torch.tensor([recv1.data_ptr()], dtype=torch.int64, device=DEV),
                 torch.tensor([sig1.data_ptr()], dtype=torch.int64, device=DEV), sig1, flags1,
                 ws, 1, 1_000_000_000) == 0
    torch.cuda.synchronize()
    assert _lib.read_device_error(clear=True) == 0 and int(flags1[3].item()) == 0
    err = (y1.float() - ref).abs()
    assert bool((err <= 2.0 ** -7 * ref.abs() + 2.0 ** -7 * ref.abs() + 1e-3).all())

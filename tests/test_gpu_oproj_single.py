"""The fused o_proj GEMM + all-reduce kernel (nkv_oproj_allreduce_p2p,
replacing F.linear + dist.all_reduce, nanokvllm/layers/linear.py:151-155) as
a single-rank group on one GPU, in every tiling the launch can pick.

With one rank the all-reduce is the identity, so y must be F.linear(x, w)
rounded once to bf16 (the reference's output type). The tilings differ in
their epilogue: S > 1 sums a cluster's fp32 K-range partials through the
workspace before the bf16 send, S = 1 sends the accumulator straight from the
drained TMA ring. S = 1 runs when K is not a multiple of 128 (no K split
fits), when no workspace is passed, or when a cluster launch is refused.
Every call must leave the call's status word (flags[3]) and the device error
word at zero, and record the tiling that ran in flags[2].
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


class LocalOProj:
    """Buffers of a one-rank group: receive slots of both parities, arrival
    counters and the flags word, all on this GPU."""

    def __init__(self, T, N, workspace=True):
        self.T, self.N = T, N
        self.recv = torch.zeros(2 * T * N, dtype=torch.bfloat16, device=DEV)
        self.sig = torch.zeros(4, dtype=torch.int32, device=DEV)
        self.flags = torch.zeros(5, dtype=torch.int32, device=DEV)
        self.ws = torch.empty(4 * 512 * N, dtype=torch.float32, device=DEV) if workspace else None
        self.recv_ptrs = torch.tensor([self.recv.data_ptr()], dtype=torch.int64, device=DEV)
        self.sig_ptrs = torch.tensor([self.sig.data_ptr()], dtype=torch.int64, device=DEV)

    def __call__(self, x, w, y):
        from nanokv_b200 import _lib, ops
        T, K = x.shape
        ws_ptr = self.ws.data_ptr() if self.ws is not None else None
        ws_bytes = self.ws.numel() * 4 if self.ws is not None else 0
        _lib.check("nkv_oproj_allreduce_p2p", _lib.load().nkv_oproj_allreduce_p2p(
            x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), T, K, w.shape[0],
            self.recv_ptrs.data_ptr(), self.T * self.N, self.sig_ptrs.data_ptr(),
            self.sig.data_ptr(), self.flags.data_ptr(), 0, 1, 1_000_000_000,
            ws_ptr, ws_bytes, y.data_ptr(), y.stride(0), ops._stream(x.device)))


def _check(T, K, N, workspace=True, calls=3, expect_splits=None):
    from nanokv_b200 import _lib
    from nanokv_b200.layers.linear import oproj_tiling
    op = LocalOProj(T, N, workspace)
    for call in range(calls):
        g = torch.Generator(device=DEV).manual_seed(100 * call + T + K)
        x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
        y = torch.full((T, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        op(x, w, y)
        torch.cuda.synchronize()
        dev_err = _lib.read_device_error(clear=True)
        status = int(op.flags[3].item())
        tn, S, clustered = oproj_tiling(int(op.flags[2].item()))
        where = f"T={T} K={K} N={N} call {call} tiling TN={tn} S={S} clustered={clustered}"
        assert dev_err == 0 and status == 0, f"{where}: device error {dev_err}, status {status}"
        assert tn in (32, 64, 128) and S in (1, 2, 4) and clustered, where
        if expect_splits is not None:
            assert S == expect_splits, where
        ref = F.linear(x.float(), w.float())
        err = (y.float() - ref).abs()
        # one bf16 rounding of the fp32 product (half an ulp, <= 2^-8 relative)
        # plus fp32 accumulation-order slack
        tol = 2.0 ** -8 * ref.abs() + 1e-3
        assert bool((err <= tol).all()), f"{where}: max err {err.max().item()}"
        # epoch and barrier target advance once per call
        assert int(op.flags[4].item()) == call + 1, where


@pytest.mark.parametrize("T,K,N", [(32, 512, 1024), (256, 2048, 4096), (1, 4096, 4096),
                                   (129, 1024, 5120), (512, 512, 2048)])
def test_oproj_single_rank_default_tiling(cuda_lib, T, K, N):
    _check(T, K, N)


@pytest.mark.parametrize("T,K,N", [(32, 576, 1024), (200, 192, 4096), (512, 576, 1024)])
def test_oproj_single_rank_unsplit_k(cuda_lib, T, K, N):
    # K % 128 != 0: no K split divides it, so the single-CTA tiling (S = 1) runs
    _check(T, K, N, expect_splits=1)


@pytest.mark.parametrize("T,K,N", [(32, 512, 1024), (256, 2048, 4096)])
def test_oproj_single_rank_without_workspace(cuda_lib, T, K, N):
    # no split-K workspace: S = 1 even where a split would be chosen
    _check(T, K, N, workspace=False, expect_splits=1)

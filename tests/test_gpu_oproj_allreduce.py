"""The o_proj GEMM fused with the tensor-parallel all-reduce
(nkv_oproj_allreduce, replacing nanokvllm/layers/linear.py:151-155) on two
GPUs: every rank's result equals the fp32 sum over ranks of x_r @ w_r^T
within the reference's two roundings -- each rank's partial to bf16 (the
F.linear output type; our fp32 accumulation order differs from cuBLAS's, so
one bf16 ulp of each partial) and the sum to bf16 -- over consecutive calls
(both epoch parities, the buffers cleared between uses) and token counts
1..512, which select different split-K cluster shapes, in both modes
(one-shot peer stores, two-shot NVLink SHARP). Needs >= 2 GPUs (skipped
otherwise); the ranks run as spawned processes over NCCL."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, hidden, k_local, one_shot):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(repo / "nanokv-llm_b200"))
    import datetime
    import torch.distributed as dist
    import torch.nn.functional as F
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    errors = []
    try:
        from nanokv_b200 import _lib
        from nanokv_b200.layers.linear import OProjAllReduce
        op = OProjAllReduce(hidden, 512, device=dev, one_shot=one_shot)
        if one_shot is not None and op.one_shot != one_shot:
            errors.append(f"rank {rank}: asked one_shot={one_shot}, got {op.one_shot}")
        for call, T in enumerate([256, 7, 512, 256, 129]):
            g = torch.Generator(device=dev).manual_seed(1000 * call + rank)
            x = torch.randn(T, k_local, device=dev, generator=g).to(torch.bfloat16)
            w = (torch.randn(hidden, k_local, device=dev, generator=g) * 0.05).to(torch.bfloat16)
            y = op(x, w)
            try:
                op.check()  # the call's status word: no bounded wait gave up
            except RuntimeError as e:
                errors.append(f"rank {rank} call {call}: {e}")
            part = F.linear(x.float(), w.float())
            ref = part.clone()
            dist.all_reduce(ref)
            mag = part.abs()
            dist.all_reduce(mag)  # sum over ranks of |partial|
            torch.cuda.synchronize(dev)
            if _lib.read_device_error(clear=True) != 0:
                errors.append(f"rank {rank} call {call}: device error")
            err = (y.float() - ref).abs()
            # one bf16 ulp of the output (<= 2^-7 relative) + one ulp of each
            # bf16 partial (<= 2^-7 of its magnitude) + fp32 order slack
            tol = 2.0 ** -7 * ref.abs() + 2.0 ** -7 * mag + 1e-4
            if not bool((err <= tol).all()):
                errors.append(f"rank {rank} call {call} T={T}: max err {err.max().item()}")
        # every rank reaches this point and releases the symmetric (multicast-
        # bound) buffer together before any failure is raised
        torch.cuda.synchronize(dev)
        dist.barrier()
        del op
        torch.cuda.synchronize(dev)
        dist.barrier()
    finally:
        dist.destroy_process_group()
    assert not errors, errors


@pytest.mark.parametrize("hidden,k_local,one_shot", [(4096, 2048, True), (4096, 2048, False),
                                                     (5120, 1024, None), (4096, 512, False)])
def test_oproj_allreduce_two_ranks(cuda_lib, hidden, k_local, one_shot):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    torch.multiprocessing.spawn(_worker, args=(2, _free_port(), hidden, k_local, one_shot),
                                nprocs=2, join=True)

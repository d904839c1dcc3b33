"""o_proj of the attention block with its tensor-parallel all-reduce fused in.

The reference's RowParallelLinear.forward (nanokvllm/layers/linear.py:151-155)
runs F.linear on the rank's weight shard and then dist.all_reduce of the
bf16 result (NCCL). OProjAllReduce does both in ONE kernel per rank
(nkv_oproj_allreduce_p2p / nkv_oproj_allreduce): a split-K tcgen05 GEMM (a
cluster of CTAs per output tile, their fp32 partial tiles summed through an
L2-resident workspace) whose bf16 partials -- the reference's F.linear output
type -- go either into every rank's receive buffer (one-shot: one in-kernel
barrier, then a local fp32 sum in rank order) or to a symmetric buffer summed
in fp32 through NVLink SHARP (two-shot: multimem.ld_reduce, multimem.st, two
barriers).
It serves decode-sized steps (tokens <= 512); RowParallelOProj falls back to
the reference's own two calls for larger (prefill) steps or groups without
NVLink multicast.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import _lib, ops

MAX_FUSED_TOKENS = 512

# Bits of a call's status word (flags[3] of the kernel, sticky): which
# bounded wait gave up. The kernel turns the affected data into NaN instead of
# returning a plausible wrong sum.
OPROJ_STATUS_BITS = {
    1: "TMA ring slot never freed",
    2: "a stage's TMA load never landed",
    4: "accumulator never completed",
    8: "cross-rank barrier timed out",
}


def oproj_status_text(status: int) -> str:
    return ", ".join(t for b, t in OPROJ_STATUS_BITS.items() if status & b) or "ok"


def oproj_tiling(word: int) -> tuple[int, int, bool]:
    """(TN output columns per tile, S K ranges per tile, clustered) from
    flags[2]. clustered is False when the launch lacked its thread-block
    clusters (a profiler that relaunches kernels can drop them) and every
    tile therefore ran unsplit (S = 1): same result, slower."""
    w = int(word)
    return (w >> 8) & 0xFF, w & 0xFF, not (w >> 16) & 1


class OProjAllReduceError(RuntimeError):
    """A fused o_proj call whose bounded waits gave up (its output holds NaN)."""


class OProjAllReduce:
    """Fused y = all_reduce(x @ w_shard^T) for one process group.

    Two modes, one kernel (nkv_oproj_allreduce / nkv_oproj_allreduce_p2p):
    one-shot -- every rank stores its bf16 partial from the GEMM epilogue
    into every rank's receive buffer over NVLink, one in-kernel barrier, a
    local sum -- which moves (world - 1) partials per rank and suits small
    groups; and two-shot through NVLink SHARP (NVLS multicast: each rank sums
    its slice in the switch and broadcasts it, two barriers), whose traffic
    does not grow with the group. one_shot=None picks one-shot for groups of
    at most four ranks (measured faster there: 23.5 vs 34.5 us at 2 ranks,
    30.8 vs 33.6 us at 4, config 2's decode shape) and whenever the group
    has no multicast.

    Failure: a bounded wait that gives up (a rank that never arrives within
    timeout_s, or a TMA / MMA stage that never completes) sets the call's
    status word and turns the affected output into NaN. Outside CUDA-graph
    capture every call queues a 8-byte copy of (tiling, status) to pinned host
    memory; the next call (without waiting) or check() (waiting) raises
    OProjAllReduceError once it sees a nonzero status, and the object then
    refuses further calls: the ranks' counters no longer agree, so the group
    must build a new one.

    Collective construction (every rank of `group` constructs it, in the same
    order): allocates a symmetric buffer (one-shot: [2 parities][world]
    receive slots of max_tokens x hidden bf16; two-shot: bf16 partials and
    the bf16 result, max_tokens x hidden each; plus the epoch slots) and
    rendezvouses it (torch symmetric memory) for the peers' addresses and the
    multicast address. Every rank must then make the same sequence of calls;
    the call counter lives on the device, so the calls can be captured in and
    replayed from a CUDA graph.
    """

    def __init__(self, hidden: int, max_tokens: int = MAX_FUSED_TOKENS, group=None,
                 device: torch.device | None = None, timeout_s: float = 2.0,
                 one_shot: bool | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        group = group if group is not None else dist.group.WORLD
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        name = group.group_name
        E = max_tokens * hidden
        W = self.world
        sig_words = (2 * W + 3) // 4 * 4
        want_one_shot = W <= 4 if one_shot is None else bool(one_shot)
        # one-shot needs W * E words of receive slots, two-shot E words
        # (partials + result); unless two-shot was asked for, room for
        # one-shot (the fallback without multicast); epoch slots after them
        data_words = W * E if one_shot is not False else E
        self.buf = symm_mem.empty(data_words + sig_words, dtype=torch.float32, device=self.device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, name)
        offset = self.buf.data_ptr() - int(self.handle.buffer_ptrs[self.rank])
        mc = int(self.handle.multicast_ptr)
        if not want_one_shot and mc == 0:
            if one_shot is False:
                raise RuntimeError("OProjAllReduce: no NVLink multicast (NVLS) on this process group")
            want_one_shot = True
        self.one_shot = want_one_shot
        self._sig_off = 4 * data_words
        if self.one_shot:
            peers = [int(self.handle.buffer_ptrs[q]) + offset for q in range(W)]
            self.slot_stride = E
            self.recv_ptrs = torch.tensor(peers, dtype=torch.int64, device=self.device)
            self.sig_ptrs = torch.tensor([b + self._sig_off for b in peers], dtype=torch.int64,
                                         device=self.device)
        else:
            self.mc_base = mc + offset
            self._part_off, self._out_off = 0, 2 * E
        # [barrier 1 target, barrier 2 target, tiling, status, epoch]
        self.flags = torch.zeros(5, dtype=torch.int32, device=self.device)
        self._status_host = torch.zeros(2, dtype=torch.int32, pin_memory=True)
        self._status_event = None
        self.failed = 0
        # split-K partial tiles: up to 4 K ranges x max_tokens (rounded up to
        # 128-row tiles) x hidden fp32, L2-resident at decode sizes
        self.workspace = torch.empty(4 * ((max_tokens + 127) // 128 * 128) * hidden,
                                     dtype=torch.float32, device=self.device)
        self.timeout_ns = int(timeout_s * 1e9)
        torch.cuda.synchronize(self.device)
        dist.barrier(group)

    def _poll(self, wait: bool) -> None:
        ev = self._status_event
        if ev is None:
            return
        if wait:
            ev.synchronize()
        elif not ev.query():
            return
        self._status_event = None
        st = int(self._status_host[1])
        if st:
            self.failed = st
            raise OProjAllReduceError(
                f"rank {self.rank}: fused o_proj + all-reduce failed ({oproj_status_text(st)}); "
                "its output is NaN and this object must be rebuilt")

    def check(self) -> None:
        """Raises OProjAllReduceError if any call so far gave up a wait
        (synchronises with the last call, and reads the device status word
        itself, so it also covers calls replayed from a CUDA graph)."""
        if self.failed:
            raise OProjAllReduceError(f"rank {self.rank}: an earlier call failed "
                                      f"({oproj_status_text(self.failed)})")
        self._poll(wait=True)
        st = int(self.flags[3].item())
        if st:
            self.failed = st
            raise OProjAllReduceError(
                f"rank {self.rank}: fused o_proj + all-reduce failed ({oproj_status_text(st)})")

    def tiling(self) -> tuple[int, int, bool]:
        """(TN, S, clustered) of the last call's launch (synchronises)."""
        return oproj_tiling(int(self.flags[2].item()))

    def __call__(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None):
        if self.failed:
            raise OProjAllReduceError(f"rank {self.rank}: an earlier call failed "
                                      f"({oproj_status_text(self.failed)}); rebuild the object")
        capturing = torch.cuda.is_current_stream_capturing()
        if not capturing:
            self._poll(wait=False)
        out = self._launch(x, w, out)
        if not capturing:
            self._status_host.copy_(self.flags[2:4], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(x.device))
            self._status_event = ev
        return out

    def _launch(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None):
        T, K = x.shape
        N = w.shape[0]
        assert N == self.hidden and T <= self.max_tokens and w.shape[1] == K
        assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
        assert x.stride(-1) == 1 and w.stride(-1) == 1
        if out is None:
            out = torch.empty(T, N, dtype=torch.bfloat16, device=x.device)
        assert out.stride(-1) == 1
        base = self.buf.data_ptr()
        lib = _lib.load()
        if self.one_shot:
            _lib.check("nkv_oproj_allreduce_p2p", lib.nkv_oproj_allreduce_p2p(
                x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), T, K, N,
                self.recv_ptrs.data_ptr(), self.slot_stride, self.sig_ptrs.data_ptr(),
                base + self._sig_off, self.flags.data_ptr(), self.rank, self.world,
                self.timeout_ns, self.workspace.data_ptr(), self.workspace.numel() * 4,
                out.data_ptr(), out.stride(0), ops._stream(x.device)))
            return out
        mc = self.mc_base
        _lib.check("nkv_oproj_allreduce", lib.nkv_oproj_allreduce(
            x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), T, K, N,
            mc + self._part_off, base + self._part_off, mc + self._out_off, base + self._out_off,
            mc + self._sig_off, base + self._sig_off, self.flags.data_ptr(), self.rank,
            self.world, self.timeout_ns, self.workspace.data_ptr(), self.workspace.numel() * 4,
            out.data_ptr(), out.stride(0), ops._stream(x.device)))
        return out


class RowParallelOProj:
    """Drop-in forward of the attention block's o_proj (RowParallelLinear
    without bias, nanokvllm/layers/linear.py:133-155): with fused=True the
    fused kernel for decode-sized steps, otherwise (and for larger steps) the
    reference's F.linear + dist.all_reduce. The fused kernel is opt-in."""

    def __init__(self, weight: torch.Tensor, group=None, max_tokens: int = MAX_FUSED_TOKENS,
                 fused: bool = False):
        self.weight = weight
        self.group = group
        self.fused = None
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        if fused and world > 1:
            try:
                self.fused = OProjAllReduce(weight.shape[0], max_tokens, group, weight.device)
            except RuntimeError:
                self.fused = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused is not None and x.size(0) <= self.fused.max_tokens:
            return self.fused(x, self.weight)
        y = F.linear(x, self.weight)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(y, group=self.group)
        return y

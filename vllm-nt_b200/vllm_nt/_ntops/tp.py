"""Row-parallel projection with its all-reduce over peer memory (tensor parallelism).

Under TP, vLLM's RowParallelLinear (o_proj, down) computes a partial product on every
rank and sums the partials with an NCCL all-reduce
(vllm:model_executor/layers/linear.py, RowParallelLinear.forward ->
tensor_model_parallel_all_reduce).  Here the GEMM writes its partial into local memory and
``ntb200_allreduce_oneshot`` pushes it over NVLink into every rank's peer-mapped buffer
(torch symmetric memory), meets the other ranks at one barrier and sums the pushed
partials; for larger messages ``ntb200_allreduce_twoshot`` reduce-scatters and
all-gathers over the same buffers instead.  Two kernels of this library back to back (the
second launched as a programmatic dependent of the first), no NCCL call.

Every rank must make the same sequence of calls on its buffer.  The call count lives in
the buffer on the device, so the GEMM + all-reduce pair can be captured in a CUDA graph.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from vllm_nt._ntops.torch._ext import ops


class PeerAllReduce:
    """A peer-mapped buffer for ``capacity`` bf16/f16 elements per rank."""

    def __init__(self, group: dist.ProcessGroup | None, capacity: int, device: torch.device | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.capacity = int(capacity)
        world = dist.get_world_size(self.group)
        nbytes = int(ops().allreduce_buffer_size(self.capacity, 2, world))
        self.buffer = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.buffer.zero_()
        torch.cuda.synchronize(self.device)
        self.handle = symm_mem.rendezvous(self.buffer, self.group)
        self.rank = int(self.handle.rank)
        self.world_size = int(self.handle.world_size)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=self.device)
        # The one-shot push moves (W-1) x bytes per rank over NVLink and needs one barrier;
        # the two-shot form moves 2 (W-1)/W x bytes and needs two.  Measured on B200s (GEMM +
        # all-reduce of a [M, 4096] bf16 partial): at 8 ranks the one-shot is fastest up to
        # 1 MB (13 us at 8 KB against 32 us for NCCL) and the two-shot from 8 MB (60 against
        # 82 us at 8 MB, 266 against 320 us at 64 MB); at 2 ranks the one-shot is ahead at
        # every size measured.  Hence one-shot up to 8 MB / (W - 1), two-shot beyond, NCCL
        # past the buffer's capacity.
        self.oneshot_max_bytes = (8 << 20) // max(1, self.world_size - 1)
        # no rank may write a peer's flags before every rank has cleared its own buffer
        dist.barrier(group=self.group)

    def method_for(self, partial: torch.Tensor) -> str:
        """The path ``reduce`` takes for ``partial`` by default; the same on every rank,
        since the sizes are."""
        if partial.numel() > self.capacity:
            return "nccl"
        if partial.numel() * partial.element_size() <= self.oneshot_max_bytes or partial.numel() % 8:
            return "oneshot"
        return "twoshot"

    def reduce(self, partial: torch.Tensor, out: torch.Tensor | None = None, oneshot: bool | None = None,
               method: str | None = None, check: bool = False) -> torch.Tensor:
        """Sums ``partial`` (contiguous) over all ranks into ``out``.  ``method`` is
        "oneshot", "twoshot" or "nccl" (default: ``method_for``); ``oneshot=True/False`` is
        the older spelling of "oneshot"/"nccl".  Every rank must call with the same method.

        A peer that does not reach a call within ~2 s makes the kernel give up the wait: it
        sets the device error word (NTB200_DEVERR_WAIT_TIMEOUT) and ``out`` is then not the
        sum.  Read the word at a step boundary (``capi.read_device_error``), or pass
        ``check=True``, which synchronises the stream after the call and raises on it."""
        if out is None:
            out = torch.empty_like(partial)
        if method is None:
            method = self.method_for(partial) if oneshot is None else ("oneshot" if oneshot else "nccl")
        if method != "nccl" and partial.numel() > self.capacity:
            method = "nccl"
        if method == "twoshot" and partial.numel() % 8:
            method = "oneshot"
        if method == "nccl":
            out.copy_(partial)
            dist.all_reduce(out, group=self.group)
            return out
        fn = ops().allreduce_twoshot if method == "twoshot" else ops().allreduce_oneshot
        fn(out, partial, self.peers, self.capacity, self.rank, self.world_size)
        if check:
            from vllm_nt._ntops import capi

            word = capi.read_device_error(torch.cuda.current_stream(self.device).cuda_stream)
            if word & capi.DEVERR_WAIT_TIMEOUT:
                raise RuntimeError(f"peer all-reduce on rank {self.rank}: a peer did not arrive (device error {word})")
        return out

    def linear(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
               out: torch.Tensor | None = None, partial: torch.Tensor | None = None) -> torch.Tensor:
        """sum over ranks of x_r @ weight_r^T, plus bias once (on rank 0, as vLLM's
        RowParallelLinear adds it before the reduction).  ``partial`` and ``out`` may be
        given to keep the call free of allocations (e.g. for CUDA-graph capture)."""
        shape = (*x.shape[:-1], weight.shape[0])
        if partial is None:
            partial = x.new_empty(shape)
        ops().linear(partial, x, weight, bias if self.rank == 0 else None, None)
        return self.reduce(partial, out)

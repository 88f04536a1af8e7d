"""One rank of the peer-memory all-reduce test (run by tests/test_tp_allreduce_gpu.py
under torch.distributed.run, one process per GPU).

Each rank computes a row-parallel projection through PeerAllReduce (our GEMM, then the
one-shot and the two-shot all-reduce over peer memory, alternating on one buffer) and
compares it with the same partials summed by NCCL: bf16 partial per rank, bias on rank 0,
as vLLM's RowParallelLinear does.  Exits non-zero on a mismatch or a device-side timeout."""

import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "vllm-nt_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    from vllm_nt._ntops import capi
    from vllm_nt._ntops.torch._ext import ops
    from vllm_nt._ntops.tp import PeerAllReduce

    stream = torch.cuda.current_stream().cuda_stream
    capi.read_device_error(stream)
    par = PeerAllReduce(None, capacity=256 * 4096)
    # decode and odd shapes; the same (M, N) twice in a row and alternating slots
    cases = [(1, 4096, 4096), (256, 14336, 4096), (37, 520, 264), (256, 4096, 4096), (3, 64, 8), (256, 4096, 4096),
             (128, 14336, 4096)]
    bad = []
    for step, (m, k_total, n) in enumerate(cases + [(256, 4096, 4096)]):
        k = max(8, (k_total // world) // 8 * 8)
        g = torch.Generator().manual_seed(1000 * step + rank)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        w = (0.05 * torch.randn(n, k, generator=g)).to(torch.bfloat16).to(dev)
        b = torch.randn(n, generator=torch.Generator().manual_seed(step)).to(torch.bfloat16).to(dev)
        partial = x.new_empty(m, n)
        ops().linear(partial, x, w, b if rank == 0 else None, None)
        # the same partial through both kernels, alternating which goes first
        methods = ("oneshot", "twoshot") if step % 2 == 0 else ("twoshot", "oneshot")
        outs = {meth: par.reduce(partial, method=meth) for meth in methods if meth == "oneshot" or m * n % 8 == 0}
        ref = x.float() @ w.float().t()
        if rank == 0:
            ref = ref + b.float()
        ref = ref.to(torch.bfloat16).float()
        # the partials are rounded to bf16 on each rank (ours by the GEMM, the reference by
        # torch) and may differ by a rounding step where the fp32 sums differ in order; the
        # error bound therefore scales with the partials' magnitudes, not the sum's
        mag = ref.abs()
        dist.all_reduce(ref)
        dist.all_reduce(mag)
        torch.cuda.synchronize()
        for meth, out in outs.items():
            d = (out.float() - ref).abs()
            off = int((d > 2e-2 + 2e-2 * mag).sum())
            if off:
                bad.append(f"case {step} {(m, k, n)} {meth}: max |diff| {d.max().item():.3g}, "
                           f"{off} of {d.numel()} outside 0.02 + 0.02 * sum|partial|")
        if len(outs) == 2 and not torch.equal(outs["oneshot"], outs["twoshot"]):
            bad.append(f"case {step}: one-shot and two-shot sums differ")
    # the GEMM + all-reduce pair captured once in a CUDA graph and replayed on new inputs
    m, k, n = 64, max(8, (4096 // world) // 8 * 8), 4096
    xs = torch.empty(m, k, dtype=torch.bfloat16, device=dev)
    ws = (0.05 * torch.randn(n, k, generator=torch.Generator().manual_seed(99 + rank))).to(torch.bfloat16).to(dev)
    xs.normal_()
    gout = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    gpart = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    gout2 = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    par.linear(xs, ws, out=gout, partial=gpart)  # warm-up outside the capture
    par.reduce(gpart, gout2, method="twoshot")
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):  # both kernels, one after the other, in one graph
        par.linear(xs, ws, out=gout, partial=gpart)
        par.reduce(gpart, gout2, method="twoshot")
    for rep in range(3):
        xs.copy_(torch.randn(m, k, generator=torch.Generator().manual_seed(500 + 10 * rep + rank)).to(torch.bfloat16))
        dist.barrier()
        graph.replay()
        ref = (xs.float() @ ws.float().t()).to(torch.bfloat16).float()
        mag = ref.abs()
        dist.all_reduce(ref)
        dist.all_reduce(mag)
        torch.cuda.synchronize()
        d = (gout.float() - ref).abs()
        off = int((d > 2e-2 + 2e-2 * mag).sum())
        if off:
            bad.append(f"graph replay {rep}: {off} of {d.numel()} off, max |diff| {d.max().item():.3g}")
        if not torch.equal(gout, gout2):
            bad.append(f"graph replay {rep}: two-shot differs from one-shot")
    del graph
    word = capi.read_device_error(stream)
    if word:
        bad.append(f"device error word {word}")
    flags = torch.tensor([len(bad)], device=dev)
    dist.all_reduce(flags)
    print(f"rank {rank}/{world}: {'OK' if not bad else bad}", flush=True)
    del par
    dist.destroy_process_group()
    return 0 if int(flags.item()) == 0 else 1


if __name__ == "__main__":
    sys.exit(main())

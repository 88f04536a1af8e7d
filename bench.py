#!/usr/bin/env python
"""Benchmark of the vllm_nt B200 hot path.

Headline (one JSON line on rank 0): paged-attention decode throughput in tokens/s for the
decode workload -- 256 sequences x one query token, 32 query / 8 KV heads, head 128,
block 16, context lengths U[512, 8192], distinct block ids from a 150000-block pool, bf16
with fp32 softmax -- sharded across the N ranks by KV head (rank r owns KV heads
[r*8/N, (r+1)*8/N) of the pool and their query heads; no collective on the data path).
A step is one decode call over the whole batch; value = 256 * steps / (max over ranks of
the device time of the timed steps).

Also reported: the roofline of the decode kernel against measured HBM bandwidth, the
end-to-end rate through the plugin's public decode entry point with host buffers, the
oracle's CPU rate on a bounded sample, clocks sampled during the timed region, and (at
N = 1) a per-op table: achieved HBM GB/s for every memory-bound op at its benchmark
config and tensor TFLOP/s for the projection GEMM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-ops]
"""

from __future__ import annotations

import argparse
import itertools
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "vllm-nt_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "per-op HBM GB/s (% of B200 peak); paged-attn decode tok/s at 1/2/4/8 GPUs"
BATCH, HQ, HKV, HEAD, BLOCK, POOL, CTX_LO, CTX_HI, MAX_BLOCKS = 256, 32, 8, 128, 16, 150000, 512, 8192, 512
L2_BYTES = 126 * 1024 * 1024


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def workload(seed: int = 0, batch: int = BATCH, pool: int = POOL):
    """Context lengths and block tables of the decode workload (CPU, deterministic)."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(CTX_LO, CTX_HI + 1, (BATCH,), generator=g)
    q = torch.randn(BATCH, HQ, HEAD, generator=g).to(torch.bfloat16)
    ctx, q = ctx[:batch], q[:batch]
    nblk = (ctx + BLOCK - 1) // BLOCK
    if int(nblk.sum()) > pool:
        raise SystemExit(f"--pool {pool} is smaller than the {int(nblk.sum())} blocks the batch needs")
    ids = torch.randperm(pool, generator=g)[: int(nblk.sum())].to(torch.int32)
    table = torch.zeros(batch, MAX_BLOCKS, dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk.tolist()):
        table[i, :n] = ids[off : off + n]
        off += n
    return ctx.to(torch.int32), table, q


def decode_bytes(ctx: torch.Tensor, hkv_local: int) -> int:
    """Algorithmic HBM bytes of one decode call: every cached K and V row of the local
    heads once, q and out once, the block-table entries used and the sequence lengths."""
    batch = ctx.shape[0]
    tokens = int(ctx.sum())
    blocks = int(((ctx + BLOCK - 1) // BLOCK).sum())
    hq_local = hkv_local * (HQ // HKV)
    return tokens * hkv_local * HEAD * 2 * 2 + 2 * batch * hq_local * HEAD * 2 + blocks * 4 + batch * 4


class ClockSampler:
    """nvidia-smi sampling (200 ms) of SM clock and throttle reasons during the run."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"ntb200_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        power = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        loaded = [s for s, p in zip(sm, power) if p > 300.0] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": smax,
            "reasons": reasons,
            "samples": len(rows),
            "samples_under_load": len([p for p in power if p > 300.0]),
        }


def traffic_from_profile() -> float | None:
    """Per-launch DRAM bytes of the decode split kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "paged_decode_split_b256.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# --------------------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle on a bounded sample of sequences
# --------------------------------------------------------------------------------------


def oracle_decode_rate(ctx, q, seqs_per_call: int, calls: int, seed: int = 1) -> tuple[float, int, str]:
    """Times oracle.paged_decode over `calls` calls of `seqs_per_call` sequences each
    (K/V of each sampled sequence generated ~N(0,1) in a local paged cache).  Returns
    (tokens/s, threads, sample description)."""
    import oracle

    g = torch.Generator().manual_seed(seed)
    order = torch.randperm(BATCH, generator=g).tolist()
    total_t = 0.0
    done = 0
    k = 0
    for _ in range(calls):
        pick = [order[(k + i) % BATCH] for i in range(seqs_per_call)]
        k += seqs_per_call
        lens = ctx[pick]
        nblk = int(((lens + BLOCK - 1) // BLOCK).sum())
        kc = torch.randn(nblk, BLOCK, HKV, HEAD, generator=g).to(torch.bfloat16)
        vc = torch.randn(nblk, BLOCK, HKV, HEAD, generator=g).to(torch.bfloat16)
        table = torch.zeros(len(pick), MAX_BLOCKS, dtype=torch.int32)
        off = 0
        for i, n in enumerate(((lens + BLOCK - 1) // BLOCK).tolist()):
            table[i, :n] = torch.arange(off, off + n, dtype=torch.int32)
            off += n
        t0 = time.perf_counter()
        oracle.paged_decode(q[pick], kc, vc, lens, table, 1.0 / math.sqrt(HEAD))
        total_t += time.perf_counter() - t0
        done += len(pick)
    sample = f"{done} sequences of the decode workload ({calls} calls x {seqs_per_call}), torch CPU oracle"
    return done / total_t, torch.get_num_threads(), sample


def run_reference(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    ctx, table, q = workload()
    # size each step so warmup + steps take about two minutes
    t_one, _, _ = oracle_decode_rate(ctx, q, 1, 1)
    budget = 120.0 / max(1, args.steps + args.warmup)
    per_step = max(1, min(BATCH, int(budget * t_one)))
    oracle_decode_rate(ctx, q, per_step, args.warmup)
    value, threads, sample = oracle_decode_rate(ctx, q, per_step, args.steps, seed=2)
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": value,
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * per_step / value,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(n: int) -> dict:
    return {
        "workload": "paged decode 256 seqs x 1 tok, 32q/8kv heads, d128, block 16, ctx U[512,8192], "
        "150000-block pool, bf16",
        "global_batch": BATCH,
        "seq_len": "U[512,8192]",
        "parallelism": f"kv-head shard x{n}" if n > 1 else "single GPU",
        "kv_heads_per_gpu": HKV // n,
        "l2": "inputs > L2 (>=570 MB K/V per step per GPU)",
    }


# --------------------------------------------------------------------------------------
# per-op table (N = 1)
# --------------------------------------------------------------------------------------


def time_graph(fn_list, iters: int) -> float:
    """Average device ms per call of a round-robin over fn_list, captured in a CUDA graph
    (launch gaps minimal); the set of buffers the calls touch exceeds L2."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fn_list:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(iters):
            fn_list[i % len(fn_list)]()
    graph.replay()
    torch.cuda.synchronize()
    # best of 5 replays (each replay = `iters` launches timed with CUDA events)
    best = float("inf")
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) / iters)
    return best


def per_op_table(dev, peaks) -> dict:
    from vllm_nt._ntops.torch._ext import ops

    o = ops()
    hbm = peaks["hbm_gbs"]
    tens = peaks["bf16_tflops"]
    g = torch.Generator(device=dev).manual_seed(7)
    res = {}

    def copies(nbytes):
        return max(2, math.ceil(3 * L2_BYTES / nbytes))

    def report(name, nbytes, ms, extra=None):
        gbs = nbytes / (ms * 1e-3) / 1e9
        d = {"bytes": nbytes, "us": ms * 1e3, "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 3)}
        if extra:
            d.update(extra)
        res[name] = d

    # The same shapes through the kernels vLLM itself ships (its _C extension, cuBLAS via
    # F.linear, F.embedding): reported beside ours for comparison only.
    try:
        import vllm._custom_ops as vops
    except Exception:  # noqa: BLE001 - the comparison column is optional
        vops = None

    def floor(name, fn):
        """The same kernel on a single-row input: what one launch costs with no data to
        move (CUDA graph of back-to-back launches)."""
        res[name]["floor_us"] = round(time_graph([fn], 40) * 1e3, 2)

    def lib(name, label, fns, iters):
        if fns is None:
            return
        try:
            us = time_graph(fns, iters) * 1e3
        except Exception as exc:  # noqa: BLE001
            res[name]["lib"] = f"{label}: unavailable ({type(exc).__name__})"
            return
        res[name]["lib"] = label
        res[name]["lib_us"] = round(us, 2)
        res[name]["ours_vs_lib"] = round(us / res[name]["us"], 3)

    # (a) fused_add_rms_norm fp32 [128, 4096]
    M, H = 128, 4096
    nb = 4 * M * H * 4 + H * 4
    r = copies(nb)
    xs = [torch.randn(M, H, device=dev, generator=g) for _ in range(r)]
    rs = [torch.randn(M, H, device=dev, generator=g) for _ in range(r)]
    w = 1 + 0.1 * torch.randn(H, device=dev, generator=g)
    outs = [torch.empty(M, H, device=dev) for _ in range(r)]
    fns = [lambda i=i: o.fused_add_rms_norm(outs[i], rs[i], xs[i], w, 1e-6) for i in range(r)]
    report("fused_add_rms_norm f32 [128,4096]", nb, time_graph(fns, 20 * r))
    floor("fused_add_rms_norm f32 [128,4096]", lambda: o.fused_add_rms_norm(outs[0][:1], rs[0][:1], xs[0][:1], w, 1e-6))
    lib("fused_add_rms_norm f32 [128,4096]", "vllm _C.fused_add_rms_norm (in place)",
        vops and [lambda i=i: vops.fused_add_rms_norm(xs[i], rs[i], w, 1e-6) for i in range(r)], 20 * r)
    # bf16 M-sweep point at a size where launch latency no longer dominates
    M2 = 8192
    nb2 = 4 * M2 * H * 2 + H * 2
    r2 = copies(nb2)
    xs2 = [torch.randn(M2, H, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(r2)]
    rs2 = [torch.randn(M2, H, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(r2)]
    w2 = w.to(torch.bfloat16)
    outs2 = [torch.empty_like(xs2[0]) for _ in range(r2)]
    fns = [lambda i=i: o.fused_add_rms_norm(outs2[i], rs2[i], xs2[i], w2, 1e-6) for i in range(r2)]
    report("fused_add_rms_norm bf16 [8192,4096]", nb2, time_graph(fns, 10 * r2))
    lib("fused_add_rms_norm bf16 [8192,4096]", "vllm _C.fused_add_rms_norm (in place)",
        vops and [lambda i=i: vops.fused_add_rms_norm(xs2[i], rs2[i], w2, 1e-6) for i in range(r2)], 10 * r2)
    del xs, rs, outs, xs2, rs2, outs2

    # (b) silu_and_mul fp32 [128,22016] -> [128,11008]
    nb = 128 * 22016 * 4 + 128 * 11008 * 4
    r = copies(nb)
    xs = [torch.randn(128, 22016, device=dev, generator=g) for _ in range(r)]
    outs = [torch.empty(128, 11008, device=dev) for _ in range(r)]
    fns = [lambda i=i: o.silu_and_mul(outs[i], xs[i]) for i in range(r)]
    report("silu_and_mul f32 [128,22016]", nb, time_graph(fns, 20 * r))
    floor("silu_and_mul f32 [128,22016]", lambda: o.silu_and_mul(outs[0][:1], xs[0][:1]))
    lib("silu_and_mul f32 [128,22016]", "vllm _C.silu_and_mul",
        vops and [lambda i=i: torch.ops._C.silu_and_mul(outs[i], xs[i]) for i in range(r)], 20 * r)
    del xs, outs

    # (c) RoPE fp32 q [128,32,128], k [128,8,128], positions U[0,4096)
    T = 128
    nb = 2 * T * (32 + 8) * 128 * 4 + T * 128 * 4 + T * 8
    r = copies(nb)
    qs = [torch.randn(T, 32, 128, device=dev, generator=g) for _ in range(r)]
    ks = [torch.randn(T, 8, 128, device=dev, generator=g) for _ in range(r)]
    pos = [torch.randint(0, 4096, (T,), device=dev, generator=g) for _ in range(r)]
    import oracle

    cache = oracle.build_cos_sin_cache(128, 4096, 10000.0).to(dev)
    fns = [lambda i=i: o.rotary_embedding_neox(pos[i], qs[i], ks[i], cache, 128, 128) for i in range(r)]
    report("rope_neox f32 q[128,32,128] k[128,8,128]", nb, time_graph(fns, 20 * r))
    floor("rope_neox f32 q[128,32,128] k[128,8,128]",
          lambda: o.rotary_embedding_neox(pos[0][:1], qs[0][:1], ks[0][:1], cache, 128, 128))
    lib("rope_neox f32 q[128,32,128] k[128,8,128]", "vllm _C.rotary_embedding (neox)",
        vops and [lambda i=i: vops.rotary_embedding(pos[i], qs[i], ks[i], 128, cache, True) for i in range(r)],
        20 * r)
    del qs, ks

    # KV store bf16: 4096 tokens x 8 x 128 into [8192,16,8,128] caches, distinct slots
    N = 4096
    nb = 2 * N * 8 * 128 * 2 * 2 + N * 8
    kc = torch.zeros(8192, 16, 8, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    r = copies(nb)
    keys = [torch.randn(N, 8, 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(r)]
    vals = [torch.randn(N, 8, 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(r)]
    slots = [torch.randperm(8192 * 16, device=dev, generator=g)[:N] for _ in range(r)]
    fns = [lambda i=i: o.reshape_and_cache(keys[i], vals[i], kc, vc, slots[i]) for i in range(r)]
    report("reshape_and_cache bf16 4096x8x128", nb, time_graph(fns, 20 * r))
    floor("reshape_and_cache bf16 4096x8x128", lambda: o.reshape_and_cache(keys[0][:1], vals[0][:1], kc, vc, slots[0][:1]))
    one = torch.ones((), device=dev)
    lib("reshape_and_cache bf16 4096x8x128", "vllm _C_cache_ops.reshape_and_cache_flash",
        vops and [lambda i=i: vops.reshape_and_cache_flash(keys[i], vals[i], kc, vc, slots[i], "auto", one, one)
                  for i in range(r)], 20 * r)
    del keys, vals, kc, vc

    # embedding bf16: 4096 ids into a [128256, 4096] table
    Tn = 4096
    wt = torch.randn(128256, 4096, device=dev, generator=g, dtype=torch.bfloat16)
    ids = [torch.randint(0, 128256, (Tn,), device=dev, generator=g) for _ in range(8)]
    outs = [torch.empty(Tn, 4096, device=dev, dtype=torch.bfloat16) for _ in range(8)]
    nb = 2 * Tn * 4096 * 2 + Tn * 8
    fns = [lambda i=i: o.embedding(outs[i], ids[i], wt) for i in range(8)]
    report("embedding bf16 4096 ids x 4096", nb, time_graph(fns, 80))
    lib("embedding bf16 4096 ids x 4096", "torch F.embedding",
        [lambda i=i: torch.nn.functional.embedding(ids[i], wt) for i in range(8)], 80)
    del wt, outs

    # the same kernels at prefill-sized inputs, where launch latency no longer hides the
    # bandwidth: silu_and_mul on a 2048-token gate_up output, RoPE over 16384 tokens of
    # a qkv buffer, the KV store of 16384 tokens
    xs3 = [torch.randn(2048, 28672, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(2)]
    outs3 = [torch.empty(2048, 14336, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    nb = 2048 * 28672 * 2 + 2048 * 14336 * 2
    report("silu_and_mul bf16 [2048,28672]", nb, time_graph([lambda i=i: o.silu_and_mul(outs3[i], xs3[i])
                                                            for i in range(2)], 10))
    lib("silu_and_mul bf16 [2048,28672]", "vllm _C.silu_and_mul",
        vops and [lambda i=i: torch.ops._C.silu_and_mul(outs3[i], xs3[i]) for i in range(2)], 10)
    del xs3, outs3
    T3 = 16384
    qkv3 = [torch.randn(T3, 48 * 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(2)]
    pos3 = torch.randint(0, 4096, (T3,), device=dev, generator=g)
    cache3 = cache.to(torch.bfloat16)
    nb = 2 * T3 * 40 * 128 * 2 + T3 * 128 * 2 + T3 * 8
    report("rope_neox bf16 16384 tokens of qkv [T,48*128]", nb,
           time_graph([lambda i=i: o.rotary_embedding_neox(pos3, qkv3[i][:, :4096], qkv3[i][:, 4096:5120], cache3,
                                                           128, 128) for i in range(2)], 10))
    lib("rope_neox bf16 16384 tokens of qkv [T,48*128]", "vllm _C.rotary_embedding (neox)",
        vops and [lambda i=i: vops.rotary_embedding(pos3, qkv3[i][:, :4096], qkv3[i][:, 4096:5120], 128, cache3, True)
                  for i in range(2)], 10)
    del qkv3
    kc3 = torch.zeros(8192, 16, 8, 128, device=dev, dtype=torch.bfloat16)
    vc3 = torch.zeros_like(kc3)
    k3 = [torch.randn(T3, 8, 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(2)]
    v3 = [torch.randn(T3, 8, 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(2)]
    sl3 = torch.randperm(8192 * 16, device=dev, generator=g)[:T3]
    nb = 2 * T3 * 8 * 128 * 2 * 2 + T3 * 8
    report("reshape_and_cache bf16 16384x8x128", nb,
           time_graph([lambda i=i: o.reshape_and_cache(k3[i], v3[i], kc3, vc3, sl3) for i in range(2)], 10))
    del kc3, vc3, k3, v3

    def rope_cache_rows():
        # RoPE fused with the KV store (one kernel) beside the two kernels it replaces (ours,
        # and vLLM's _C pair), for a Llama-3-8B layer: qkv [T, 48*128] bf16, FlashAttention
        # cache [2, 8192, 16, 8, 128], a decode step (256 tokens) and a prefill chunk (16384).
        # Bytes: q and k read and written, v read, rotated k and v written to the cache,
        # cos/sin rows, positions and slots.
        kv4 = torch.zeros(2, 8192, 16, 8, 128, device=dev, dtype=torch.bfloat16)
        for T4, iters4 in ((256, 20), (16384, 2)):
            nb = 2 * T4 * 40 * 128 * 2 + T4 * 8 * 128 * 2 + 2 * T4 * 8 * 128 * 2 + T4 * 128 * 2 + T4 * 16
            r4 = copies(nb)
            qkv4 = [torch.randn(T4, 48 * 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(r4)]
            pos4 = [torch.randint(0, 4096, (T4,), device=dev, generator=g) for _ in range(r4)]
            sl4 = [torch.randperm(8192 * 16, device=dev, generator=g)[:T4] for _ in range(r4)]
            parts = [(x[:, :4096], x[:, 4096:5120], x[:, 5120:]) for x in qkv4]
            name = f"rope_and_cache bf16 {T4} tokens of qkv [T,48*128]"
            report(name, nb, time_graph([lambda i=i: o.rope_and_cache_flash_layout(
                pos4[i], *parts[i], cache3, kv4, sl4[i], 128, 128, 0) for i in range(r4)], iters4 * r4))

            def unfused(i):
                q4, k4, v4 = parts[i]
                o.rotary_embedding_neox(pos4[i], q4, k4, cache3, 128, 128)
                o.store_flash_layout(k4, v4, kv4, sl4[i], 0)

            us = time_graph([lambda i=i: unfused(i) for i in range(r4)], iters4 * r4) * 1e3
            res[name]["unfused_us"] = round(us, 2)
            res[name]["unfused_vs_fused"] = round(us / res[name]["us"], 3)

            def vllm_pair(i):
                q4, k4, v4 = parts[i]
                vops.rotary_embedding(pos4[i], q4, k4, 128, cache3, True)
                vops.reshape_and_cache_flash(k4.view(T4, 8, 128), v4.view(T4, 8, 128), kv4[0], kv4[1], sl4[i], "auto",
                                             one, one)

            lib(name, "vllm _C rotary_embedding + reshape_and_cache_flash",
                vops and [lambda i=i: vllm_pair(i) for i in range(r4)], iters4 * r4)
            del qkv4, parts
        del kv4

    def sampler_rows():
        # sampler at a decode batch of 256 over the Llama-3 vocabulary (fp32 logits, as vLLM's
        # sampler holds them): the top-k/top-p mask (k = 50, p = 0.9 on every row) and the
        # exponential-race sample.  The mask works in place, so each call first restores its
        # logits from a pristine copy; the copy is timed alone and subtracted.  Algorithmic
        # bytes: the logits read once and written once (mask); probs and q read once (sample).
        B5, V5 = 256, 128256
        src5 = torch.randn(B5, V5, device=dev, generator=g) * 2
        lg5 = torch.empty_like(src5)
        k5 = torch.full((B5,), 50, device=dev, dtype=torch.int32)
        p5 = torch.full((B5,), 0.9, device=dev)
        copy_us = time_graph([lambda: lg5.copy_(src5)], 10) * 1e3
        name = "top_k_top_p f32 [256,128256] k=50 p=0.9"
        us = time_graph([lambda: (lg5.copy_(src5), o.top_k_top_p(lg5, k5, p5))], 10) * 1e3 - copy_us
        report(name, 2 * B5 * V5 * 4, us * 1e-3, {"note": "radix select, ~8 passes over each row (L2/HBM)"})
        try:
            from vllm.v1.sample.ops.topk_topp_sampler import apply_top_k_top_p_pytorch
            from vllm.v1.sample.ops.topk_topp_triton import apply_top_k_top_p_triton

            t_us = time_graph([lambda: (lg5.copy_(src5), apply_top_k_top_p_triton(lg5, k5, p5))], 10) * 1e3 - copy_us
            res[name].update(lib="vllm apply_top_k_top_p_triton (vLLM's choice for batch >= 8)", lib_us=round(t_us, 2),
                             ours_vs_lib=round(t_us / res[name]["us"], 3))
            s_us = time_graph([lambda: (lg5.copy_(src5), apply_top_k_top_p_pytorch(lg5, k5, p5))], 3) * 1e3 - copy_us
            res[name].update(sort_us=round(s_us, 2), ours_vs_sort=round(s_us / res[name]["us"], 3),
                             sort="torch sort + cumsum + scatter (the reference's algorithm, on the GPU)")
        except Exception as exc:  # noqa: BLE001 - the comparison columns are optional
            res[name]["lib"] = f"unavailable ({type(exc).__name__}: {exc})"[:200]
        # a small decode batch (4 rows): one cluster of CTAs per row
        lg4, src4 = torch.empty_like(src5[:4]), src5[:4].clone()
        k4, p4 = k5[:4].clone(), p5[:4].clone()
        copy4 = time_graph([lambda: lg4.copy_(src4)], 10) * 1e3
        name = "top_k_top_p f32 [4,128256] k=50 p=0.9"
        us = time_graph([lambda: (lg4.copy_(src4), o.top_k_top_p(lg4, k4, p4))], 10) * 1e3 - copy4
        report(name, 2 * 4 * V5 * 4, us * 1e-3, {"note": "one cluster of 8 CTAs per row, row slices in shared memory"})
        try:
            from vllm.v1.sample.ops.topk_topp_sampler import apply_top_k_top_p_pytorch

            s_us = time_graph([lambda: (lg4.copy_(src4), apply_top_k_top_p_pytorch(lg4, k4, p4))], 3) * 1e3 - copy4
            res[name].update(lib="vllm apply_top_k_top_p_pytorch (torch sort + cumsum + scatter)", lib_us=round(s_us, 2),
                             ours_vs_lib=round(s_us / res[name]["us"], 3))
        except Exception as exc:  # noqa: BLE001 - the comparison column is optional
            res[name]["lib"] = f"unavailable ({type(exc).__name__}: {exc})"[:200]
        del lg5, lg4, src4
        probs5 = src5.softmax(dim=-1)
        q5 = torch.empty_like(probs5).exponential_(generator=g)
        ids5 = torch.empty(B5, dtype=torch.int64, device=dev)
        name = "random_sample f32 [256,128256]"
        report(name, 2 * B5 * V5 * 4 + B5 * 8, time_graph([lambda: o.random_sample(ids5, probs5, q5)], 20))
        lib(name, "torch div + argmax (the reference's random_sample after its draws)",
            [lambda: probs5.div(q5).argmax(dim=-1)], 20)
        del src5, probs5, q5

    # rows added beside the headline kernels: a failure is recorded in the table, never
    # fatal to the bench line
    for label, rows in (("rope_and_cache", rope_cache_rows), ("sampler", sampler_rows)):
        try:
            rows()
        except Exception as exc:  # noqa: BLE001
            res[f"{label} (error)"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        torch.cuda.synchronize()

    # decode at the vLLM end-to-end shape: 256 sequences, ctx U[512, 640] (prompt 512 + up
    # to 128 generated), 32/8 heads, block 16: contexts that fit one chunk, so the split
    # kernel writes the output itself; the K/V working set (~0.6 GB) exceeds L2
    gs = torch.Generator().manual_seed(11)
    ctx_s = torch.randint(512, 641, (256,), generator=gs)
    nblk_s = (ctx_s + BLOCK - 1) // BLOCK
    pool_s = int(nblk_s.sum())
    ids_s = torch.randperm(pool_s, generator=gs).to(torch.int32)
    tab_s = torch.zeros(256, 40, dtype=torch.int32)
    off = 0
    for i, nb_i in enumerate(nblk_s.tolist()):
        tab_s[i, :nb_i] = ids_s[off : off + nb_i]
        off += nb_i
    kc_s = torch.randn(pool_s, BLOCK, HKV, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
    vc_s = torch.randn(pool_s, BLOCK, HKV, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
    q_s = torch.randn(256, HQ, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
    o_s = torch.empty_like(q_s)
    seq_s, tab_d = ctx_s.to(torch.int32).to(dev), tab_s.to(dev)
    ws_s = torch.empty(max(256, int(o.decode_workspace_size(256, HQ, HKV, HEAD, BLOCK, 640))), dtype=torch.uint8,
                       device=dev)
    nb = decode_bytes(ctx_s.to(torch.int32), HKV)
    fns = [lambda: o.paged_attention_decode(o_s, q_s, kc_s, vc_s, seq_s, tab_d, 1.0 / math.sqrt(HEAD), 640, ws_s)]
    report("paged decode bf16 B=256 ctx U[512,640] (vLLM e2e shape)", nb, time_graph(fns, 20))
    del kc_s, vc_s

    # varlen prefill over the paged cache (causal, end-aligned), Llama-3-8B heads: a full
    # scheduler batch of 32 prompts x 512 tokens, and 8 prompts of 512 new tokens after
    # 1536 cached ones.  FLOPs = 4 * D * Hq * (visible query-key pairs).
    def prefill_case(name, qlens, ctxs):
        nblk = [(c + BLOCK - 1) // BLOCK for c in ctxs]
        pool_p = sum(nblk)
        gp = torch.Generator().manual_seed(len(qlens))
        ids_p = torch.randperm(pool_p, generator=gp).to(torch.int32)
        tab_p = torch.zeros(len(ctxs), max(nblk), dtype=torch.int32)
        off = 0
        for i, n in enumerate(nblk):
            tab_p[i, :n] = ids_p[off : off + n]
            off += n
        cu_p = torch.tensor([0] + list(itertools.accumulate(qlens)), dtype=torch.int32)
        kc_p = torch.randn(pool_p, BLOCK, HKV, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
        vc_p = torch.randn(pool_p, BLOCK, HKV, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
        q_p = torch.randn(int(cu_p[-1]), HQ, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
        o_p = torch.empty_like(q_p)
        cu_d, seq_d, tab_d = cu_p.to(dev), torch.tensor(ctxs, dtype=torch.int32, device=dev), tab_p.to(dev)
        pairs = sum(sum(min(c - ql + i + 1, c) for i in range(ql)) for ql, c in zip(qlens, ctxs))
        flops = 4.0 * HEAD * HQ * pairs
        nbytes = 2 * int(cu_p[-1]) * HQ * HEAD * 2 + 2 * sum(ctxs) * HKV * HEAD * 2
        sc = 1.0 / math.sqrt(HEAD)
        ms = time_graph([lambda: o.paged_attention_prefill(o_p, q_p, kc_p, vc_p, cu_d, seq_d, tab_d, max(qlens),
                                                            sc, True)], 10)
        tf = flops / (ms * 1e-3) / 1e12
        res[name] = {"us": ms * 1e3, "TFLOP/s": round(tf, 1), "frac_of_bf16": round(tf / tens, 3),
                     "flops": flops, "bytes": nbytes}
        try:
            from vllm.vllm_flash_attn import flash_attn_varlen_func as vllm_fa
        except Exception:  # noqa: BLE001 - the comparison column is optional
            vllm_fa = None
        lib(name, "vLLM flash_attn_varlen_func (paged, causal)",
            vllm_fa and [lambda: vllm_fa(q_p, kc_p, vc_p, out=o_p, cu_seqlens_q=cu_d, max_seqlen_q=max(qlens),
                                         seqused_k=seq_d, max_seqlen_k=max(ctxs), softmax_scale=sc, causal=True,
                                         block_table=tab_d)], 10)
        del kc_p, vc_p, q_p, o_p

    prefill_case("paged prefill bf16 32 x 512 tokens (causal)", [512] * 32, [512] * 32)
    prefill_case("paged prefill bf16 8 x 512 new after 1536 cached", [512] * 8, [2048] * 8)

    # projection GEMM bf16 (fp32 accumulate)
    for (K, Nn, tag) in ((4096, 6144, "qkv"), (4096, 4096, "o_proj"), (4096, 28672, "gate_up"), (14336, 4096, "down")):
        for M in (1, 16, 128, 256, 1024, 8192):
            x = torch.randn(M, K, device=dev, generator=g, dtype=torch.bfloat16)
            wts = [0.02 * torch.randn(Nn, K, device=dev, generator=g, dtype=torch.bfloat16)
                   for _ in range(max(1, math.ceil(3 * L2_BYTES / (Nn * K * 2))) if M <= 256 else 1)]
            out = torch.empty(M, Nn, device=dev, dtype=torch.bfloat16)
            fns = [lambda w_=w_: o.linear(out, x, w_, None, None) for w_ in wts]
            iters = max(4, 2 * len(wts))
            ms = time_graph(fns, iters)
            flops = 2.0 * M * Nn * K
            nbytes = Nn * K * 2 + M * K * 2 + M * Nn * 2
            tf = flops / (ms * 1e-3) / 1e12
            name = f"linear {tag} M={M}"
            if M <= 256:
                report(name, nbytes, ms, {"TFLOP/s": round(tf, 2)})
            else:
                res[name] = {"us": ms * 1e3, "TFLOP/s": round(tf, 1), "frac_of_bf16": round(tf / tens, 3)}
            lib(name, "cuBLAS (torch.mm, the F.linear GEMM)",
                [lambda w_=w_: torch.mm(x, w_.t(), out=out) for w_ in wts], iters)
            del x, wts, out

    # residual add + RMS norm fused into the qkv projection's input (decode batches <= 16
    # tokens): one kernel against the norm kernel followed by the GEMM (ours, and vLLM's _C
    # norm with cuBLAS).  Algorithmic bytes: W, x and residual read, out and the new
    # residual written.
    from vllm_nt._ntops.torch.linear import rms_norm_linear

    for M in (1, 16):
        K, Nn = 4096, 6144
        x = torch.randn(M, K, device=dev, generator=g, dtype=torch.bfloat16)
        r = torch.randn(M, K, device=dev, generator=g, dtype=torch.bfloat16)
        gam = torch.ones(K, device=dev, dtype=torch.bfloat16)
        wts = [0.02 * torch.randn(Nn, K, device=dev, generator=g, dtype=torch.bfloat16)
               for _ in range(max(1, math.ceil(3 * L2_BYTES / (Nn * K * 2))))]
        out = torch.empty(M, Nn, device=dev, dtype=torch.bfloat16)
        new_r = torch.empty_like(x)
        h = torch.empty_like(x)
        iters = max(4, 2 * len(wts))
        ms = time_graph([lambda w_=w_: o.rms_norm_linear(out, new_r, x, r, gam, 1e-5, w_) for w_ in wts], iters)
        name = f"rms_norm+linear qkv M={M}"
        report(name, Nn * K * 2 + 3 * M * K * 2 + M * Nn * 2, ms)

        # the unfused pairs work in place, as vLLM runs them (the residual keeps growing
        # across replays; the timing does not depend on the values)
        def unfused(w_):
            o.fused_add_rms_norm(h, new_r, x, gam, 1e-5)
            o.linear(out, h, w_, None, None)

        new_r.copy_(r)
        res[name]["unfused_ntb200_us"] = round(time_graph([lambda w_=w_: unfused(w_) for w_ in wts], iters) * 1e3, 2)
        if vops is not None:

            def vllm_pair(w_):
                vops.fused_add_rms_norm(h, new_r, gam, 1e-5)
                torch.mm(h, w_.t(), out=out)

            h.copy_(x)
            new_r.copy_(r)
            lib(name, "vllm _C.fused_add_rms_norm + cuBLAS", [lambda w_=w_: vllm_pair(w_) for w_ in wts], iters)
        del x, r, wts, out, new_r, h

    # LM head + greedy sampling, vocabulary 128256 x hidden 4096 (a 1.05 GB weight, beyond
    # L2): the fused kernel keeps the logits on chip and emits the int64 token per row;
    # the unfused pair writes [M, V] logits and reads them back for torch.argmax
    V = 128256
    w_lm = 0.02 * torch.randn(V, 4096, device=dev, generator=g, dtype=torch.bfloat16)
    for M in (1, 16, 128, 256):
        x = torch.randn(M, 4096, device=dev, generator=g, dtype=torch.bfloat16)
        tok = torch.empty(M, dtype=torch.int64, device=dev)
        logits = torch.empty(M, V, device=dev, dtype=torch.bfloat16)
        name = f"lm_head+argmax V={V} M={M}"
        nbytes = V * 4096 * 2 + M * 4096 * 2 + M * 8
        ms = time_graph([lambda: o.linear_argmax(tok, x, w_lm)], 6)
        report(name, nbytes, ms, {"TFLOP/s": round(2.0 * M * V * 4096 / (ms * 1e-3) / 1e12, 2)})
        t_ours = time_graph([lambda: (o.linear(logits, x, w_lm, None, None), torch.argmax(logits, -1))], 6)
        res[name]["unfused_ntb200_linear_plus_torch_argmax_us"] = round(t_ours * 1e3, 1)
        lib(name, "cuBLAS torch.mm + torch.argmax",
            [lambda: (torch.mm(x, w_lm.t(), out=logits), torch.argmax(logits, -1))], 6)
        del x, tok, logits
    del w_lm
    return res


def _sig3(x):
    """x to three significant figures (ints stay ints)."""
    if x is None or isinstance(x, str):
        return x
    if x == 0:
        return 0
    r = float(f"{x:.3g}")
    return int(r) if r == int(r) and abs(r) >= 100 else r


# short row names of the compact per-op table, in print order: GEMMs and attention first,
# the memory-bound ops last (the end of the line is what a truncated log keeps)
_SHORT = {
    **{f"linear {t} M={m}": f"{t} {m}" for t in ("qkv", "o_proj", "gate_up", "down")
       for m in (1, 16, 128, 256, 1024, 8192)},
    **{f"lm_head+argmax V=128256 M={m}": f"lmhead+argmax {m}" for m in (1, 16, 128, 256)},
    "paged prefill bf16 32 x 512 tokens (causal)": "prefill 32x512",
    "paged prefill bf16 8 x 512 new after 1536 cached": "prefill 8x512@1536",
    "paged decode bf16 B=256 ctx U[512,640] (vLLM e2e shape)": "decode ctx512-640",
    "top_k_top_p f32 [256,128256] k=50 p=0.9": "topk_topp 256x128256",
    "top_k_top_p f32 [4,128256] k=50 p=0.9": "topk_topp 4x128256",
    "rms_norm+linear qkv M=1": "norm+qkv 1",
    "rms_norm+linear qkv M=16": "norm+qkv 16",
    "random_sample f32 [256,128256]": "sample 256x128256",
    "rope_and_cache bf16 256 tokens of qkv [T,48*128]": "rope+kv 256",
    "rope_and_cache bf16 16384 tokens of qkv [T,48*128]": "rope+kv 16384",
    "embedding bf16 4096 ids x 4096": "embed 4096",
    "silu_and_mul bf16 [2048,28672]": "silu bf16 2048x28672",
    "rope_neox bf16 16384 tokens of qkv [T,48*128]": "rope bf16 16384",
    "reshape_and_cache bf16 16384x8x128": "kv 16384",
    "fused_add_rms_norm bf16 [8192,4096]": "rms bf16 8192x4096",
    "fused_add_rms_norm f32 [128,4096]": "rms f32 cfg(a)",
    "silu_and_mul f32 [128,22016]": "silu f32 cfg(b)",
    "rope_neox f32 q[128,32,128] k[128,8,128]": "rope f32 cfg(c)",
    "reshape_and_cache bf16 4096x8x128": "kv cfg 4096",
}


def compact_ops(res: dict) -> dict:
    """The per-op table as short rows [rate, frac, x_lib, floor_us]: rate is GB/s
    (HBM-bound rows) or TFLOP/s (tensor-bound rows), frac its fraction of the measured
    peak, x_lib vLLM's kernel time / ours (>1: ours faster), floor_us the same kernel's
    time on a single-row input (its launch floor), where measured.  Microseconds per call
    are in the full table (stderr)."""
    out = {"cols": "GB/s|TF/s,frac,x_lib,floor_us"}
    order = list(_SHORT) + [k for k in res if k not in _SHORT]
    for name in order:
        d = res.get(name)
        if d is None:
            continue
        if "error" in d:
            out[_SHORT.get(name, name)] = d["error"][:80]
            continue
        if "frac_of_hbm" in d:
            row = [d["GB/s"], d["frac_of_hbm"]]
        else:
            row = [d.get("TFLOP/s"), d.get("frac_of_bf16")]
        row.append(d.get("ours_vs_lib"))
        if "floor_us" in d:
            row.append(d["floor_us"])
        while row and row[-1] is None:
            row.pop()
        out[_SHORT.get(name, name)] = [_sig3(v) for v in row]
    return out


def compact_tp(res: dict) -> dict:
    """The row-parallel table as short rows of microseconds per call."""
    cols = ("gemm_us", "allreduce_us", "serial_us", "peer_gemm_allreduce_us", "peer_twoshot_gemm_allreduce_us")
    out = {"cols": "gemm,nccl_ar,gemm+nccl,gemm+peer1,gemm+peer2 (us)"}
    for name, d in res.items():
        if name.startswith("_"):
            out[name] = d
            continue
        out[name] = [_sig3(d.get(c)) for c in cols]
    return out


def tp_projection_table(dev, n: int, rank: int, dist) -> dict:
    """Row-parallel projections (o_proj K=4096, down K=14336; N=4096) on n ranks: each rank
    multiplies its K-shard and the partial outputs are summed across ranks.  Times (max
    over ranks, CUDA events, median of 5 replays of a CUDA graph of 10 back-to-back calls,
    per call; the two-stream chunked pipeline is timed eagerly):
    - NCCL: the local GEMM, the all-reduce, the two back to back, and an M-chunked
      pipeline in which the all-reduce of chunk i (on a second stream) overlaps the GEMM of
      chunk i+1;
    - peer: the GEMM writing into this rank's peer-mapped slot followed by this library's
      one-shot all-reduce over NVLink (vllm_nt._ntops.tp.PeerAllReduce), no NCCL."""
    from vllm_nt._ntops import sharding
    from vllm_nt._ntops.torch._ext import ops
    from vllm_nt._ntops.tp import PeerAllReduce

    o = ops()
    g = torch.Generator(device=dev).manual_seed(50 + rank)
    comm = torch.cuda.Stream(device=dev)
    par = PeerAllReduce(None, capacity=8192 * 4096, device=dev)
    res = {}
    inner = 10

    def timed(fn, reps=5, graph=True) -> float:
        """Device time per call: `inner` calls captured in one CUDA graph (so that host
        launch cost does not count), replayed after a barrier, median of `reps`."""
        g_ = None
        if graph:
            torch.cuda.synchronize()
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_):
                for _ in range(inner):
                    fn()
        ts = []
        for _ in range(reps):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            if g_ is not None:
                g_.replay()
            else:
                for _ in range(inner):
                    fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / inner)
        del g_
        t = torch.tensor([statistics.median(ts)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for name, k_full in (("o_proj", 4096), ("down", 14336)):
        k0, k1 = sharding.row_range(rank, n, k_full)
        kl = k1 - k0
        w = 0.02 * torch.randn(4096, kl, device=dev, generator=g, dtype=torch.bfloat16)
        for m in (1, 128, 1024, 8192):
            x = torch.randn(m, kl, device=dev, generator=g, dtype=torch.bfloat16)
            out = torch.empty(m, 4096, device=dev, dtype=torch.bfloat16)
            chunks = 4 if m >= 1024 else 1
            rows = m // chunks

            def gemm():
                o.linear(out, x, w, None, None)

            def allreduce():
                dist.all_reduce(out)

            def serial():
                gemm()
                allreduce()

            def pipelined():
                main = torch.cuda.current_stream()
                for c in range(chunks):
                    sl = slice(c * rows, (c + 1) * rows)
                    o.linear(out[sl], x[sl], w, None, None)
                    ev = torch.cuda.Event()
                    ev.record(main)
                    comm.wait_event(ev)
                    with torch.cuda.stream(comm):
                        dist.all_reduce(out[sl])
                main.wait_stream(comm)

            out_peer = torch.empty(m, 4096, device=dev, dtype=torch.bfloat16)
            out_peer2 = torch.empty(m, 4096, device=dev, dtype=torch.bfloat16)

            part = torch.empty(m, 4096, device=dev, dtype=torch.bfloat16)

            def peer():
                o.linear(part, x, w, None, None)
                par.reduce(part, out_peer, method="oneshot")

            def peer2():
                o.linear(part, x, w, None, None)
                par.reduce(part, out_peer2, method="twoshot")

            for f in (gemm, allreduce, serial, pipelined, peer, peer2):
                f()
            torch.cuda.synchronize()
            t_gemm, t_ar, t_serial = timed(gemm), timed(allreduce), timed(serial)
            t_pipe = timed(pipelined, graph=False)
            t_peer, t_peer2 = timed(peer), timed(peer2)
            # the paths agree (each sums this rank's bf16 partial with its peers')
            serial()
            peer()
            peer2()
            torch.cuda.synchronize()
            agree = float(max((out.float() - out_peer.float()).abs().max().item(),
                              (out.float() - out_peer2.float()).abs().max().item()))
            res[f"{name} M={m}"] = {
                "gemm_us": round(t_gemm * 1e3, 1),
                "allreduce_us": round(t_ar * 1e3, 1),
                "serial_us": round(t_serial * 1e3, 1),
                "chunked_overlap_us": round(t_pipe * 1e3, 1),
                "peer_gemm_allreduce_us": round(t_peer * 1e3, 1),
                "peer_twoshot_gemm_allreduce_us": round(t_peer2 * 1e3, 1),
                "peer_vs_nccl_max_abs_diff": round(agree, 4),
                "allreduce_bytes": m * 4096 * 2,
                "chunks": chunks,
            }
            del x, out, out_peer, part
        del w
    del par
    return res


def run_linear_case(args) -> int:
    """One GEMM shape for profiling: warmup + steps eager launches (so that ncu can capture
    one), then the device time per call of CUDA-graph replays over weight copies larger
    than L2, as the per-op table times it (prints its own timings)."""
    from vllm_nt._ntops.torch._ext import ops

    m, n, k = args.linear_case
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(m, k, device=dev, generator=g, dtype=torch.bfloat16)
    copies = max(1, math.ceil(3 * L2_BYTES / (n * k * 2)))
    ws = [0.02 * torch.randn(n, k, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(copies)]
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    o = ops()
    ms = _time_calls(lambda: o.linear(out, x, ws[0], None, None), args.warmup, args.steps)
    graph_us = time_graph([lambda w_=w_: o.linear(out, x, w_, None, None) for w_ in ws], max(8, 2 * copies)) * 1e3
    print(json.dumps({"linear_case": [m, n, k], "us": ms * 1e3, "graph_us": round(graph_us, 2),
                      "TFLOP/s": round(2.0 * m * n * k / (graph_us * 1e-6) / 1e12, 1),
                      "GB/s": round((n * k * 2 + m * k * 2 + m * n * 2) / (graph_us * 1e-6) / 1e9, 1)}))
    return 0


def _time_calls(call, warmup: int, steps: int) -> float:
    """Average device ms of `steps` back-to-back calls after `warmup` untimed ones."""
    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_sampler_case(args) -> int:
    """The top-k/top-p mask (k = 50, p = 0.9 on every row) of fp32 logits [B, V], warmup +
    steps launches on one buffer, for profiling (prints its own timing).  The mask works in
    place, so calls after the first see already-masked rows: time with the per-op table."""
    from vllm_nt._ntops.torch._ext import ops

    b, v = args.sampler_case
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    logits = torch.randn(b, v, device=dev, generator=g) * 2
    k = torch.full((b,), 50, device=dev, dtype=torch.int32)
    p = torch.full((b,), 0.9, device=dev)
    o = ops()
    ms = _time_calls(lambda: o.top_k_top_p(logits, k, p), args.warmup, args.steps)
    print(json.dumps({"sampler_case": [b, v], "us": ms * 1e3}))
    return 0


def run_rope_cache_case(args) -> int:
    """RoPE + KV store of T tokens of a Llama-3-8B qkv [T, 48*128] bf16 into a
    FlashAttention cache [2, 8192, 16, 8, 128], warmup + steps launches, for profiling."""
    from vllm_nt._ntops.torch._ext import ops
    import oracle

    t = args.rope_cache_case
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(t, 48 * HEAD, device=dev, generator=g, dtype=torch.bfloat16)
    pos = torch.randint(0, 4096, (t,), device=dev, generator=g)
    slots = torch.randperm(8192 * BLOCK, device=dev, generator=g)[:t]
    kv = torch.zeros(2, 8192, BLOCK, HKV, HEAD, device=dev, dtype=torch.bfloat16)
    cache = oracle.build_cos_sin_cache(HEAD, 4096, 10000.0).to(torch.bfloat16).to(dev)
    q, k, v = qkv[:, : HQ * HEAD], qkv[:, HQ * HEAD : (HQ + HKV) * HEAD], qkv[:, (HQ + HKV) * HEAD :]
    o = ops()
    ms = _time_calls(lambda: o.rope_and_cache_flash_layout(pos, q, k, v, cache, kv, slots, HEAD, HEAD, 0),
                     args.warmup, args.steps)

    def pair():
        o.rotary_embedding_neox(pos, q, k, cache, HEAD, HEAD)
        o.store_flash_layout(k, v, kv, slots, 0)

    fused_us = time_graph([lambda: o.rope_and_cache_flash_layout(pos, q, k, v, cache, kv, slots, HEAD, HEAD, 0)],
                          10) * 1e3
    pair_us = time_graph([pair], 10) * 1e3
    print(json.dumps({"rope_cache_case": t, "us": ms * 1e3, "graph_us": round(fused_us, 2),
                      "pair_graph_us": round(pair_us, 2)}))
    return 0


OP_CASES = ("rms_f32", "rms_bf16", "silu_f32", "silu_bf16", "rope_f32", "rope_bf16", "kv_store", "kv_store_16k",
            "embedding", "random_sample")


def op_case_calls(name: str, dev, g) -> tuple[int, list]:
    """(algorithmic bytes per call, calls over rotating input sets) for one memory-bound op
    at its benchmark size: rms_f32 / silu_f32 / rope_f32 are the fp32 decoder configs
    (x, r [128, 4096]; [128, 22016] -> [128, 11008]; q [128, 32, 128], k [128, 8, 128]),
    kv_store the bf16 4096 x 8 x 128 store into [8192, 16, 8, 128] caches; rms_bf16 /
    silu_bf16 / rope_bf16 / kv_store_16k / embedding are the prefill-sized points
    ([8192, 4096]; [2048, 28672]; 16384 tokens of a [T, 48*128] qkv; 16384 tokens; 4096
    ids into a [128256, 4096] table); random_sample is [256, 128256] fp32."""
    from vllm_nt._ntops.torch._ext import ops
    import oracle

    o = ops()
    bf = torch.bfloat16

    def sets(nbytes):
        return max(2, math.ceil(3 * L2_BYTES / nbytes))

    if name in ("rms_f32", "rms_bf16"):
        m, dt = (128, torch.float32) if name == "rms_f32" else (8192, bf)
        es = 4 if dt == torch.float32 else 2
        nb = 4 * m * 4096 * es + 4096 * es
        r = sets(nb)
        xs = [torch.randn(m, 4096, device=dev, generator=g).to(dt) for _ in range(r)]
        rs = [torch.randn(m, 4096, device=dev, generator=g).to(dt) for _ in range(r)]
        w = (1 + 0.1 * torch.randn(4096, device=dev, generator=g)).to(dt)
        outs = [torch.empty_like(xs[0]) for _ in range(r)]
        return nb, [lambda i=i: o.fused_add_rms_norm(outs[i], rs[i], xs[i], w, 1e-6) for i in range(r)]
    if name in ("silu_f32", "silu_bf16"):
        m, d, dt = (128, 11008, torch.float32) if name == "silu_f32" else (2048, 14336, bf)
        es = 4 if dt == torch.float32 else 2
        nb = 3 * m * d * es
        r = sets(nb)
        xs = [torch.randn(m, 2 * d, device=dev, generator=g).to(dt) for _ in range(r)]
        outs = [torch.empty(m, d, device=dev, dtype=dt) for _ in range(r)]
        return nb, [lambda i=i: o.silu_and_mul(outs[i], xs[i]) for i in range(r)]
    if name in ("rope_f32", "rope_bf16"):
        t, dt, base = (128, torch.float32, 10000.0) if name == "rope_f32" else (16384, bf, 500000.0)
        es = 4 if dt == torch.float32 else 2
        nb = 2 * t * 40 * 128 * es + t * 128 * es + t * 8
        r = sets(nb)
        qkv = [torch.randn(t, 48 * 128, device=dev, generator=g).to(dt) for _ in range(r)]
        pos = [torch.randint(0, 4096, (t,), device=dev, generator=g) for _ in range(r)]
        cache = oracle.build_cos_sin_cache(128, 4096, base).to(dt).to(dev)
        return nb, [lambda i=i: o.rotary_embedding_neox(pos[i], qkv[i][:, :4096], qkv[i][:, 4096:5120], cache, 128, 128)
                    for i in range(r)]
    if name in ("kv_store", "kv_store_16k"):
        n = 4096 if name == "kv_store" else 16384
        nb = 2 * n * 8 * 128 * 2 * 2 + n * 8
        r = sets(nb)
        kc = torch.zeros(8192, 16, 8, 128, device=dev, dtype=bf)
        vc = torch.zeros_like(kc)
        keys = [torch.randn(n, 8, 128, device=dev, generator=g).to(bf) for _ in range(r)]
        vals = [torch.randn(n, 8, 128, device=dev, generator=g).to(bf) for _ in range(r)]
        slots = [torch.randperm(8192 * 16, device=dev, generator=g)[:n] for _ in range(r)]
        return nb, [lambda i=i: o.reshape_and_cache(keys[i], vals[i], kc, vc, slots[i]) for i in range(r)]
    if name == "embedding":
        wt = torch.randn(128256, 4096, device=dev, generator=g).to(bf)
        ids = [torch.randint(0, 128256, (4096,), device=dev, generator=g) for _ in range(8)]
        outs = [torch.empty(4096, 4096, device=dev, dtype=bf) for _ in range(8)]
        return 2 * 4096 * 4096 * 2 + 4096 * 8, [lambda i=i: o.embedding(outs[i], ids[i], wt) for i in range(8)]
    if name == "random_sample":
        probs = torch.randn(256, 128256, device=dev, generator=g).softmax(dim=-1)
        q = torch.empty_like(probs).exponential_(generator=g)
        ids = torch.empty(256, dtype=torch.int64, device=dev)
        return 2 * 256 * 128256 * 4 + 256 * 8, [lambda: o.random_sample(ids, probs, q)]
    raise SystemExit(f"--op-case: unknown op {name!r} (one of {', '.join(OP_CASES)})")


def run_op_case(args) -> int:
    """One memory-bound op at its benchmark size, warmup + steps launches rotating over
    input sets larger than L2, for profiling (prints its own timing)."""
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    nb, calls = op_case_calls(args.op_case, dev, g)
    i = iter(itertools.cycle(calls))
    ms = _time_calls(lambda: next(i)(), args.warmup, args.steps)
    gbs = nb / (ms * 1e-3) / 1e9
    print(json.dumps({"op_case": args.op_case, "bytes": nb, "us": round(ms * 1e3, 2), "GB/s": round(gbs, 1)}))
    return 0


def run_prefill_case(args) -> int:
    """NSEQ sequences of Q new tokens after CTX - Q cached ones (Llama-3-8B heads, paged
    cache), warmup + steps launches of the prefill kernel, for profiling."""
    from vllm_nt._ntops.torch._ext import ops

    q_len, ctx, nseq = args.prefill_case
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    nblk = (ctx + BLOCK - 1) // BLOCK
    table = torch.randperm(nseq * nblk, device=dev, generator=g).to(torch.int32).view(nseq, nblk)
    kc = torch.randn(nseq * nblk, BLOCK, HKV, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(nseq * q_len, HQ, HEAD, device=dev, generator=g, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    cu = torch.arange(0, nseq + 1, device=dev, dtype=torch.int32) * q_len
    seq = torch.full((nseq,), ctx, device=dev, dtype=torch.int32)
    o = ops()

    def call():
        o.paged_attention_prefill(out, q, kc, vc, cu, seq, table, q_len, 1.0 / math.sqrt(HEAD), True)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    pairs = nseq * sum(ctx - q_len + i + 1 for i in range(q_len))
    print(json.dumps({"prefill_case": [q_len, ctx, nseq], "us": ms * 1e3,
                      "TFLOP/s": 4.0 * HEAD * HQ * pairs / (ms * 1e-3) / 1e12}))
    return 0


# --------------------------------------------------------------------------------------
# main arm
# --------------------------------------------------------------------------------------


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-op table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--decode-batch", type=int, default=BATCH, help="profiling: fewer sequences than the workload")
    ap.add_argument("--pool", type=int, default=POOL, help="profiling: smaller block pool")
    ap.add_argument("--linear-case", type=int, nargs=3, metavar=("M", "N", "K"),
                    help="profiling: run only the GEMM out[M,N] = x[M,K] W[N,K]^T, warmup+steps times")
    ap.add_argument("--prefill-case", type=int, nargs=3, metavar=("Q", "CTX", "NSEQ"),
                    help="profiling: run only the paged prefill kernel, warmup+steps times")
    ap.add_argument("--sampler-case", type=int, nargs=2, metavar=("B", "V"),
                    help="profiling: run only the top-k/top-p mask over [B, V] logits, warmup+steps times")
    ap.add_argument("--rope-cache-case", type=int, metavar="T",
                    help="profiling: run only the fused RoPE + KV store over T tokens, warmup+steps times")
    ap.add_argument("--shard-of", type=int, default=0, metavar="S",
                    help="profiling: one process runs rank 0's share of an S-way KV-head split of the decode")
    ap.add_argument("--op-case", choices=OP_CASES,
                    help="profiling: run only one memory-bound op at its benchmark size, warmup+steps times")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.linear_case:
        return run_linear_case(args)
    if args.prefill_case:
        return run_prefill_case(args)
    if args.sampler_case:
        return run_sampler_case(args)
    if args.rope_cache_case:
        return run_rope_cache_case(args)
    if args.op_case:
        return run_op_case(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = world
    if HKV % n != 0:
        raise SystemExit(f"--gpus {n}: the 8 KV heads must divide evenly across ranks")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from vllm_nt import oot  # noqa: F401  (the plugin's public surface)
    from vllm_nt._ntops.torch.attention import decode_workspace_bytes, paged_decode

    peaks, peak_kind = load_peaks()
    batch, pool = args.decode_batch, args.pool
    ctx, table, q_all = workload(0, batch, pool)
    from vllm_nt._ntops import sharding

    # --shard-of S (profiling, one process): run rank 0's share of an S-way KV-head split
    split = args.shard_of if args.shard_of else n
    h0, h1 = sharding.kv_head_range(rank, split, HKV)
    q0, q1 = sharding.q_head_range(rank, split, HQ, HKV)
    hkv, hq = h1 - h0, q1 - q0
    q = q_all[:, q0:q1].contiguous()
    gk = torch.Generator(device=dev).manual_seed(1000 + rank)
    kc = torch.randn(pool, BLOCK, hkv, HEAD, device=dev, generator=gk, dtype=torch.bfloat16)
    vc = torch.randn(pool, BLOCK, hkv, HEAD, device=dev, generator=gk, dtype=torch.bfloat16)
    qd, sd, td = q.to(dev), ctx.to(dev), table.to(dev)
    out = torch.empty_like(qd)
    scale = 1.0 / math.sqrt(HEAD)
    ws = torch.empty(decode_workspace_bytes(batch, hq, hkv, CTX_HI), dtype=torch.uint8, device=dev)

    def step():
        paged_decode(out, qd, kc, vc, sd, td, scale, CTX_HI, ws)

    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    clocks = sampler.stop()
    ms_max = ms
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = batch * args.steps / (ms_max * 1e-3)

    # the same call replayed from a CUDA graph (launch gaps removed): against the eager
    # time above it separates the kernels' device time from the host's launch cost, per rank
    graph_ms = time_graph([step], 20)
    per_rank = torch.tensor([ms / args.steps, graph_ms, decode_bytes(ctx, hkv) / (graph_ms * 1e-3) / 1e9], device=dev)
    if dist:
        gathered = [torch.zeros_like(per_rank) for _ in range(n)]
        dist.all_gather(gathered, per_rank)
    else:
        gathered = [per_rank]
    rank_split = {
        "eager_us_max": round(max(float(t[0]) for t in gathered) * 1e3, 1),
        "graph_us_max": round(max(float(t[1]) for t in gathered) * 1e3, 1),
        "graph_GB/s_min": round(min(float(t[2]) for t in gathered), 1),
    }

    # roofline of this rank's decode call (split + combine launches)
    algo = decode_bytes(ctx, hkv)
    achieved = algo / (ms / args.steps * 1e-3) / 1e9
    traffic = traffic_from_profile()
    roofline = {
        "bound": "hbm",
        "achieved": round(achieved, 1),
        "peak": peaks["hbm_gbs"],
        "unit": "GB/s",
        "frac": round(achieved / peaks["hbm_gbs"], 3),
        "traffic": traffic * (hkv / HKV) if traffic is not None else None,
        "peak_source": "measured hbm_gbs" if peak_kind == "measured" else "fallback 6.65 TB/s",
        "algorithmic_bytes_per_launch": algo,
    }

    # e2e: the plugin's public decode entry point with host buffers
    from vllm_nt.oot import paged_attention_decode

    q_host = q.view(batch, 1, hq, HEAD).pin_memory()
    s_host = ctx.pin_memory()
    t_host = table.pin_memory()
    o_host = torch.empty(batch, 1, hq, HEAD, dtype=torch.bfloat16).pin_memory()
    e2e_steps = 0 if args.no_e2e else max(10, min(args.steps, 200))

    def e2e_step():
        qq = q_host.to(dev, non_blocking=True)
        ss = s_host.to(dev, non_blocking=True)
        tt = t_host.to(dev, non_blocking=True)
        res = paged_attention_decode(qq, kc, vc, ss, tt, softmax_scale=scale, max_seq_len=CTX_HI)
        o_host.copy_(res, non_blocking=True)

    for _ in range(3 if e2e_steps else 0):
        e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max(e0.elapsed_time(e1), 1e3 * (time.perf_counter() - t0), 1e-6)
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = None if not e2e_steps else {
        "value": round(batch * e2e_steps / (e2e_ms * 1e-3), 1),
        "unit": "tok/s",
        "h2d_bytes_per_step": q_host.numel() * 2 + s_host.numel() * 4 + t_host.numel() * 4,
        "d2h_bytes_per_step": o_host.numel() * 2,
        "steps": e2e_steps,
        "path": "oot.paged_attention_decode, pinned host in/out",
    }

    per_op = None
    tp_table = None
    if rank == 0 and n == 1 and not args.no_ops:
        del kc, vc, ws
        torch.cuda.empty_cache()
        per_op = per_op_table(dev, peaks)
    elif n > 1 and not args.no_ops:
        del kc, vc, ws
        torch.cuda.empty_cache()
        tp_table = tp_projection_table(dev, n, rank, dist)

    cpu = None
    if rank == 0 and n == 1 and not args.no_cpu and batch == BATCH:
        torch.set_num_threads(os.cpu_count() or 1)
        t_one, _, _ = oracle_decode_rate(ctx, q_all, 1, 1)
        per_call = max(1, min(BATCH, int(4.0 * t_one)))
        calls = max(1, min(64, int(15.0 / max(per_call / t_one, 1e-3))))
        v, threads, sample = oracle_decode_rate(ctx, q_all, per_call, calls)
        cpu = {"value": round(v, 2), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tok/s",
        "n_gpus": n,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(n) if batch == BATCH and pool == POOL and not args.shard_of else
        {**workload_config(n), "profiling_case": f"batch {batch}, pool {pool}, shard 1 of {args.shard_of or 1}"},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 2 * args.steps,  # split + combine per timed step
        "clocks": clocks,
        "per_rank": rank_split,
    }
    # the full tables go to stderr; the line carries their compact form, so that the whole
    # line stays within a few thousand characters
    if per_op is not None:
        print("per_op " + json.dumps(per_op), file=sys.stderr, flush=True)
        line["ops"] = compact_ops(per_op)
    if tp_table is not None:
        print("tp_projection " + json.dumps(tp_table), file=sys.stderr, flush=True)
        line["tp"] = compact_tp(tp_table)
    print(json.dumps(line, separators=(",", ":")), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

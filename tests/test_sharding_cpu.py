"""Multi-rank partitioning of the hot path, as world-size-2 gloo process groups on CPU
(the oracle stands in for the kernels): KV-head-sharded decode needs no exchange and its
head slices concatenate to the full output; column-parallel projections all-gather;
row-parallel projections all-reduce."""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from vllm_nt._ntops import sharding


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        # decode, KV-head sharded
        hq, hkv, d = 8, 4, 16
        q = torch.randn(3, hq, d, generator=g)
        kc = torch.randn(10, 4, hkv, d, generator=g)
        vc = torch.randn(10, 4, hkv, d, generator=g)
        seq = torch.tensor([5, 1, 12], dtype=torch.int32)
        table = torch.tensor([[0, 1, 2], [3, 4, 5], [6, 7, 8]], dtype=torch.int32)
        h0, h1 = sharding.kv_head_range(rank, world, hkv)
        q0, q1 = sharding.q_head_range(rank, world, hq, hkv)
        local = oracle.paged_decode(q[:, q0:q1], kc[:, :, h0:h1], vc[:, :, h0:h1], seq, table, 1 / math.sqrt(d))
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        full = oracle.paged_decode(q, kc, vc, seq, table, 1 / math.sqrt(d))
        ok_decode = torch.allclose(torch.cat(parts, dim=1), full, atol=1e-6)
        # column-parallel (qkv / gate_up) and row-parallel (o_proj / down) projections
        x = torch.randn(5, 32, generator=g)
        w = torch.randn(24, 32, generator=g)
        n0, n1 = sharding.column_range(rank, world, 24)
        col = oracle.linear(x, w[n0:n1])
        cols = [torch.empty_like(col) for _ in range(world)]
        dist.all_gather(cols, col)
        ok_col = torch.allclose(torch.cat(cols, dim=1), oracle.linear(x, w), atol=1e-5)
        k0, k1 = sharding.row_range(rank, world, 32)
        row = oracle.linear(x[:, k0:k1], w[:, k0:k1])
        dist.all_reduce(row)
        ok_row = torch.allclose(row, oracle.linear(x, w), atol=1e-4)
        results[rank] = (ok_decode, ok_col, ok_row)
    finally:
        dist.destroy_process_group()


def test_two_rank_partitioning_reproduces_single_rank_results():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}


def test_ranges_reject_uneven_splits():
    assert sharding.kv_head_range(3, 8, 8) == (3, 4)
    assert sharding.q_head_range(1, 2, 32, 8) == (16, 32)
    with pytest.raises(ValueError):
        sharding.kv_head_range(0, 3, 8)
    with pytest.raises(ValueError):
        sharding.row_range(0, 3, 4096)

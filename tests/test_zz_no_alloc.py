"""The decode entry point for callers that cannot allocate device memory at the call (a
serving loop that must not call cudaMalloc while decoding, code recorded into a CUDA graph,
a host with no device allocator of its own): ntb200_paged_attention_decode_noalloc keeps
its split-K partials in a fixed array inside the library instead of a caller workspace.

Checked through the C ABI against the workspace entry point, on two calls in a row with
different inputs (the second call must not see the first call's leftovers), within the
decode tolerance of the other tests (2e-2).  The file name sorts last so that a run that
stops at the first failure has already run every other test; the test needs nothing from
them and also passes alone in a fresh process."""

import math

import pytest
import torch

from _util import cuda_device, ptr, seeded, stream
from vllm_nt._ntops import capi

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _case(ctx, hq, hkv, num_blocks, seed):
    g = seeded(seed)
    nblk = [(c + 15) // 16 for c in ctx]
    width = max(1, max(nblk))
    ids = torch.randperm(num_blocks, generator=g)[: sum(nblk)].to(torch.int32)
    table = torch.zeros(len(ctx), width, dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk):
        table[i, :n] = ids[off : off + n]
        off += n
    q = torch.randn(len(ctx), hq, 128, generator=g).to(torch.bfloat16)
    kc = torch.randn(num_blocks, 16, hkv, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(num_blocks, 16, hkv, 128, generator=g).to(torch.bfloat16)
    return [t.cuda() for t in (q, kc, vc, torch.tensor(ctx, dtype=torch.int32), table)]


def _common_args(q, kc, seq, table, out, hq, hkv, max_seq_len):
    b = q.shape[0]
    return [ptr(out), ptr(q), ptr(kc), None, ptr(seq), ptr(table), b, hq, hkv, 128, 16, kc.shape[0],
            table.shape[1], table.stride(0), max_seq_len, 1.0 / math.sqrt(128), q.stride(0), q.stride(1),
            out.stride(0), out.stride(1), kc.stride(0), kc.stride(1), kc.stride(2)]


def _with_workspace(q, kc, vc, seq, table, hq, hkv, max_seq_len):
    out = torch.empty_like(q)
    args = _common_args(q, kc, seq, table, out, hq, hkv, max_seq_len)
    args[3] = ptr(vc)
    ws_bytes = capi.lib().ntb200_paged_attention_decode_workspace_size(q.shape[0], hq, hkv, 128, 16, max_seq_len)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    capi.call("ntb200_paged_attention_decode", *args, ptr(ws), ws_bytes, 1, stream())
    return out


def _no_alloc(q, kc, vc, seq, table, hq, hkv, max_seq_len):
    out = torch.empty_like(q)
    args = _common_args(q, kc, seq, table, out, hq, hkv, max_seq_len)
    args[3] = ptr(vc)
    capi.call("ntb200_paged_attention_decode_noalloc", *args, 1, stream())
    return out


def test_no_alloc_decode_matches_workspace_decode_two_calls_in_a_row():
    cuda_device()
    # call 1: long contexts, many splits; call 2: different shapes and shorter contexts,
    # so stale partials of call 1 would show up if the second call read any
    first = _case([4097, 1, 2048, 700, 16, 3000], 32, 8, 1200, seed=21)
    second = _case([33, 5000, 0, 1025], 16, 4, 800, seed=22)
    for (q, kc, vc, seq, table), (hq, hkv) in ((first, (32, 8)), (second, (16, 4))):
        msl = table.shape[1] * 16
        ref = _with_workspace(q, kc, vc, seq, table, hq, hkv, msl)
        got = _no_alloc(q, kc, vc, seq, table, hq, hkv, msl)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), ref.float(), rtol=TOL, atol=TOL)
    assert capi.read_device_error(stream()) == 0


def test_no_alloc_decode_rejects_calls_beyond_the_static_scratch():
    cuda_device()
    q = torch.zeros(4096, 32, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(1, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
    seq = torch.ones(4096, dtype=torch.int32, device="cuda")
    table = torch.zeros(4096, 8192, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    args = _common_args(q, kc, seq, table, out, 32, 8, 131072)
    args[3] = ptr(kc)
    with pytest.raises(capi.NtB200Error) as e:
        capi.call("ntb200_paged_attention_decode_noalloc", *args, 1, stream())
    assert e.value.status == -4 and "static scratch" in str(e.value)

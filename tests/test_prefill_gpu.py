"""GPU parity of the tcgen05 varlen prefill kernel against the CPU oracle (tolerance 2e-2:
bf16/f16 in, fp32 softmax and accumulation, P rounded to the input type for P.V), over the
paged cache (torch.ops.ntb200.paged_attention_prefill and the vLLM-layout entry) and over
contiguous K/V (flash_attn_varlen_func, the reference's signature)."""

import math

import pytest
import torch

import oracle
from _util import cuda_device, seeded, stream
from vllm_nt._ntops import capi

pytestmark = pytest.mark.gpu
TOL = 2e-2
INDEX_RANGE = 2


@pytest.fixture(autouse=True)
def _clean_device_error():
    cuda_device()
    torch.cuda.synchronize()
    capi.read_device_error(stream())
    yield


def make_paged(qlens, ctxs, hq, hkv, seed, dtype=torch.bfloat16, spare_blocks=7):
    """Random queries and a shuffled paged cache holding ctx tokens per sequence (the
    sequence's own keys last).  Cache rows past each context are random too, so a kernel
    that let them through would fail."""
    g = seeded(seed)
    nblk = [(c + 15) // 16 for c in ctxs]
    num_blocks = sum(nblk) + spare_blocks
    ids = torch.randperm(num_blocks, generator=g)[: sum(nblk)].to(torch.int32)
    width = max(1, max(nblk))
    table = torch.zeros(len(ctxs), width + 2, dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk):
        table[i, :n] = ids[off : off + n]
        off += n
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0).tolist()), dtype=torch.int32)
    q = torch.randn(int(cu[-1]), hq, 128, generator=g).to(dtype)
    kc = torch.randn(num_blocks, 16, hkv, 128, generator=g).to(dtype)
    vc = torch.randn(num_blocks, 16, hkv, 128, generator=g).to(dtype)
    return q, kc, vc, cu, torch.tensor(ctxs, dtype=torch.int32), table


def run_paged(q, kc, vc, cu, seq, table, scale, causal=True, max_q=None):
    from vllm_nt._ntops.torch.attention import paged_prefill

    dev = cuda_device()
    out = torch.full_like(q, float("nan")).to(dev)
    mq = int((cu[1:] - cu[:-1]).max()) if max_q is None else max_q
    paged_prefill(out, q.to(dev), kc.to(dev), vc.to(dev), cu.to(dev), seq.to(dev), table.to(dev), mq, scale, causal)
    torch.cuda.synchronize()
    return out.float().cpu()


CASES = {
    "prompts": ([1, 5, 127, 128, 129, 300], [1, 5, 127, 128, 129, 300]),
    "prefix": ([64, 200, 3, 130], [600, 1000, 37, 259]),
    "decode_rows": ([1, 1, 2, 1], [700, 17, 2, 129]),
    "long": ([512, 1024], [2048, 1024]),
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (4, 1)])
def test_paged_prefill_matches_oracle(case, hq, hkv):
    qlens, ctxs = CASES[case]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, hq, hkv, seed=hq + 3 * hkv + len(case))
    scale = 1.0 / math.sqrt(128)
    ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, scale)
    out = run_paged(q, kc, vc, cu, seq, table, scale)
    torch.testing.assert_close(out, ref, rtol=TOL, atol=TOL)
    assert capi.read_device_error(stream()) == 0


def test_paged_prefill_f16_and_non_causal():
    qlens, ctxs = [77, 130, 1], [300, 130, 40]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, 8, 2, seed=11, dtype=torch.float16)
    for causal in (True, False):
        ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, 0.1, causal=causal)
        out = run_paged(q, kc, vc, cu, seq, table, 0.1, causal=causal)
        torch.testing.assert_close(out, ref, rtol=TOL, atol=TOL)


def test_paged_prefill_empty_sequences_and_rows_without_keys():
    """q_len 0 writes nothing; a context shorter than the queries leaves the first rows
    with no visible key (zeros), as does an empty context."""
    qlens, ctxs = [0, 4, 3, 2], [20, 2, 0, 2]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, 4, 2, seed=12)
    ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, 0.125)
    out = run_paged(q, kc, vc, cu, seq, table, 0.125)
    torch.testing.assert_close(out, ref, rtol=TOL, atol=TOL)
    assert not out[4:7].any()  # the empty context: zero rows


def test_paged_prefill_stale_cache_rows_do_not_leak():
    """Rows of the last page past the context hold inf/nan: they are masked and zeroed."""
    qlens, ctxs = [5, 19], [21, 19]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, 8, 8, seed=13)
    for b, n in enumerate(ctxs):
        blk = int(table[b, (n - 1) // 16])
        kc[blk, n % 16 :] = float("inf")
        vc[blk, n % 16 :] = float("nan")
    ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, 0.09)
    out = run_paged(q, kc, vc, cu, seq, table, 0.09)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out, ref, rtol=TOL, atol=TOL)


def test_paged_prefill_head_major_cache():
    """A cache stored [blocks, heads, 16, D] (FlashInfer's HND) viewed as [blocks, 16, heads,
    D]: the kernel follows the strides."""
    qlens, ctxs = [100, 33], [140, 33]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, 16, 4, seed=14)
    ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, 0.08)
    dev = cuda_device()
    kh = kc.permute(0, 2, 1, 3).contiguous().to(dev).permute(0, 2, 1, 3)
    vh = vc.permute(0, 2, 1, 3).contiguous().to(dev).permute(0, 2, 1, 3)
    assert kh.stride(2) > kh.stride(1)
    from vllm_nt._ntops.torch.attention import paged_prefill

    out = torch.empty_like(q).to(dev)
    paged_prefill(out, q.to(dev), kh, vh, cu.to(dev), seq.to(dev), table.to(dev), 100, 0.08)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)


def test_paged_prefill_bad_block_id_is_reported_not_read():
    qlens, ctxs = [20], [40]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, 4, 4, seed=15)
    table[0, 1] = kc.shape[0] + 5
    run_paged(q, kc, vc, cu, seq, table, 0.1)
    assert capi.read_device_error(stream()) & INDEX_RANGE


def test_prefill_flash_layout_entry():
    """vLLM's FlashAttention cache [2, blocks, 16, H, D] and padded [capacity, H*D]
    activations: only the first num_tokens rows are touched."""
    from vllm_nt._ntops.oot_support import paged_attention_prefill_flash

    qlens, ctxs = [40, 90], [40, 200]
    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, 8, 2, seed=16)
    ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, 0.07)
    dev = cuda_device()
    kv = torch.stack([kc, vc]).to(dev)
    n = q.shape[0]
    qpad = torch.zeros(n + 16, 8 * 128, dtype=q.dtype, device=dev)
    qpad[:n] = q.reshape(n, -1).to(dev)
    opad = torch.full_like(qpad, 3.0)
    paged_attention_prefill_flash(opad, qpad, kv, cu.to(dev), seq.to(dev), table.to(dev), n, 90, 0.07)
    torch.testing.assert_close(opad[:n].view(n, 8, 128).float().cpu(), ref, rtol=TOL, atol=TOL)
    assert (opad[n:] == 3.0).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_flash_attn_varlen_func_contiguous(dtype):
    """The reference's flash_attn_varlen_func signature over contiguous K/V, with sequences
    whose keys outnumber their queries (a cached prefix) and equal-length ones."""
    from vllm_nt._ntops.torch.attention import flash_attn_varlen_func

    g = seeded(17)
    qlens, klens = [3, 150, 1, 64, 2], [3, 150, 90, 400, 2]
    cu_q = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32)
    cu_k = torch.tensor([0] + torch.tensor(klens).cumsum(0).tolist(), dtype=torch.int32)
    q = torch.randn(int(cu_q[-1]), 8, 128, generator=g).to(dtype)
    k = torch.randn(int(cu_k[-1]) + 9, 2, 128, generator=g).to(dtype)  # rows past the last sequence
    v = torch.randn(int(cu_k[-1]) + 9, 2, 128, generator=g).to(dtype)
    k[int(cu_k[-1]) :] = float("nan")
    v[int(cu_k[-1]) :] = float("nan")
    ref = oracle.varlen_attention(q, k, v, cu_q, cu_k)
    dev = cuda_device()
    out = flash_attn_varlen_func(q.to(dev), k.to(dev), v.to(dev), cu_q.to(dev), cu_k.to(dev), max(qlens))
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)
    assert capi.read_device_error(stream()) == 0


def test_reference_varlen_known_answer_on_gpu():
    """vllm_nt/tests/test_attention.py:57-72 at head size 128: cu_q = cu_k = [0, 2, 5]."""
    from vllm_nt._ntops.oot_support import paged_attention_prefill

    g = seeded(18)
    q = torch.randn(5, 2, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(5, 2, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(5, 2, 128, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0, 2, 5], dtype=torch.int32)
    dev = cuda_device()
    out = paged_attention_prefill(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), cu.to(dev), 3)
    ref = oracle.varlen_attention(q, k, v, cu, cu)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)


def _run_vllm_layout(qlens, ctxs, hq, hkv, seed, scale):
    from vllm_nt._ntops.oot_support import paged_attention_flash

    q, kc, vc, cu, seq, table = make_paged(qlens, ctxs, hq, hkv, seed=seed)
    ref = oracle.paged_prefill(q, kc, vc, cu, seq, table, scale)
    dev = cuda_device()
    kv = torch.stack([kc, vc]).to(dev)
    n = q.shape[0]
    qpad = torch.zeros(n + 8, hq * 128, dtype=q.dtype, device=dev)
    qpad[:n] = q.reshape(n, -1).to(dev)
    opad = torch.full_like(qpad, 5.0)
    paged_attention_flash(opad, qpad, kv, cu.to(dev), seq.to(dev), table.to(dev), n, max(qlens), max(ctxs), scale)
    torch.cuda.synchronize()
    torch.testing.assert_close(opad[:n].view(n, hq, 128).float().cpu(), ref, rtol=TOL, atol=TOL)
    assert (opad[n:] == 5.0).all()
    assert capi.read_device_error(stream()) == 0


def test_mixed_batch_through_vllm_layout():
    """Decodes (one query), a chunk of a prefill after a cached prefix and fresh prompts in
    one batch on the FlashAttention cache: decode rows on the split-K kernel, the rest on
    the prefill kernel, every row against the oracle."""
    _run_vllm_layout([1, 130, 1, 1, 64, 300, 1, 2], [700, 500, 1, 33, 64, 300, 129, 2], 32, 8, 19, 0.088)


def test_decode_only_and_uniform_prefill_batches_through_vllm_layout():
    _run_vllm_layout([1] * 9, [5, 17, 600, 1, 64, 33, 2000, 16, 128], 8, 2, 20, 0.1)
    _run_vllm_layout([64] * 5, [64, 100, 700, 64, 129], 8, 2, 21, 0.1)

"""GPU parity of the split-K paged-decode kernel against the CPU oracle (tolerance 2e-2,
bf16 in / fp32 softmax), through the C ABI and torch.ops.ntb200."""

import math

import pytest
import torch

import oracle
from _util import cuda_device, ptr, seeded, stream
from vllm_nt._ntops import capi

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(autouse=True)
def _clean_device_error():
    cuda_device()
    torch.cuda.synchronize()
    capi.read_device_error(stream())
    yield


def make_case(ctx, hq, hkv, num_blocks, seed, dtype=torch.bfloat16, dev="cuda"):
    g = seeded(seed)
    b = len(ctx)
    nblk = [(c + 15) // 16 for c in ctx]
    width = max(1, max(nblk))
    assert sum(nblk) <= num_blocks
    ids = torch.randperm(num_blocks, generator=g)[: sum(nblk)].to(torch.int32)
    table = torch.zeros(b, width, dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk):
        table[i, :n] = ids[off : off + n]
        off += n
    q = torch.randn(b, hq, 128, generator=g).to(dtype)
    kc = torch.randn(num_blocks, 16, hkv, 128, generator=g).to(dtype)
    vc = torch.randn(num_blocks, 16, hkv, 128, generator=g).to(dtype)
    seq = torch.tensor(ctx, dtype=torch.int32)
    return q, kc, vc, seq, table


def run_torch(q, kc, vc, seq, table, scale, max_seq_len=None):
    from vllm_nt._ntops.torch.attention import paged_decode

    out = torch.empty_like(q)
    paged_decode(out, q, kc, vc, seq, table, scale, max_seq_len)
    return out


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (16, 8), (8, 1), (4, 2)])
def test_decode_edge_lengths_and_gqa_groups(hq, hkv):
    ctx = [1, 15, 16, 17, 255, 1023, 1024, 1025, 2048, 4097]
    q, kc, vc, seq, table = make_case(ctx, hq, hkv, 700, seed=hq * 10 + hkv)
    scale = 1.0 / math.sqrt(128)
    ref = oracle.paged_decode(q, kc, vc, seq, table, scale)
    dev = cuda_device()
    out = run_torch(q.to(dev), kc.to(dev), vc.to(dev), seq.to(dev), table.to(dev), scale)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)
    assert capi.read_device_error(stream()) == 0


def test_decode_capi_empty_sequence_fp16_and_strided_query():
    dev = cuda_device()
    ctx = [0, 40, 300, 16]
    q, kc, vc, seq, table = make_case(ctx, 8, 2, 64, seed=5, dtype=torch.float16)
    scale = 0.07
    ref = oracle.paged_decode(q, kc, vc, seq, table, scale)
    # query as a view into a wider per-token buffer (q heads, then k/v heads)
    wide = torch.zeros(4, 12, 128, dtype=torch.float16)
    wide[:, :8] = q
    qd = wide.to(dev)[:, :8]
    out = torch.full((4, 8, 128), 7.0, dtype=torch.float16, device=dev)
    kd, vd, sd, td = kc.to(dev), vc.to(dev), seq.to(dev), table.to(dev)
    msl = table.shape[1] * 16
    ws_bytes = capi.lib().ntb200_paged_attention_decode_workspace_size(4, 8, 2, 128, 16, msl)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    capi.call("ntb200_paged_attention_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(sd), ptr(td),
              4, 8, 2, 128, 16, 64, table.shape[1], table.shape[1], msl, scale,
              12 * 128, 128, 8 * 128, 128, kc.stride(0), kc.stride(1), kc.stride(2),
              ptr(ws), ws_bytes, 2, stream())
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)
    assert not out[0].any()  # empty sequence -> zeros
    assert capi.read_device_error(stream()) == 0


def test_decode_rejects_small_workspace_and_bad_shapes():
    """A context of 600 tokens splits into several chunks (the partials need a workspace);
    a 40-token one is a single chunk, written directly, and needs none."""
    dev = cuda_device()
    q, kc, vc, seq, table = make_case([600], 4, 1, 40, seed=6)
    qd, kd, vd, sd, td = (t.to(dev) for t in (q, kc, vc, seq, table))
    out = torch.empty_like(qd)
    ws = torch.empty(256, dtype=torch.uint8, device=dev)
    width = table.shape[1]  # 38 blocks
    msl = width * 16
    assert capi.lib().ntb200_paged_attention_decode_workspace_size(1, 4, 1, 128, 16, msl) > 256
    assert capi.lib().ntb200_paged_attention_decode_workspace_size(1, 4, 1, 128, 16, 48) == 0
    with pytest.raises(capi.NtB200Error) as e:
        capi.call("ntb200_paged_attention_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(sd), ptr(td),
                  1, 4, 1, 128, 16, 40, width, width, msl, 0.1, 512, 128, 512, 128, kd.stride(0), kd.stride(1),
                  kd.stride(2), ptr(ws), 16, 1, stream())
    assert e.value.status == -4
    with pytest.raises(capi.NtB200Error) as e:
        capi.call("ntb200_paged_attention_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(sd), ptr(td),
                  1, 4, 1, 64, 16, 40, width, width, msl, 0.1, 512, 128, 512, 128, kd.stride(0), kd.stride(1),
                  kd.stride(2), ptr(ws), 256, 1, stream())
    assert e.value.status == -6


def _full_config(dev, seed=0):
    """Decode config: B=256, 32/8 heads, D=128, block 16, ctx U[512, 8192], distinct block
    ids from a 150000-block pool, q/K/V ~N(0,1) bf16 (caches generated on the device)."""
    g = seeded(seed)
    ctx = torch.randint(512, 8193, (256,), generator=g)
    nblk = (ctx + 15) // 16
    ids = torch.randperm(150000, generator=g)[: int(nblk.sum())].to(torch.int32)
    table = torch.zeros(256, 512, dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk.tolist()):
        table[i, :n] = ids[off : off + n]
        off += n
    q = torch.randn(256, 32, 128, generator=g).to(torch.bfloat16)
    gd = torch.Generator(device=dev).manual_seed(seed)
    kc = torch.randn(150000, 16, 8, 128, generator=gd, device=dev, dtype=torch.bfloat16)
    vc = torch.randn(150000, 16, 8, 128, generator=gd, device=dev, dtype=torch.bfloat16)
    return q, kc, vc, ctx.to(torch.int32), table


def test_decode_full_config_subset_and_properties():
    dev = cuda_device()
    q, kc, vc, seq, table = _full_config(dev)
    scale = 1.0 / math.sqrt(128)
    qd, sd, td = q.to(dev), seq.to(dev), table.to(dev)
    out = run_torch(qd, kc, vc, sd, td, scale, 8192)
    torch.cuda.synchronize()
    assert capi.read_device_error(stream()) == 0
    # oracle on a seeded subset of sequences (the shortest, the longest, and random ones)
    pick = sorted({int(seq.argmin()), int(seq.argmax()), *torch.randperm(256, generator=seeded(9))[:6].tolist()})
    for b in pick:
        n = int(seq[b])
        blocks = table[b, : (n + 15) // 16].long().to(dev)
        kb = kc[blocks].cpu()
        vb = vc[blocks].cpu()
        local_table = torch.arange(kb.shape[0], dtype=torch.int32).unsqueeze(0)
        ref = oracle.paged_decode(q[b : b + 1], kb, vb, seq[b : b + 1], local_table, scale)
        torch.testing.assert_close(out[b].float().cpu(), ref[0], rtol=TOL, atol=TOL)
    # property: permuting the batch permutes the output (same split choice -> bit-exact)
    perm = torch.randperm(256, generator=seeded(10))
    out_p = run_torch(qd[perm.to(dev)], kc, vc, sd[perm.to(dev)], td[perm.to(dev)], scale, 8192)
    assert torch.equal(out_p.cpu(), out.cpu()[perm])
    # property: constant V rows give that constant (softmax weights sum to one)
    vconst = torch.full((1024, 16, 8, 128), 0.375, dtype=torch.bfloat16, device=dev)
    t2 = (td[:64] % 1024).contiguous()
    out_c = run_torch(qd[:64], kc[:1024], vconst, sd[:64], t2, scale, 8192)
    torch.testing.assert_close(out_c.float().cpu(), torch.full((64, 32, 128), 0.375), rtol=1e-3, atol=1e-3)


def test_decode_kv_head_sharding_matches_unsharded():
    """The multi-GPU layout: a rank owning KV heads [h0, h1) runs the kernel on its head
    slice of the cache and of q; concatenating the shards reproduces the full output."""
    dev = cuda_device()
    q, kc, vc, seq, table = make_case([700, 33, 2000, 1], 32, 8, 400, seed=11)
    scale = 1.0 / math.sqrt(128)
    qd, kd, vd, sd, td = (t.to(dev) for t in (q, kc, vc, seq, table))
    full = run_torch(qd, kd, vd, sd, td, scale)
    for shards in (2, 4, 8):
        parts = []
        for r in range(shards):
            h0, h1 = r * 8 // shards, (r + 1) * 8 // shards
            parts.append(run_torch(qd[:, h0 * 4 : h1 * 4].contiguous(), kd[:, :, h0:h1].contiguous(),
                                   vd[:, :, h0:h1].contiguous(), sd, td, scale))
        # the split size depends on the head count, so shards may round differently
        torch.testing.assert_close(torch.cat(parts, dim=1).float(), full.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("ctx", [[0, 40, 200, 16, 255], [1, 256]])
def test_decode_single_chunk_writes_output_directly(ctx):
    """Contexts that fit one chunk: the split kernel writes the output rows (no partials,
    no combine kernel, no workspace); an empty sequence gives a zero row."""
    dev = cuda_device()
    q, kc, vc, seq, table = make_case(ctx, 32, 8, 64, seed=17)
    ref = oracle.paged_decode(q, kc, vc, seq, table, 0.09)
    qd, kd, vd, sd, td = (t.to(dev) for t in (q, kc, vc, seq, table))
    out = torch.full_like(qd, 3.0)
    msl = table.shape[1] * 16
    assert capi.lib().ntb200_paged_attention_decode_workspace_size(len(ctx), 32, 8, 128, 16, msl) == 0
    capi.call("ntb200_paged_attention_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(sd), ptr(td),
              len(ctx), 32, 8, 128, 16, 64, table.shape[1], table.shape[1], msl, 0.09,
              32 * 128, 128, 32 * 128, 128, kd.stride(0), kd.stride(1), kd.stride(2), None, 0, 1, stream())
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)
    if ctx[0] == 0:
        assert not out[0].any()
    assert capi.read_device_error(stream()) == 0


def test_decode_direct_mode_flags_a_sequence_longer_than_max_seq_len():
    """max_seq_len = 256 at a batch of 2 makes the call a single-chunk (direct) decode; a
    sequence of 600 tokens breaks that contract and must raise the index-range flag (its
    row covers only the first chunk), while the sequence within the bound is exact."""
    dev = cuda_device()
    ctx = [600, 100]
    q, kc, vc, seq, table = make_case(ctx, 32, 8, 64, seed=23)
    ref = oracle.paged_decode(q, kc, vc, seq, table, 0.09)
    qd, kd, vd, sd, td = (t.to(dev) for t in (q, kc, vc, seq, table))
    out = torch.empty_like(qd)
    assert capi.lib().ntb200_paged_attention_decode_workspace_size(2, 32, 8, 128, 16, 256) == 0
    capi.call("ntb200_paged_attention_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(sd), ptr(td),
              2, 32, 8, 128, 16, 64, table.shape[1], table.shape[1], 256, 0.09,
              32 * 128, 128, 32 * 128, 128, kd.stride(0), kd.stride(1), kd.stride(2), None, 0, 1, stream())
    torch.cuda.synchronize()
    torch.testing.assert_close(out[1].float().cpu(), ref[1], rtol=TOL, atol=TOL)
    assert capi.read_device_error(stream()) == capi.DEVERR_INDEX_RANGE

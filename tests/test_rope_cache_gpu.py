"""GPU parity of the fused RoPE + paged KV-cache store (ntb200_rope_and_cache) against the
CPU oracle (rope_neox followed by reshape_and_cache) and against this library's own two
unfused kernels.  Everything is checked bit for bit: q, k, the untouched v and both
caches."""

import pytest
import torch

import oracle
from _util import bits_equal, cuda_device, ptr, seeded, stream
from vllm_nt._ntops import capi
from vllm_nt._ntops.torch._ext import ops
from vllm_nt._ntops.torch.rotary_emb import rotary_embedding_and_cache

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_device_error():
    dev = cuda_device()
    torch.cuda.synchronize(dev)
    capi.read_device_error(stream())
    yield
    torch.cuda.synchronize(dev)


def _qkv(t, hq, hk, d, dtype, seed, pad_cols=0):
    """A fused qkv projection output [t, (hq + 2 hk) d] (row stride + pad_cols) and its
    q/k/v column slices, as vLLM's attention layer hands them to RoPE and the KV store."""
    g = seeded(seed)
    width = (hq + 2 * hk) * d
    buf = torch.randn(t, width + pad_cols, generator=g).to(dtype)
    qkv = buf[:, :width]
    return buf, qkv[:, : hq * d], qkv[:, hq * d : (hq + hk) * d], qkv[:, (hq + hk) * d :]


def _oracle(pos, q, k, v, cache_f32, kc, vc, slots, d, rot):
    kc, vc = kc.clone(), vc.clone()
    rq, rk = oracle.rope_and_cache(pos, q.contiguous(), k.contiguous(), v.contiguous(), cache_f32, kc, vc, slots, d,
                                   rot)
    return rq, rk, kc, vc


def test_llama_decode_batch_flash_layout_bit_exact():
    """256 decode tokens of a Llama-3-8B layer (32/8 heads, head 128, theta 5e5, positions
    up to 8192) into vLLM's FlashAttention cache [2, blocks, 16, 8, 128], every 17th slot
    a -1 padding slot: the 16-byte vector path."""
    dev = cuda_device()
    t, hq, hk, d = 256, 32, 8, 128
    buf, q, k, v = _qkv(t, hq, hk, d, torch.bfloat16, 21)
    g = seeded(22)
    pos = torch.randint(0, 8192, (t,), generator=g)
    cache = oracle.build_cos_sin_cache(d, 8192, 500000.0)
    blocks = 64
    slots = torch.randperm(blocks * 16, generator=g)[:t]
    slots[::17] = -1
    kv = torch.zeros(2, blocks, 16, hk, d, dtype=torch.bfloat16)
    rq, rk, rkc, rvc = _oracle(pos, q, k, v, cache, kv[0], kv[1], slots, d, d)

    bufd, kvd = buf.to(dev), kv.to(dev)
    width = (hq + 2 * hk) * d
    qd, kd, vd = bufd[:, : hq * d], bufd[:, hq * d : (hq + hk) * d], bufd[:, (hq + hk) * d : width]
    ops().rope_and_cache_flash_layout(pos.to(dev), qd, kd, vd, cache.to(torch.bfloat16).to(dev), kvd, slots.to(dev),
                                      d, d, 0)
    torch.cuda.synchronize()
    assert bits_equal(qd.cpu().contiguous(), rq)
    assert bits_equal(kd.cpu().contiguous(), rk)
    assert bits_equal(vd.cpu().contiguous(), v.contiguous())  # v is read only
    assert bits_equal(kvd[0].cpu(), rkc)
    assert bits_equal(kvd[1].cpu(), rvc)
    assert capi.read_device_error(stream()) == 0


def test_config_c_fp32_capi_separate_caches():
    """Config (c) shapes in fp32 (q [128, 32x128], k and v [128, 8x128], base 1e4,
    positions < 4096) through the C ABI, with separate K and V caches."""
    dev = cuda_device()
    g = seeded(23)
    t, hq, hk, d = 128, 32, 8, 128
    q = torch.randn(t, hq * d, generator=g)
    k = torch.randn(t, hk * d, generator=g)
    v = torch.randn(t, hk * d, generator=g)
    pos = torch.randint(0, 4096, (t,), generator=g)
    cache = oracle.build_cos_sin_cache(d, 4096, 10000.0)
    blocks = 16
    slots = torch.randperm(blocks * 16, generator=g)[:t]
    kc = torch.zeros(blocks, 16, hk, d)
    vc = torch.zeros_like(kc)
    rq, rk, rkc, rvc = _oracle(pos, q, k, v, cache, kc, vc, slots, d, d)
    qd, kd, vd, kcd, vcd = q.to(dev), k.to(dev), v.to(dev), kc.to(dev), vc.to(dev)
    posd, sd, cd = pos.to(dev), slots.to(dev), cache.to(dev)
    capi.call("ntb200_rope_and_cache", ptr(posd), 4, ptr(qd), ptr(kd), ptr(vd), ptr(cd), ptr(kcd), ptr(vcd), ptr(sd),
              4, t, t, hq, hk, d, d, hq * d, d, hk * d, d, hk * d, d, d, 4096, 16, blocks * 16, 16 * hk * d, hk * d,
              d, 0, stream())
    torch.cuda.synchronize()
    assert bits_equal(qd.cpu(), rq) and bits_equal(kd.cpu(), rk)
    assert bits_equal(kcd.cpu(), rkc) and bits_equal(vcd.cpu(), rvc)
    assert bits_equal(vd.cpu(), v)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_partial_rotary_scalar_path_int32_padded_rows(dtype):
    """rotary_dim 64 < head 128 (the k dims past it are copied into the cache as they
    are); an odd row stride forces the scalar path; int32 positions and slots; the slot
    mapping covers only the first t - 3 rows (vLLM's padded rows are rotated only)."""
    dev = cuda_device()
    t, hq, hk, d, rot = 37, 8, 2, 128, 64
    buf, q, k, v = _qkv(t, hq, hk, d, dtype, 24, pad_cols=1)
    g = seeded(25)
    pos = torch.randint(0, 2048, (t,), generator=g).to(torch.int32)
    cache = oracle.build_cos_sin_cache(rot, 2048, 500000.0)
    blocks = 8
    slots = torch.randperm(blocks * 16, generator=g)[: t - 3].to(torch.int32)
    slots[[2, 9]] = -1
    kc = torch.zeros(blocks, 16, hk, d, dtype=dtype)
    vc = torch.zeros_like(kc)
    rq, rk, rkc, rvc = _oracle(pos, q, k, v, cache, kc, vc, slots, d, rot)
    bufd, kcd, vcd = buf.to(dev), kc.to(dev), vc.to(dev)
    width = (hq + 2 * hk) * d
    qd, kd, vd = bufd[:, : hq * d], bufd[:, hq * d : (hq + hk) * d], bufd[:, (hq + hk) * d : width]
    assert qd.stride(0) % 8 != 0
    rotary_embedding_and_cache(pos.to(dev), qd, kd, vd, d, cache.to(dtype).to(dev), kcd, vcd, slots.to(dev), rot)
    torch.cuda.synchronize()
    assert bits_equal(qd.cpu().contiguous(), rq) and bits_equal(kd.cpu().contiguous(), rk)
    assert bits_equal(kcd.cpu(), rkc) and bits_equal(vcd.cpu(), rvc)
    assert bits_equal(bufd[:, width:].cpu(), buf[:, width:])  # the pad column is untouched
    assert capi.read_device_error(stream()) == 0


@pytest.mark.parametrize("t", [1024, 4096])
def test_flashinfer_hnd_cache_matches_oracle_and_unfused_kernels(t):
    """FlashInfer's cache [blocks, 2, 16, H, D] in HND memory order (kv_dim 1, head stride
    16 x 128) at prefill-sized steps: 1024 tokens (the fused kernel) and 4096 tokens (the
    entry point launches the RoPE and KV-store kernels from 4096 tokens on).  Both leave the
    oracle's bits, and the same bits as calling the two kernels directly."""
    dev = cuda_device()
    hq, hk, d = 32, 8, 128
    buf, q, k, v = _qkv(t, hq, hk, d, torch.bfloat16, 26)
    g = seeded(27)
    pos = torch.randint(0, 16384, (t,), generator=g)
    cache = oracle.build_cos_sin_cache(d, 16384, 500000.0)
    cache_d = cache.to(torch.bfloat16).to(dev)
    blocks = 512
    slots = torch.randperm(blocks * 16, generator=g)[:t]
    width = (hq + 2 * hk) * d
    zeros = torch.zeros(blocks, 16, hk, d, dtype=torch.bfloat16)
    rq, rk, rkc, rvc = _oracle(pos, q, k, v, cache, zeros, zeros, slots, d, d)

    def fresh():
        b = buf.to(dev)
        kv = torch.zeros(blocks, 2, hk, 16, d, dtype=torch.bfloat16, device=dev).permute(0, 1, 3, 2, 4)
        return b, b[:, : hq * d], b[:, hq * d : (hq + hk) * d], b[:, (hq + hk) * d : width], kv

    b1, q1, k1, v1, kv1 = fresh()
    ops().rope_and_cache_flash_layout(pos.to(dev), q1, k1, v1, cache_d, kv1, slots.to(dev), d, d, 1)
    b2, q2, k2, v2, kv2 = fresh()
    ops().rotary_embedding_neox(pos.to(dev), q2, k2, cache_d, d, d)
    ops().store_flash_layout(k2, v2, kv2, slots.to(dev), 1)
    torch.cuda.synchronize()
    assert kv1.stride(3) == 16 * d  # HND: heads outermost inside a page
    assert bits_equal(b1.cpu(), b2.cpu())
    assert bits_equal(kv1.contiguous().cpu(), kv2.contiguous().cpu())
    assert bits_equal(q1.cpu().contiguous(), rq) and bits_equal(k1.cpu().contiguous(), rk)
    assert bits_equal(kv1[:, 0].contiguous().cpu(), rkc) and bits_equal(kv1[:, 1].contiguous().cpu(), rvc)
    assert capi.read_device_error(stream()) == 0


def test_out_of_range_position_and_slot_are_flagged_and_skipped():
    """As the two kernels in sequence: a position past the cos/sin cache leaves its token's
    q/k unrotated (its unrotated k and its v are still stored); a slot past the cache is
    rotated but not stored; both raise the index-range bit."""
    dev = cuda_device()
    t, hq, hk, d = 4, 2, 1, 128
    buf, q, k, v = _qkv(t, hq, hk, d, torch.bfloat16, 28)
    cache = oracle.build_cos_sin_cache(d, 64, 10000.0)
    pos = torch.tensor([3, 99, 5, 7])
    slots = torch.tensor([0, 1, 32, 2])  # 32 == num_slots (2 blocks of 16)
    kc = torch.zeros(2, 16, hk, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    bufd, kcd, vcd = buf.to(dev), kc.to(dev), vc.to(dev)
    width = (hq + 2 * hk) * d
    qd, kd, vd = bufd[:, : hq * d], bufd[:, hq * d : (hq + hk) * d], bufd[:, (hq + hk) * d : width]
    ops().rope_and_cache(pos.to(dev), qd, kd, vd, cache.to(torch.bfloat16).to(dev), kcd, vcd, slots.to(dev), d, d)
    torch.cuda.synchronize()
    assert capi.read_device_error(stream()) & capi.DEVERR_INDEX_RANGE
    ok = [0, 2, 3]
    rq, rk = oracle.rope_neox(pos[ok], q[ok].contiguous(), k[ok].contiguous(), cache, d, d)
    assert bits_equal(qd[ok].cpu(), rq) and bits_equal(kd[ok].cpu(), rk)
    assert bits_equal(qd[1].cpu(), q[1]) and bits_equal(kd[1].cpu(), k[1])  # token 1 unrotated
    kflat, vflat = kcd.view(32, hk * d).cpu(), vcd.view(32, hk * d).cpu()
    assert bits_equal(kflat[0], rk[0]) and bits_equal(kflat[2], rk[2])
    assert bits_equal(vflat[0], v[0]) and bits_equal(vflat[2], v[3])
    assert bits_equal(kflat[1], k[1]) and bits_equal(vflat[1], v[1])  # token 1 stored unrotated
    assert kflat[3:].count_nonzero() == 0 and vflat[3:].count_nonzero() == 0  # token 2 (slot 32) not stored

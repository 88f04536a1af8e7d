"""Pins the CPU oracle against (a) golden outputs of the real reference implementations
(tests/golden/make_golden.py) and (b) the known-answer cases of the reference's own tests.
CPU only."""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from _util import bits_equal, golden, seeded


@pytest.mark.parametrize("tag", ["f32", "bf16", "f16"])
def test_rms_norm_matches_vllm_native(tag):
    g = golden(f"rms_norm_{tag}")
    y, res = oracle.fused_add_rms_norm(g["x"], g["residual"], g["weight"], 1e-6)
    assert bits_equal(res, g["residual_out"])
    torch.testing.assert_close(y, g["out"], rtol=0, atol=0)
    torch.testing.assert_close(oracle.rms_norm(g["x"], g["weight"], 1e-6), g["out_plain"], rtol=0, atol=0)


@pytest.mark.parametrize("tag", ["f32", "bf16", "f16"])
def test_gemma_rms_norm_matches_vllm_native(tag):
    """GemmaRMSNorm.forward_native outputs (tests/golden/gemma_rms_norm.npz), bit for bit,
    including the fp32 residual vLLM hands back for fp16 inputs."""
    g = golden("gemma_rms_norm")
    x, r, w = g[f"{tag}_x"], g[f"{tag}_residual"], g[f"{tag}_weight"]
    assert bits_equal(oracle.gemma_rms_norm(x, w, 1e-6), g[f"{tag}_out_plain"])
    out, res = oracle.gemma_rms_norm(x, w, 1e-6, r)
    assert bits_equal(out, g[f"{tag}_out"]) and bits_equal(res, g[f"{tag}_residual_out"])


@pytest.mark.parametrize("tag", ["f32", "bf16", "f16"])
def test_silu_and_mul_matches_vllm_native(tag):
    g = golden(f"silu_and_mul_{tag}")
    out = oracle.silu_and_mul(g["x"])
    tol = 1e-6 if tag == "f32" else 0.0  # exp rounding may differ by an ulp in fp32
    torch.testing.assert_close(out, g["out"], rtol=tol, atol=tol)


@pytest.mark.parametrize("tag", ["f32", "bf16", "f16"])
def test_rope_matches_vllm_forward_static(tag):
    g = golden(f"rope_{tag}")
    cache = oracle.build_cos_sin_cache(64, 128, 10000.0)
    assert bits_equal(cache, g["cos_sin_cache"])
    qo, ko = oracle.rope_neox(g["positions"], g["query"], g["key"], g["cos_sin_cache"], 64, 64)
    assert bits_equal(qo, g["query_out"]) and bits_equal(ko, g["key_out"])
    qp, kp = oracle.rope_neox(g["positions"], g["query"], g["key"], g["cos_sin_cache_rot32"], 64, 32)
    assert bits_equal(qp, g["query_out_rot32"]) and bits_equal(kp, g["key_out_rot32"])



@pytest.mark.parametrize("tag", ["f32", "bf16"])
@pytest.mark.parametrize("rot", [64, 32])
def test_rope_and_cache_is_rope_then_store(tag, rot):
    """The fused restatement against the RoPE golden outputs (vLLM forward_static): q/k
    rotated as the fixture says, the rotated key rows and the value rows at their slots,
    padding slots and rows past the slot mapping not stored."""
    g = golden(f"rope_{tag}")
    suffix = "" if rot == 64 else "_rot32"
    value = g["key"].flip(0).contiguous()
    slots = torch.tensor([5, -1, 0, 13, 7])  # 5 of 6 rows: the last is a padded row
    kc = torch.zeros(4, 4, 2, 64, dtype=value.dtype)
    vc = torch.zeros_like(kc)
    qo, ko = oracle.rope_and_cache(g["positions"], g["query"], g["key"], value, g["cos_sin_cache" + suffix], kc, vc,
                                   slots, 64, rot)
    assert bits_equal(qo, g["query_out" + suffix]) and bits_equal(ko, g["key_out" + suffix])
    kflat, vflat = kc.reshape(16, 2, 64), vc.reshape(16, 2, 64)
    stored = [(t, int(sl)) for t, sl in enumerate(slots) if sl >= 0]
    for t, sl in stored:
        assert bits_equal(kflat[sl], g["key_out" + suffix][t].reshape(2, 64))
        assert bits_equal(vflat[sl], value[t].reshape(2, 64))
    untouched = sorted(set(range(16)) - {sl for _, sl in stored})
    assert not kflat[untouched].any() and not vflat[untouched].any()

def test_kv_store_matches_reference_torch_store():
    g = golden("kv_store_bf16")
    kc = np.zeros((8, 4, 2, 16), dtype=np.uint16)
    vc = np.zeros_like(kc)
    k16 = g["key"].view(torch.int16).numpy().view(np.uint16)
    v16 = g["value"].view(torch.int16).numpy().view(np.uint16)
    oracle.reshape_and_cache(k16, v16, kc, vc, g["slot_mapping"].numpy())
    assert np.array_equal(kc, g["key_cache_out"].view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(vc, g["value_cache_out"].view(torch.int16).numpy().view(np.uint16))


def test_kv_store_reference_known_answer():
    """vllm_nt/tests/test_kv_cache.py:26-45: 3 tokens x 2 heads x 4 dims into an 8x8 flat
    cache at slots [1, 4, 6] (a flat cache is block_size 1)."""
    rng = np.random.default_rng(0)
    key = rng.standard_normal((3, 2, 4)).astype(np.float32)
    value = rng.standard_normal((3, 2, 4)).astype(np.float32)
    kc = np.zeros((8, 1, 2, 4), np.float32)
    vc = np.zeros_like(kc)
    oracle.reshape_and_cache(key, value, kc, vc, np.array([1, 4, 6], np.int32))
    for t, s in enumerate([1, 4, 6]):
        assert np.array_equal(kc[s, 0], key[t]) and np.array_equal(vc[s, 0], value[t])
    assert not kc[[0, 2, 3, 5, 7]].any()


def test_embedding_matches_f_embedding():
    g = golden("embedding_bf16")
    w16 = g["weight"].view(torch.int16).numpy()
    out = oracle.embedding(g["ids"].numpy(), w16)
    assert np.array_equal(out, g["out"].view(torch.int16).numpy())


def test_paged_decode_matches_sdpa_golden():
    g = golden("paged_decode_bf16")
    out = oracle.paged_decode(g["query"], g["key_cache"], g["value_cache"], g["seq_lens"], g["block_table"])
    torch.testing.assert_close(out, g["out"], rtol=1e-5, atol=1e-5)


def test_paged_decode_reference_known_answer():
    """vllm_nt/tests/test_attention.py:75-104: q (2,1,2,8), cache (4 blocks, bs 2, 2 heads,
    8), seqlens [3, 4], tables [[0,1],[2,3]], checked against SDPA over gathered tokens."""
    g = seeded(1)
    q = torch.randn((2, 2, 8), generator=g)
    kc = torch.randn((4, 2, 2, 8), generator=g)
    vc = torch.randn((4, 2, 2, 8), generator=g)
    seq = torch.tensor([3, 4], dtype=torch.int32)
    table = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32)
    out = oracle.paged_decode(q, kc, vc, seq, table)
    for b in range(2):
        n = int(seq[b])
        k = kc[table[b].long()].reshape(-1, 2, 8)[:n].transpose(0, 1).unsqueeze(0)
        v = vc[table[b].long()].reshape(-1, 2, 8)[:n].transpose(0, 1).unsqueeze(0)
        ref = F.scaled_dot_product_attention(q[b].unsqueeze(0).unsqueeze(2), k, v)[0, :, 0]
        torch.testing.assert_close(out[b], ref, rtol=1e-5, atol=1e-5)


def test_paged_decode_empty_sequence_is_zero():
    q = torch.randn(2, 4, 16)
    kc = torch.randn(3, 4, 2, 16)
    out = oracle.paged_decode(q, kc, kc, torch.tensor([0, 2], dtype=torch.int32), torch.tensor([[0], [1]], dtype=torch.int32))
    assert not out[0].any() and out[1].abs().sum() > 0


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_linear_matches_f_linear(tag):
    g = golden(f"linear_{tag}")
    torch.testing.assert_close(oracle.linear(g["x"], g["weight"], g["bias"]), g["out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("m,k,n", [(1, 4096, 512), (5, 1032, 700), (16, 2048, 256)])
@pytest.mark.parametrize("with_residual", [False, True])
def test_fused_norm_linear_rounding_is_no_less_accurate_than_the_pair(m, k, n, with_residual):
    """The fused entry point's rounding points (s * w rounded once, 1/rms on the fp32
    products): the new residual is the pair's bit for bit, the output differs from the
    pair's (vLLM's RMSNorm rounded, then F.linear) by rounding only, and its RMS error
    against the unrounded fp64 value is no larger than the pair's."""
    g = seeded(100 * m + k + n + with_residual)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    res = torch.randn(m, k, generator=g).to(torch.bfloat16) if with_residual else None
    gamma = (1.0 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, generator=g)).to(torch.bfloat16)
    out, new_res = oracle.rms_norm_linear(x, gamma, 1e-5, w, res)
    if with_residual:
        h, res_pair = oracle.fused_add_rms_norm(x, res, gamma, 1e-5)
        assert bits_equal(new_res, res_pair)
    else:
        h = oracle.rms_norm(x, gamma, 1e-5)
        assert new_res is None
    pair = oracle.linear(h, w)
    torch.testing.assert_close(out, pair, rtol=2e-2, atol=2e-2)
    exact = oracle.rms_norm_linear_exact(x, gamma, 1e-5, w, res)
    err = (out.to(torch.bfloat16).double() - exact).pow(2).mean().sqrt()
    err_pair = (pair.to(torch.bfloat16).double() - exact).pow(2).mean().sqrt()
    assert err <= err_pair


def test_rope_reference_known_answer():
    """vllm_nt/tests/test_rope.py:26-46: x (5,4,8), per-token cos/sin (5,1,4); reference
    cat(x1*cos - x2*sin, x2*cos + x1*sin)."""
    g = seeded(2)
    x = torch.randn(5, 4, 8, generator=g)
    cos = torch.randn(5, 4, generator=g)
    sin = torch.randn(5, 4, generator=g)
    table = torch.cat((cos, sin), dim=-1)
    out, _ = oracle.rope_neox(torch.arange(5), x, None, table, 8, 8)
    x1, x2 = x[..., :4], x[..., 4:]
    ref = torch.cat((x1 * cos[:, None] - x2 * sin[:, None], x2 * cos[:, None] + x1 * sin[:, None]), dim=-1)
    assert bits_equal(out, ref)


def test_rms_norm_reference_known_answer():
    """vllm_nt/tests/test_oot.py:33-77 reference: fp32 statistics, cast back."""
    g = seeded(3)
    for shape in [(1, 4096), (32, 4096), (1, 32, 4096)]:
        x = torch.randn(shape, generator=g)
        w = torch.randn(shape[-1], generator=g)
        ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
        torch.testing.assert_close(oracle.rms_norm(x, w, 1e-6), ref, rtol=0, atol=0)


def test_silu_reference_known_answer():
    g = seeded(4)
    for shape in [(1, 8192), (32, 8192), (1, 32, 8192)]:
        x = torch.randn(shape, generator=g)
        d = shape[-1] // 2
        torch.testing.assert_close(oracle.silu_and_mul(x), F.silu(x[..., :d]) * x[..., d:], rtol=1e-6, atol=1e-6)


def test_cos_sin_cache_matches_vllm_definition():
    c = oracle.build_cos_sin_cache(128, 4096, 500000.0)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    assert c.shape == (4096, 128)
    torch.testing.assert_close(c[:, :64], torch.cos(torch.arange(4096).float()[:, None] * inv), rtol=0, atol=0)
    assert math.isclose(float(c[0, 0]), 1.0)


def test_paged_prefill_matches_sdpa_golden():
    g = golden("paged_prefill_bf16")
    out = oracle.paged_prefill(g["query"], g["key_cache"], g["value_cache"], g["query_start_loc"], g["seq_lens"],
                               g["block_table"])
    torch.testing.assert_close(out, g["out"], rtol=1e-5, atol=1e-5)


def test_varlen_reference_known_answer():
    """vllm_nt/tests/test_attention.py:57-72: q/k/v (5, 2, 8), cu_q = cu_k = [0, 2, 5],
    causal, checked against SDPA(is_causal=True) per sequence (equal q and k lengths, where
    the start- and end-aligned masks coincide)."""
    g = seeded(3)
    q = torch.randn((5, 2, 8), generator=g)
    k = torch.randn((5, 2, 8), generator=g)
    v = torch.randn((5, 2, 8), generator=g)
    cu = torch.tensor([0, 2, 5], dtype=torch.int32)
    out = oracle.varlen_attention(q, k, v, cu, cu)
    for b in range(2):
        sl = slice(int(cu[b]), int(cu[b + 1]))
        ref = F.scaled_dot_product_attention(q[sl].transpose(0, 1)[None], k[sl].transpose(0, 1)[None],
                                             v[sl].transpose(0, 1)[None], is_causal=True)[0].transpose(0, 1)
        torch.testing.assert_close(out[sl], ref, rtol=1e-5, atol=1e-5)


def test_varlen_end_aligned_mask_with_prefix():
    """With a cached prefix (ctx > q_len) the last query sees every key (a decode step) and
    the first sees ctx - q_len + 1 of them; the result equals attention over that prefix of
    the keys."""
    g = seeded(4)
    q = torch.randn((3, 4, 16), generator=g)
    k = torch.randn((10, 2, 16), generator=g)
    v = torch.randn((10, 2, 16), generator=g)
    out = oracle.varlen_attention(q, k, v, torch.tensor([0, 3], dtype=torch.int32),
                                  torch.tensor([0, 10], dtype=torch.int32))
    for i in range(3):
        n = 10 - 3 + i + 1
        kk = k[:n].repeat_interleave(2, dim=1).transpose(0, 1)  # [Hq, n, D]
        vv = v[:n].repeat_interleave(2, dim=1).transpose(0, 1)
        ref = F.scaled_dot_product_attention(q[i][:, None], kk, vv)[:, 0]
        torch.testing.assert_close(out[i], ref, rtol=1e-5, atol=1e-5)


def test_paged_prefill_equals_varlen_over_gathered_tokens():
    g = seeded(5)
    kc = torch.randn(9, 4, 2, 16, generator=g)
    vc = torch.randn(9, 4, 2, 16, generator=g)
    seq = torch.tensor([5, 9], dtype=torch.int32)
    table = torch.tensor([[3, 7, 0], [8, 1, 5]], dtype=torch.int32)
    cu_q = torch.tensor([0, 5, 8], dtype=torch.int32)
    q = torch.randn(8, 4, 16, generator=g)
    k, v, cu_k = oracle.gather_paged_kv(kc, vc, seq, table)
    assert cu_k.tolist() == [0, 5, 14]
    assert torch.equal(k[5:9], kc[8].reshape(4, 2, 16)) and torch.equal(k[13], kc[5, 0])
    torch.testing.assert_close(oracle.paged_prefill(q, kc, vc, cu_q, seq, table),
                               oracle.varlen_attention(q, k, v, cu_q, cu_k))


def test_sampler_matches_the_reference_torch_sampler():
    """tests/golden/sampler_f32.npz holds the reference's own apply_top_k_top_p and
    random_sample outputs (and vLLM's native top-k/top-p, identical on it): the oracle
    reproduces them bit for bit, ties at a top-k cut and -inf entries included."""
    g = golden("sampler_f32")
    logits, k, p = g["logits"], g["k"], g["p"]
    assert bits_equal(oracle.apply_top_k_top_p(logits, k, None), g["top_k_out"])
    assert bits_equal(oracle.apply_top_k_top_p(logits, None, p), g["top_p_out"])
    assert bits_equal(oracle.apply_top_k_top_p(logits, k, p), g["top_k_top_p_out"])
    assert bits_equal(g["top_k_top_p_out_vllm"], g["top_k_top_p_out"])
    assert bits_equal(oracle.apply_top_k_top_p(logits, None, None), logits)
    assert torch.equal(oracle.random_sample_from_draws(g["probs"], g["q"]), g["sample"])
    # ties at the top-k cut of row 5 are all kept: more than k survive
    assert int((g["top_k_out"][5] != float("-inf")).sum()) > int(k[5])


def test_top_p_cumulative_is_the_quantity_top_p_compares():
    """Every logit the reference drops for top-p has a running probability <= 1 - p (up to
    fp32 summation error) and every survivor but the row maximum one above it."""
    g = golden("sampler_f32")
    run = oracle.top_p_cumulative(g["logits"], g["k"])
    both = g["top_k_top_p_out"]
    topk = g["top_k_out"]
    for b in range(both.shape[0]):
        limit = 1 - float(g["p"][b])
        dropped = (both[b] == float("-inf")) & (topk[b] != float("-inf"))
        kept = both[b] != float("-inf")
        assert (run[b][dropped] <= limit + 1e-6).all()
        top = int(topk[b].argmax())
        kept[top] = False
        assert (run[b][kept] > limit - 1e-6).all()

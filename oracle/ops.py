"""CPU restatements of the hooked ops (test infrastructure; see oracle/__init__.py).

All functions take and return CPU tensors / numpy arrays; nothing here touches a GPU."""

from __future__ import annotations

import math

import numpy as np
import torch


def _round(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 -> storage dtype -> fp32 (round-to-nearest-even), a torch op's rounding point."""
    return t.to(dtype).to(torch.float32)


# --------------------------------------------------------------------------------------
# RMS norm  (vllm:ir/ops/layernorm.py:10-62; vllm_nt/_ntops/oot_support.py:32-48)
# --------------------------------------------------------------------------------------


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) in fp32; normalised value rounded to the weight dtype,
    multiplied by the weight, rounded to x's dtype."""
    dtype = x.dtype
    xf = x.to(torch.float32)
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    y = xf * torch.rsqrt(var + eps)
    if weight is not None:
        y = _round(y, weight.dtype) * weight.to(torch.float32)
    return y.to(dtype)


def fused_add_rms_norm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor | None, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """s = x + residual in fp32; returns (rms_norm of the fp32 s, s rounded to x's dtype).

    (vLLM adds in fp32, vllm:ir/ops/layernorm.py:40-62; the reference's adapter adds in the
    input dtype first, vllm_nt/_ntops/oot_support.py:39-41 -- parity is defined against
    vLLM's native path.)"""
    dtype = x.dtype
    s = x.to(torch.float32) + residual.to(torch.float32)
    new_residual = s.to(dtype)
    var = s.pow(2).mean(dim=-1, keepdim=True)
    y = s * torch.rsqrt(var + eps)
    if weight is not None:
        y = _round(y, weight.dtype) * weight.to(torch.float32)
    return y.to(dtype), new_residual


def gemma_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
                   residual: torch.Tensor | None = None):
    """GemmaRMSNorm.forward_native (vllm:model_executor/layers/layernorm.py:153-170):
    w1 = weight.float() + 1 (fp32); with a residual s = x + residual in x's dtype (fp16 sums
    in fp32 and keeps an fp32 residual); out = x_f32 * rsqrt(mean(x_f32^2) + eps) * w1,
    rounded once to x's dtype.  Returns out, or (out, s)."""
    dtype = x.dtype
    w1 = weight.to(torch.float32) + 1.0
    if residual is not None:
        if dtype == torch.float16:
            x = x.to(torch.float32) + residual.to(torch.float32)
        else:
            x = (x.to(torch.float32) + residual.to(torch.float32)).to(dtype)
        residual = x
    xf = x.to(torch.float32)
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    out = (xf * torch.rsqrt(var + eps) * w1).to(dtype)
    return out if residual is None else (out, residual)


# --------------------------------------------------------------------------------------
# SiluAndMul  (vllm:model_executor/layers/activation.py:137-141;
#              vllm_nt/_ntops/oot_support.py:51-56, vllm_nt/_ntops/kernels/silu.py:9-18)
# --------------------------------------------------------------------------------------


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """silu(gate) rounded to x's dtype, times up, rounded again."""
    d = x.shape[-1] // 2
    g = x[..., :d].to(torch.float32)
    u = x[..., d:].to(torch.float32)
    a = _round(g / (1.0 + torch.exp(-g)), x.dtype)
    return (a * u).to(x.dtype)


# --------------------------------------------------------------------------------------
# NeoX RoPE  (vllm:model_executor/layers/rotary_embedding/base.py:69-92 (cache),
#             base.py:140-180 + common.py:144-183 (apply);
#             vllm_nt/_ntops/oot_support.py:134-204, vllm_nt/_ntops/kernels/rotary_emb.py:6-37)
# --------------------------------------------------------------------------------------


def build_cos_sin_cache(rotary_dim: int, max_position: int, base: float) -> torch.Tensor:
    """[max_position, rotary_dim] fp32 table cat(cos, sin) of position * inv_freq."""
    inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.einsum("i,j->ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def rope_neox(
    positions: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor | None,
    cos_sin_cache: torch.Tensor,
    head_size: int,
    rotary_dim: int,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Returns rotated copies of query/key ([tokens, heads*head_size] or 3-D).  Each torch
    op of the native path is one rounding point: x1*c, x2*s, their difference, ..."""

    def rot(x: torch.Tensor) -> torch.Tensor:
        dtype = x.dtype
        n = positions.numel()
        cs = cos_sin_cache.index_select(0, positions.reshape(-1).long()).to(dtype)
        c = cs[:, : rotary_dim // 2].to(torch.float32).unsqueeze(1)
        s = cs[:, rotary_dim // 2 : rotary_dim].to(torch.float32).unsqueeze(1)
        v = x.reshape(n, -1, head_size)
        r = v[..., :rotary_dim].to(torch.float32)
        x1, x2 = r[..., : rotary_dim // 2], r[..., rotary_dim // 2 :]
        o1 = (_round(x1 * c, dtype) - _round(x2 * s, dtype)).to(dtype)
        o2 = (_round(x2 * c, dtype) + _round(x1 * s, dtype)).to(dtype)
        out = v.clone()
        out[..., : rotary_dim // 2] = o1
        out[..., rotary_dim // 2 : rotary_dim] = o2
        return out.reshape(x.shape)

    return rot(query), (rot(key) if key is not None else None)


# --------------------------------------------------------------------------------------
# KV-cache store  (vllm_nt/_ntops/kernels/kv_cache.py:4-45, vllm_nt/_ntops/torch/kv_cache.py:7-21;
#                  negative padding slots skipped as vllm_nt/_ntops/patching.py:1752-1770 does)
# --------------------------------------------------------------------------------------


def reshape_and_cache(
    key: np.ndarray,
    value: np.ndarray,
    key_cache: np.ndarray,
    value_cache: np.ndarray,
    slot_mapping: np.ndarray,
) -> None:
    """In place on numpy arrays: cache[slot // bs, slot % bs] = key[t] for slot >= 0.
    key/value [T, H, D]; caches [blocks, bs, H, D]; any element type (a byte copy)."""
    bs = key_cache.shape[1]
    slots = np.asarray(slot_mapping).reshape(-1).astype(np.int64)
    t = np.nonzero(slots >= 0)[0]
    s = slots[t]
    key_cache[s // bs, s % bs] = key[t]
    value_cache[s // bs, s % bs] = value[t]


# --------------------------------------------------------------------------------------
# RoPE followed by the KV-cache store: the two hooks of one attention layer in vLLM's
# order (vllm:model_executor/models/llama.py:228-231 rotates q/k, then
# vllm:model_executor/layers/attention/attention.py:498-518 stores the rotated k and v);
# vllm_nt reaches them as vllm_nt/_ntops/patching.py:1323-1354 then 532-562.
# --------------------------------------------------------------------------------------


def _bits(t: torch.Tensor) -> np.ndarray:
    """numpy view of a contiguous CPU tensor's raw bits (shares memory)."""
    width = {1: torch.int8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.view(width).numpy()


def rope_and_cache(
    positions: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    head_size: int,
    rotary_dim: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns rotated copies of query/key (rope_neox) and stores the rotated key and the
    value into the contiguous CPU caches [blocks, bs, Hkv, D] in place (reshape_and_cache,
    a bit copy): rows t < slot_mapping.numel() with slot >= 0."""
    q, k = rope_neox(positions, query, key, cos_sin_cache, head_size, rotary_dim)
    n = slot_mapping.numel()
    k3 = k.reshape(k.shape[0], -1, head_size)[:n].contiguous()
    v3 = value.reshape(value.shape[0], -1, head_size)[:n].contiguous()
    reshape_and_cache(_bits(k3), _bits(v3), _bits(key_cache), _bits(value_cache), slot_mapping.numpy())
    return q, k


# --------------------------------------------------------------------------------------
# Embedding  (vllm_nt/_ntops/kernels/wpe.py:11-67, vllm_nt/_ntops/torch/embedding.py:7-30;
#             vllm:model_executor/layers/vocab_parallel_embedding.py:77-78 = F.embedding)
# --------------------------------------------------------------------------------------


def embedding(ids: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """weight[ids] (a row gather, exact)."""
    return weight[np.asarray(ids).astype(np.int64)]


# --------------------------------------------------------------------------------------
# Paged decode  (vllm_nt/tests/test_attention.py:41-102 -- the reference's oracle for
#                vllm_nt/_ntops/kernels/attention.py:97-197)
# --------------------------------------------------------------------------------------


def paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    seq_lens: torch.Tensor,
    block_table: torch.Tensor,
    scale: float | None = None,
    seqs: list[int] | None = None,
) -> torch.Tensor:
    """query [B, Hq, D]; caches [blocks, bs, Hkv, D]; returns fp32 [B, Hq, D] (rows of
    sequences outside ``seqs`` are left zero).  For each sequence: gather its first
    seq_len cached tokens block by block, s = scale * q . k in fp32, softmax, o = p . v.
    A sequence with no cached tokens yields zeros."""
    b_total, hq, d = query.shape
    hkv = key_cache.shape[2]
    bs = key_cache.shape[1]
    group = hq // hkv
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    out = torch.zeros((b_total, hq, d), dtype=torch.float32)
    for b in range(b_total) if seqs is None else seqs:
        n = int(seq_lens[b])
        if n <= 0:
            continue
        nblk = (n + bs - 1) // bs
        ids = block_table[b, :nblk].long()
        k = key_cache[ids].reshape(nblk * bs, hkv, d)[:n].to(torch.float32)  # [n, Hkv, D]
        v = value_cache[ids].reshape(nblk * bs, hkv, d)[:n].to(torch.float32)
        q = query[b].to(torch.float32).reshape(hkv, group, d)
        s = torch.einsum("hgd,nhd->hgn", q, k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hgn,nhd->hgd", p, v).reshape(hq, d)
    return out


def varlen_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    scale: float | None = None,
    causal: bool = True,
) -> torch.Tensor:
    """query [Tq, Hq, D], key/value [Tk, Hkv, D]; returns fp32 [Tq, Hq, D].  Sequence b's
    queries are rows cu_seqlens_q[b] .. [b+1], its keys rows cu_seqlens_k[b] .. [b+1]
    (q_len and ctx of them).  s = scale * q . k in fp32; with ``causal`` query i sits at
    position ctx - q_len + i and sees keys 0 .. that position (vLLM's FlashAttention rule);
    softmax; o = p . v.  A row that sees no key is zero.  Follows the online-softmax
    recurrence of vllm_nt/_ntops/kernels/attention.py:40-82 in closed form, with the mask
    aligned to the end of the keys instead of the start (attention.py:61-63); the two agree
    when ctx == q_len, the case the reference's own test (tests/test_attention.py:57-72)
    covers."""
    tq, hq, d = query.shape
    hkv = key.shape[1]
    group = hq // hkv
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    out = torch.zeros((tq, hq, d), dtype=torch.float32)
    for b in range(cu_seqlens_q.numel() - 1):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        k0, k1 = int(cu_seqlens_k[b]), int(cu_seqlens_k[b + 1])
        q_len, ctx = q1 - q0, k1 - k0
        if q_len <= 0 or ctx <= 0:
            continue
        q = query[q0:q1].to(torch.float32).reshape(q_len, hkv, group, d)
        k = key[k0:k1].to(torch.float32)  # [ctx, Hkv, D]
        v = value[k0:k1].to(torch.float32)
        s = torch.einsum("qhgd,khd->hgqk", q, k) * scale
        if causal:
            pos = torch.arange(q_len) + (ctx - q_len)
            visible = torch.arange(ctx)[None, :] <= pos[:, None]  # [q_len, ctx]
            s = s.masked_fill(~visible, float("-inf"))
            seen = visible.any(dim=1)
        else:
            seen = torch.ones(q_len, dtype=torch.bool)
        p = torch.softmax(s, dim=-1).nan_to_num(0.0)
        o = torch.einsum("hgqk,khd->qhgd", p, v).reshape(q_len, hq, d)
        out[q0:q1] = o * seen[:, None, None]
    return out


def gather_paged_kv(key_cache: torch.Tensor, value_cache: torch.Tensor, seq_lens: torch.Tensor,
                    block_table: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Each sequence's first seq_lens[b] cached tokens, block by block, concatenated:
    (key [sum, Hkv, D], value, cu_seqlens [B + 1] int32), as
    vllm_nt/_ntops/torch/kv_cache.py:24-63 gathers them for the reference's prefill."""
    bs = key_cache.shape[1]
    ks, vs, cu = [], [], [0]
    for b in range(seq_lens.numel()):
        n = max(int(seq_lens[b]), 0)
        nblk = (n + bs - 1) // bs
        ids = block_table[b, :nblk].long()
        ks.append(key_cache[ids].reshape(nblk * bs, *key_cache.shape[2:])[:n])
        vs.append(value_cache[ids].reshape(nblk * bs, *value_cache.shape[2:])[:n])
        cu.append(cu[-1] + n)
    return torch.cat(ks), torch.cat(vs), torch.tensor(cu, dtype=torch.int32)


def paged_prefill(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    query_start_loc: torch.Tensor,
    seq_lens: torch.Tensor,
    block_table: torch.Tensor,
    scale: float | None = None,
    causal: bool = True,
) -> torch.Tensor:
    """query [T, Hq, D]; caches [blocks, bs, Hkv, D]: the reference's prefill path over the
    cache (vllm_nt/_ntops/patching.py:652-667: gather the cached tokens, then varlen
    attention) with vLLM's end-aligned causal mask.  Returns fp32 [T, Hq, D]."""
    k, v, cu_k = gather_paged_kv(key_cache, value_cache, seq_lens, block_table)
    return varlen_attention(query, k, v, query_start_loc, cu_k, scale, causal)


# --------------------------------------------------------------------------------------
# Dense projection  (vllm_nt/_ntops/kernels/linear.py:9-85; vllm:model_executor/layers/utils.py
#                    -> F.linear)
# --------------------------------------------------------------------------------------


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """x @ weight^T (+ bias) with fp32 inputs and accumulation; returns fp32."""
    y = x.to(torch.float32) @ weight.to(torch.float32).t()
    if bias is not None:
        y = y + bias.to(torch.float32)
    return y


def rms_norm_linear(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, weight: torch.Tensor,
                    residual: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """The fused decode entry point's arithmetic for RMSNorm followed by a projection (the
    reference runs the two as separate ops: vllm_nt/_ntops/oot_support.py:32-48, then
    vllm_nt/_ntops/torch/linear.py:7-21).  s = x (+ residual) in fp32; the GEMM input is
    s * norm_weight rounded once to x's dtype; the 1 / rms of each row, rsqrt(mean(s^2) + eps),
    scales the fp32 products.  Returns (fp32 output before its final rounding, s rounded to
    x's dtype or None)."""
    s = x.to(torch.float32)
    if residual is not None:
        s = s + residual.to(torch.float32)
    rstd = torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    y = _round(s * norm_weight.to(torch.float32), x.dtype)
    out = rstd * (y @ weight.to(torch.float32).t())
    return out, (s.to(x.dtype) if residual is not None else None)


def rms_norm_linear_exact(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, weight: torch.Tensor,
                          residual: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm then the projection in fp64 with no intermediate rounding: the value both the
    fused entry point and the reference's unfused pair approximate."""
    s = x.to(torch.float64)
    if residual is not None:
        s = s + residual.to(torch.float64)
    h = s * torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps) * norm_weight.to(torch.float64)
    return h @ weight.to(torch.float64).t()


# --------------------------------------------------------------------------------------
# Sampler  (vllm_nt/_ntops/torch/sampler.py:4-42; vllm:v1/sample/ops/topk_topp_sampler.py
#           apply_top_k_top_p_pytorch and random_sample)
# --------------------------------------------------------------------------------------


def apply_top_k_top_p(logits: torch.Tensor, k: torch.Tensor | None, p: torch.Tensor | None) -> torch.Tensor:
    """Masked copy of fp32 logits [B, V] by the reference's sort-based rule: sort each row
    ascending; top-k sets every value below the (V - k)-th sorted value to -inf (k clamped
    to [1, V]); top-p takes the softmax of the sorted (top-k masked) row, its running sum
    from the smallest value up, and sets to -inf every position whose running sum is
    <= 1 - p, except the last (largest) one; the row is scattered back."""
    out = logits.clone()
    if k is None and p is None:
        return out
    vocab = out.shape[-1]
    ordered, order = out.sort(dim=-1)
    if k is not None:
        kk = k.to(torch.long).clamp(1, vocab)
        kth = ordered.gather(1, (vocab - kk).unsqueeze(1))
        ordered = ordered.masked_fill(ordered < kth, float("-inf"))
    if p is not None:
        running = ordered.softmax(dim=-1, dtype=torch.float32).cumsum(dim=-1)
        drop = running <= 1 - p.to(torch.float32).unsqueeze(1)
        drop[:, -1] = False
        ordered = ordered.masked_fill(drop, float("-inf"))
    return out.scatter(-1, order, ordered)


def random_sample_from_draws(probs: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """argmax_i probs[b, i] / q[b, i] per row (int64 [B]): the reference's random_sample
    once its exponential draws q are fixed (torch.argmax: first index on ties)."""
    return torch.div(probs, q).argmax(dim=-1).view(-1)


def top_p_cumulative(logits: torch.Tensor, k: torch.Tensor | None) -> torch.Tensor:
    """fp64 running probability, per logit, of the rows after the top-k mask, summed from the
    smallest logit up to and including each one (the quantity the top-p rule compares with
    1 - p), returned in the logits' own positions: the yardstick for logits whose fate
    depends on fp32 summation order."""
    masked = apply_top_k_top_p(logits, k, None) if k is not None else logits
    ordered, order = masked.double().sort(dim=-1)
    running = ordered.softmax(dim=-1).cumsum(dim=-1)
    return torch.empty_like(running).scatter(-1, order, running)


def linear_argmax(x: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Greedy token of an LM head: argmax over the vocabulary of the logits rounded to x's
    dtype (vLLM's compute_logits writes them in the model dtype; its greedy sampler takes
    torch.argmax, which returns the first index among equal maxima).  Returns
    (token ids, the fp32 logits) -- the logits let a caller bound a disagreement."""
    logits = linear(x, weight)
    return torch.argmax(logits.to(x.dtype), dim=-1), logits

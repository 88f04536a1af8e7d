"""Paged-attention decode (split-K kernel) and varlen prefill (tcgen05 flash-attention
kernel) on sm_100a; replaces vllm_nt/_ntops/torch/attention.py:9-77."""

from __future__ import annotations

import math

import torch

from vllm_nt._ntops.torch._ext import ops

BLOCK_SIZE = 16
HEAD_DIM = 128


def decode_workspace_bytes(
    num_seqs: int, num_q_heads: int, num_kv_heads: int, max_seq_len: int
) -> int:
    return int(
        ops().decode_workspace_size(num_seqs, num_q_heads, num_kv_heads, HEAD_DIM, BLOCK_SIZE, max_seq_len)
    )


def paged_decode(
    out: torch.Tensor,
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    seq_lens: torch.Tensor,
    block_table: torch.Tensor,
    scale: float,
    max_seq_len: int | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """out[b, h] = softmax(scale * q[b, h] K_b^T) V_b for query [B, Hq, D] and caches
    [blocks, 16, Hkv, 128].  ``max_seq_len`` bounds seq_lens (None: the block table's
    capacity).  ``workspace`` may be passed to avoid an allocation per call."""
    num_seqs, hq, _ = query.shape
    hkv = key_cache.shape[2]
    cap = block_table.shape[1] * key_cache.shape[1]
    msl = cap if max_seq_len is None or max_seq_len <= 0 else min(int(max_seq_len), cap)
    need = decode_workspace_bytes(num_seqs, hq, hkv, msl) if num_seqs > 0 else 0
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=query.device)
    seq_lens = seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)
    block_table = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    ops().paged_attention_decode(
        out, query, key_cache, value_cache, seq_lens.contiguous(), block_table, float(scale), msl, workspace
    )
    return out


def flash_attn_with_kvcache(
    q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale=None, causal=True, max_seq_len=None
):
    """Reference signature: q [B, 1, Hq, D] (one new token per sequence) -> [B, 1, Hq, D].
    ``causal`` is irrelevant for a single query token (every cached token is visible)."""
    del causal
    scale = 1.0 / math.sqrt(q.shape[-1]) if softmax_scale is None else softmax_scale
    b = q.shape[0]
    q3 = q.reshape(b, q.shape[-2], q.shape[-1])
    out = torch.empty_like(q3)
    paged_decode(out, q3, k_cache, v_cache, cache_seqlens, block_table, scale, max_seq_len)
    return out.view(q.shape)


def flash_attn_varlen_func(
    q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale=None, causal=True, out=None, **kwargs
):
    """Reference signature (vllm_nt/_ntops/torch/attention.py:9-46): q [Tq, Hq, D], k/v
    [Tk, Hkv, D] with cu_seqlens_q/k [B + 1]; returns [Tq, Hq, D].  Causal masking is aligned
    to the end of each sequence's keys (vLLM's FlashAttention rule; the reference aligns to
    the start, which is the same whenever a sequence has as many keys as queries)."""
    del kwargs
    scale = 1.0 / math.sqrt(q.shape[-1]) if softmax_scale is None else float(softmax_scale)
    out = torch.empty_like(q) if out is None else out
    cu_q = cu_seqlens_q if cu_seqlens_q.dtype == torch.int32 else cu_seqlens_q.to(torch.int32)
    cu_k = cu_seqlens_k if cu_seqlens_k.dtype == torch.int32 else cu_seqlens_k.to(torch.int32)
    ops().flash_attn_varlen(out, q, k, v, cu_q.contiguous(), cu_k.contiguous(), int(max_seqlen_q), scale,
                            bool(causal))
    return out


def paged_prefill(
    out: torch.Tensor,
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    query_start_loc: torch.Tensor,
    seq_lens: torch.Tensor,
    block_table: torch.Tensor,
    max_query_len: int,
    scale: float,
    causal: bool = True,
) -> torch.Tensor:
    """Varlen attention straight over the paged cache: query/out [T, Hq, 128] (sequence b's
    queries at rows query_start_loc[b] .. [b + 1]), caches [blocks, 16, Hkv, 128] holding
    seq_lens[b] tokens of b (its queries' own keys last)."""
    ops().paged_attention_prefill(out, query, key_cache, value_cache, query_start_loc, seq_lens, block_table,
                                  int(max_query_len), float(scale), bool(causal))
    return out

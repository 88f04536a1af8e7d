"""Paged KV-cache store on the sm_100a kernel (replaces vllm_nt/_ntops/torch/kv_cache.py)."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def _as_paged(cache: torch.Tensor, num_heads: int, head_dim: int) -> torch.Tensor:
    """[blocks, block_size, heads, dim] view of a paged cache, or of the reference's flat
    [slots, heads * dim] cache (one slot per row, i.e. block_size 1)."""
    if cache.dim() == 4:
        return cache
    if cache.dim() == 2 and cache.shape[1] == num_heads * head_dim and cache.stride(1) == 1:
        return cache.as_strided(
            (cache.shape[0], 1, num_heads, head_dim),
            (cache.stride(0), cache.stride(0), head_dim, 1),
        )
    raise ValueError(f"unsupported cache shape {tuple(cache.shape)}")


def store_kvcache(key, value, k_cache, v_cache, slot_mapping):
    """k_cache[slot] = key[t], v_cache[slot] = value[t] for every t with slot >= 0
    (reference signature: vllm_nt/_ntops/torch/kv_cache.py:7-21).  The number of tokens
    stored is ``slot_mapping.numel()`` (vLLM pads key/value, not the slot mapping)."""
    num_heads, head_dim = key.shape[-2], key.shape[-1]
    key3 = key.view(-1, num_heads, head_dim)
    value3 = value.view(-1, num_heads, head_dim)
    slots = slot_mapping.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    ops().reshape_and_cache(
        key3, value3, _as_paged(k_cache, num_heads, head_dim), _as_paged(v_cache, num_heads, head_dim), slots
    )


def get_kv_from_cache(k_cache, v_cache, seq_lens, block_table):
    """Prefill helper of the reference (vllm_nt/_ntops/torch/kv_cache.py:24-63: copies each
    sequence's cached tokens out of the paged cache).  This backend's prefill kernel reads
    the paged cache in place through the block table (paged_attention_prefill), so nothing
    is gathered and this helper has no implementation here."""
    raise NotImplementedError("the B200 prefill reads the paged cache in place; use paged_attention_prefill")

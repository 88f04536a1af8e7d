"""In-place NeoX rotary embedding on the sm_100a kernel (replaces
vllm_nt/_ntops/torch/rotary_emb.py and the cos/sin gather of
vllm_nt/_ntops/oot_support.py:164-204)."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def _heads(t: torch.Tensor, num_tokens: int, head_size: int) -> torch.Tensor:
    v = t.view(num_tokens, -1, head_size)
    if v.stride(-1) != 1:
        raise ValueError("rotary_embedding needs unit stride in the head dimension")
    return v


def rotary_embedding(
    positions: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor | None,
    head_size: int,
    cos_sin_cache: torch.Tensor,
    rotary_dim: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Rotates the first ``rotary_dim`` dims of every head of query (and key) in place,
    NeoX style, with cos/sin = cos_sin_cache[positions] split in halves.  The cache must
    already have query's dtype (vLLM's _match_cos_sin_cache_dtype)."""
    rot = cos_sin_cache.shape[-1] if rotary_dim is None else rotary_dim
    if (positions.is_contiguous() and cos_sin_cache.is_contiguous() and query.dim() == 2
            and query.stride(-1) == 1 and (key is None or (key.dim() == 2 and key.stride(-1) == 1))):
        # vLLM's [tokens, heads * head_size] slices of the qkv projection go straight in
        ops().rotary_embedding_neox(positions, query, key, cos_sin_cache, head_size, rot)
        return query, key
    positions = positions.reshape(-1)
    if not positions.is_contiguous():
        positions = positions.contiguous()
    n = positions.shape[0]
    cache = cos_sin_cache if cos_sin_cache.stride(-1) == 1 else cos_sin_cache.contiguous()
    q = _heads(query, n, head_size)
    k = _heads(key, n, head_size) if key is not None else None
    ops().rotary_embedding_neox(positions, q, k, cache, int(head_size), int(rot))
    return query, key


def rotary_embedding_and_cache(
    positions: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    head_size: int,
    cos_sin_cache: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    rotary_dim: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """rotary_embedding(positions, query, key, ...) followed by
    store_kvcache(key, value, key_cache, value_cache, slot_mapping) in one kernel: q/k are
    rotated in place and the rotated key rows and the value rows land in the paged caches
    [blocks, block_size, kv_heads, head_size].  Bit-identical to the two calls in sequence.
    Tokens past ``slot_mapping.numel()`` (vLLM's padded rows) are rotated only."""
    rot = cos_sin_cache.shape[-1] if rotary_dim is None else rotary_dim
    positions = positions.reshape(-1)
    if not positions.is_contiguous():
        positions = positions.contiguous()
    slots = slot_mapping.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    cache = cos_sin_cache if cos_sin_cache.stride(-1) == 1 else cos_sin_cache.contiguous()
    n = positions.shape[0]
    q = query if query.dim() == 2 and query.stride(-1) == 1 else _heads(query, n, head_size)
    k = key if key.dim() == 2 and key.stride(-1) == 1 else _heads(key, n, head_size)
    v = value if value.dim() == 2 and value.stride(-1) == 1 else _heads(value, n, head_size)
    ops().rope_and_cache(positions, q, k, v, cache, key_cache, value_cache, slots, int(head_size), int(rot))
    return query, key


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Reference signature (vllm_nt/_ntops/torch/rotary_emb.py:7-9): x [T, H, R] rotated in
    place with per-token cos/sin [T, 1, R/2] (or [T, R/2]).  Implemented by handing the
    kernel a per-token cos|sin table and positions 0..T-1."""
    t, _, r = x.shape
    table = torch.cat((cos.reshape(t, r // 2), sin.reshape(t, r // 2)), dim=-1).to(x.dtype)
    pos = torch.arange(t, device=x.device, dtype=torch.int64)
    if x.stride(-1) != 1:
        raise ValueError("apply_rotary_emb needs unit stride in the last dimension")
    ops().rotary_embedding_neox(pos, x, None, table.contiguous(), r, r)
    return x

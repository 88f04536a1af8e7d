"""Op adapters between the vLLM hooks and the B200 kernels.

Same function names and argument meanings as vllm_nt/_ntops/oot_support.py:32-208; each
adapter now lands on one sm_100a kernel (for example ``norm`` with a residual is the
fused add+RMS-norm kernel instead of a torch add followed by a norm kernel, and ``rope``
gathers cos/sin inside the kernel)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import torch

from vllm_nt._ntops.torch._ext import ops
from vllm_nt._ntops.torch.attention import flash_attn_varlen_func as nt_flash_attn_varlen_func
from vllm_nt._ntops.torch.attention import flash_attn_with_kvcache as nt_flash_attn_with_kvcache
from vllm_nt._ntops.torch.attention import paged_decode as nt_paged_decode
from vllm_nt._ntops.torch.embedding import embedding as nt_embedding
from vllm_nt._ntops.torch.kv_cache import get_kv_from_cache as nt_get_kv_from_cache
from vllm_nt._ntops.torch.kv_cache import store_kvcache as nt_store_kvcache
from vllm_nt._ntops.torch.linear import linear as nt_linear
from vllm_nt._ntops.torch.linear import linear_silu_and_mul as nt_linear_silu_and_mul
from vllm_nt._ntops.torch.linear import rms_norm_linear as nt_rms_norm_linear
from vllm_nt._ntops.torch.rms_norm import fused_add_rms_norm as nt_fused_add_rms_norm
from vllm_nt._ntops.torch.rms_norm import gemma_rms_norm as nt_gemma_rms_norm
from vllm_nt._ntops.torch.rms_norm import rms_norm as nt_rms_norm
from vllm_nt._ntops.torch.rotary_emb import apply_rotary_emb as nt_apply_rotary_emb
from vllm_nt._ntops.torch.rotary_emb import rotary_embedding as nt_rotary_embedding
from vllm_nt._ntops.torch.silu import silu_and_mul as nt_silu_and_mul
from vllm_nt._ntops.torch.sampler import apply_top_k_top_p as nt_apply_top_k_top_p  # noqa: F401
from vllm_nt._ntops.torch.sampler import random_sample as nt_random_sample  # noqa: F401


@dataclass
class OperatorStats:
    """Per-operator accounting: kernel hits, whether the first hit was logged, the
    strongest registration path that installed the op, and the calls the kernels did not
    serve, counted by reason."""

    hits: int = 0
    logged: bool = False
    registered_via: str | None = None
    declined: dict[str, int] = field(default_factory=dict)


def norm(self, x: torch.Tensor, weight: torch.Tensor | None, residual: torch.Tensor | None = None, gemma: bool = False):
    """RMSNorm.forward contract: returns ``out`` or ``(out, new_residual)``.

    With a residual the sum is formed in fp32 inside the kernel and written into the
    residual buffer (vLLM's CUDA convention), the norm is taken of the fp32 sum.  With
    ``gemma=True`` ``weight`` is the raw Gemma parameter w: the kernel forms (1 + w) in fp32
    and rounds as GemmaRMSNorm.forward_native does, and returns new tensors."""
    eps = self.variance_epsilon
    if gemma:
        return nt_gemma_rms_norm(x, weight, eps, residual)
    if residual is not None:
        return nt_fused_add_rms_norm(x, residual, weight, eps, inplace=True)
    hidden = weight.shape[0] if weight is not None else self.hidden_size
    return nt_rms_norm(x, hidden, weight=weight, eps=eps)


def act_and_mul(x: torch.Tensor, act: Callable[[torch.Tensor], torch.Tensor] | None = None, reverse: bool = False) -> torch.Tensor:
    """silu(x[..., :d]) * x[..., d:] as one kernel.  Other activations (or the reversed
    MulAndSilu order) compose ``act`` with a multiply, as the reference does."""
    if act is None and not reverse:
        return nt_silu_and_mul(x)
    d = x.shape[-1] // 2
    left, right = (x[..., d:], x[..., :d]) if reverse else (x[..., :d], x[..., d:])
    fn = act if act is not None else torch.nn.functional.silu
    return fn(left) * right


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    return nt_linear(x, weight, bias)


def gate_up_silu_and_mul(x: torch.Tensor, gate_up_weight: torch.Tensor) -> torch.Tensor:
    """silu(x W_gate^T) * (x W_up^T) for a merged [2I, K] gate_up weight in one kernel."""
    return nt_linear_silu_and_mul(x, gate_up_weight)


def norm_linear(norm_layer: torch.nn.Module, x: torch.Tensor, residual: torch.Tensor | None,
                weight: torch.Tensor):
    """RMSNorm(x [+ residual]) followed by the projection by ``weight`` in one kernel (at
    most 16 rows); returns the projection, or (projection, new residual)."""
    return nt_rms_norm_linear(x, norm_layer.weight, norm_layer.variance_epsilon, weight, residual)


def embedding(layer: torch.nn.Module, input_: torch.Tensor) -> torch.Tensor:
    return nt_embedding(input_, layer.weight)


def rope(
    positions: torch.Tensor,
    query: torch.Tensor,
    key: torch.Tensor | None,
    *,
    cos_sin_cache: torch.Tensor,
    head_size: int,
    rotary_dim: int,
    is_neox_style: bool,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """In-place NeoX rotary embedding of query/key (reference: oot_support.py:164-204)."""
    if not is_neox_style:
        raise NotImplementedError("Only NeoX-style RoPE is supported.")
    if rotary_dim % 2:
        raise ValueError("rotary_dim must be even.")
    cache = cos_sin_cache
    if cache.dtype != query.dtype:
        cache = cache.to(query.dtype)
    return nt_rotary_embedding(positions, query, key, head_size, cache, rotary_dim)


def store_kv_cache(key, value, k_cache, v_cache, slot_mapping):
    return nt_store_kvcache(key, value, k_cache, v_cache, slot_mapping)


def rope_and_store_kv_cache_flash(positions, query, key, value, cos_sin_cache, head_size, rotary_dim, kv_cache,
                                  slot_mapping, kv_dim=0):
    """NeoX RoPE of q/k (in place) and the slot-mapped store of the rotated k and the v into
    vLLM's combined cache tensor (kv_dim as in store_kv_cache_flash), one kernel for a
    decode step: the RoPE hook and the KV-store hook of one attention layer fused."""
    cache = cos_sin_cache if cos_sin_cache.dtype == query.dtype else cos_sin_cache.to(query.dtype)
    ops().rope_and_cache_flash_layout(positions.reshape(-1), query, key, value, cache, kv_cache, slot_mapping,
                                      int(head_size), int(rotary_dim), int(kv_dim))


def store_kv_cache_flash(key, value, kv_cache, slot_mapping, kv_dim=0):
    """The KV store on vLLM's combined cache tensor in one op call: kv_dim 0 is
    FlashAttention's [2, blocks, block_size, kv_heads, head_size], kv_dim 1 FlashInfer's
    [blocks, 2, ...]; the K/V split and views happen in the op."""
    ops().store_flash_layout(key, value, kv_cache, slot_mapping, kv_dim)


def paged_attention_decode_flash(output, query, kv_cache, seq_lens, block_table, num_tokens, scale, max_seq_len,
                                 kv_dim=0):
    """Decode attention for the first ``num_tokens`` rows of vLLM's padded activations on
    its combined cache tensor (kv_dim as in store_kv_cache_flash), in one op call (views,
    slicing and the split-K workspace are made inside the op)."""
    ops().decode_flash_layout(output, query, kv_cache, seq_lens, block_table, num_tokens, scale, max_seq_len,
                              kv_dim)


def paged_attention_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale=None, causal=True, max_seq_len=None):
    return nt_flash_attn_with_kvcache(
        q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale=softmax_scale, causal=causal, max_seq_len=max_seq_len
    )


def paged_attention_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale=None, causal=True,
                            **kwargs):
    """Reference signature (vllm_nt/_ntops/oot_support.py:88-109): varlen attention over
    contiguous K/V on the tcgen05 prefill kernel."""
    return nt_flash_attn_varlen_func(
        q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale=softmax_scale, causal=causal, **kwargs
    )


def paged_attention_flash(output, query, kv_cache, query_start_loc, seq_lens, block_table, num_tokens,
                          max_query_len, max_seq_len, scale, kv_dim=0):
    """Causal attention for any vLLM batch (decodes, prefills, chunked prefills, mixed) on
    its combined cache: single-query sequences on the split-K decode kernel, the others on
    the tcgen05 prefill kernel; the first ``num_tokens`` rows of the padded activations."""
    ops().attention_flash_layout(output, query, kv_cache, query_start_loc, seq_lens, block_table, num_tokens,
                                 max_query_len, max_seq_len, scale, kv_dim)


def paged_attention_prefill_flash(output, query, kv_cache, query_start_loc, seq_lens, block_table, num_tokens,
                                  max_query_len, scale, causal=True, kv_dim=0):
    """Varlen attention for the first ``num_tokens`` rows of vLLM's padded activations,
    reading K/V from its combined cache tensor in place (kv_dim as in store_kv_cache_flash)."""
    ops().prefill_flash_layout(output, query, kv_cache, query_start_loc, seq_lens, block_table, num_tokens,
                               max_query_len, scale, causal, kv_dim)


def get_kv_from_cache(k_cache, v_cache, seq_lens, block_table):
    return nt_get_kv_from_cache(k_cache, v_cache, seq_lens, block_table)


def sdpa(*args, **kwargs):
    """Dense SDPA (vision/encoder models) is outside this backend; vLLM's path serves it."""
    raise NotImplementedError("SDPA is served by vLLM's original path")

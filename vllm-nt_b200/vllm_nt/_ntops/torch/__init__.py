"""Torch-level entry points of the B200 kernels (names follow vllm_nt/_ntops/torch)."""

from vllm_nt._ntops.torch.attention import (
    flash_attn_varlen_func,
    flash_attn_with_kvcache,
    paged_decode,
)
from vllm_nt._ntops.torch.embedding import embedding
from vllm_nt._ntops.torch.kv_cache import get_kv_from_cache, store_kvcache
from vllm_nt._ntops.torch.linear import linear, matmul
from vllm_nt._ntops.torch.rms_norm import fused_add_rms_norm, rms_norm
from vllm_nt._ntops.torch.sampler import apply_top_k_top_p, random_sample
from vllm_nt._ntops.torch.rotary_emb import apply_rotary_emb, rotary_embedding, rotary_embedding_and_cache
from vllm_nt._ntops.torch.silu import silu_and_mul

__all__ = [
    "apply_rotary_emb",
    "apply_top_k_top_p",
    "embedding",
    "flash_attn_varlen_func",
    "flash_attn_with_kvcache",
    "fused_add_rms_norm",
    "get_kv_from_cache",
    "linear",
    "matmul",
    "paged_decode",
    "random_sample",
    "rms_norm",
    "rotary_embedding",
    "rotary_embedding_and_cache",
    "silu_and_mul",
    "store_kvcache",
]

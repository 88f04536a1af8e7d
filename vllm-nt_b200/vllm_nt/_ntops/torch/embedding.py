"""Embedding gather on the sm_100a kernel (replaces vllm_nt/_ntops/torch/embedding.py)."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def embedding(input_ids: torch.Tensor, weight: torch.Tensor, *unused, **unused_kw) -> torch.Tensor:
    """out[..., :] = weight[input_ids[...], :] (bit-exact)."""
    ids = input_ids.reshape(-1)
    if not ids.is_contiguous():
        ids = ids.contiguous()
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    out = torch.empty((ids.shape[0], w.shape[-1]), dtype=w.dtype, device=w.device)
    ops().embedding(out, ids, w)
    return out.view(*input_ids.shape, w.shape[-1])

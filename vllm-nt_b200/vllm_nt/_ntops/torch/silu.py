"""silu_and_mul on the sm_100a kernel.

The reference exposes an elementwise ``silu`` and multiplies by the up half in torch
(vllm_nt/_ntops/torch/silu.py:7-17, vllm_nt/_ntops/oot_support.py:51-56); here the gate,
the up half and the product are one kernel."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """out[..., i] = silu(x[..., i]) * x[..., d + i] with d = x.shape[-1] // 2."""
    shape = x.shape
    two_d = shape[-1]
    if two_d % 2:
        raise ValueError("silu_and_mul needs an even last dimension")
    d = two_d // 2
    if x.is_contiguous():
        # the op takes any-rank row layouts itself
        out = x.new_empty((*shape[:-1], d))
        ops().silu_and_mul(out, x)
        return out
    x2 = x.reshape(-1, two_d)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty((x2.shape[0], d), dtype=x.dtype, device=x.device)
    ops().silu_and_mul(out, x2)
    return out.view(*shape[:-1], d)

"""Top-k / top-p masking and exponential-race sampling on the sm_100a kernels (replaces
vllm_nt/_ntops/torch/sampler.py; same function names, arguments and results)."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def apply_top_k_top_p(
    logits: torch.Tensor,
    k: torch.Tensor | None,
    p: torch.Tensor | None,
) -> torch.Tensor:
    """Masks fp32 logits [B, V] in place and returns them (reference signature:
    vllm_nt/_ntops/torch/sampler.py:4-31): logits below each row's k-th largest become
    -inf (k clamped to [1, V]), then, among the survivors, those whose cumulative
    probability from the smallest upwards is <= 1 - p.  Per-row radix selection on the
    GPU instead of a full sort; the largest logit of a row always survives."""
    if k is None and p is None:
        return logits
    if k is not None:
        if k.dtype not in (torch.int32, torch.int64) or k.device != logits.device:
            k = k.to(device=logits.device, dtype=torch.int64)
        if not k.is_contiguous():
            k = k.contiguous()
    if p is not None:
        p = p.to(device=logits.device, dtype=torch.float32).contiguous()
    ops().top_k_top_p(logits, k, p)
    return logits


def random_sample(
    probs: torch.Tensor,
    generators: dict[int, torch.Generator],
) -> torch.Tensor:
    """argmax(probs / q) per row for q ~ Exp(1) (reference signature:
    vllm_nt/_ntops/torch/sampler.py:34-42).  q is drawn exactly as the reference draws it
    (the device's default generator for every row, then each request's own generator for
    its row), so the sample is the one the reference returns; the division and the argmax
    are one kernel pass that never writes the [B, V] quotient."""
    q = torch.empty_like(probs)
    q.exponential_()
    for i, generator in generators.items():
        q[i].exponential_(generator=generator)
    out = torch.empty(probs.shape[0], dtype=torch.int64, device=probs.device)
    ops().random_sample(out, probs, q)
    return out

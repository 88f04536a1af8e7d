"""RMS norm on the sm_100a kernel (replaces vllm_nt/_ntops/torch/rms_norm.py)."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def _rows(t: torch.Tensor, hidden: int) -> torch.Tensor:
    t2 = t.reshape(-1, hidden)
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


def _weight(weight: torch.Tensor | None, hidden: int, dtype: torch.dtype) -> torch.Tensor | None:
    if weight is None:
        return None
    w = weight.reshape(-1)[:hidden] if weight.numel() != hidden else weight.reshape(hidden)
    if w.dtype != dtype:
        w = w.to(dtype)
    return w.contiguous()


def _weight_ok(weight: torch.Tensor | None, x: torch.Tensor) -> bool:
    return weight is None or (weight.dtype == x.dtype and weight.dim() == 1 and weight.is_contiguous())


def rms_norm(input, normalized_shape, weight=None, eps=None):
    """y = input * rsqrt(mean(input^2, -1) + eps) * weight over the last dimension.

    Same signature as vllm_nt/_ntops/torch/rms_norm.py:36-61; only normalisation over
    the last dimension is supported (the case every vLLM layer uses)."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    normalized_shape = tuple(normalized_shape)
    if len(normalized_shape) != 1 or normalized_shape[0] != input.shape[-1]:
        raise NotImplementedError("ntb200.rms_norm normalises over the last dimension only")
    if eps is None:
        eps = torch.finfo(input.dtype).eps
    if input.is_contiguous() and _weight_ok(weight, input):
        # the op takes any-rank row layouts itself
        out = torch.empty_like(input)
        ops().rms_norm(out, input, weight, float(eps))
        return out
    hidden = input.shape[-1]
    x = _rows(input, hidden)
    out = torch.empty_like(x)
    ops().rms_norm(out, x, _weight(weight, hidden, input.dtype), float(eps))
    return out.view(input.shape)


def fused_add_rms_norm(x, residual, weight, eps, inplace=False):
    """Returns (rms_norm(x + residual), x + residual) with the sum and statistics in
    fp32, as vLLM's fused_add_rms_norm (vllm/ir/ops/layernorm.py:40-62).

    With ``inplace=True`` both inputs are overwritten, vLLM's CUDA convention
    (vllm/_custom_ops.py fused_add_rms_norm): the normalised rows go into ``x`` and the
    sum into ``residual``, and those two tensors are returned; no memory is allocated.
    Otherwise neither input is modified."""
    if inplace and x.is_contiguous() and residual.is_contiguous() and _weight_ok(weight, x):
        ops().fused_add_rms_norm(x, residual, x, weight, float(eps))
        return x, residual
    hidden = x.shape[-1]
    x2 = _rows(x, hidden)
    res = residual.reshape(-1, hidden)
    if not inplace or res.stride(-1) != 1:
        res = res.clone(memory_format=torch.contiguous_format)
    out = x2 if inplace and x2.data_ptr() == x.data_ptr() else torch.empty_like(x2)
    ops().fused_add_rms_norm(out, res, x2, _weight(weight, hidden, x.dtype), float(eps))
    return out.view(x.shape), res.view(residual.shape)


def gemma_rms_norm(x, weight, eps, residual=None):
    """vLLM's GemmaRMSNorm.forward_native (vllm/model_executor/layers/layernorm.py:153-170)
    on one kernel: out = x * rsqrt(mean(x^2) + eps) * (1 + w) with (1 + w) in fp32 and one
    rounding of the product; ``weight`` is the raw Gemma parameter w.  With a residual the
    sum is taken in the input dtype and ``(out, sum)`` is returned as new tensors, as vLLM's
    native code returns them (neither input is modified).  fp16 with a residual is not
    served (vLLM hands back an fp32 residual there)."""
    if residual is None:
        if x.is_contiguous() and _weight_ok(weight, x):
            out = torch.empty_like(x)
            ops().gemma_rms_norm(out, x, weight, float(eps))
            return out
        hidden = x.shape[-1]
        x2 = _rows(x, hidden)
        out = torch.empty_like(x2)
        ops().gemma_rms_norm(out, x2, _weight(weight, hidden, x.dtype), float(eps))
        return out.view(x.shape)
    hidden = x.shape[-1]
    x2 = _rows(x, hidden)
    res = residual.reshape(-1, hidden).clone(memory_format=torch.contiguous_format)
    out = torch.empty_like(x2)
    ops().gemma_fused_add_rms_norm(out, res, x2, _weight(weight, hidden, x.dtype), float(eps))
    return out.view(x.shape), res.view(residual.shape)

"""Dense projection on the tcgen05 GEMM (replaces vllm_nt/_ntops/torch/linear.py and
vllm_nt/_ntops/torch/matmul.py)."""

from __future__ import annotations

import torch

from vllm_nt._ntops.torch._ext import ops


def _k_contiguous(t: torch.Tensor) -> torch.Tensor:
    ok = t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def linear(input: torch.Tensor, other: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """out = input @ other^T (+ bias) for input [..., K] and other [N, K] (vLLM layout)."""
    if input.is_contiguous() and other.is_contiguous() and (bias is None or bias.is_contiguous()):
        # the op views [..., K] as rows and realigns an unaligned x itself
        out = input.new_empty((*input.shape[:-1], other.shape[0]))
        ops().linear(out, input, other, bias, None)
        return out
    x = _k_contiguous(input.reshape(-1, input.shape[-1]))
    w = _k_contiguous(other)
    out = torch.empty((x.shape[0], w.shape[0]), dtype=x.dtype, device=x.device)
    if bias is not None and not bias.is_contiguous():
        bias = bias.contiguous()
    ops().linear(out, x, w, bias, None)
    return out.view(*input.shape[:-1], w.shape[0])


def linear_silu_and_mul(input: torch.Tensor, gate_up: torch.Tensor) -> torch.Tensor:
    """silu(input @ gate_up[:I]^T) * (input @ gate_up[I:]^T) for vLLM's merged gate_up
    weight [2I, K], as one GEMM whose epilogue applies SiluAndMul (no [.., 2I] tensor is
    written)."""
    w = _k_contiguous(gate_up)
    out = input.new_empty((*input.shape[:-1], w.shape[0] // 2))
    x = input if input.is_contiguous() else input.contiguous()
    ops().linear_silu_and_mul(out, x, w)
    return out


def rms_norm_linear(input: torch.Tensor, norm_weight: torch.Tensor, eps: float, weight: torch.Tensor,
                    residual: torch.Tensor | None = None):
    """RMSNorm (after adding residual, when given) of a decode batch of at most 16 rows,
    then the projection by weight [N, K], as one kernel: the GEMM input round(s *
    norm_weight) is formed in shared memory and never written, and each row's 1/rms scales
    the fp32 products before the output's one rounding.  Returns out [M, N], or
    (out, new_residual) with a residual (new_residual = input + residual, a new tensor)."""
    x = input if input.is_contiguous() else input.contiguous()
    x2 = x.reshape(-1, x.shape[-1])
    w = _k_contiguous(weight)
    out = torch.empty((x2.shape[0], w.shape[0]), dtype=x.dtype, device=x.device)
    if residual is None:
        ops().rms_norm_linear(out, None, x2, None, norm_weight.contiguous(), float(eps), w)
        return out.view(*input.shape[:-1], w.shape[0])
    r2 = residual.reshape(-1, residual.shape[-1])
    r2 = r2 if r2.is_contiguous() else r2.contiguous()
    new_res = torch.empty_like(x2)
    ops().rms_norm_linear(out, new_res, x2, r2, norm_weight.contiguous(), float(eps), w)
    return out.view(*input.shape[:-1], w.shape[0]), new_res.view(input.shape)


def linear_argmax(input: torch.Tensor, lm_head: torch.Tensor) -> torch.Tensor:
    """Greedy next tokens: argmax over the vocabulary of input @ lm_head^T (int64, one per
    row of input), with the logits compared at input's dtype and the first index winning
    ties; for up to 256 rows the logits are never written to memory."""
    w = _k_contiguous(lm_head)
    x = input if input.is_contiguous() else input.contiguous()
    out = torch.empty(x.shape[:-1], dtype=torch.int64, device=x.device)
    ops().linear_argmax(out, x, w)
    return out


def matmul(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    """lhs [M, K] @ rhs [K, N]; rhs is transposed once into the [N, K] operand layout."""
    return linear(lhs, rhs.t().contiguous())

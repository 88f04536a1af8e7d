"""Shared test helpers: golden fixtures, CUDA gating, C-ABI argument plumbing."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden(name: str) -> dict[str, torch.Tensor]:
    """Loads tests/golden/<name>.npz; keys ending in __bf16 are uint16 bit patterns."""
    out = {}
    with np.load(GOLDEN / f"{name}.npz") as z:
        for key in z.files:
            arr = z[key]
            if key.endswith("__bf16"):
                out[key[: -len("__bf16")]] = torch.from_numpy(arr.astype(np.uint16).view(np.int16)).view(torch.bfloat16)
            else:
                out[key] = torch.from_numpy(arr)
    return out


def cuda_device() -> torch.device:
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def dtype_code(dt: torch.dtype) -> int:
    return {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2, torch.int32: 3, torch.int64: 4}[dt]


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def seeded(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality of two same-shape tensors (NaN-safe, -0 != +0)."""
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    ia = a.contiguous().view(torch.uint8)
    ib = b.contiguous().view(torch.uint8)
    return bool(torch.equal(ia, ib))

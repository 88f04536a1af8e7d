"""Loads the in-tree sm_100a kernel library and its torch binding.

There is exactly one implementation of every op: the CUDA kernels in ``libntb200.so``.
If the library is missing this module raises; nothing falls back to a CPU or torch
path (the plugin's router may still choose vLLM's ``original`` backend after a failure,
and counts that as a failure)."""

from __future__ import annotations

import threading
from pathlib import Path

import torch

LIB_DIR = Path(__file__).resolve().parents[2] / "_lib"
BINDING = LIB_DIR / "_ntb200_C.so"
LIBRARY = LIB_DIR / "libntb200.so"

_lock = threading.Lock()
_loaded = False


def _register_fakes() -> None:
    """Shape-only implementations so torch.compile can trace through the ops (they
    mutate their outputs and return nothing)."""

    def nothing(*args, **kwargs):
        return None

    for name in (
        "rms_norm",
        "fused_add_rms_norm",
        "silu_and_mul",
        "rotary_embedding_neox",
        "reshape_and_cache",
        "rope_and_cache",
        "rope_and_cache_flash_layout",
        "embedding",
        "paged_attention_decode",
        "decode_flash_layout",
        "store_flash_layout",
        "linear",
        "allreduce_oneshot",
        "linear_silu_and_mul",
        "linear_argmax",
        "paged_attention_prefill",
        "prefill_flash_layout",
        "flash_attn_varlen",
        "attention_flash_layout",
        "top_k_top_p",
        "random_sample",
    ):
        torch.library.register_fake(f"ntb200::{name}")(nothing)


def ops():
    """Returns ``torch.ops.ntb200`` after loading the binding once per process."""
    global _loaded
    if not _loaded:
        with _lock:
            if not _loaded:
                if not BINDING.exists() or not LIBRARY.exists():
                    raise RuntimeError(
                        f"vllm_nt B200 kernels are not built ({BINDING} missing); "
                        "run `python vllm-nt_b200/csrc/build.py`"
                    )
                torch.ops.load_library(str(BINDING))
                _register_fakes()
                _loaded = True
    return torch.ops.ntb200


def loaded_paths() -> list[str]:
    return [str(LIBRARY), str(BINDING)] if _loaded else []

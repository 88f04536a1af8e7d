"""The C-ABI library loads and exports every entry point include/ntb200.h declares, and
its host-side argument checks reject bad calls before touching a device.  CPU only (no
kernel is launched)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from vllm_nt._ntops import capi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ntb200.h"


def declared_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(ntb200_\w+)\s*\(", text))


def test_header_declarations_are_all_exported():
    names = declared_functions()
    assert {"ntb200_rms_norm", "ntb200_paged_attention_decode", "ntb200_linear"} <= names
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIBRARY)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (ntb200_\w+)", out.stdout))
    assert names <= exported, names - exported


def test_ctypes_view_covers_the_header():
    assert declared_functions() == set(capi.SIGNATURES)
    lib = capi.lib()
    for name in capi.SIGNATURES:
        assert hasattr(lib, name)


def test_status_strings_and_version():
    lib = capi.lib()
    assert lib.ntb200_version() >= 1
    assert lib.ntb200_status_string(0) == b"ok"
    assert lib.ntb200_status_string(-4).startswith(b"workspace")


@pytest.mark.parametrize(
    "name,args,status",
    [
        ("ntb200_rms_norm", (1, 1, None, -1, 8, 8, 8, 1e-6, 0, None), -1),
        ("ntb200_rms_norm", (1, 1, None, 4, 8, 8, 8, 1e-6, 9, None), -2),
        ("ntb200_fused_add_rms_norm", (1, None, 1, None, 4, 8, 8, 8, 8, 1e-6, 1, None), -1),
        ("ntb200_silu_and_mul", (1, 1, 4, 8, 16, 8, 7, None), -2),
        ("ntb200_silu_and_mul", (1, 1, 4, 8, 8, 8, 1, None), -1),
        ("ntb200_rotary_embedding_neox", (1, 4, 1, None, 1, 4, 2, 0, 64, 63, 128, 64, 0, 0, 64, 10, 1, None), -1),
        ("ntb200_reshape_and_cache", (1, 1, 1, 1, 1, 4, 4, 2, 128, 16, 64, 256, 128, 256, 128, 4096, 256, 128, 3, None), -2),
        # rope_and_cache: odd rotary_dim; more store tokens than tokens; null key; fp8 dtype code
        ("ntb200_rope_and_cache", (1, 4, 1, 1, 1, 1, 1, 1, 1, 4, 4, 4, 2, 1, 128, 127) + (128,) * 6 + (128, 64, 16, 64, 2048, 128, 128, 1, None), -1),
        ("ntb200_rope_and_cache", (1, 4, 1, 1, 1, 1, 1, 1, 1, 4, 4, 5, 2, 1, 128, 128) + (128,) * 6 + (128, 64, 16, 64, 2048, 128, 128, 1, None), -1),
        ("ntb200_rope_and_cache", (1, 4, 1, None, 1, 1, 1, 1, 1, 4, 4, 4, 2, 1, 128, 128) + (128,) * 6 + (128, 64, 16, 64, 2048, 128, 128, 1, None), -1),
        ("ntb200_rope_and_cache", (1, 4, 1, 1, 1, 1, 1, 1, 1, 4, 4, 4, 2, 1, 128, 128) + (128,) * 6 + (128, 64, 16, 64, 2048, 128, 128, 7, None), -2),
        ("ntb200_embedding", (1, 1, 4, 1, 4, 10, 16, 8, 16, 2, None), -1),
        # top_k_top_p: row stride below the vocabulary; a k dtype that is not an integer code
        ("ntb200_top_k_top_p", (1, 4, 100, 99, 1, 4, None, None), -1),
        ("ntb200_top_k_top_p", (1, 4, 100, 100, 1, 1, None, None), -2),
        ("ntb200_top_k_top_p", (None, 4, 100, 100, 1, 4, None, None), -1),
        # random_sample: empty vocabulary; q row stride below it; null output
        ("ntb200_random_sample", (1, 1, 1, 4, 0, 8, 8, None), -1),
        ("ntb200_random_sample", (1, 1, 1, 4, 8, 8, 7, None), -1),
        ("ntb200_random_sample", (None, 1, 1, 4, 8, 8, 8, None), -1),
        ("ntb200_linear", (1, 1, 1, None, 4, 8, 16, 16, 16, 8, None, 0, 0, None), -2),
        # linear_silu_and_mul: fp32; x row stride below K; x not 16-byte aligned
        ("ntb200_linear_silu_and_mul", (16, 16, 16, 4, 8, 64, 64, 64, 8, 0, None), -2),
        ("ntb200_linear_silu_and_mul", (16, 16, 16, 4, 8, 64, 32, 64, 8, 1, None), -1),
        ("ntb200_linear_silu_and_mul", (16, 8, 16, 4, 8, 64, 64, 64, 8, 1, None), -3),
        # rms_norm_linear (out, residual_out, x, residual, norm_weight, eps, weight, M, N, K,
        # strides x / residual / residual_out / weight / out, dtype, stream): fp32; 17 rows;
        # a residual without residual_out; residual_out aliasing x; K not a multiple of 8
        ("ntb200_rms_norm_linear", (16, None, 16, None, 16, 1e-5, 16, 4, 8, 64, 64, 0, 0, 64, 8, 0, None), -2),
        ("ntb200_rms_norm_linear", (16, None, 16, None, 16, 1e-5, 16, 17, 8, 64, 64, 0, 0, 64, 8, 1, None), -6),
        ("ntb200_rms_norm_linear", (16, None, 16, 32, 16, 1e-5, 16, 4, 8, 64, 64, 64, 64, 64, 8, 1, None), -1),
        ("ntb200_rms_norm_linear", (16, 16, 16, 32, 16, 1e-5, 16, 4, 8, 64, 64, 64, 64, 64, 8, 1, None), -1),
        ("ntb200_rms_norm_linear", (16, None, 16, None, 16, 1e-5, 16, 4, 8, 60, 64, 0, 0, 64, 8, 1, None), -3),
        ("ntb200_paged_attention_decode",
         (1, 1, 1, 1, 1, 1, 2, 4, 1, 64, 16, 8, 4, 4, 64, 0.1, 512, 128, 512, 128, 2048, 128, 128, None, 0, 1, None), -6),
        # Gemma norms: the raw weight is required; fp16 with a residual (vLLM keeps it fp32);
        # a row stride below hidden
        ("ntb200_gemma_rms_norm", (16, 16, None, 4, 8, 8, 8, 1e-6, 1, None), -1),
        ("ntb200_gemma_fused_add_rms_norm", (16, 16, 16, 16, 4, 8, 8, 8, 8, 1e-6, 2, None), -2),
        ("ntb200_gemma_fused_add_rms_norm", (16, 16, 16, 16, 4, 8, 8, 4, 8, 1e-6, 1, None), -1),
        # paged prefill (out, query, k/v cache, query_start_loc, seq_lens, block_tables,
        # seqs, tokens, q/kv heads, head_size, block_size, blocks, max blocks, table stride,
        # max_query_len, scale, causal, q/out token+head strides, cache strides, dtype,
        # stream): fp32; head_size 64; 30 q heads over 8 kv heads; null query; out 8-aligned
        ("ntb200_paged_attention_prefill", (16, 16, 16, 16, 16, 16, 16, 2, 8, 32, 8, 128, 16, 64, 4, 4, 4, 0.1, 1,
                                            4096, 128, 4096, 128, 16384, 1024, 128, 0, None), -2),
        ("ntb200_paged_attention_prefill", (16, 16, 16, 16, 16, 16, 16, 2, 8, 32, 8, 64, 16, 64, 4, 4, 4, 0.1, 1,
                                            4096, 128, 4096, 128, 16384, 1024, 128, 1, None), -6),
        ("ntb200_paged_attention_prefill", (16, 16, 16, 16, 16, 16, 16, 2, 8, 30, 8, 128, 16, 64, 4, 4, 4, 0.1, 1,
                                            4096, 128, 4096, 128, 16384, 1024, 128, 1, None), -1),
        ("ntb200_paged_attention_prefill", (16, None, 16, 16, 16, 16, 16, 2, 8, 32, 8, 128, 16, 64, 4, 4, 4, 0.1, 1,
                                            4096, 128, 4096, 128, 16384, 1024, 128, 1, None), -1),
        ("ntb200_paged_attention_prefill", (8, 16, 16, 16, 16, 16, 16, 2, 8, 32, 8, 128, 16, 64, 4, 4, 4, 0.1, 1,
                                            4096, 128, 4096, 128, 16384, 1024, 128, 1, None), -3),
        # contiguous varlen (out, query, key, value, cu_q, cu_k, seqs, q tokens, k tokens,
        # q/kv heads, head_size, max_query_len, scale, causal, q/k/v/out token+head strides,
        # dtype, stream): fp32; head_size 96; negative key count; null cu_seqlens_k; a key
        # row stride that is not a multiple of 8
        ("ntb200_flash_attn_varlen", (16, 16, 16, 16, 16, 16, 2, 8, 8, 32, 8, 128, 4, 0.1, 1,
                                      4096, 128, 1024, 128, 1024, 128, 4096, 128, 0, None), -2),
        ("ntb200_flash_attn_varlen", (16, 16, 16, 16, 16, 16, 2, 8, 8, 32, 8, 96, 4, 0.1, 1,
                                      4096, 128, 1024, 128, 1024, 128, 4096, 128, 1, None), -6),
        ("ntb200_flash_attn_varlen", (16, 16, 16, 16, 16, 16, 2, 8, -1, 32, 8, 128, 4, 0.1, 1,
                                      4096, 128, 1024, 128, 1024, 128, 4096, 128, 1, None), -1),
        ("ntb200_flash_attn_varlen", (16, 16, 16, 16, 16, None, 2, 8, 8, 32, 8, 128, 4, 0.1, 1,
                                      4096, 128, 1024, 128, 1024, 128, 4096, 128, 1, None), -1),
        ("ntb200_flash_attn_varlen", (16, 16, 16, 16, 16, 16, 2, 8, 8, 32, 8, 128, 4, 0.1, 1,
                                      4096, 128, 1028, 128, 1024, 128, 4096, 128, 1, None), -3),
        # decode for the single-query rows of a varlen batch: null query_start_loc; GQA
        # group 16; a block table stride below its width
        ("ntb200_paged_attention_decode_varlen", (16, 16, 16, 16, None, 16, 16, 2, 32, 8, 128, 16, 64, 4, 4, 64, 0.1,
                                                  4096, 128, 4096, 128, 16384, 1024, 128, None, 0, 1, None), -1),
        ("ntb200_paged_attention_decode_varlen", (16, 16, 16, 16, 16, 16, 16, 2, 128, 8, 128, 16, 64, 4, 4, 64, 0.1,
                                                  4096, 128, 4096, 128, 16384, 1024, 128, None, 0, 1, None), -6),
        ("ntb200_paged_attention_decode_varlen", (16, 16, 16, 16, 16, 16, 16, 2, 32, 8, 128, 16, 64, 4, 3, 64, 0.1,
                                                  4096, 128, 4096, 128, 16384, 1024, 128, None, 0, 1, None), -1),
        # peer all-reduce (out, partial, peer_buffers, numel, capacity, rank, world_size,
        # dtype, stream): more elements than the capacity; rank outside the world; nine
        # ranks; out 8-aligned; fp32; a two-shot count that is not a multiple of 8
        ("ntb200_allreduce_oneshot", (16, 16, 16, 2000, 1000, 0, 2, 1, None), -1),
        ("ntb200_allreduce_oneshot", (16, 16, 16, 8, 1000, 2, 2, 1, None), -1),
        ("ntb200_allreduce_oneshot", (16, 16, 16, 8, 1000, 0, 9, 1, None), -1),
        ("ntb200_allreduce_oneshot", (8, 16, 16, 8, 1000, 0, 2, 1, None), -3),
        ("ntb200_allreduce_oneshot", (16, 16, 16, 8, 1000, 0, 2, 0, None), -2),
        ("ntb200_allreduce_twoshot", (16, 16, 16, 12, 1000, 0, 2, 1, None), -1),
        ("ntb200_paged_attention_decode",
         (1, 1, 1, 1, 1, 1, 2, 36, 4, 128, 16, 8, 4, 4, 64, 0.1, 512, 128, 512, 128, 2048, 128, 128, None, 0, 1, None), -6),
    ],
)
def test_host_validation_rejects_before_launch(name, args, status):
    with pytest.raises(capi.NtB200Error) as e:
        capi.call(name, *args)
    assert e.value.status == status
    assert capi.lib().ntb200_last_error()  # a detail message was recorded


def test_zero_sized_calls_are_no_ops():
    assert capi.call("ntb200_rms_norm", 1, 1, None, 0, 8, 8, 8, 1e-6, 0, None) == 0
    assert capi.call("ntb200_silu_and_mul", 1, 1, 0, 8, 16, 8, 1, None) == 0
    assert capi.call("ntb200_linear", 1, 1, 1, None, 0, 8, 16, 16, 16, 8, None, 0, 1, None) == 0
    assert capi.call("ntb200_rope_and_cache", 1, 4, 1, 1, 1, 1, 1, 1, 1, 4, 0, 0, 2, 1, 128, 128, *(128,) * 6,
                     128, 64, 16, 64, 2048, 128, 128, 1, None) == 0
    # no rows, no filter: nothing to do (no device is touched)
    assert capi.call("ntb200_top_k_top_p", 1, 0, 100, 100, 1, 4, None, None) == 0
    assert capi.call("ntb200_top_k_top_p", 1, 4, 100, 100, None, 4, None, None) == 0
    assert capi.call("ntb200_random_sample", 1, 1, 1, 0, 8, 8, 8, None) == 0
    assert capi.call("ntb200_linear_silu_and_mul", 16, 16, 16, 0, 8, 64, 64, 64, 8, 1, None) == 0
    assert capi.call("ntb200_rms_norm_linear", 16, None, 16, None, 16, 1e-5, 16, 0, 8, 64, 64, 0, 0, 64, 8, 1,
                     None) == 0
    assert capi.call("ntb200_gemma_rms_norm", 16, 16, 16, 0, 8, 8, 8, 1e-6, 1, None) == 0
    assert capi.call("ntb200_paged_attention_prefill", 16, 16, 16, 16, 16, 16, 16, 0, 0, 32, 8, 128, 16, 64, 4, 4,
                     4, 0.1, 1, 4096, 128, 4096, 128, 16384, 1024, 128, 1, None) == 0
    assert capi.call("ntb200_flash_attn_varlen", 16, 16, 16, 16, 16, 16, 2, 0, 8, 32, 8, 128, 4, 0.1, 1,
                     4096, 128, 1024, 128, 1024, 128, 4096, 128, 1, None) == 0
    assert capi.call("ntb200_allreduce_oneshot", 16, 16, 16, 0, 1000, 0, 2, 1, None) == 0
    assert capi.call("ntb200_allreduce_twoshot", 16, 16, 16, 0, 1000, 0, 2, 1, None) == 0


def test_workspace_queries():
    lib = capi.lib()
    ws = lib.ntb200_paged_attention_decode_workspace_size(256, 32, 8, 128, 16, 8192)
    # 256 seqs x 32 heads x 8 chunks of 1024 tokens x (128 fp32 partials + 1 lse), 256-aligned
    assert ws == 256 * 32 * 8 * 128 * 4 + 256 * 32 * 8 * 4
    assert lib.ntb200_paged_attention_decode_workspace_size(256, 32, 8, 64, 16, 8192) == 0
    assert lib.ntb200_linear_workspace_size(1, 4096, 4096) == 0
    # peer all-reduce buffer: 8 KiB of flags + a 256-byte header + two parities x W ranks
    # of the capacity rounded to 256 B
    # two flag arrays, the header, the one-shot parity slots (2 x 4 x 2048 B: 1000 bf16
    # rounded to 256 B), then the two-shot scatter slots and reduced chunk (5 x 512 B:
    # ceil(1000 / 4) = 250 -> 256 elements)
    assert lib.ntb200_allreduce_buffer_size(1000, 2, 4) == 2 * 8192 + 256 + 2 * 4 * 2048 + 5 * 512
    assert lib.ntb200_allreduce_buffer_size(1000, 2, 9) == 0
    # LM-head argmax: one 8-byte key per row (256-aligned) while the logits stay on chip
    # (M <= 256); beyond, the [M, V] logits as well
    assert lib.ntb200_linear_argmax_workspace_size(256, 128256, 4096) == 2048
    assert lib.ntb200_linear_argmax_workspace_size(300, 1000, 64) == 2560 + 600064
    assert lib.ntb200_linear_argmax_workspace_size(0, 1000, 64) == 0


def test_read_device_error_rejects_null():
    with pytest.raises(capi.NtB200Error):
        capi.call("ntb200_read_device_error", ctypes.POINTER(ctypes.c_int)(), None)


def test_torch_ops_refuse_host_tensors():
    """The product path has no CPU fallback: each torch-facing wrapper, given host tensors,
    raises instead of computing anything (the ntb200 ops are registered for the CUDA
    dispatch key only, so torch's dispatcher refuses the CPU call)."""
    import torch

    from vllm_nt._ntops.torch.embedding import embedding
    from vllm_nt._ntops.torch.linear import linear, linear_argmax, linear_silu_and_mul, rms_norm_linear
    from vllm_nt._ntops.torch.rms_norm import fused_add_rms_norm, gemma_rms_norm, rms_norm
    from vllm_nt._ntops.torch.silu import silu_and_mul

    x = torch.randn(4, 64).to(torch.bfloat16)
    w = torch.randn(32, 64).to(torch.bfloat16)
    g = torch.ones(64, dtype=torch.bfloat16)
    ids = torch.tensor([0, 3, 5])
    calls = {
        "linear": lambda: linear(x, w),
        "linear_silu_and_mul": lambda: linear_silu_and_mul(x, w),
        "linear_argmax": lambda: linear_argmax(x, w),
        "rms_norm_linear": lambda: rms_norm_linear(x, g, 1e-5, w, x.clone()),
        "rms_norm": lambda: rms_norm(x, 64, g, 1e-5),
        "fused_add_rms_norm": lambda: fused_add_rms_norm(x, x.clone(), g, 1e-5),
        "gemma_rms_norm": lambda: gemma_rms_norm(x, g, 1e-6),
        "silu_and_mul": lambda: silu_and_mul(x),
        "embedding": lambda: embedding(ids, w),
    }
    for name, call in calls.items():
        with pytest.raises((RuntimeError, NotImplementedError), match="'CPU' backend|CUDA tensor"):
            call()
            pytest.fail(f"{name} ran on host tensors")

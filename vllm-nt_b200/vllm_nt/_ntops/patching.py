"""Registers the B200 kernels into vLLM and keeps the plugin's usage statistics.

Public surface (same names as vllm_nt/_ntops/patching.py): ``ensure_registered``,
``get_usage_summary``, ``format_usage_summary``, ``maybe_print_usage_summary``,
``_reset_usage_state``, ``_OPERATOR_SPECS``, ``_FUNCTION_PATCH_SPECS`` and the
``_nt_*`` forwards.  Mechanisms, in the order ``ensure_registered`` applies them:

1. CustomOp out-of-tree registration (``cls.register_oot``) of an ``NT<op>`` subclass for
   RMSNorm / GemmaRMSNorm / SiluAndMul.  On a CUDA platform vLLM dispatches
   ``forward_cuda`` (vllm/model_executor/custom_op.py:174-207), and ``forward_native`` when
   the op is disabled; the reference overrides only ``forward_oot``, which CUDA never
   calls.  The subclasses here override all three.
2. Leaf-method patches of ``UnquantizedLinearMethod.apply`` (MatMul) and
   ``UnquantizedEmbeddingMethod.embedding`` / ``.apply`` (Embedding / LMHead).
3. Function patches (``FunctionPatchSpec``): ``RotaryEmbedding.forward_{cuda,oot,native}``
   (RoPE) and, because on CUDA attention runs inside the opaque custom ops
   ``unified_kv_cache_update`` / ``unified_attention_with_output`` which call
   ``impl.do_kv_cache_update`` / ``impl.forward``, ``FlashAttentionImpl.do_kv_cache_update``
   (StoreKVCache) and ``FlashAttentionImpl.forward`` (PagedAttentionDecode for pure-decode
   batches; prefill stays on vLLM's FlashAttention).

Each hook checks that the call is one the kernels implement (dtype, head size, layout);
other calls go to vLLM's implementation directly.  Eligible calls go through
``backends.route`` so the YAML config, ``VLLM_NT_DISABLE_OPS``, first-failure disabling
and the hit/failure/fallback counters behave as in the reference.
"""

from __future__ import annotations

import atexit
import importlib
import inspect
import logging
import os
import sys
from dataclasses import dataclass
from typing import Any, Callable, cast

import torch
from vllm.model_executor.layers import activation, layernorm
from vllm.model_executor.layers.linear import UnquantizedLinearMethod
from vllm.model_executor.layers.vocab_parallel_embedding import UnquantizedEmbeddingMethod

from vllm_nt._ntops import backends
from vllm_nt._ntops.config import canonical_op_name, load_backend_config, reset_backend_config_cache
from vllm_nt._ntops.oot_support import (
    OperatorStats,
    act_and_mul,
    embedding,
    gate_up_silu_and_mul,
    linear,
    norm,
    nt_apply_top_k_top_p,
    nt_paged_decode,
    nt_random_sample,
    paged_attention_decode_flash,
    paged_attention_flash,
    rope,
    store_kv_cache,
    store_kv_cache_flash,
)

logger = logging.getLogger("vllm_nt")
_PARENT_PID_ENV = "VLLM_NT_PARENT_PID"
os.environ.setdefault(_PARENT_PID_ENV, str(os.getpid()))
_TRUE = frozenset({"1", "true", "yes", "on"})
_FEATURE_ENV_VARS = {"FA": "VLLM_NT_ENABLE_FA", "MM": "VLLM_NT_ENABLE_MM"}
_FUNCTION_PATCH_FEATURES = {
    "StoreKVCache": "FA",
    "UnifiedAttentionWithOutput": "FA",
    "PagedAttentionPrefill": "FA",
    "PagedAttentionDecode": "FA",
    "SDPA": "FA",
}
_OPERATOR_FEATURES = {"MatMul": "MM", "LMHead": "MM"}
_REGISTERED_VIA_PRIORITY = {
    None: 0,
    "oot": 1,
    "monkey_patch": 2,
    "function_patch": 3,
    "custom_op_rebind": 4,
    "custom_op_intercept": 5,
}
_HALF_TYPES = (torch.bfloat16, torch.float16)


@dataclass(frozen=True)
class FunctionPatchSpec:
    patch_id: str
    module_path: str
    attr_name: str
    object_name: str | None = None
    required: bool = True
    builder: Callable[[object], object] | None = None


@dataclass
class _AppliedFunctionPatch:
    spec: FunctionPatchSpec
    target_obj: object
    original: object


# --------------------------------------------------------------------------------------
# small helpers
# --------------------------------------------------------------------------------------


def _mark_function_patch(fn: object, patch_id: str) -> object:
    try:
        setattr(fn, "_vllm_nt_patch_id", patch_id)
    except Exception:
        pass
    return fn


def _is_function_patch(fn: object, patch_id: str) -> bool:
    return getattr(fn, "_vllm_nt_patch_id", None) == patch_id


def _env_flag(name: str, default: bool) -> bool:
    value = os.environ.get(name)
    return default if value is None else value.strip().lower() in _TRUE


def _nt_feature_enabled(feature: str | None = None) -> bool:
    if not _env_flag("VLLM_NT_ENABLE_ALL", True):
        return False
    return feature is None or _env_flag(_FEATURE_ENV_VARS[feature], True)


def _disabled_ops() -> set[str]:
    return backends.disabled_ops()


def _operator_enabled(name: str) -> bool:
    return name not in _disabled_ops() and _nt_feature_enabled(_OPERATOR_FEATURES.get(name))


# Patches this build adds beyond the reference's op set: applied only when the config
# names the op with a kernel backend, so configs written for the reference run unchanged.
_OPT_IN_PATCHES = frozenset({"GateUpSiluAndMul"})


def _function_patch_enabled(spec: FunctionPatchSpec) -> bool:
    if spec.patch_id in _disabled_ops():
        return False
    key = canonical_op_name(spec.patch_id)
    if key in _OPT_IN_PATCHES and not (key in load_backend_config().ops and backends.backend_enabled(key)):
        return False
    if key == "UnifiedAttentionWithOutput":
        key = "PagedAttentionDecode"
    if spec.module_path.startswith("vllm") and key in load_backend_config().ops and not backends.backend_enabled(key):
        return False
    return _nt_feature_enabled(_FUNCTION_PATCH_FEATURES.get(spec.patch_id))


def _route(op_name: str, call_original: Callable[[], Any], call_b200: Callable[[], Any]) -> Any:
    return backends.route(op_name, call_original, call_ninetoothed=call_b200, call_b200=call_b200)


def _record_hit(name: str, x: torch.Tensor) -> None:
    if not backends.stats_enabled():
        return
    stats = _OPERATOR_STATS[name]
    stats.hits += 1
    backends.record_hit(name)
    if not stats.logged:
        logger.info("vllm-nt: %s %s kernel invoked (shape=%s)", backends.active_backend(name), name, tuple(x.shape))
        stats.logged = True


def _set_registered_via(name: str, value: str) -> None:
    stats = _OPERATOR_STATS[name]
    if _REGISTERED_VIA_PRIORITY.get(value, 0) >= _REGISTERED_VIA_PRIORITY.get(stats.registered_via, 0):
        stats.registered_via = value


def _unbound(cls: type, attr: str) -> Callable[..., Any] | None:
    """``cls.attr`` as a callable taking (self, *args), unwrapping staticmethods, so the
    hooks can call vLLM's own implementation of an op they replaced."""
    try:
        raw = inspect.getattr_static(cls, attr)
    except AttributeError:
        return None
    if isinstance(raw, staticmethod):
        fn = raw.__func__
        return lambda self, *a, **k: fn(*a, **k)
    if callable(raw):
        return raw
    return None


# --------------------------------------------------------------------------------------
# CustomOp forwards
# --------------------------------------------------------------------------------------

# name -> {"native": f(self, ...), "cuda": f(self, ...)} captured before registration
_ORIGINAL_OPERATOR_FORWARDS: dict[str, dict[str, Callable[..., Any]]] = {}


def _call_original_operator(name: str, self, *args: Any) -> Any:
    impls = _ORIGINAL_OPERATOR_FORWARDS.get(name)
    if not impls:
        raise RuntimeError(f"original {name} forward is unavailable")
    first = args[0] if args else None
    if isinstance(first, torch.Tensor) and first.is_cuda and "cuda" in impls:
        return impls["cuda"](self, *args)
    return impls["native"](self, *args)


def _norm_eligible(x: torch.Tensor, weight: torch.Tensor | None, residual: torch.Tensor | None) -> bool:
    return (
        x.is_cuda
        and x.dtype in (torch.float32, *_HALF_TYPES)
        and (weight is None or weight.dtype == x.dtype)
        and (residual is None or (residual.dtype == x.dtype and residual.shape == x.shape))
    )


def _nt_rms_norm_forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
    has_weight = getattr(self, "has_weight", True)
    weight = self.weight.data if has_weight and getattr(self, "weight", None) is not None else None
    if "RMSNorm" not in _ORIGINAL_OPERATOR_FORWARDS:
        _record_hit("RMSNorm", x)
        return norm(self, x, weight, residual)
    if getattr(self, "variance_size_override", None) is not None or not _norm_eligible(x, weight, residual):
        return _call_original_operator("RMSNorm", self, x, residual)

    def kernels():
        _record_hit("RMSNorm", x)
        return norm(self, x, weight, residual)

    return _route("RMSNorm", lambda: _call_original_operator("RMSNorm", self, x, residual), kernels)


def _nt_gemma_rms_norm_forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
    weight = (1.0 + self.weight.data.float()).to(x.dtype)
    if "GemmaRMSNorm" not in _ORIGINAL_OPERATOR_FORWARDS:
        _record_hit("GemmaRMSNorm", x)
        return norm(self, x, weight, residual, gemma=True)
    if not _norm_eligible(x, weight, residual):
        return _call_original_operator("GemmaRMSNorm", self, x, residual)

    def kernels():
        _record_hit("GemmaRMSNorm", x)
        return norm(self, x, weight, residual, gemma=True)

    return _route("GemmaRMSNorm", lambda: _call_original_operator("GemmaRMSNorm", self, x, residual), kernels)


def _nt_silu_and_mul_forward(self, x: torch.Tensor) -> torch.Tensor:
    if "SiluAndMul" not in _ORIGINAL_OPERATOR_FORWARDS:
        _record_hit("SiluAndMul", x)
        return act_and_mul(x)
    if not (x.is_cuda and x.dtype in (torch.float32, *_HALF_TYPES)):
        return _call_original_operator("SiluAndMul", self, x)

    def kernels():
        _record_hit("SiluAndMul", x)
        return act_and_mul(x)

    return _route("SiluAndMul", lambda: _call_original_operator("SiluAndMul", self, x), kernels)


def _nt_mul_and_silu_forward(self, x: torch.Tensor) -> torch.Tensor:
    """MulAndSilu is not one of this backend's kernels: vLLM's implementation runs."""
    return _call_original_operator("MulAndSilu", self, x)


def _nt_gelu_and_mul_forward(self, x: torch.Tensor) -> torch.Tensor:
    """GeluAndMul is not one of this backend's kernels: vLLM's implementation runs."""
    return _call_original_operator("GeluAndMul", self, x)


# --------------------------------------------------------------------------------------
# leaf methods: MatMul / Embedding / LMHead
# --------------------------------------------------------------------------------------


def _gemm_eligible(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> bool:
    return (
        x.is_cuda
        and x.dtype in _HALF_TYPES
        and weight.dtype == x.dtype
        and weight.dim() == 2
        and weight.shape[1] % 8 == 0
        and weight.stride(-1) == 1
        and (bias is None or bias.dtype == x.dtype)
    )


def _nt_unquantized_linear_apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None, **kwargs):
    original = getattr(_nt_unquantized_linear_apply, "_original", None)

    def finish(out: torch.Tensor) -> torch.Tensor:
        residual = kwargs.get("residual")
        return out + residual if residual is not None else out

    def kernels():
        _record_hit("MatMul", x)
        return finish(linear(x, layer.weight, bias))

    if original is None or not isinstance(self, UnquantizedLinearMethod):
        return kernels()
    call = lambda: original(self, layer, x, bias, **kwargs)  # noqa: E731
    if not _gemm_eligible(x, layer.weight, bias):
        return call()
    return _route("MatMul", call, kernels)


def _nt_unquantized_embedding(self, layer: torch.nn.Module, input_: torch.Tensor) -> torch.Tensor:
    original = getattr(_nt_unquantized_embedding, "_original", None)

    def kernels():
        _record_hit("Embedding", input_)
        return embedding(layer, input_)

    if original is None or not isinstance(self, UnquantizedEmbeddingMethod):
        return kernels()
    call = lambda: original(self, layer, input_)  # noqa: E731
    if not (input_.is_cuda and layer.weight.is_cuda and input_.dtype in (torch.int32, torch.int64)):
        return call()
    return _route("Embedding", call, kernels)


def _nt_unquantized_embedding_apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None, **kwargs):
    original = getattr(_nt_unquantized_embedding_apply, "_original", None)

    def finish(out: torch.Tensor) -> torch.Tensor:
        residual = kwargs.get("residual")
        return out + residual if residual is not None else out

    def kernels():
        _record_hit("LMHead", x)
        return finish(linear(x, layer.weight, bias))

    if original is None or not isinstance(self, UnquantizedEmbeddingMethod):
        return kernels()
    call = lambda: original(self, layer, x, bias, **kwargs)  # noqa: E731
    if not _gemm_eligible(x, layer.weight, bias):
        return call()
    return _route("LMHead", call, kernels)


def _nt_layer_norm(*args, **kwargs):
    raise NotImplementedError("LayerNorm (GPT-2) is outside the B200 backend; vLLM's path serves it")


# --------------------------------------------------------------------------------------
# function-patch builders
# --------------------------------------------------------------------------------------


def _build_rotary_forward(original: object) -> object:
    """Replacement for RotaryEmbedding.forward_{cuda,oot,native}(positions, query, key)."""
    if _is_function_patch(original, "RoPE"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor | None = None, *rest, **kw):
        call = lambda: original_fn(self, positions, query, key, *rest, **kw)  # noqa: E731
        if (
            rest
            or kw
            or not self.is_neox_style
            or self.rotary_dim % 2
            or not query.is_cuda
            or query.dtype not in (torch.float32, *_HALF_TYPES)
        ):
            return call()

        def kernels():
            cache = self._match_cos_sin_cache_dtype(query)
            if cache is None:  # older vLLM returned nothing and updated the attribute
                cache = self.cos_sin_cache
            result = rope(
                positions,
                query,
                key,
                cos_sin_cache=cache,
                head_size=self.head_size,
                rotary_dim=self.rotary_dim,
                is_neox_style=self.is_neox_style,
            )
            _record_hit("RoPE", query)
            return result

        return _route("RoPE", call, kernels)

    return _mark_function_patch(forward, "RoPE")


def _attn_impl_supported(impl: Any, dtype: torch.dtype, kv_cache: torch.Tensor, kv_dim: int = 0) -> bool:
    """Whether the B200 attention kernels serve this attention impl and cache.  kv_dim is
    the cache dimension that separates K from V: 0 for FlashAttention's
    [2, blocks, 16, H, D], 1 for FlashInfer's [blocks, 2, 16, H, D] (whose memory order may
    be NHD or HND; the kernels take the strides).  The answer is kept on the impl (its
    configuration is fixed after construction), keyed by the dtypes and the cache shape, so
    the per-layer check is one attribute read."""
    key = (dtype, kv_cache.dtype, kv_cache.shape, kv_dim)
    cached = getattr(impl, "_ntb200_supported", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    ok = _attn_impl_check(impl, dtype, kv_cache, kv_dim)
    try:
        impl._ntb200_supported = (key, ok)
    except AttributeError:
        pass
    return ok


def _attn_impl_check(impl: Any, dtype: torch.dtype, kv_cache: torch.Tensor, kv_dim: int = 0) -> bool:
    attn_type = getattr(impl, "attn_type", "decoder")
    sliding = getattr(impl, "sliding_window", None)
    return (
        str(getattr(attn_type, "value", attn_type)).lower() == "decoder"
        and getattr(impl, "kv_cache_dtype", "auto") == "auto"
        and getattr(impl, "alibi_slopes", None) is None
        and not getattr(impl, "logits_soft_cap", None)
        and getattr(impl, "sinks", None) is None
        and (sliding is None or tuple(sliding) == (-1, -1))
        and getattr(impl, "dcp_world_size", 1) == 1
        and getattr(impl, "head_size", 0) == 128
        and dtype in _HALF_TYPES
        and getattr(impl, "kv_sharing_target_layer_name", None) is None
        and kv_cache.dim() == 5
        and kv_cache.shape[kv_dim] == 2
        and kv_cache.shape[2] == 16
        and kv_cache.stride(-1) == 1
        and kv_cache.dtype == dtype
    )


def _build_flash_attn_kv_update(original: object) -> object:
    """Replacement for FlashAttentionImpl.do_kv_cache_update(layer, key, value, kv_cache,
    slot_mapping): the slot-mapped store runs on the B200 kernel."""
    if _is_function_patch(original, "StoreKVCache"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        call = lambda: original_fn(self, layer, key, value, kv_cache, slot_mapping)  # noqa: E731
        if not (key.is_cuda and _attn_impl_supported(self, key.dtype, kv_cache)):
            return call()

        def kernels():
            _record_hit("StoreKVCache", key)
            store_kv_cache_flash(key, value, kv_cache, slot_mapping)

        return _route("StoreKVCache", call, kernels)

    return _mark_function_patch(do_kv_cache_update, "StoreKVCache")


def _build_flash_attn_forward(original: object) -> object:
    """Replacement for FlashAttentionImpl.forward: pure-decode batches (one query token
    per request) run on the split-K paged-decode kernel; prefill, chunked-prefill and mixed
    batches on the tcgen05 prefill kernel (its single-query requests on the decode kernel),
    reading K/V from the paged cache in place.  Cascade attention and non-causal metadata
    stay on vLLM's FlashAttention."""
    if _is_function_patch(original, "PagedAttentionDecode"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None, output_block_scale=None, *rest, **kw):
        call = lambda: original_fn(  # noqa: E731
            self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale, *rest, **kw
        )
        meta = attn_metadata
        if (
            meta is None
            or rest
            or kw
            or output_scale is not None
            or output_block_scale is not None
            or getattr(meta, "use_cascade", False)
            or not getattr(meta, "causal", True)
            or getattr(meta, "max_query_len", 0) < 1
            or not query.is_cuda
            or not _attn_impl_supported(self, query.dtype, kv_cache)
        ):
            return call()
        n = int(meta.num_actual_tokens)
        qsl = getattr(meta, "query_start_loc", None)
        max_q = int(meta.max_query_len)
        if max_q == 1 and (qsl is None or qsl.shape[0] - 1 == n):

            def kernels():
                _record_hit("PagedAttentionDecode", query)
                paged_attention_decode_flash(
                    output, query, kv_cache, meta.seq_lens, meta.block_table, n, self.scale, int(meta.max_seq_len)
                )
                return output

            return _route("PagedAttentionDecode", call, kernels)
        if qsl is None:
            return call()

        def varlen():
            _record_hit("PagedAttentionPrefill", query)
            paged_attention_flash(
                output, query, kv_cache, qsl, meta.seq_lens, meta.block_table, n, max_q, int(meta.max_seq_len),
                self.scale,
            )
            return output

        return _route("PagedAttentionPrefill", call, varlen)

    return _mark_function_patch(forward, "PagedAttentionDecode")


def _build_flashinfer_kv_update(original: object) -> object:
    """Replacement for FlashInferImpl.do_kv_cache_update: the same slot-mapped store on
    FlashInfer's [blocks, 2, 16, H, D] cache."""
    if _is_function_patch(original, "StoreKVCache"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        call = lambda: original_fn(self, layer, key, value, kv_cache, slot_mapping)  # noqa: E731
        if not (key.is_cuda and _attn_impl_supported(self, key.dtype, kv_cache, 1)):
            return call()

        def kernels():
            _record_hit("StoreKVCache", key)
            store_kv_cache_flash(key, value, kv_cache, slot_mapping, 1)

        return _route("StoreKVCache", call, kernels)

    return _mark_function_patch(do_kv_cache_update, "StoreKVCache")


def _build_flashinfer_forward(original: object) -> object:
    """Replacement for FlashInferImpl.forward: a pure-decode batch (one query token per
    request) whose metadata carries the decode block table and lengths (vLLM's TRT-LLM
    decode metadata on Blackwell) runs on the split-K paged-decode kernel; prefill, mixed
    batches, cascade and FlashInfer's own planned decode stay on FlashInfer."""
    if _is_function_patch(original, "PagedAttentionDecode"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None, output_block_scale=None, *rest, **kw):
        call = lambda: original_fn(  # noqa: E731
            self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale, *rest, **kw
        )
        meta = attn_metadata
        dec = getattr(meta, "decode", None)
        if (
            meta is None
            or rest
            or kw
            or output_scale is not None
            or output_block_scale is not None
            or getattr(meta, "use_cascade", False)
            or getattr(meta, "num_prefills", 1) != 0
            or getattr(dec, "block_tables", None) is None
            or getattr(dec, "seq_lens", None) is None
            or not query.is_cuda
            or not _attn_impl_supported(self, query.dtype, kv_cache, 1)
        ):
            return call()
        n = int(meta.num_actual_tokens)
        if int(getattr(meta, "num_decodes", -1)) != n or int(getattr(meta, "num_decode_tokens", -1)) != n:
            return call()

        def kernels():
            _record_hit("PagedAttentionDecode", query)
            paged_attention_decode_flash(
                output, query, kv_cache, dec.seq_lens, dec.block_tables, n, self.scale, int(dec.max_seq_len), 1
            )
            return output

        return _route("PagedAttentionDecode", call, kernels)

    return _mark_function_patch(forward, "PagedAttentionDecode")


def _fused_mlp_eligible(mlp: Any, x: torch.Tensor) -> bool:
    """gate_up_proj -> SiluAndMul -> down_proj with an unquantised, bias-free merged
    gate_up weight whose output stays on this rank (no gather)."""
    gu = getattr(mlp, "gate_up_proj", None)
    act = getattr(mlp, "act_fn", None)
    w = getattr(gu, "weight", None)
    return (
        isinstance(act, activation.SiluAndMul)
        and hasattr(mlp, "down_proj")
        and isinstance(getattr(gu, "quant_method", None), UnquantizedLinearMethod)
        and getattr(gu, "bias", None) is None
        and not getattr(gu, "gather_output", False)
        and isinstance(w, torch.Tensor)
        and w.dim() == 2
        and w.shape[0] % 2 == 0
        and w.shape[1] % 8 == 0
        and w.stride(-1) == 1
        and x.is_cuda
        and x.dtype in _HALF_TYPES
        and w.dtype == x.dtype
        and x.shape[-1] == w.shape[1]
    )


def _build_mlp_forward(original: object) -> object:
    """Replacement for LlamaMLP.forward (and MLPs of the same shape): gate_up_proj and
    SiluAndMul become one GEMM whose epilogue applies silu(gate) * up, so the [T, 2I]
    gate_up activation is never written; down_proj runs through its own hook."""
    if _is_function_patch(original, "GateUpSiluAndMul"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, x):
        if not _fused_mlp_eligible(self, x):
            return original_fn(self, x)

        def kernels():
            _record_hit("GateUpSiluAndMul", x)
            out, _ = self.down_proj(gate_up_silu_and_mul(x, self.gate_up_proj.weight))
            return out

        return _route("GateUpSiluAndMul", lambda: original_fn(self, x), kernels)

    return _mark_function_patch(forward, "GateUpSiluAndMul")



def _sampler_logits_eligible(x: torch.Tensor) -> bool:
    """fp32 rows on a CUDA device with unit stride in the vocabulary dimension."""
    return x.is_cuda and x.dtype == torch.float32 and x.dim() == 2 and x.stride(-1) == 1


def _build_apply_top_k_top_p_patch(original: object) -> object:
    """Replacement for vLLM's topk_topp_sampler.apply_top_k_top_p(logits, k, p) (the
    reference's TopKTopP patch, vllm_nt/_ntops/patching.py:1446-1463): the mask is the
    radix-select kernel instead of a sort of every row.  vLLM's TopKTopPSampler reaches it
    on its native path (per-request generators, or FlashInfer sampling turned off)."""
    if _is_function_patch(original, "TopKTopP"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def wrapped(logits: torch.Tensor, k: torch.Tensor | None, p: torch.Tensor | None):
        call = lambda: original_fn(logits, k, p)  # noqa: E731
        if (k is None and p is None) or not _sampler_logits_eligible(logits):
            return call()

        def kernels():
            _record_hit("TopKTopP", logits)
            return nt_apply_top_k_top_p(logits, k, p)

        return _route("TopKTopP", call, kernels)

    return _mark_function_patch(wrapped, "TopKTopP")


def _build_random_sample_patch(original: object) -> object:
    """Replacement for vLLM's topk_topp_sampler.random_sample(probs, generators) (the
    reference's RandomSample patch, vllm_nt/_ntops/patching.py:1466-1479): the division by
    the exponential draws and the argmax are one kernel pass."""
    if _is_function_patch(original, "RandomSample"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def wrapped(probs: torch.Tensor, generators: dict[int, torch.Generator]):
        call = lambda: original_fn(probs, generators)  # noqa: E731
        if not _sampler_logits_eligible(probs):
            return call()

        def kernels():
            _record_hit("RandomSample", probs)
            return nt_random_sample(probs, generators)

        return _route("RandomSample", call, kernels)

    return _mark_function_patch(wrapped, "RandomSample")


def _build_rejection_sample_patch(original: object) -> object:
    """Counts vLLM's rejection_sample calls under RejectionSample and runs vLLM's own code,
    as the reference's patch does (vllm_nt/_ntops/patching.py:1482-1497).  The hit is
    recorded against the target distribution: the ``target_logits`` (older vLLM:
    ``target_probs``) keyword, else the sixth positional argument."""
    if _is_function_patch(original, "RejectionSample"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def wrapped(*args: Any, **kwargs: Any):
        candidates = (kwargs.get("target_logits"), kwargs.get("target_probs"), args[5] if len(args) > 5 else None)
        target = next((c for c in candidates if isinstance(c, torch.Tensor)), None)
        if target is not None:
            _record_hit("RejectionSample", target)
        return original_fn(*args, **kwargs)

    return _mark_function_patch(wrapped, "RejectionSample")

_OPERATOR_SPECS: dict[str, tuple[type, Callable[..., Any]]] = {
    "RMSNorm": (layernorm.RMSNorm, _nt_rms_norm_forward),
    "SiluAndMul": (activation.SiluAndMul, _nt_silu_and_mul_forward),
}
if getattr(layernorm, "GemmaRMSNorm", None) is not None:
    _OPERATOR_SPECS["GemmaRMSNorm"] = (layernorm.GemmaRMSNorm, _nt_gemma_rms_norm_forward)

_OPERATOR_STATS: dict[str, OperatorStats] = {name: OperatorStats() for name in _OPERATOR_SPECS} | {
    name: OperatorStats()
    for name in (
        "MulAndSilu",
        "GeluAndMul",
        "GELU",
        "LayerNorm",
        "MatMul",
        "Embedding",
        "WPE",
        "NTWPEKernel",
        "LMHead",
        "PagedAttentionPrefill",
        "PagedAttentionDecode",
        "StoreKVCache",
        "GateUpSiluAndMul",
        "RoPE",
        "SDPA",
        "TopKTopP",
        "RandomSample",
        "RejectionSample",
    )
}

for _name, (_cls, _fwd) in _OPERATOR_SPECS.items():
    _impls = {}
    for _key, _attr in (("native", "forward_native"), ("cuda", "forward_cuda")):
        _fn = _unbound(_cls, _attr)
        if _fn is not None:
            _impls[_key] = _fn
    if _impls:
        _ORIGINAL_OPERATOR_FORWARDS[_name] = _impls
for _name, _attr_cls in (("MulAndSilu", "MulAndSilu"), ("GeluAndMul", "GeluAndMul")):
    _cls = getattr(activation, _attr_cls, None)
    if _cls is not None:
        _ORIGINAL_OPERATOR_FORWARDS[_name] = {
            k: f for k, f in (("native", _unbound(_cls, "forward_native")), ("cuda", _unbound(_cls, "forward_cuda"))) if f
        }

_ROPE_MODULES = ("vllm.model_executor.layers.rotary_embedding.base",)
_FA_MODULE = "vllm.v1.attention.backends.flash_attn"
_FI_MODULE = "vllm.v1.attention.backends.flashinfer"
_SAMPLER_MODULE = "vllm.v1.sample.ops.topk_topp_sampler"
_FUNCTION_PATCH_SPECS: tuple[FunctionPatchSpec, ...] = (
    *(
        FunctionPatchSpec("RoPE", mod, attr, "RotaryEmbedding", False, _build_rotary_forward)
        for mod in _ROPE_MODULES
        for attr in ("forward_cuda", "forward_oot", "forward_native")
    ),
    FunctionPatchSpec("StoreKVCache", _FA_MODULE, "do_kv_cache_update", "FlashAttentionImpl", False, _build_flash_attn_kv_update),
    FunctionPatchSpec("PagedAttentionDecode", _FA_MODULE, "forward", "FlashAttentionImpl", False, _build_flash_attn_forward),
    FunctionPatchSpec("StoreKVCache", _FI_MODULE, "do_kv_cache_update", "FlashInferImpl", False, _build_flashinfer_kv_update),
    FunctionPatchSpec("PagedAttentionDecode", _FI_MODULE, "forward", "FlashInferImpl", False, _build_flashinfer_forward),
    FunctionPatchSpec("TopKTopP", _SAMPLER_MODULE, "apply_top_k_top_p", None, False, _build_apply_top_k_top_p_patch),
    FunctionPatchSpec("RandomSample", _SAMPLER_MODULE, "random_sample", None, False, _build_random_sample_patch),
    FunctionPatchSpec(
        "RejectionSample", "vllm.v1.sample.rejection_sampler", "rejection_sample", None, False,
        _build_rejection_sample_patch,
    ),
    *(
        FunctionPatchSpec("GateUpSiluAndMul", mod, "forward", cls, False, _build_mlp_forward)
        for mod, cls in (
            ("vllm.model_executor.models.llama", "LlamaMLP"),
            ("vllm.model_executor.models.qwen2", "Qwen2MLP"),
        )
    ),
)

_summary_printed = False
_registered = False
_APPLIED_FUNCTION_PATCHES: list[_AppliedFunctionPatch] = []


# --------------------------------------------------------------------------------------
# registration
# --------------------------------------------------------------------------------------


def _nt_subclass(name: str, cls: type, forward: Callable[..., Any]) -> type:
    return type(f"NT{name}", (cls,), {"forward_oot": forward, "forward_cuda": forward, "forward_native": forward})


def _try_register_oot() -> bool:
    try:
        for name, (cls, forward) in _OPERATOR_SPECS.items():
            if not _operator_enabled(name):
                continue
            cls.register_oot(name=name)(_nt_subclass(name, cls, forward))
            _set_registered_via(name, "oot")
        logger.info("vllm-nt: OOT registration succeeded for %s", ", ".join(_OPERATOR_SPECS))
        return True
    except Exception as exc:
        logger.warning("OOT registration failed (%s), will monkey-patch", exc)
        return False


def _monkey_patch() -> None:
    for name, (cls, forward) in _OPERATOR_SPECS.items():
        if not _operator_enabled(name):
            continue
        cls.forward_oot = forward
        cls.forward_cuda = forward
        cls.forward_native = forward
        _set_registered_via(name, "monkey_patch")
    logger.info("vllm-nt: monkey-patched %s", ", ".join(_OPERATOR_SPECS))


def _patch_leaf_methods() -> None:
    if _operator_enabled("MatMul"):
        setattr(_nt_unquantized_linear_apply, "_original", UnquantizedLinearMethod.apply)
        UnquantizedLinearMethod.apply = _nt_unquantized_linear_apply
        _set_registered_via("MatMul", "monkey_patch")
    if _operator_enabled("Embedding"):
        setattr(_nt_unquantized_embedding, "_original", UnquantizedEmbeddingMethod.embedding)
        UnquantizedEmbeddingMethod.embedding = _nt_unquantized_embedding
        _set_registered_via("Embedding", "monkey_patch")
    if _operator_enabled("LMHead"):
        setattr(_nt_unquantized_embedding_apply, "_original", UnquantizedEmbeddingMethod.apply)
        UnquantizedEmbeddingMethod.apply = _nt_unquantized_embedding_apply
        _set_registered_via("LMHead", "monkey_patch")


def _resolve_function_patch_target(spec: FunctionPatchSpec) -> tuple[object, object]:
    module = importlib.import_module(spec.module_path)
    target = getattr(module, spec.object_name) if spec.object_name else module
    return target, getattr(target, spec.attr_name)


def _apply_function_patches() -> None:
    global _APPLIED_FUNCTION_PATCHES
    applied: list[_AppliedFunctionPatch] = []
    try:
        for spec in _FUNCTION_PATCH_SPECS:
            if not _function_patch_enabled(spec):
                continue
            try:
                target, original = _resolve_function_patch_target(spec)
                replacement = original if spec.builder is None else spec.builder(original)
                setattr(target, spec.attr_name, replacement)
                applied.append(_AppliedFunctionPatch(spec, target, original))
                if spec.patch_id in _OPERATOR_STATS:
                    _set_registered_via(spec.patch_id, "function_patch")
            except Exception as exc:
                if spec.required:
                    raise
                logger.debug("Skipping optional function patch %s: %s", spec.patch_id, exc)
    except Exception:
        for patch in reversed(applied):
            setattr(patch.target_obj, patch.spec.attr_name, patch.original)
        raise
    _APPLIED_FUNCTION_PATCHES = applied


def _apply_custom_op_rebindings() -> None:
    """The reference can rebind vLLM's attention custom ops (VLLM_NT_ENABLE_CUSTOM_OP_REBIND)
    to reach its kernels on vendor platforms.  On CUDA the FlashAttentionImpl methods those
    ops call are patched instead, so the flag is accepted and has nothing left to do."""
    if os.environ.get("VLLM_NT_ENABLE_CUSTOM_OP_REBIND") == "1":
        logger.info("vllm-nt: attention is hooked through FlashAttentionImpl; custom-op rebind not needed")


# --------------------------------------------------------------------------------------
# usage summary
# --------------------------------------------------------------------------------------


def get_usage_summary() -> dict[str, object]:
    if not backends.stats_enabled():
        return {"registered_ops": [], "hit_ops": [], "missed_ops": [], "operators": {}, "disabled": []}
    operators: dict[str, dict[str, Any]] = {}
    for name, stats in _OPERATOR_STATS.items():
        per_backend = {
            backend: {"attempts": s.attempts, "hits": s.hits, "failures": s.failures, "fallbacks": s.fallbacks}
            for backend, s in sorted(backends.backend_stats(name).items())
        }
        operators[name] = {
            "configured_backend": backends.configured_backend(name),
            "active_backend": backends.active_backend(name),
            "hits": max(stats.hits, sum(v["hits"] for v in per_backend.values())),
            "failures": sum(v["failures"] for v in per_backend.values()),
            "fallbacks": sum(v["fallbacks"] for v in per_backend.values()),
            "registered_via": stats.registered_via,
            "backends": per_backend,
        }
    hit_ops = [name for name, d in operators.items() if d["hits"] > 0]
    return {
        "registered_ops": list(_OPERATOR_STATS),
        "hit_ops": hit_ops,
        "missed_ops": [name for name in _OPERATOR_STATS if name not in hit_ops],
        "operators": operators,
        "disabled": sorted(backends.disabled_ops()),
    }


def format_usage_summary(use_color: bool = True) -> str:
    blue, reset = ("\033[94m", "\033[0m") if use_color else ("", "")
    summary = get_usage_summary()
    lines = [f"{blue}Operator usage summary{reset}"]
    for name, d in cast(dict[str, dict[str, Any]], summary["operators"]).items():
        lines.append(
            f"{blue}- {name}: backend={d['active_backend']} hits={d['hits']} failures={d['failures']} "
            f"fallbacks={d['fallbacks']} ({d['registered_via'] or 'unregistered'}){reset}"
        )
    missed = cast(list[str], summary["missed_ops"])
    lines.append(f"{blue}Missed operators: {', '.join(missed) or 'None'}{reset}")
    return "\n".join(lines)


def maybe_print_usage_summary(*, include_empty: bool = False) -> bool:
    global _summary_printed
    if not backends.stats_enabled():
        return False
    summary = get_usage_summary()
    if _summary_printed or (not include_empty and not summary["hit_ops"]):
        return False
    print(format_usage_summary(), file=sys.stderr)
    _summary_printed = True
    return True


def _reset_usage_state() -> None:
    global _summary_printed
    for stats in _OPERATOR_STATS.values():
        stats.hits = 0
        stats.logged = False
    backends.reset_backend_state()
    reset_backend_config_cache()
    _summary_printed = False


def _print_worker_summary_on_exit() -> None:
    if os.getpid() != int(os.environ.get(_PARENT_PID_ENV, os.getpid())):
        maybe_print_usage_summary(include_empty=True)


atexit.register(_print_worker_summary_on_exit)


def ensure_registered() -> None:
    """Idempotent; applies every hook enabled by the env flags and the backend config."""
    global _registered
    if _registered:
        return
    if not _nt_feature_enabled():
        logger.info("vllm-nt: registration skipped because VLLM_NT_ENABLE_ALL is disabled")
        _registered = True
        return
    load_backend_config()
    _registered = True
    if not _try_register_oot():
        _monkey_patch()
    _patch_leaf_methods()
    _apply_function_patches()
    _apply_custom_op_rebindings()

"""Registers the B200 kernels into vLLM and keeps the plugin's usage statistics.

Public surface (the names vllm_nt/_ntops/patching.py exports, which configs, tests and
scripts written against vllm_nt use): ``ensure_registered``, ``get_usage_summary``,
``format_usage_summary``, ``maybe_print_usage_summary``, ``_reset_usage_state``,
``OperatorStats``, ``_OPERATOR_STATS``, ``_OPERATOR_SPECS``, ``FunctionPatchSpec``,
``_FUNCTION_PATCH_SPECS`` and the ``_nt_*`` forwards.

How the hooks reach vLLM, in the order ``ensure_registered`` installs them:

1. CustomOp out-of-tree registration (``cls.register_oot``) of an ``NT<op>`` subclass for
   RMSNorm / GemmaRMSNorm / SiluAndMul.  On a CUDA platform vLLM dispatches
   ``forward_cuda`` (vllm/model_executor/custom_op.py:174-207), and ``forward_native`` when
   the op is disabled; the reference overrides only ``forward_oot``, which CUDA never calls,
   so the subclasses here override all three.  An op whose registration raises gets the
   three methods assigned on vLLM's class instead.
2. Leaf-method replacements of ``UnquantizedLinearMethod.apply`` (MatMul) and
   ``UnquantizedEmbeddingMethod.embedding`` / ``.apply`` (Embedding / LMHead).
3. Function patches (``FunctionPatchSpec`` table): RoPE, the FlashAttention and FlashInfer
   impls' ``forward`` / ``do_kv_cache_update`` (on CUDA attention runs inside opaque custom
   ops that call these methods), the sampler functions and the opt-in fused MLP.

Every replaced attribute is written through one journal, so a required patch that fails
undoes the batch it belongs to.  Replacement functions are remembered in a weak map (the
mark that keeps registration idempotent).

Accounting.  Each hook first decides whether the kernels serve the call (dtype, layout,
head size, metadata).  A call they serve goes through ``backends.route`` (YAML config,
``VLLM_NT_DISABLE_OPS``, first-failure disabling, the attempts / hits / failures / fallbacks
counters).  A call they do not serve runs vLLM's implementation and is recorded as a
fallback to ``original`` together with the reason, so the usage summary shows every call
that did not reach a kernel: an operator's ``declined`` map counts them by reason.
"""

from __future__ import annotations

import atexit
import importlib
import inspect
import logging
import os
import sys
import weakref
from dataclasses import dataclass
from typing import Any, Callable, Iterable, cast

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
    norm_linear,
    nt_apply_top_k_top_p,
    nt_paged_decode,  # noqa: F401  (re-exported for callers of the reference's module)
    nt_random_sample,
    paged_attention_decode_flash,
    paged_attention_flash,
    rope,
    rope_and_store_kv_cache_flash,
    store_kv_cache,  # noqa: F401
    store_kv_cache_flash,
)

logger = logging.getLogger("vllm_nt")

# ======================================================================================
# switches
# ======================================================================================

_PARENT_PID_ENV = "VLLM_NT_PARENT_PID"
os.environ.setdefault(_PARENT_PID_ENV, str(os.getpid()))
_FEATURE_ENV_VARS = {"FA": "VLLM_NT_ENABLE_FA", "MM": "VLLM_NT_ENABLE_MM"}
# feature group of each patch / operator that has one
_FUNCTION_PATCH_FEATURES = dict.fromkeys(
    ("StoreKVCache", "UnifiedAttentionWithOutput", "PagedAttentionPrefill", "PagedAttentionDecode", "SDPA"), "FA"
)
_OPERATOR_FEATURES = {"MatMul": "MM", "LMHead": "MM"}
# Patches this build adds beyond the reference's op set: applied only when the config
# names the op with a kernel backend, so configs written for the reference run unchanged.
_OPT_IN_PATCHES = frozenset({"GateUpSiluAndMul", "RoPEKVCache", "RMSNormQKV"})
_HALF_TYPES = (torch.bfloat16, torch.float16)
_FLOAT_TYPES = (torch.float32, torch.bfloat16, torch.float16)


def _env_on(name: str, default: bool) -> bool:
    raw = os.environ.get(name)
    return default if raw is None else raw.strip().lower() in ("1", "true", "yes", "on")


def _nt_feature_enabled(feature: str | None = None) -> bool:
    """VLLM_NT_ENABLE_ALL gates everything; VLLM_NT_ENABLE_FA / _MM gate their groups."""
    return _env_on("VLLM_NT_ENABLE_ALL", True) and (feature is None or _env_on(_FEATURE_ENV_VARS[feature], True))


def _disabled_ops() -> set[str]:
    return backends.disabled_ops()


def _operator_enabled(name: str) -> bool:
    return name not in _disabled_ops() and _nt_feature_enabled(_OPERATOR_FEATURES.get(name))


def _function_patch_enabled(spec: FunctionPatchSpec) -> bool:
    """Whether ``spec`` is installed: not disabled, its feature group on, and -- for a
    patch on vLLM itself -- its op not configured to run on ``original``."""
    if spec.patch_id in _disabled_ops() or not _nt_feature_enabled(_FUNCTION_PATCH_FEATURES.get(spec.patch_id)):
        return False
    op = canonical_op_name(spec.patch_id)
    configured = load_backend_config().ops
    if op in _OPT_IN_PATCHES:
        return op in configured and backends.backend_enabled(op)
    if op == "UnifiedAttentionWithOutput":
        op = "PagedAttentionDecode"
    return not (spec.module_path.startswith("vllm") and op in configured and not backends.backend_enabled(op))


# ======================================================================================
# ledger: one OperatorStats per operator name
# ======================================================================================

# registration paths from weakest to strongest; an operator reports the strongest one
# that installed it
_VIA_ORDER = (None, "oot", "monkey_patch", "function_patch", "custom_op_rebind", "custom_op_intercept")
_REGISTERED_VIA_PRIORITY = {via: rank for rank, via in enumerate(_VIA_ORDER)}

_OPERATOR_NAMES = (
    "RMSNorm", "SiluAndMul", "GemmaRMSNorm", "MulAndSilu", "GeluAndMul", "GELU", "LayerNorm", "MatMul", "Embedding",
    "WPE", "NTWPEKernel", "LMHead", "PagedAttentionPrefill", "PagedAttentionDecode", "StoreKVCache",
    "GateUpSiluAndMul", "RoPE", "RoPEKVCache", "RMSNormQKV", "SDPA", "TopKTopP", "RandomSample", "RejectionSample",
)
_OPERATOR_STATS: dict[str, OperatorStats] = {}


def _stats(name: str) -> OperatorStats:
    entry = _OPERATOR_STATS.get(name)
    if entry is None:
        entry = _OPERATOR_STATS[name] = OperatorStats()
    return entry


def _record_hit(name: str, x: torch.Tensor) -> None:
    """A kernel served ``name``; the first hit of an op is logged with its shape."""
    if not backends.stats_enabled():
        return
    entry = _stats(name)
    entry.hits += 1
    backends.record_hit(name)
    if not entry.logged:
        entry.logged = True
        logger.info("vllm-nt: %s %s kernel invoked (shape=%s)", backends.active_backend(name), name, tuple(x.shape))


def _decline(name: str, reason: str, run_vllm: Callable[[], Any]) -> Any:
    """Runs vLLM's implementation of a call the kernels do not serve, recording it as a
    fallback to ``original`` with ``reason``."""
    if backends.stats_enabled():
        entry = _stats(name)
        entry.declined[reason] = entry.declined.get(reason, 0) + 1
        backends.record_fallback(name, "original")
    return run_vllm()


def _note_registration(name: str, via: str) -> None:
    entry = _stats(name)
    if _REGISTERED_VIA_PRIORITY.get(via, 0) >= _REGISTERED_VIA_PRIORITY.get(entry.registered_via, 0):
        entry.registered_via = via


def _route(op_name: str, call_original: Callable[[], Any], call_b200: Callable[[], Any]) -> Any:
    return backends.route(op_name, call_original, call_ninetoothed=call_b200, call_b200=call_b200)


# ======================================================================================
# patch marks and the replacement journal
# ======================================================================================

_PATCH_MARKS: "weakref.WeakKeyDictionary[Any, str]" = weakref.WeakKeyDictionary()


def _mark_function_patch(fn: object, patch_id: str) -> object:
    try:
        _PATCH_MARKS[fn] = patch_id
    except TypeError:  # not weak-referenceable: such a replacement is simply not marked
        pass
    return fn


def _is_function_patch(fn: object, patch_id: str) -> bool:
    try:
        return _PATCH_MARKS.get(fn) == patch_id
    except TypeError:
        return False


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


class _Journal:
    """Every attribute the plugin replaced, oldest first, with the value it replaced."""

    def __init__(self) -> None:
        self.entries: list[tuple[object, str, object]] = []

    def replace(self, owner: object, attr: str, value: object) -> object:
        before = getattr(owner, attr)
        setattr(owner, attr, value)
        self.entries.append((owner, attr, before))
        return before

    def mark(self) -> int:
        return len(self.entries)

    def undo_to(self, mark: int) -> None:
        while len(self.entries) > mark:
            owner, attr, before = self.entries.pop()
            setattr(owner, attr, before)


_JOURNAL = _Journal()


# ======================================================================================
# CustomOp forwards
# ======================================================================================


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
    return raw if callable(raw) else None


# name -> {"native": f(self, ...), "cuda": f(self, ...)}, captured before registration
_ORIGINAL_OPERATOR_FORWARDS: dict[str, dict[str, Callable[..., Any]]] = {}


def _call_original_operator(name: str, self, *args: Any) -> Any:
    impls = _ORIGINAL_OPERATOR_FORWARDS.get(name)
    if not impls:
        raise RuntimeError(f"original {name} forward is unavailable")
    first = args[0] if args else None
    if isinstance(first, torch.Tensor) and first.is_cuda and "cuda" in impls:
        return impls["cuda"](self, *args)
    return impls["native"](self, *args)


def _why_not_norm(x: torch.Tensor, weight: torch.Tensor | None, residual: torch.Tensor | None) -> str | None:
    if not x.is_cuda:
        return "not a CUDA tensor"
    if x.dtype not in _FLOAT_TYPES:
        return f"dtype {x.dtype}"
    if weight is not None and weight.dtype != x.dtype:
        return "weight dtype differs"
    if residual is not None and (residual.dtype != x.dtype or residual.shape != x.shape):
        return "residual dtype/shape differs"
    return None


def _nt_rms_norm_forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
    has_weight = getattr(self, "has_weight", True)
    weight = self.weight.data if has_weight and getattr(self, "weight", None) is not None else None
    if "RMSNorm" not in _ORIGINAL_OPERATOR_FORWARDS:
        _record_hit("RMSNorm", x)
        return norm(self, x, weight, residual)
    vllm_path = lambda: _call_original_operator("RMSNorm", self, x, residual)  # noqa: E731
    if getattr(self, "variance_size_override", None) is not None:
        return _decline("RMSNorm", "variance_size_override", vllm_path)
    reason = _why_not_norm(x, weight, residual)
    if reason:
        return _decline("RMSNorm", reason, vllm_path)

    def kernels():
        _record_hit("RMSNorm", x)
        return norm(self, x, weight, residual)

    return _route("RMSNorm", vllm_path, kernels)


def _nt_gemma_rms_norm_forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
    """GemmaRMSNorm on the Gemma variant of the norm kernel: the raw parameter w goes to
    the kernel, which forms (1 + w) in fp32 and rounds as GemmaRMSNorm.forward_native
    (vllm/model_executor/layers/layernorm.py:153-170)."""
    weight = self.weight.data
    if "GemmaRMSNorm" not in _ORIGINAL_OPERATOR_FORWARDS:
        _record_hit("GemmaRMSNorm", x)
        return norm(self, x, weight, residual, gemma=True)
    vllm_path = lambda: _call_original_operator("GemmaRMSNorm", self, x, residual)  # noqa: E731
    reason = _why_not_norm(x, weight, residual)
    if reason is None and residual is not None and x.dtype == torch.float16:
        reason = "fp16 with a residual (vLLM returns an fp32 residual)"
    if reason:
        return _decline("GemmaRMSNorm", reason, vllm_path)

    def kernels():
        _record_hit("GemmaRMSNorm", x)
        return norm(self, x, weight, residual, gemma=True)

    return _route("GemmaRMSNorm", vllm_path, kernels)


def _nt_silu_and_mul_forward(self, x: torch.Tensor) -> torch.Tensor:
    if "SiluAndMul" not in _ORIGINAL_OPERATOR_FORWARDS:
        _record_hit("SiluAndMul", x)
        return act_and_mul(x)
    vllm_path = lambda: _call_original_operator("SiluAndMul", self, x)  # noqa: E731
    if not x.is_cuda or x.dtype not in _FLOAT_TYPES:
        return _decline("SiluAndMul", "not a CUDA float tensor", vllm_path)

    def kernels():
        _record_hit("SiluAndMul", x)
        return act_and_mul(x)

    return _route("SiluAndMul", vllm_path, kernels)


def _nt_mul_and_silu_forward(self, x: torch.Tensor) -> torch.Tensor:
    """MulAndSilu has no kernel in this backend: vLLM's implementation runs."""
    return _decline("MulAndSilu", "no B200 kernel", lambda: _call_original_operator("MulAndSilu", self, x))


def _nt_gelu_and_mul_forward(self, x: torch.Tensor) -> torch.Tensor:
    """GeluAndMul has no kernel in this backend: vLLM's implementation runs."""
    return _decline("GeluAndMul", "no B200 kernel", lambda: _call_original_operator("GeluAndMul", self, x))


# ======================================================================================
# leaf methods: MatMul / Embedding / LMHead
# ======================================================================================


def _why_not_gemm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> str | None:
    if not x.is_cuda:
        return "not a CUDA tensor"
    if x.dtype not in _HALF_TYPES or weight.dtype != x.dtype:
        return f"dtype {x.dtype} / weight {weight.dtype}"
    if weight.dim() != 2 or weight.stride(-1) != 1:
        return "weight layout"
    if weight.shape[1] % 8:
        return "K not a multiple of 8"
    if bias is not None and bias.dtype != x.dtype:
        return "bias dtype differs"
    return None


def _with_residual(out: torch.Tensor, kwargs: dict[str, Any]) -> torch.Tensor:
    residual = kwargs.get("residual")
    return out if residual is None else out + residual


def _linear_hook(op: str, method_cls: type, self, layer: torch.nn.Module, x: torch.Tensor,
                 bias: torch.Tensor | None, kwargs: dict[str, Any], original: Callable[..., Any] | None) -> Any:
    """Shared body of the MatMul and LMHead hooks (both are x @ W^T (+ bias))."""

    def kernels():
        _record_hit(op, x)
        return _with_residual(linear(x, layer.weight, bias), kwargs)

    if original is None or not isinstance(self, method_cls):
        return kernels()
    vllm_path = lambda: original(self, layer, x, bias, **kwargs)  # noqa: E731
    reason = _why_not_gemm(x, layer.weight, bias)
    if reason:
        return _decline(op, reason, vllm_path)
    return _route(op, vllm_path, kernels)


def _nt_unquantized_linear_apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None,
                                 **kwargs):
    return _linear_hook("MatMul", UnquantizedLinearMethod, self, layer, x, bias, kwargs,
                        getattr(_nt_unquantized_linear_apply, "_original", None))


def _nt_unquantized_embedding_apply(self, layer: torch.nn.Module, x: torch.Tensor,
                                    bias: torch.Tensor | None = None, **kwargs):
    return _linear_hook("LMHead", UnquantizedEmbeddingMethod, self, layer, x, bias, kwargs,
                        getattr(_nt_unquantized_embedding_apply, "_original", None))


def _nt_unquantized_embedding(self, layer: torch.nn.Module, input_: torch.Tensor) -> torch.Tensor:
    original = getattr(_nt_unquantized_embedding, "_original", None)

    def kernels():
        _record_hit("Embedding", input_)
        return embedding(layer, input_)

    if original is None or not isinstance(self, UnquantizedEmbeddingMethod):
        return kernels()
    vllm_path = lambda: original(self, layer, input_)  # noqa: E731
    if not (input_.is_cuda and layer.weight.is_cuda and input_.dtype in (torch.int32, torch.int64)):
        return _decline("Embedding", "not CUDA int ids", vllm_path)
    return _route("Embedding", vllm_path, kernels)


def _nt_layer_norm(*args, **kwargs):
    raise NotImplementedError("LayerNorm (GPT-2) is outside the B200 backend; vLLM's path serves it")


# ======================================================================================
# function-patch builders
# ======================================================================================


def _already(original: object, patch_id: str) -> bool:
    return _is_function_patch(original, patch_id)


def _build_rotary_forward(original: object) -> object:
    """Replacement for RotaryEmbedding.forward_{cuda,oot,native}(positions, query, key)."""
    if _already(original, "RoPE"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor | None = None, *rest, **kw):
        vllm_path = lambda: original_fn(self, positions, query, key, *rest, **kw)  # noqa: E731
        if rest or kw:
            return _decline("RoPE", "extra arguments", vllm_path)
        if not self.is_neox_style:
            return _decline("RoPE", "not NeoX style", vllm_path)
        if self.rotary_dim % 2:
            return _decline("RoPE", "odd rotary_dim", vllm_path)
        if not query.is_cuda or query.dtype not in _FLOAT_TYPES:
            return _decline("RoPE", "not a CUDA float tensor", vllm_path)

        def kernels():
            cache = self._match_cos_sin_cache_dtype(query)
            if cache is None:  # older vLLM returned nothing and updated the attribute
                cache = self.cos_sin_cache
            result = rope(positions, query, key, cos_sin_cache=cache, head_size=self.head_size,
                          rotary_dim=self.rotary_dim, is_neox_style=self.is_neox_style)
            _record_hit("RoPE", query)
            return result

        return _route("RoPE", vllm_path, kernels)

    return _mark_function_patch(forward, "RoPE")


def _attn_impl_reason(impl: Any, dtype: torch.dtype, kv_cache: torch.Tensor, kv_dim: int = 0) -> str | None:
    """Why the attention kernels do not serve this impl and cache (None: they do).
    kv_dim is the cache dimension that separates K from V: 0 for FlashAttention's
    [2, blocks, 16, H, D], 1 for FlashInfer's [blocks, 2, 16, H, D] (whose memory order may
    be NHD or HND; the kernels take the strides).  An impl's configuration is fixed after
    construction, so the answer is kept on the impl, keyed by the dtypes and cache shape."""
    key = (dtype, kv_cache.dtype, kv_cache.shape, kv_dim)
    cached = getattr(impl, "_ntb200_reason", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    reason = _attn_impl_check(impl, dtype, kv_cache, kv_dim)
    try:
        impl._ntb200_reason = (key, reason)
    except AttributeError:
        pass
    return reason


def _attn_impl_supported(impl: Any, dtype: torch.dtype, kv_cache: torch.Tensor, kv_dim: int = 0) -> bool:
    return _attn_impl_reason(impl, dtype, kv_cache, kv_dim) is None


def _attn_impl_check(impl: Any, dtype: torch.dtype, kv_cache: torch.Tensor, kv_dim: int = 0) -> str | None:
    attn_type = getattr(impl, "attn_type", "decoder")
    sliding = getattr(impl, "sliding_window", None)
    checks = (
        (str(getattr(attn_type, "value", attn_type)).lower() == "decoder", "not decoder attention"),
        (getattr(impl, "kv_cache_dtype", "auto") == "auto", "quantised KV cache"),
        (getattr(impl, "alibi_slopes", None) is None, "ALiBi"),
        (not getattr(impl, "logits_soft_cap", None), "logits soft cap"),
        (getattr(impl, "sinks", None) is None, "attention sinks"),
        (sliding is None or tuple(sliding) == (-1, -1), "sliding window"),
        (getattr(impl, "dcp_world_size", 1) == 1, "decode context parallel"),
        (getattr(impl, "head_size", 0) == 128, "head size not 128"),
        (dtype in _HALF_TYPES, f"dtype {dtype}"),
        (getattr(impl, "kv_sharing_target_layer_name", None) is None, "shared KV layer"),
        (kv_cache.dim() == 5 and kv_cache.shape[kv_dim] == 2 and kv_cache.shape[2] == 16, "cache layout / block size"),
        (kv_cache.stride(-1) == 1 and kv_cache.dtype == dtype, "cache strides / dtype"),
    )
    return next((why for ok, why in checks if not ok), None)


def _kv_update_builder(patch_id: str, kv_dim: int) -> Callable[[object], object]:
    """Replacement builder for ``<Impl>.do_kv_cache_update(layer, key, value, kv_cache,
    slot_mapping)``: the slot-mapped store runs on the B200 kernel."""

    def build(original: object) -> object:
        if _already(original, patch_id):
            return original
        original_fn = cast(Callable[..., Any], original)

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            if getattr(layer, "_ntb200_kv_stored", False):
                # the fused RoPE + KV-store kernel of this layer's forward stored these rows
                layer._ntb200_kv_stored = False
                _record_hit("StoreKVCache", key)
                return None
            vllm_path = lambda: original_fn(self, layer, key, value, kv_cache, slot_mapping)  # noqa: E731
            reason = "not a CUDA tensor" if not key.is_cuda else _attn_impl_reason(self, key.dtype, kv_cache, kv_dim)
            if reason:
                return _decline("StoreKVCache", reason, vllm_path)

            def kernels():
                _record_hit("StoreKVCache", key)
                store_kv_cache_flash(key, value, kv_cache, slot_mapping, kv_dim)

            return _route("StoreKVCache", vllm_path, kernels)

        return _mark_function_patch(do_kv_cache_update, patch_id)

    return build


_build_flash_attn_kv_update = _kv_update_builder("StoreKVCache", 0)
_build_flashinfer_kv_update = _kv_update_builder("StoreKVCache", 1)


def _attention_common_reason(self, query, kv_cache, meta, rest, kw, output_scale, output_block_scale,
                             kv_dim: int) -> str | None:
    if meta is None:
        return "no attention metadata (profiling run)"
    if rest or kw:
        return "extra arguments"
    if output_scale is not None or output_block_scale is not None:
        return "quantised output"
    if getattr(meta, "use_cascade", False):
        return "cascade attention"
    if not query.is_cuda:
        return "not a CUDA tensor"
    return _attn_impl_reason(self, query.dtype, kv_cache, kv_dim)


def _build_flash_attn_forward(original: object) -> object:
    """Replacement for FlashAttentionImpl.forward: pure-decode batches (one query token
    per request) run on the split-K paged-decode kernel; prefill, chunked-prefill and mixed
    batches on the tcgen05 prefill kernel (its single-query requests on the decode kernel),
    reading K/V from the paged cache in place.  Cascade attention and non-causal metadata
    stay on vLLM's FlashAttention."""
    if _already(original, "PagedAttentionDecode"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None, *rest, **kw):
        vllm_path = lambda: original_fn(  # noqa: E731
            self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale,
            *rest, **kw)
        meta = attn_metadata
        max_q = int(getattr(meta, "max_query_len", 0)) if meta is not None else 0
        op = "PagedAttentionDecode" if max_q == 1 else "PagedAttentionPrefill"
        reason = _attention_common_reason(self, query, kv_cache, meta, rest, kw, output_scale, output_block_scale, 0)
        if reason is None and not getattr(meta, "causal", True):
            reason = "non-causal"
        if reason is None and max_q < 1:
            reason = "empty batch"
        if reason:
            return _decline(op, reason, vllm_path)
        n = int(meta.num_actual_tokens)
        qsl = getattr(meta, "query_start_loc", None)
        if max_q == 1 and (qsl is None or qsl.shape[0] - 1 == n):

            def decode():
                _record_hit("PagedAttentionDecode", query)
                paged_attention_decode_flash(output, query, kv_cache, meta.seq_lens, meta.block_table, n, self.scale,
                                             int(meta.max_seq_len))
                return output

            return _route("PagedAttentionDecode", vllm_path, decode)
        if qsl is None:
            return _decline("PagedAttentionPrefill", "no query_start_loc", vllm_path)

        def varlen():
            _record_hit("PagedAttentionPrefill", query)
            paged_attention_flash(output, query, kv_cache, qsl, meta.seq_lens, meta.block_table, n, max_q,
                                  int(meta.max_seq_len), self.scale)
            return output

        return _route("PagedAttentionPrefill", vllm_path, varlen)

    return _mark_function_patch(forward, "PagedAttentionDecode")


def _build_flashinfer_forward(original: object) -> object:
    """Replacement for FlashInferImpl.forward: a pure-decode batch (one query token per
    request) whose metadata carries the decode block table and lengths (vLLM's TRT-LLM
    decode metadata on Blackwell) runs on the split-K paged-decode kernel; prefill, mixed
    batches, cascade and FlashInfer's own planned decode stay on FlashInfer."""
    if _already(original, "PagedAttentionDecode"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None, *rest, **kw):
        vllm_path = lambda: original_fn(  # noqa: E731
            self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale,
            *rest, **kw)
        meta = attn_metadata
        reason = _attention_common_reason(self, query, kv_cache, meta, rest, kw, output_scale, output_block_scale, 1)
        if reason is None and getattr(meta, "num_prefills", 1) != 0:
            return _decline("PagedAttentionPrefill", "prefill on FlashInfer (not hooked)", vllm_path)
        dec = getattr(meta, "decode", None)
        if reason is None and (getattr(dec, "block_tables", None) is None or getattr(dec, "seq_lens", None) is None):
            reason = "FlashInfer planned decode (no TRT-LLM decode metadata)"
        n = int(getattr(meta, "num_actual_tokens", 0)) if meta is not None else 0
        if reason is None and (int(getattr(meta, "num_decodes", -1)) != n or
                               int(getattr(meta, "num_decode_tokens", -1)) != n):
            reason = "decode count mismatch"
        if reason:
            return _decline("PagedAttentionDecode", reason, vllm_path)

        def kernels():
            _record_hit("PagedAttentionDecode", query)
            paged_attention_decode_flash(output, query, kv_cache, dec.seq_lens, dec.block_tables, n, self.scale,
                                         int(dec.max_seq_len), 1)
            return output

        return _route("PagedAttentionDecode", vllm_path, kernels)

    return _mark_function_patch(forward, "PagedAttentionDecode")


def _why_not_fused_mlp(mlp: Any, x: torch.Tensor) -> str | None:
    """gate_up_proj -> SiluAndMul -> down_proj with an unquantised, bias-free merged
    gate_up weight whose output stays on this rank (no gather)."""
    gu = getattr(mlp, "gate_up_proj", None)
    w = getattr(gu, "weight", None)
    if not isinstance(getattr(mlp, "act_fn", None), activation.SiluAndMul) or not hasattr(mlp, "down_proj"):
        return "not gate_up -> SiluAndMul -> down"
    if not isinstance(getattr(gu, "quant_method", None), UnquantizedLinearMethod):
        return "quantised gate_up"
    if getattr(gu, "bias", None) is not None or getattr(gu, "gather_output", False):
        return "gate_up bias or gathered output"
    if not (isinstance(w, torch.Tensor) and w.dim() == 2 and w.shape[0] % 2 == 0 and w.shape[1] % 8 == 0
            and w.stride(-1) == 1):
        return "gate_up weight layout"
    if not (x.is_cuda and x.dtype in _HALF_TYPES and w.dtype == x.dtype and x.shape[-1] == w.shape[1]):
        return "activation dtype / device"
    return None


def _build_mlp_forward(original: object) -> object:
    """Replacement for LlamaMLP.forward (and MLPs of the same shape): gate_up_proj and
    SiluAndMul become one GEMM whose epilogue applies silu(gate) * up, so the [T, 2I]
    gate_up activation is never written; down_proj runs through its own hook."""
    if _already(original, "GateUpSiluAndMul"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, x):
        vllm_path = lambda: original_fn(self, x)  # noqa: E731
        reason = _why_not_fused_mlp(self, x)
        if reason:
            return _decline("GateUpSiluAndMul", reason, vllm_path)

        def kernels():
            _record_hit("GateUpSiluAndMul", x)
            out, _ = self.down_proj(gate_up_silu_and_mul(x, self.gate_up_proj.weight))
            return out

        return _route("GateUpSiluAndMul", vllm_path, kernels)

    return _mark_function_patch(forward, "GateUpSiluAndMul")


_KV_DIM_BY_IMPL = {"FlashAttentionImpl": 0, "FlashInferImpl": 1}


def _why_not_fused_rope_kv(attn_mod: Any, q: torch.Tensor) -> str | None:
    """The attention module's RoPE is the plain NeoX RotaryEmbedding whose forward the RoPE
    hook serves, and its attention layer stores K/V through one of the hooked impls."""
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding

    rot = getattr(attn_mod, "rotary_emb", None)
    layer = getattr(attn_mod, "attn", None)
    impl = getattr(layer, "impl", None)
    if not isinstance(rot, RotaryEmbedding) or type(rot).forward_cuda is not RotaryEmbedding.forward_cuda:
        return "not the base RotaryEmbedding"
    if not rot.is_neox_style or rot.rotary_dim % 2:
        return "not NeoX style / odd rotary_dim"
    if type(impl).__name__ not in _KV_DIM_BY_IMPL:
        return "attention impl without a hooked KV store"
    if getattr(layer, "kv_sharing_target_layer_name", None) is not None or getattr(
            getattr(layer, "attn_backend", None), "forward_includes_kv_cache_update", False):
        return "layer does not store its own K/V"
    if not q.is_cuda or q.dtype not in _HALF_TYPES:
        return "not a CUDA 16-bit tensor"
    if not backends.backend_enabled("StoreKVCache") or "StoreKVCache" in _disabled_ops():
        return "KV-store hook disabled"
    return None


def _opt_in_active(op: str) -> bool:
    """Whether the opt-in patch ``op`` is configured with a kernel backend (and not disabled)."""
    return op not in _disabled_ops() and op in load_backend_config().ops and backends.backend_enabled(op)


def _attention_after_qkv(self: Any, positions: torch.Tensor, qkv: torch.Tensor) -> torch.Tensor:
    """LlamaAttention.forward after its qkv projection: with the RoPEKVCache patch, the RoPE
    of q/k and the KV store as one kernel (the layer's own KV-store call then finds its rows
    stored); otherwise the module's RoPE and attention calls, as vLLM makes them."""
    q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
    reason = None if _opt_in_active("RoPEKVCache") else "RoPEKVCache not configured"
    if reason is None:
        reason = _why_not_fused_rope_kv(self, q)
    slot_mapping = kv_cache = None
    if reason is None:
        from vllm.model_executor.layers.attention.attention import get_attention_context

        try:
            _, _, kv_cache, slot_mapping = get_attention_context(self.attn.layer_name)
        except Exception:  # noqa: BLE001 - no forward context (e.g. a bare module call)
            reason = "no forward context"
        if reason is None and slot_mapping is None:
            reason = "no slot mapping (profiling run)"
        if reason is None:
            reason = _attn_impl_reason(self.attn.impl, q.dtype, kv_cache, _KV_DIM_BY_IMPL[type(self.attn.impl).__name__])
    if reason:
        if backends.stats_enabled():
            entry = _stats("RoPEKVCache")
            entry.declined[reason] = entry.declined.get(reason, 0) + 1
            backends.record_fallback("RoPEKVCache", "original")
        q, k = self.rotary_emb(positions, q, k)
        attn_output = self.attn(q, k, v)
    else:
        rot = self.rotary_emb
        cache = rot._match_cos_sin_cache_dtype(q)
        if cache is None:
            cache = rot.cos_sin_cache
        kv_dim = _KV_DIM_BY_IMPL[type(self.attn.impl).__name__]

        def kernels():
            _record_hit("RoPEKVCache", q)
            rope_and_store_kv_cache_flash(positions, q, k, v, cache, rot.head_size, rot.rotary_dim, kv_cache,
                                          slot_mapping, kv_dim)
            self.attn._ntb200_kv_stored = True
            return q, k

        q, k = _route("RoPEKVCache", lambda: self.rotary_emb(positions, q, k), kernels)
        attn_output = self.attn(q, k, v)
    output, _ = self.o_proj(attn_output)
    return output


def _build_attention_rope_kv_forward(original: object) -> object:
    """Replacement for LlamaAttention.forward (and attention modules of the same shape):
    the RoPE of q/k and the KV store of the rotated k and the v become one kernel
    (ntb200_rope_and_cache); the layer's own KV-store call then finds its rows stored and
    returns.  Prefill-sized calls take the two kernels inside the same entry point."""
    if _already(original, "RoPEKVCache"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, positions, hidden_states):
        qkv, _ = self.qkv_proj(hidden_states)
        return _attention_after_qkv(self, positions, qkv)

    return _mark_function_patch(forward, "RoPEKVCache")


# ntb200_rms_norm_linear takes up to 16 rows, but only batches of one or two tokens run
# faster than the separate norm and projection kernels (Llama-3-8B qkv with x and the
# residual just written, as in a decoder layer: 15.3 against 17.4 us at one token, 17.0
# against 17.5 at two, 18.4 against 17.8 at four), so larger batches decline.
_NORM_LINEAR_MAX_ROWS = 2


def _why_not_norm_qkv(layer: Any, hidden: torch.Tensor, residual: torch.Tensor | None) -> str | None:
    """input_layernorm is a plain RMSNorm and self_attn.qkv_proj an unquantised, bias-free
    projection whose output stays on this rank, for a decode batch of one or two tokens."""
    ln = getattr(layer, "input_layernorm", None)
    qkv = getattr(getattr(layer, "self_attn", None), "qkv_proj", None)
    if not isinstance(ln, layernorm.RMSNorm) or not getattr(ln, "has_weight", True) or \
            getattr(ln, "variance_size_override", None) is not None:
        return "input_layernorm is not a plain RMSNorm"
    if not isinstance(getattr(qkv, "quant_method", None), UnquantizedLinearMethod):
        return "quantised qkv_proj"
    if getattr(qkv, "bias", None) is not None or getattr(qkv, "gather_output", False):
        return "qkv_proj bias or gathered output"
    w, g = getattr(qkv, "weight", None), getattr(ln, "weight", None)
    if not (isinstance(w, torch.Tensor) and w.dim() == 2 and w.shape[1] % 8 == 0 and w.stride(-1) == 1):
        return "qkv_proj weight layout"
    if hidden.dim() != 2 or hidden.shape[-1] != w.shape[1]:
        return "hidden states are not [tokens, hidden]"
    if hidden.shape[0] > _NORM_LINEAR_MAX_ROWS:
        return f"batch above {_NORM_LINEAR_MAX_ROWS} token(s)"
    if not (hidden.is_cuda and hidden.dtype in _HALF_TYPES and w.dtype == hidden.dtype and
            isinstance(g, torch.Tensor) and g.dtype == hidden.dtype):
        return "activation / weight dtype or device"
    if residual is not None and (residual.shape != hidden.shape or residual.dtype != hidden.dtype):
        return "residual shape or dtype"
    return None


def _build_decoder_norm_qkv_forward(original: object) -> object:
    """Replacement for LlamaDecoderLayer.forward: for a decode batch of one or two tokens the
    input RMSNorm (with its residual add) and the qkv projection become one kernel
    (ntb200_rms_norm_linear), whose normalised rows never leave shared memory; the rest of
    the layer runs as vLLM's code does (attention through the hooks, with the RoPEKVCache
    fusion when that patch is configured)."""
    if _already(original, "RMSNormQKV"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def forward(self, positions, hidden_states, residual):
        vllm_path = lambda: original_fn(self, positions, hidden_states, residual)  # noqa: E731
        reason = _why_not_norm_qkv(self, hidden_states, residual)
        if reason:
            return _decline("RMSNormQKV", reason, vllm_path)

        def kernels():
            _record_hit("RMSNormQKV", hidden_states)
            attn = self.self_attn
            if residual is None:
                qkv = norm_linear(self.input_layernorm, hidden_states, None, attn.qkv_proj.weight)
                res = hidden_states
            else:
                qkv, res = norm_linear(self.input_layernorm, hidden_states, residual, attn.qkv_proj.weight)
            h = _attention_after_qkv(attn, positions, qkv)
            h, res = self.post_attention_layernorm(h, res)
            return self.mlp(h), res

        return _route("RMSNormQKV", vllm_path, kernels)

    return _mark_function_patch(forward, "RMSNormQKV")


def _why_not_sampler_rows(x: torch.Tensor) -> str | None:
    """The sampler kernels take fp32 rows on a CUDA device with unit vocabulary stride."""
    if not x.is_cuda:
        return "not a CUDA tensor"
    if x.dtype != torch.float32 or x.dim() != 2 or x.stride(-1) != 1:
        return "not fp32 [rows, vocab] with unit stride"
    return None


def _build_apply_top_k_top_p_patch(original: object) -> object:
    """Replacement for vLLM's topk_topp_sampler.apply_top_k_top_p(logits, k, p) (the
    reference's TopKTopP patch, vllm_nt/_ntops/patching.py:1446-1463): the mask is the
    radix-select kernel instead of a sort of every row.  vLLM's TopKTopPSampler reaches it
    on its native path (per-request generators, or FlashInfer sampling turned off)."""
    if _already(original, "TopKTopP"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def wrapped(logits: torch.Tensor, k: torch.Tensor | None, p: torch.Tensor | None):
        vllm_path = lambda: original_fn(logits, k, p)  # noqa: E731
        reason = "neither top-k nor top-p set" if k is None and p is None else _why_not_sampler_rows(logits)
        if reason:
            return _decline("TopKTopP", reason, vllm_path)

        def kernels():
            _record_hit("TopKTopP", logits)
            return nt_apply_top_k_top_p(logits, k, p)

        return _route("TopKTopP", vllm_path, kernels)

    return _mark_function_patch(wrapped, "TopKTopP")


def _build_random_sample_patch(original: object) -> object:
    """Replacement for vLLM's topk_topp_sampler.random_sample(probs, generators) (the
    reference's RandomSample patch, vllm_nt/_ntops/patching.py:1466-1479): the division by
    the exponential draws and the argmax are one kernel pass."""
    if _already(original, "RandomSample"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def wrapped(probs: torch.Tensor, generators: dict[int, torch.Generator]):
        vllm_path = lambda: original_fn(probs, generators)  # noqa: E731
        reason = _why_not_sampler_rows(probs)
        if reason:
            return _decline("RandomSample", reason, vllm_path)

        def kernels():
            _record_hit("RandomSample", probs)
            return nt_random_sample(probs, generators)

        return _route("RandomSample", vllm_path, kernels)

    return _mark_function_patch(wrapped, "RandomSample")


def _build_rejection_sample_patch(original: object) -> object:
    """Counts vLLM's rejection_sample calls under RejectionSample and runs vLLM's own code,
    as the reference's patch does (vllm_nt/_ntops/patching.py:1482-1497).  The hit is
    recorded against the target distribution: the ``target_logits`` (older vLLM:
    ``target_probs``) keyword, else the sixth positional argument."""
    if _already(original, "RejectionSample"):
        return original
    original_fn = cast(Callable[..., Any], original)

    def wrapped(*args: Any, **kwargs: Any):
        candidates = (kwargs.get("target_logits"), kwargs.get("target_probs"), args[5] if len(args) > 5 else None)
        target = next((c for c in candidates if isinstance(c, torch.Tensor)), None)
        if target is not None:
            _record_hit("RejectionSample", target)
        return original_fn(*args, **kwargs)

    return _mark_function_patch(wrapped, "RejectionSample")


# ======================================================================================
# what gets installed
# ======================================================================================

_OPERATOR_SPECS: dict[str, tuple[type, Callable[..., Any]]] = {
    "RMSNorm": (layernorm.RMSNorm, _nt_rms_norm_forward),
    "SiluAndMul": (activation.SiluAndMul, _nt_silu_and_mul_forward),
}
if getattr(layernorm, "GemmaRMSNorm", None) is not None:
    _OPERATOR_SPECS["GemmaRMSNorm"] = (layernorm.GemmaRMSNorm, _nt_gemma_rms_norm_forward)

for _name in _OPERATOR_NAMES:
    _stats(_name)


def _capture_original_forwards(names_and_classes: Iterable[tuple[str, type | None]]) -> None:
    for name, cls in names_and_classes:
        if cls is None:
            continue
        impls = {key: fn for key, fn in (("native", _unbound(cls, "forward_native")),
                                         ("cuda", _unbound(cls, "forward_cuda"))) if fn is not None}
        if impls:
            _ORIGINAL_OPERATOR_FORWARDS[name] = impls


_capture_original_forwards([(name, cls) for name, (cls, _) in _OPERATOR_SPECS.items()] +
                           [(name, getattr(activation, name, None)) for name in ("MulAndSilu", "GeluAndMul")])

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
    FunctionPatchSpec("StoreKVCache", _FA_MODULE, "do_kv_cache_update", "FlashAttentionImpl", False,
                      _build_flash_attn_kv_update),
    FunctionPatchSpec("PagedAttentionDecode", _FA_MODULE, "forward", "FlashAttentionImpl", False,
                      _build_flash_attn_forward),
    FunctionPatchSpec("StoreKVCache", _FI_MODULE, "do_kv_cache_update", "FlashInferImpl", False,
                      _build_flashinfer_kv_update),
    FunctionPatchSpec("PagedAttentionDecode", _FI_MODULE, "forward", "FlashInferImpl", False,
                      _build_flashinfer_forward),
    FunctionPatchSpec("TopKTopP", _SAMPLER_MODULE, "apply_top_k_top_p", None, False, _build_apply_top_k_top_p_patch),
    FunctionPatchSpec("RandomSample", _SAMPLER_MODULE, "random_sample", None, False, _build_random_sample_patch),
    FunctionPatchSpec("RejectionSample", "vllm.v1.sample.rejection_sampler", "rejection_sample", None, False,
                      _build_rejection_sample_patch),
    *(
        FunctionPatchSpec("GateUpSiluAndMul", mod, "forward", cls, False, _build_mlp_forward)
        for mod, cls in (("vllm.model_executor.models.llama", "LlamaMLP"),
                         ("vllm.model_executor.models.qwen2", "Qwen2MLP"))
    ),
    FunctionPatchSpec("RoPEKVCache", "vllm.model_executor.models.llama", "forward", "LlamaAttention", False,
                      _build_attention_rope_kv_forward),
    FunctionPatchSpec("RMSNormQKV", "vllm.model_executor.models.llama", "forward", "LlamaDecoderLayer", False,
                      _build_decoder_norm_qkv_forward),
)

_APPLIED_FUNCTION_PATCHES: list[_AppliedFunctionPatch] = []


# ======================================================================================
# installation
# ======================================================================================


def _register_custom_ops() -> None:
    """Step 1: an NT subclass per enabled CustomOp, through vLLM's out-of-tree registry; an
    op whose registration raises gets the forwards assigned on vLLM's class instead."""
    for name, (cls, forward) in _OPERATOR_SPECS.items():
        if not _operator_enabled(name):
            continue
        methods = dict.fromkeys(("forward_oot", "forward_cuda", "forward_native"), forward)
        try:
            cls.register_oot(name=name)(type(f"NT{name}", (cls,), methods))
            _note_registration(name, "oot")
        except Exception as exc:  # noqa: BLE001 - any registry failure takes the direct route
            logger.warning("vllm-nt: out-of-tree registration of %s failed (%s); assigning its forwards", name, exc)
            for attr, fn in methods.items():
                _JOURNAL.replace(cls, attr, fn)
            _note_registration(name, "monkey_patch")
    logger.info("vllm-nt: CustomOp hooks for %s", ", ".join(n for n in _OPERATOR_SPECS if _operator_enabled(n)))


# leaf method replacements: (operator, class attribute name on the vLLM method class, hook)
_LEAF_HOOKS = (
    ("MatMul", "UnquantizedLinearMethod", "apply", _nt_unquantized_linear_apply),
    ("Embedding", "UnquantizedEmbeddingMethod", "embedding", _nt_unquantized_embedding),
    ("LMHead", "UnquantizedEmbeddingMethod", "apply", _nt_unquantized_embedding_apply),
)


def _patch_leaf_methods() -> None:
    """Step 2: the unquantised linear and embedding methods (the hook keeps vLLM's method
    on its ``_original`` attribute)."""
    owners = {"UnquantizedLinearMethod": UnquantizedLinearMethod,
              "UnquantizedEmbeddingMethod": UnquantizedEmbeddingMethod}
    here = sys.modules[__name__]
    for op, owner_name, attr, hook in _LEAF_HOOKS:
        if not _operator_enabled(op):
            continue
        owner = getattr(here, owner_name, owners[owner_name])  # a test may swap the class
        hook._original = getattr(owner, attr)
        _JOURNAL.replace(owner, attr, hook)
        _note_registration(op, "monkey_patch")


def _resolve_function_patch_target(spec: FunctionPatchSpec) -> tuple[object, object]:
    module = importlib.import_module(spec.module_path)
    owner = getattr(module, spec.object_name) if spec.object_name else module
    return owner, getattr(owner, spec.attr_name)


def _apply_function_patches() -> None:
    """Step 3: the FunctionPatchSpec table.  An optional patch whose target is missing is
    skipped; a required one that fails undoes every patch of this step and re-raises."""
    global _APPLIED_FUNCTION_PATCHES
    start = _JOURNAL.mark()
    applied: list[_AppliedFunctionPatch] = []
    for spec in filter(_function_patch_enabled, _FUNCTION_PATCH_SPECS):
        try:
            owner, current = _resolve_function_patch_target(spec)
            _JOURNAL.replace(owner, spec.attr_name, spec.builder(current) if spec.builder else current)
        except Exception as exc:
            if spec.required:
                _JOURNAL.undo_to(start)
                raise
            logger.debug("vllm-nt: optional patch %s not applied: %s", spec.patch_id, exc)
            continue
        applied.append(_AppliedFunctionPatch(spec, owner, current))
        if spec.patch_id in _OPERATOR_STATS:
            _note_registration(spec.patch_id, "function_patch")
        if spec.patch_id == "PagedAttentionDecode" and spec.module_path == _FA_MODULE:
            # the FlashAttention forward patch serves prefill batches too
            _note_registration("PagedAttentionPrefill", "function_patch")
    _APPLIED_FUNCTION_PATCHES = applied


def _apply_custom_op_rebindings() -> None:
    """The reference can rebind vLLM's attention custom ops (VLLM_NT_ENABLE_CUSTOM_OP_REBIND)
    to reach its kernels on vendor platforms.  On CUDA the FlashAttention / FlashInfer impl
    methods those ops call are patched instead, so the flag has nothing left to do."""
    if os.environ.get("VLLM_NT_ENABLE_CUSTOM_OP_REBIND") == "1":
        logger.info("vllm-nt: attention is hooked through the impl methods; custom-op rebind not needed")


_registered = False


def ensure_registered() -> None:
    """Installs every hook the env flags and the backend config enable (idempotent)."""
    global _registered
    if _registered:
        return
    if not _nt_feature_enabled():
        logger.info("vllm-nt: registration skipped because VLLM_NT_ENABLE_ALL is disabled")
        _registered = True
        return
    load_backend_config()  # a bad config raises here, before anything is installed
    _registered = True
    for step in (_register_custom_ops, _patch_leaf_methods, _apply_function_patches, _apply_custom_op_rebindings):
        step()


# ======================================================================================
# usage summary
# ======================================================================================

_EMPTY_SUMMARY_KEYS = ("registered_ops", "hit_ops", "missed_ops", "operators", "disabled")
_COUNTERS = ("attempts", "hits", "failures", "fallbacks")
_summary_printed = False


def _operator_view(name: str, entry: OperatorStats) -> dict[str, Any]:
    per_backend = {backend: {c: getattr(s, c) for c in _COUNTERS}
                   for backend, s in sorted(backends.backend_stats(name).items())}
    totals = {c: sum(v[c] for v in per_backend.values()) for c in ("hits", "failures", "fallbacks")}
    view = {
        "configured_backend": backends.configured_backend(name),
        "active_backend": backends.active_backend(name),
        "hits": max(entry.hits, totals["hits"]),
        "failures": totals["failures"],
        "fallbacks": totals["fallbacks"],
        "registered_via": entry.registered_via,
        "backends": per_backend,
    }
    if entry.declined:
        view["declined"] = dict(entry.declined)
    return view


def get_usage_summary() -> dict[str, object]:
    """Per-operator counters (the reference's JSON shape); an operator whose calls did not
    all reach a kernel also carries ``declined``: {reason: calls}."""
    if not backends.stats_enabled():
        return {key: ({} if key == "operators" else []) for key in _EMPTY_SUMMARY_KEYS}
    operators = {name: _operator_view(name, entry) for name, entry in _OPERATOR_STATS.items()}
    hit_ops = [name for name, view in operators.items() if view["hits"] > 0]
    return {
        "registered_ops": list(operators),
        "hit_ops": hit_ops,
        "missed_ops": [name for name in operators if name not in hit_ops],
        "operators": operators,
        "disabled": sorted(backends.disabled_ops()),
    }


def format_usage_summary(use_color: bool = True) -> str:
    on, off = ("\033[94m", "\033[0m") if use_color else ("", "")
    summary = get_usage_summary()
    rows = ["Operator usage summary"]
    for name, v in cast(dict[str, dict[str, Any]], summary["operators"]).items():
        row = (f"- {name}: backend={v['active_backend']} hits={v['hits']} failures={v['failures']} "
               f"fallbacks={v['fallbacks']} ({v['registered_via'] or 'unregistered'})")
        if v.get("declined"):
            row += " declined: " + ", ".join(f"{why}={n}" for why, n in v["declined"].items())
        rows.append(row)
    rows.append(f"Missed operators: {', '.join(cast(list[str], summary['missed_ops'])) or 'None'}")
    return "\n".join(f"{on}{row}{off}" for row in rows)


def maybe_print_usage_summary(*, include_empty: bool = False) -> bool:
    """Prints the summary to stderr once per process (only when something was hit, unless
    ``include_empty``); returns whether it printed."""
    global _summary_printed
    if _summary_printed or not backends.stats_enabled():
        return False
    if not include_empty and not get_usage_summary()["hit_ops"]:
        return False
    print(format_usage_summary(), file=sys.stderr)
    _summary_printed = True
    return True


def _reset_usage_state() -> None:
    global _summary_printed
    for entry in _OPERATOR_STATS.values():
        entry.hits = 0
        entry.logged = False
        entry.declined.clear()
    backends.reset_backend_state()
    reset_backend_config_cache()
    _summary_printed = False


@atexit.register
def _print_worker_summary_on_exit() -> None:
    """vLLM worker processes print their own summary when they exit (the parent prints
    through maybe_print_usage_summary)."""
    if str(os.getpid()) != os.environ.get(_PARENT_PID_ENV, str(os.getpid())):
        maybe_print_usage_summary(include_empty=True)

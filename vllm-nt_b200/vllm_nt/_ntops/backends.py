"""Backend router and per-(op, backend) counters.

``route`` runs an op on its configured backend; if that raises, it records the failure,
optionally disables the op's backend for the rest of the process, and runs the fallback
backend instead (re-raising when the fallback is the backend that just failed).  This is
the contract of vllm_nt/_ntops/backends.py:96-161, kept so that configs, env flags and
usage summaries behave the same.  The ``b200`` backend (alias ``ninetoothed``) is the
hand-written sm_100a kernel set; ``infinicore*`` adapters are not part of this build, so
selecting them fails over to the configured fallback exactly as the reference does on a
machine without InfiniCore.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Any, Callable

from vllm_nt._ntops.config import config_for, op_name_variants

LOG = logging.getLogger("vllm_nt")
DISABLE_OPS_ENV = "VLLM_NT_DISABLE_OPS"
ENABLE_STATS_ENV = "VLLM_NT_ENABLE_STATS"
_TRUE = frozenset({"1", "true", "yes", "on"})

Thunk = Callable[[], Any]


@dataclass
class BackendStats:
    attempts: int = 0
    hits: int = 0
    failures: int = 0
    fallbacks: int = 0


_DISABLED: set[str] = set()
_STATS: dict[str, dict[str, BackendStats]] = {}

# The hooks sit on every decoder op, so the env flags are parsed once per distinct raw
# value (and per change of the runtime-disabled set), not once per call.  The raw value
# is read from os.environ's underlying bytes mapping (a dict lookup; os.environ.get
# re-encodes the key and decodes the value on every call), which setenv/putenv keep current.
_ENV_BYTES = getattr(os.environ, "_data", None)
_disabled_version = 0
_disabled_cache: tuple[object, int, frozenset[str]] = (object(), -1, frozenset())
_stats_cache: tuple[object, bool] = (object(), False)


def _raw_env(name: str, name_b: bytes) -> object:
    if isinstance(_ENV_BYTES, dict):
        return _ENV_BYTES.get(name_b)
    return os.environ.get(name)


def _decode(raw: object) -> str:
    if raw is None:
        return ""
    return raw.decode(errors="replace") if isinstance(raw, bytes) else str(raw)


def stats_enabled() -> bool:
    global _stats_cache
    raw = _raw_env(ENABLE_STATS_ENV, b"VLLM_NT_ENABLE_STATS")
    if raw != _stats_cache[0]:
        _stats_cache = (raw, _decode(raw).strip().lower() in _TRUE)
    return _stats_cache[1]


def disabled_ops() -> set[str]:
    global _disabled_cache
    raw_key = _raw_env(DISABLE_OPS_ENV, b"VLLM_NT_DISABLE_OPS")
    if raw_key != _disabled_cache[0] or _disabled_version != _disabled_cache[1]:
        raw = _decode(raw_key)
        listed = {n.strip() for n in raw.split(",") if n.strip()}
        out: set[str] = set()
        for name in listed | _DISABLED:
            out |= op_name_variants(name)
        _disabled_cache = (raw_key, _disabled_version, frozenset(out))
    return _disabled_cache[2]  # type: ignore[return-value]


def _disable(op_name: str) -> None:
    global _disabled_version
    _DISABLED.add(op_name)
    _disabled_version += 1


def configured_backend(op_name: str) -> str:
    return config_for(op_name).backend


def fallback_backend(op_name: str) -> str:
    return config_for(op_name).fallback_backend


def active_backend(op_name: str) -> str:
    cfg = config_for(op_name)
    return cfg.fallback_backend if op_name in disabled_ops() else cfg.backend


def backend_enabled(op_name: str) -> bool:
    return active_backend(op_name) != "original"


def _entry(op_name: str, backend: str) -> BackendStats:
    per_op = _STATS.get(op_name)
    if per_op is None:
        per_op = _STATS[op_name] = {}
    entry = per_op.get(backend)
    if entry is None:
        entry = per_op[backend] = BackendStats()
    return entry


def record_attempt(op_name: str, backend: str) -> None:
    if stats_enabled():
        _entry(op_name, backend).attempts += 1


def record_hit(op_name: str, backend: str | None = None) -> None:
    if stats_enabled():
        _entry(op_name, backend or active_backend(op_name)).hits += 1


def record_failure(op_name: str, backend: str | None = None) -> None:
    if stats_enabled():
        _entry(op_name, backend or active_backend(op_name)).failures += 1


def record_fallback(op_name: str, backend: str | None = None) -> None:
    if stats_enabled():
        _entry(op_name, backend or fallback_backend(op_name)).fallbacks += 1


def backend_stats(op_name: str) -> dict[str, BackendStats]:
    return _STATS.get(op_name, {})


def reset_backend_state() -> None:
    global _disabled_version
    _DISABLED.clear()
    _STATS.clear()
    _disabled_version += 1


def _dispatch(op_name: str, backend: str, fn: Thunk | None, original: Thunk) -> Any:
    if backend == "original":
        record_fallback(op_name, backend)
        return original()
    if fn is None:
        raise RuntimeError(f"{op_name} has no adapter for backend {backend}")
    record_attempt(op_name, backend)
    result = fn()
    if backend.startswith("infinicore"):
        record_hit(op_name, backend)
    return result


def _adapter(backend: str, original: Thunk, infinicore: Thunk | None, ninetoothed: Thunk | None,
             infinicore_flash_attn: Thunk | None, kernels: Thunk | None) -> Thunk | None:
    if backend == "b200":
        return kernels
    if backend == "ninetoothed":
        return ninetoothed if ninetoothed is not None else kernels
    if backend == "infinicore":
        return infinicore
    if backend == "infinicore-flash-attn":
        return infinicore_flash_attn
    return original if backend == "original" else None


def route(
    op_name: str,
    call_original: Thunk,
    *,
    call_infinicore: Thunk | None = None,
    call_ninetoothed: Thunk | None = None,
    call_infinicore_flash_attn: Thunk | None = None,
    call_b200: Thunk | None = None,
) -> Any:
    """Runs ``op_name`` on its active backend with failure fallback (see module doc).

    ``call_b200`` defaults to ``call_ninetoothed``: in this build both names select the
    sm_100a kernels."""
    kernels = call_b200 if call_b200 is not None else call_ninetoothed
    cfg = config_for(op_name)
    backend = cfg.fallback_backend if op_name in disabled_ops() else cfg.backend
    try:
        fn = _adapter(backend, call_original, call_infinicore, call_ninetoothed, call_infinicore_flash_attn, kernels)
        return _dispatch(op_name, backend, fn, call_original)
    except Exception as exc:
        record_failure(op_name, backend)
        if cfg.disable_backend_on_first_failure and backend != "original":
            _disable(op_name)
            LOG.warning(
                "vllm-nt: %s backend %s disabled after failure; falling back to %s: %s",
                op_name,
                backend,
                cfg.fallback_backend,
                exc,
            )
        if cfg.fallback_backend == backend:
            raise
        fb = cfg.fallback_backend
        fn = _adapter(fb, call_original, call_infinicore, call_ninetoothed, call_infinicore_flash_attn, kernels)
        return _dispatch(op_name, fb, fn, call_original)

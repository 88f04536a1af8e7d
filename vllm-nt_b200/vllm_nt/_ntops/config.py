"""Per-op backend selection read from a YAML file.

Schema (kept identical to vllm_nt's, vllm_nt/_ntops/config.py:8-206, so existing config
files keep working)::

    version: 1
    defaults:
      backend: original                 # backend used by ops not listed below
      fallback_backend: original        # backend used after a failure
      disable_backend_on_first_failure: true
    ops:
      RMSNorm: b200                     # short form
      MatMul:                           # long form
        backend: b200
        fallback_backend: original

The file comes from ``VLLM_NT_BACKEND_CONFIG`` (or the legacy
``VLLM_INFINI_PATCH_CONFIG``); without either, ``configs/hybrid-default.yaml`` next to this
package is used.  ``metax`` is accepted as a spelling of ``original``.  ``RoPE`` is an
alias of ``ApplyRotaryEmb``.  Besides the reference's backend names this build adds
``b200``: the hand-written sm_100a kernels.  ``ninetoothed`` selects the same kernels, so
a config written for the reference runs unchanged.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

CONFIG_ENV = "VLLM_NT_BACKEND_CONFIG"
LEGACY_CONFIG_ENV = "VLLM_INFINI_PATCH_CONFIG"
DEFAULT_CONFIG_PATH = Path(__file__).resolve().parent.parent / "configs" / "hybrid-default.yaml"

_BACKEND_NAMES = frozenset(
    {"original", "metax", "b200", "ninetoothed", "infinicore", "infinicore-flash-attn"}
)
_ALIASES = {"RoPE": "ApplyRotaryEmb"}


@dataclass(frozen=True)
class OpConfig:
    backend: str
    fallback_backend: str
    disable_backend_on_first_failure: bool


@dataclass(frozen=True)
class BackendConfig:
    version: int
    default_backend: str
    default_fallback_backend: str
    default_disable_backend_on_first_failure: bool
    ops: dict[str, OpConfig] = field(default_factory=dict)
    path: str | None = None

    def default_op(self) -> OpConfig:
        return OpConfig(
            self.default_backend,
            self.default_fallback_backend,
            self.default_disable_backend_on_first_failure,
        )


_cached: BackendConfig | None = None


def _backend(value: object, where: str) -> str:
    if not isinstance(value, str):
        raise RuntimeError(f"{where} must be a string backend name")
    name = value.strip().lower()
    if name not in _BACKEND_NAMES:
        raise RuntimeError(
            f"{where} has unsupported backend {name!r}; expected one of {sorted(_BACKEND_NAMES)}"
        )
    return "original" if name == "metax" else name


def _scalar(text: str) -> object:
    low = text.lower()
    if low in ("true", "false"):
        return low == "true"
    try:
        return int(text)
    except ValueError:
        return text.strip("'\"")


def _parse_mapping_yaml(text: str) -> dict[str, Any]:
    """Indentation-based reader for the nested-mapping subset the schema needs; used only
    when PyYAML is not importable."""
    root: dict[str, Any] = {}
    parents: list[tuple[int, dict[str, Any]]] = [(-1, root)]
    for line in text.splitlines():
        body = line.strip()
        if not body or body.startswith("#"):
            continue
        if ":" not in body:
            raise RuntimeError("simple backend YAML parser only supports mappings")
        indent = len(line) - len(line.lstrip(" "))
        key, _, rest = body.partition(":")
        key, rest = key.strip(), rest.strip()
        while parents[-1][0] >= indent:
            parents.pop()
        target = parents[-1][1]
        if rest:
            target[key] = _scalar(rest)
        else:
            target[key] = {}
            parents.append((indent, target[key]))
    return root


def _read(path: Path) -> dict[str, Any]:
    text = path.read_text(encoding="utf-8")
    try:
        import yaml
    except ModuleNotFoundError:
        data: Any = _parse_mapping_yaml(text)
    else:
        data = yaml.safe_load(text) or {}
    if not isinstance(data, dict):
        raise RuntimeError(f"backend config {path} must contain a YAML mapping")
    return data


def _locate() -> tuple[Path, str | None]:
    for env in (CONFIG_ENV, LEGACY_CONFIG_ENV):
        value = os.environ.get(env)
        if value:
            return Path(value), env
    return DEFAULT_CONFIG_PATH, None


def load_backend_config() -> BackendConfig:
    """Parses (once) and returns the active backend configuration."""
    global _cached
    if _cached is not None:
        return _cached
    path, env = _locate()
    if env is not None and not path.exists():
        raise RuntimeError(f"backend config file not found: {path} (set via {env})")
    raw = _read(path) if path.exists() else {}

    version = int(raw.get("version", 1))
    if version != 1:
        raise RuntimeError(f"unsupported backend config version {version}; expected 1")
    defaults = raw.get("defaults") or {}
    if not isinstance(defaults, dict):
        raise RuntimeError("backend config defaults must be a mapping")
    d_backend = _backend(defaults.get("backend", "original"), "defaults.backend")
    d_fallback = _backend(defaults.get("fallback_backend", "original"), "defaults.fallback_backend")
    d_disable = bool(defaults.get("disable_backend_on_first_failure", True))

    entries = raw.get("ops") or {}
    if not isinstance(entries, dict):
        raise RuntimeError("backend config ops must be a mapping")
    ops: dict[str, OpConfig] = {}
    for name, entry in entries.items():
        if not isinstance(name, str):
            raise RuntimeError("backend config op names must be strings")
        if entry is None:
            entry = {}
        elif isinstance(entry, str):
            entry = {"backend": entry}
        elif not isinstance(entry, dict):
            raise RuntimeError(f"backend config for {name} must be a mapping or backend string")
        ops[name] = OpConfig(
            backend=_backend(entry.get("backend", d_backend), f"ops.{name}.backend"),
            fallback_backend=_backend(
                entry.get("fallback_backend", d_fallback), f"ops.{name}.fallback_backend"
            ),
            disable_backend_on_first_failure=bool(
                entry.get("disable_backend_on_first_failure", d_disable)
            ),
        )
    _cached = BackendConfig(
        version=version,
        default_backend=d_backend,
        default_fallback_backend=d_fallback,
        default_disable_backend_on_first_failure=d_disable,
        ops=ops,
        path=str(path) if path.exists() else None,
    )
    return _cached


def canonical_op_name(op_name: str) -> str:
    return _ALIASES.get(op_name, op_name)


def op_name_variants(op_name: str) -> set[str]:
    """The canonical name plus every alias that points at it."""
    canon = canonical_op_name(op_name)
    return {canon} | {alias for alias, target in _ALIASES.items() if target == canon}


def config_for(op_name: str) -> OpConfig:
    cfg = load_backend_config()
    return cfg.ops.get(canonical_op_name(op_name)) or cfg.default_op()


def reset_backend_config_cache() -> None:
    global _cached
    _cached = None

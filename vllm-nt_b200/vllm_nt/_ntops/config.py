"""Per-op backend selection read from a YAML file.

The file format is the one vllm_nt's configs use (vllm_nt/_ntops/config.py:8-206), so
existing config files keep working::

    version: 1
    defaults:
      backend: original                 # backend used by ops not listed below
      fallback_backend: original        # backend used after a failure
      disable_backend_on_first_failure: true
    ops:
      RMSNorm: b200                     # short form: the backend alone
      MatMul:                           # long form: any of the three settings
        backend: b200
        fallback_backend: original

The file is named by ``VLLM_NT_BACKEND_CONFIG`` (or the legacy ``VLLM_INFINI_PATCH_CONFIG``);
with neither set, ``configs/hybrid-default.yaml`` beside this package is read.  ``metax`` is
accepted as a spelling of ``original``, and ``RoPE`` names the same op as
``ApplyRotaryEmb``.  Besides the reference's backend names this build accepts ``b200``,
the hand-written sm_100a kernels; ``ninetoothed`` selects the same kernels, so a config
written for the reference runs unchanged.

How it is built: every op setting is an ``OpConfig``; the ``defaults`` mapping is resolved
over the built-in default (``original`` / ``original`` / disable on first failure), and each
``ops`` entry over the resolved defaults, by one field table (``_FIELDS``).  The parsed
file is memoised until ``reset_backend_config_cache``.
"""

from __future__ import annotations

import dataclasses
import functools
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable

CONFIG_ENV = "VLLM_NT_BACKEND_CONFIG"
LEGACY_CONFIG_ENV = "VLLM_INFINI_PATCH_CONFIG"
DEFAULT_CONFIG_PATH = Path(__file__).resolve().parent.parent / "configs" / "hybrid-default.yaml"

# accepted spellings -> the backend they select
_BACKEND_SPELLINGS = {
    "original": "original",
    "metax": "original",
    "b200": "b200",
    "ninetoothed": "ninetoothed",
    "infinicore": "infinicore",
    "infinicore-flash-attn": "infinicore-flash-attn",
}
_ALIASES = {"RoPE": "ApplyRotaryEmb"}


@dataclass(frozen=True)
class OpConfig:
    backend: str
    fallback_backend: str
    disable_backend_on_first_failure: bool


_BUILTIN = OpConfig("original", "original", True)


@dataclass(frozen=True)
class BackendConfig:
    version: int
    default_backend: str
    default_fallback_backend: str
    default_disable_backend_on_first_failure: bool
    ops: dict[str, OpConfig] = field(default_factory=dict)
    path: str | None = None

    def default_op(self) -> OpConfig:
        return OpConfig(self.default_backend, self.default_fallback_backend,
                        self.default_disable_backend_on_first_failure)


# ------------------------------------------------------------------------- field table


def _as_backend(value: object, where: str) -> str:
    if not isinstance(value, str):
        raise RuntimeError(f"{where} must be a string backend name")
    spelled = value.strip().lower()
    if spelled not in _BACKEND_SPELLINGS:
        raise RuntimeError(
            f"{where} has unsupported backend {spelled!r}; expected one of {sorted(_BACKEND_SPELLINGS)}"
        )
    return _BACKEND_SPELLINGS[spelled]


def _as_flag(value: object, where: str) -> bool:  # noqa: ARG001 - same shape as _as_backend
    return bool(value)


_FIELDS: tuple[tuple[str, Callable[[object, str], Any]], ...] = (
    ("backend", _as_backend),
    ("fallback_backend", _as_backend),
    ("disable_backend_on_first_failure", _as_flag),
)


def _overlay(base: OpConfig, settings: dict[str, Any], prefix: str) -> OpConfig:
    """``base`` with every field that ``settings`` names replaced by its checked value."""
    changes = {name: check(settings[name], f"{prefix}.{name}") for name, check in _FIELDS if name in settings}
    return dataclasses.replace(base, **changes)


# ------------------------------------------------------------------------- YAML reading


def _coerce(token: str) -> object:
    if token.lower() in ("true", "false"):
        return token.lower() == "true"
    if token.lstrip("+-").isdigit():
        return int(token)
    return token.strip("'\"")


def _indented(text: str) -> list[tuple[int, str]]:
    """(indent, content) of every meaningful line."""
    rows = []
    for line in text.splitlines():
        content = line.strip()
        if content and not content.startswith("#"):
            rows.append((len(line) - len(line.lstrip(" ")), content))
    return rows


def _block(rows: list[tuple[int, str]]) -> dict[str, Any]:
    """A mapping from a run of lines that share the first line's indent; a ``key:`` line
    with nothing after the colon owns the deeper-indented lines that follow it."""
    out: dict[str, Any] = {}
    i = 0
    while i < len(rows):
        indent, content = rows[i]
        key, colon, value = content.partition(":")
        if not colon:
            raise RuntimeError("simple backend YAML parser only supports mappings")
        j = i + 1
        while j < len(rows) and rows[j][0] > indent:
            j += 1
        value = value.strip()
        out[key.strip()] = _coerce(value) if value else _block(rows[i + 1 : j])
        i = j
    return out


def _parse_mapping_yaml(text: str) -> dict[str, Any]:
    """Reader for the nested-mapping subset of YAML the format uses; used only when PyYAML
    cannot be imported."""
    return _block(_indented(text))


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
    """The config file and the variable that named it (None for the packaged default)."""
    named = [env for env in (CONFIG_ENV, LEGACY_CONFIG_ENV) if os.environ.get(env)]
    if not named:
        return DEFAULT_CONFIG_PATH, None
    return Path(os.environ[named[0]]), named[0]


def _mapping(raw: dict[str, Any], key: str) -> dict[str, Any]:
    value = raw.get(key) or {}
    if not isinstance(value, dict):
        raise RuntimeError(f"backend config {key} must be a mapping")
    return value


def _op_entry(name: object, entry: object) -> dict[str, Any]:
    if not isinstance(name, str):
        raise RuntimeError("backend config op names must be strings")
    if entry is None:
        return {}
    if isinstance(entry, str):
        return {"backend": entry}
    if isinstance(entry, dict):
        return entry
    raise RuntimeError(f"backend config for {name} must be a mapping or backend string")


@functools.lru_cache(maxsize=1)
def _load() -> BackendConfig:
    path, env = _locate()
    exists = path.exists()
    if env is not None and not exists:
        raise RuntimeError(f"backend config file not found: {path} (set via {env})")
    raw = _read(path) if exists else {}
    version = int(raw.get("version", 1))
    if version != 1:
        raise RuntimeError(f"unsupported backend config version {version}; expected 1")
    defaults = _overlay(_BUILTIN, _mapping(raw, "defaults"), "defaults")
    ops = {name: _overlay(defaults, _op_entry(name, entry), f"ops.{name}")
           for name, entry in _mapping(raw, "ops").items()}
    return BackendConfig(
        version=version,
        default_backend=defaults.backend,
        default_fallback_backend=defaults.fallback_backend,
        default_disable_backend_on_first_failure=defaults.disable_backend_on_first_failure,
        ops=ops,
        path=str(path) if exists else None,
    )


def load_backend_config() -> BackendConfig:
    """The active backend configuration (parsed on first use)."""
    return _load()


def reset_backend_config_cache() -> None:
    _load.cache_clear()


def canonical_op_name(op_name: str) -> str:
    return _ALIASES.get(op_name, op_name)


def op_name_variants(op_name: str) -> set[str]:
    """The canonical name plus every alias that points at it."""
    canon = canonical_op_name(op_name)
    return {canon, *(alias for alias, target in _ALIASES.items() if target == canon)}


def config_for(op_name: str) -> OpConfig:
    cfg = load_backend_config()
    return cfg.ops.get(canonical_op_name(op_name)) or cfg.default_op()

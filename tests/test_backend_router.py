"""Config schema and router semantics (the reference's contract: vllm_nt/tests/
test_backend_router.py).  CPU only."""

from pathlib import Path

import pytest

import vllm_nt._ntops.backends as backends
import vllm_nt._ntops.config as config

CONFIGS = Path(__file__).resolve().parents[1] / "vllm-nt_b200" / "vllm_nt" / "configs"


@pytest.fixture(autouse=True)
def _reset(monkeypatch):
    monkeypatch.delenv("VLLM_NT_BACKEND_CONFIG", raising=False)
    monkeypatch.delenv("VLLM_INFINI_PATCH_CONFIG", raising=False)
    monkeypatch.delenv("VLLM_NT_DISABLE_OPS", raising=False)
    config.reset_backend_config_cache()
    backends.reset_backend_state()
    yield
    config.reset_backend_config_cache()
    backends.reset_backend_state()


def _use(monkeypatch, tmp_path, text):
    path = tmp_path / "backend.yaml"
    path.write_text(text, encoding="utf-8")
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(path))
    config.reset_backend_config_cache()


def test_default_config_is_hybrid_default():
    cfg = config.load_backend_config()
    assert cfg.path.endswith("vllm_nt/configs/hybrid-default.yaml")
    expect = {
        "RMSNorm": "infinicore",
        "GemmaRMSNorm": "infinicore",
        "SiluAndMul": "ninetoothed",
        "ApplyRotaryEmb": "ninetoothed",
        "RoPE": "ninetoothed",
        "Embedding": "ninetoothed",
        "MatMul": "original",
        "LMHead": "original",
        "StoreKVCache": "original",
        "PagedAttentionPrefill": "original",
        "PagedAttentionDecode": "original",
        "SDPA": "original",
    }
    for op, backend in expect.items():
        assert config.config_for(op).backend == backend, op


def test_all_b200_config_routes_every_hot_op_to_b200(monkeypatch):
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(CONFIGS / "all-b200.yaml"))
    config.reset_backend_config_cache()
    for op in ("RMSNorm", "SiluAndMul", "RoPE", "Embedding", "MatMul", "LMHead", "StoreKVCache", "PagedAttentionDecode",
               "PagedAttentionPrefill"):
        assert config.config_for(op).backend == "b200", op
        assert config.config_for(op).fallback_backend == "original"
    assert config.config_for("SDPA").backend == "original"


def test_defaults_and_string_form(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\ndefaults:\n  backend: original\n  fallback_backend: metax\nops:\n  RMSNorm: b200\n")
    cfg = config.load_backend_config()
    assert cfg.default_fallback_backend == "original"  # metax spells original
    assert config.config_for("RMSNorm").backend == "b200"
    assert config.config_for("UnknownOp").backend == "original"


def test_unknown_backend_rejected(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  RMSNorm: cuda\n")
    with pytest.raises(RuntimeError, match="unsupported backend"):
        config.load_backend_config()


def test_bad_version_rejected(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 2\n")
    with pytest.raises(RuntimeError, match="unsupported backend config version"):
        config.load_backend_config()


def test_missing_explicit_config_raises(monkeypatch, tmp_path):
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(tmp_path / "nope.yaml"))
    with pytest.raises(RuntimeError, match="backend config file not found"):
        config.load_backend_config()


def test_legacy_env_name(monkeypatch, tmp_path):
    path = tmp_path / "legacy.yaml"
    path.write_text("version: 1\nops:\n  MatMul: ninetoothed\n", encoding="utf-8")
    monkeypatch.setenv("VLLM_INFINI_PATCH_CONFIG", str(path))
    assert config.config_for("MatMul").backend == "ninetoothed"


def test_simple_yaml_parser_matches_pyyaml():
    text = (CONFIGS / "hybrid-default.yaml").read_text()
    import yaml

    assert config._parse_mapping_yaml(text) == yaml.safe_load(text)


def test_failure_falls_back_and_disables(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  MatMul:\n    backend: b200\n    fallback_backend: original\n")
    calls = []

    def boom():
        calls.append("b200")
        raise RuntimeError("kernel failed")

    assert backends.route("MatMul", lambda: "orig", call_b200=boom) == "orig"
    assert backends.active_backend("MatMul") == "original"
    s = backends.backend_stats("MatMul")
    assert s["b200"].attempts == 1 and s["b200"].failures == 1 and s["original"].fallbacks == 1
    # disabled: the kernel is not attempted again
    assert backends.route("MatMul", lambda: "orig", call_b200=boom) == "orig"
    assert calls == ["b200"]


def test_failure_reraises_when_fallback_is_same_backend(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  MatMul:\n    backend: b200\n    fallback_backend: b200\n")
    with pytest.raises(RuntimeError, match="boom"):
        backends.route("MatMul", lambda: "orig", call_b200=lambda: (_ for _ in ()).throw(RuntimeError("boom")))


def test_ninetoothed_name_selects_the_b200_kernels(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  SiluAndMul: ninetoothed\n")
    assert backends.route("SiluAndMul", lambda: "orig", call_b200=lambda: "kern") == "kern"
    assert backends.backend_stats("SiluAndMul")["ninetoothed"].attempts == 1


def test_infinicore_absent_fails_over(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  RMSNorm:\n    backend: infinicore\n    fallback_backend: b200\n")
    assert backends.route("RMSNorm", lambda: "orig", call_b200=lambda: "kern") == "kern"
    assert backends.active_backend("RMSNorm") == "b200"
    assert backends.backend_stats("RMSNorm")["infinicore"].failures == 1


def test_stats_off_by_default_but_disable_still_happens(monkeypatch, tmp_path):
    monkeypatch.delenv("VLLM_NT_ENABLE_STATS", raising=False)
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  MatMul:\n    backend: b200\n")
    assert backends.route("MatMul", lambda: "orig", call_b200=lambda: 1 / 0) == "orig"
    assert backends.active_backend("MatMul") == "original"
    assert backends.backend_stats("MatMul") == {}


@pytest.mark.parametrize("name", ["RoPE", "ApplyRotaryEmb"])
def test_disable_ops_env_with_rope_aliases(monkeypatch, tmp_path, name):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  ApplyRotaryEmb:\n    backend: b200\n")
    monkeypatch.setenv("VLLM_NT_DISABLE_OPS", name)
    assert backends.active_backend("RoPE") == "original"
    assert {"RoPE", "ApplyRotaryEmb"} <= backends.disabled_ops()


def test_rope_alias_reads_apply_rotary_emb(monkeypatch, tmp_path):
    _use(monkeypatch, tmp_path, "version: 1\nops:\n  ApplyRotaryEmb:\n    backend: b200\n    fallback_backend: original\n")
    assert backends.configured_backend("RoPE") == "b200"
    assert backends.fallback_backend("RoPE") == "original"

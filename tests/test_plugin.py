"""Plugin registration and hook behaviour with vLLM imported, no GPU: which methods are
replaced, what the hooks route where, and the usage-summary contract of the reference
(vllm_nt/tests/test_plugin_integration.py).  Kernels are replaced by fakes here; the GPU
versions of these paths are in test_hooks_gpu.py."""

import re
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytest.importorskip("vllm")

import vllm_nt  # noqa: E402
from vllm_nt._ntops import backends, config, patching  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(autouse=True)
def _fresh(monkeypatch):
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml"))
    patching._reset_usage_state()
    yield
    patching._reset_usage_state()


def test_entry_point_declared():
    text = (ROOT / "pyproject.toml").read_text()
    assert '[project.entry-points."vllm.general_plugins"]' in text
    assert 'vllm_nt = "vllm_nt:register"' in text


def test_vllm_plugin_loader_finds_the_entry_point(tmp_path, monkeypatch):
    """A dist-info with the same entry point makes vLLM's loader call vllm_nt.register."""
    dist = tmp_path / "vllm_nt-0.2.0.dist-info"
    dist.mkdir()
    (dist / "METADATA").write_text("Metadata-Version: 2.1\nName: vllm-nt\nVersion: 0.2.0\n")
    (dist / "entry_points.txt").write_text("[vllm.general_plugins]\nvllm_nt = vllm_nt:register\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    from vllm.plugins import load_plugins_by_group

    plugins = load_plugins_by_group("vllm.general_plugins")
    assert "vllm_nt" in plugins and plugins["vllm_nt"] is vllm_nt.register


def test_register_is_idempotent_and_hooks_cuda_dispatch():
    from vllm.model_executor.custom_op import op_registry_oot
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding
    from vllm.model_executor.layers.vocab_parallel_embedding import UnquantizedEmbeddingMethod

    vllm_nt.register()
    vllm_nt.register()
    for name, fwd in (("RMSNorm", patching._nt_rms_norm_forward), ("SiluAndMul", patching._nt_silu_and_mul_forward)):
        cls = op_registry_oot[name]
        # CUDA platforms dispatch forward_cuda; disabled ops dispatch forward_native
        assert cls.forward_cuda is fwd and cls.forward_native is fwd and cls.forward_oot is fwd
    assert UnquantizedLinearMethod.apply is patching._nt_unquantized_linear_apply
    assert UnquantizedEmbeddingMethod.embedding is patching._nt_unquantized_embedding
    assert UnquantizedEmbeddingMethod.apply is patching._nt_unquantized_embedding_apply
    assert patching._is_function_patch(RotaryEmbedding.forward_cuda, "RoPE")


def test_usage_summary_shape_and_registered_ops():
    vllm_nt.register()
    s = patching.get_usage_summary()
    assert set(s) == {"registered_ops", "hit_ops", "missed_ops", "operators", "disabled"}
    for op in ("RMSNorm", "SiluAndMul", "RoPE", "MatMul", "LMHead", "Embedding", "StoreKVCache", "PagedAttentionDecode"):
        assert op in s["registered_ops"]
    assert s["hit_ops"] == [] and set(s["missed_ops"]) == set(s["registered_ops"])
    d = s["operators"]["MatMul"]
    # the reference's keys; "declined" appears only once a call was not served
    assert set(d) == {"configured_backend", "active_backend", "hits", "failures", "fallbacks", "registered_via", "backends"}
    assert d["configured_backend"] == "b200"


def test_summary_empty_when_stats_disabled(monkeypatch, capsys):
    monkeypatch.setenv("VLLM_NT_ENABLE_STATS", "0")
    patching._record_hit("RMSNorm", torch.ones(1, 4))
    assert patching.get_usage_summary() == {"registered_ops": [], "hit_ops": [], "missed_ops": [], "operators": {}, "disabled": []}
    assert patching.maybe_print_usage_summary(include_empty=True) is False
    assert capsys.readouterr().err == ""


def test_feature_toggles(monkeypatch):
    assert patching._nt_feature_enabled("FA") and patching._nt_feature_enabled("MM")
    monkeypatch.setenv("VLLM_NT_ENABLE_FA", "0")
    disabled = {s.patch_id for s in patching._FUNCTION_PATCH_SPECS if not patching._function_patch_enabled(s)}
    assert {"StoreKVCache", "PagedAttentionDecode"} <= disabled and "RoPE" not in disabled
    monkeypatch.setenv("VLLM_NT_ENABLE_ALL", "0")
    monkeypatch.setenv("VLLM_NT_ENABLE_FA", "1")
    assert not patching._operator_enabled("RMSNorm")


def test_mm_toggle_skips_linear_and_lmhead(monkeypatch):
    class FakeLinear:
        apply = object()

    class FakeEmbedding:
        embedding = object()
        apply = object()

    monkeypatch.setattr(patching, "UnquantizedLinearMethod", FakeLinear)
    monkeypatch.setattr(patching, "UnquantizedEmbeddingMethod", FakeEmbedding)
    monkeypatch.setenv("VLLM_NT_ENABLE_MM", "0")
    keep_lin, keep_apply = FakeLinear.apply, FakeEmbedding.apply
    patching._patch_leaf_methods()
    assert FakeLinear.apply is keep_lin and FakeEmbedding.apply is keep_apply
    assert FakeEmbedding.embedding is patching._nt_unquantized_embedding


def test_default_config_gates_attention_patches_off(monkeypatch):
    monkeypatch.delenv("VLLM_NT_BACKEND_CONFIG")
    config.reset_backend_config_cache()
    enabled = {s.patch_id for s in patching._FUNCTION_PATCH_SPECS if patching._function_patch_enabled(s)}
    assert "StoreKVCache" not in enabled and "PagedAttentionDecode" not in enabled
    assert "RoPE" in enabled  # ApplyRotaryEmb -> ninetoothed (= these kernels) by default


# ---------------------------------------------------------------------------- hook routing


class _Norm:
    variance_epsilon = 1e-6
    has_weight = True
    hidden_size = 8

    def __init__(self):
        self.weight = torch.nn.Parameter(torch.ones(8))


def test_rms_norm_hook_hits_and_falls_back_on_failure(monkeypatch):
    monkeypatch.setattr(patching, "_why_not_norm", lambda *a: None)
    monkeypatch.setattr(patching, "norm", lambda self, x, w, r=None, gemma=False: "kernel")
    monkeypatch.setitem(patching._ORIGINAL_OPERATOR_FORWARDS, "RMSNorm", {"native": lambda self, x, r=None: "native"})
    assert patching._nt_rms_norm_forward(_Norm(), torch.ones(2, 8)) == "kernel"
    assert patching.get_usage_summary()["operators"]["RMSNorm"]["hits"] == 1

    def boom(*a, **k):
        raise RuntimeError("kernel failed")

    monkeypatch.setattr(patching, "norm", boom)
    assert patching._nt_rms_norm_forward(_Norm(), torch.ones(2, 8)) == "native"
    op = patching.get_usage_summary()["operators"]["RMSNorm"]
    assert op["failures"] == 1 and op["active_backend"] == "original"


def test_ineligible_calls_go_to_vllm_and_are_counted_as_declined():
    """CPU tensors are not eligible: vLLM's own forward runs, no hit is counted, and the
    call shows in the summary as a fallback to original with its reason."""
    from vllm.model_executor.layers.layernorm import RMSNorm
    from vllm import ir

    vllm_nt.register()
    x, r = torch.randn(3, 16), torch.randn(3, 16)
    layer = SimpleNamespace(weight=torch.nn.Parameter(torch.ones(16)), has_weight=True, variance_epsilon=1e-6,
                            variance_size_override=None, hidden_size=16, pass_weight=True, pass_weight_add=True)
    out, res = patching._nt_rms_norm_forward(layer, x.clone(), r.clone())
    ref, ref_r = ir.ops.fused_add_rms_norm(x.clone(), r.clone(), layer.weight.data, 1e-6)
    torch.testing.assert_close(out, ref)
    op = patching.get_usage_summary()["operators"]["RMSNorm"]
    assert op["hits"] == 0 and op["fallbacks"] == 1
    assert op["declined"] == {"not a CUDA tensor": 1} and op["backends"]["original"]["fallbacks"] == 1
    assert "declined: not a CUDA tensor=1" in patching.format_usage_summary(use_color=False)
    assert RMSNorm is not None


def test_linear_hook_routes_and_handles_residual(monkeypatch):
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod

    monkeypatch.setattr(patching, "_why_not_gemm", lambda *a: None)
    monkeypatch.setattr(patching, "linear", lambda x, w, b=None: x @ w.t())
    setattr(patching._nt_unquantized_linear_apply, "_original", lambda *a, **k: "vllm")
    layer = SimpleNamespace(weight=torch.ones(3, 4))
    x = torch.ones(2, 4)
    out = patching._nt_unquantized_linear_apply(UnquantizedLinearMethod(), layer, x, None, residual=torch.ones(2, 3))
    assert torch.equal(out, torch.full((2, 3), 5.0))
    assert patching.get_usage_summary()["operators"]["MatMul"]["hits"] == 1


def test_rope_hook_uses_matched_cache_and_counts(monkeypatch):
    captured = {}

    def fake_rope(positions, query, key, **kw):
        captured.update(kw)
        return query, key

    monkeypatch.setattr(patching, "rope", fake_rope)

    class Rot:
        is_neox_style = True
        rotary_dim = 4
        head_size = 4

        def __init__(self):
            self.cos_sin_cache = torch.ones(8, 4)

        def _match_cos_sin_cache_dtype(self, q):
            self.cos_sin_cache = self.cos_sin_cache.to(q.dtype)
            return self.cos_sin_cache

    fwd = patching._build_rotary_forward(lambda *a, **k: (_ for _ in ()).throw(AssertionError("fallback")))
    q = torch.zeros(2, 4, dtype=torch.float16)
    # CPU tensors are ineligible -> the original (here: raising) is called
    with pytest.raises(AssertionError):
        fwd(Rot(), torch.tensor([0, 1]), q, q.clone())
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    res = fwd(Rot(), torch.tensor([0, 1]), q, q.clone())
    assert res[0] is q and captured["cos_sin_cache"].dtype == torch.float16 and captured["rotary_dim"] == 4
    assert patching.get_usage_summary()["operators"]["RoPE"]["hits"] == 1


def test_attention_hooks_route_decode_prefill_and_kv_store(monkeypatch):
    calls = {}
    monkeypatch.setattr(patching, "_attn_impl_reason", lambda *a: None)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))

    def fake_decode(out, q, kv, seq, table, n, scale, msl, kv_dim=0):
        calls["decode"] = (tuple(out.shape), tuple(q.shape), tuple(kv.shape), tuple(seq.shape), n, scale, msl)
        out[:n].fill_(1.0)

    def fake_store(key, value, kv, slots, kv_dim=0):
        calls["store"] = (tuple(key.shape), tuple(kv.shape), tuple(slots.shape))

    def fake_varlen(out, q, kv, qsl, seq, table, n, max_q, msl, scale, kv_dim=0):
        calls["varlen"] = (tuple(qsl.shape), n, max_q, msl, scale)
        out[:n].fill_(2.0)

    monkeypatch.setattr(patching, "paged_attention_decode_flash", fake_decode)
    monkeypatch.setattr(patching, "paged_attention_flash", fake_varlen)
    monkeypatch.setattr(patching, "store_kv_cache_flash", fake_store)
    orig = lambda *a, **k: "flash-attn"  # noqa: E731
    fwd = patching._build_flash_attn_forward(orig)
    upd = patching._build_flash_attn_kv_update(orig)
    impl = SimpleNamespace(num_heads=4, head_size=128, scale=0.1)
    kv = torch.zeros(2, 6, 16, 2, 128)
    q = torch.zeros(5, 4, 128)  # 3 real decode tokens + 2 padding rows
    out = torch.zeros(5, 4 * 128)
    meta = SimpleNamespace(num_actual_tokens=3, max_query_len=1, use_cascade=False, max_seq_len=40,
                           query_start_loc=torch.tensor([0, 1, 2, 3]), seq_lens=torch.tensor([4, 9, 40]),
                           block_table=torch.zeros(3, 3, dtype=torch.int32))
    assert fwd(impl, None, q, q, q, kv, meta, out) is out
    assert calls["decode"] == ((5, 4 * 128), (5, 4, 128), (2, 6, 16, 2, 128), (3,), 3, 0.1, 40)
    assert out[:3].eq(1).all() and out[3:].eq(0).all()
    # a mixed batch (two decodes and a 3-token chunk of a prefill) goes to the varlen entry
    mixed = SimpleNamespace(**{**vars(meta), "max_query_len": 3, "num_actual_tokens": 5,
                               "query_start_loc": torch.tensor([0, 1, 2, 5])})
    assert fwd(impl, None, q, q, q, kv, mixed, out) is out
    assert calls["varlen"] == ((4,), 5, 3, 40, 0.1) and out[:5].eq(2).all()
    # cascade and non-causal metadata stay on vLLM's FlashAttention
    for bad in ({"use_cascade": True}, {"causal": False}):
        assert fwd(impl, None, q, q, q, kv, SimpleNamespace(**{**vars(mixed), **bad}), out) == "flash-attn"
    upd(impl, None, torch.zeros(5, 2, 128), torch.zeros(5, 2, 128), kv, torch.tensor([1, 2, 3]))
    assert calls["store"] == ((5, 2, 128), (2, 6, 16, 2, 128), (3,))
    ops = patching.get_usage_summary()["operators"]
    assert ops["PagedAttentionDecode"]["hits"] == 1 and ops["StoreKVCache"]["hits"] == 1
    assert ops["PagedAttentionPrefill"]["hits"] == 1


def test_no_vendor_imports_in_package():
    """Like the reference's structural test: nothing in the package imports a vendor
    accelerator stack or the reference's DSL."""
    pkg = ROOT / "vllm-nt_b200" / "vllm_nt"
    bad = re.compile(r"^\s*(import|from)\s+(torch_mlu|torch_musa|vllm_mlu|vllm_musa|vllm_metax|ninetoothed|triton|infinicore)\b", re.M)
    offenders = [str(p) for p in pkg.rglob("*.py") if bad.search(p.read_text())]
    assert offenders == []


def test_fused_mlp_hook_routes_gate_up_silu_and_down(monkeypatch):
    """LlamaMLP.forward replacement: one fused gate_up+SiluAndMul call, then down_proj; an
    ineligible MLP (quantised gate_up) runs vLLM's forward."""
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod

    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    calls = {}

    def fake_fused(x, w):
        calls["fused"] = (tuple(x.shape), tuple(w.shape))
        return torch.ones(x.shape[0], w.shape[0] // 2, dtype=x.dtype)

    monkeypatch.setattr(patching, "gate_up_silu_and_mul", fake_fused)
    fwd = patching._build_mlp_forward(lambda self, x: "vllm")
    w = torch.zeros(2 * 24, 16, dtype=torch.bfloat16)
    down = lambda h: (h.sum(-1, keepdim=True), None)  # noqa: E731
    mlp = SimpleNamespace(gate_up_proj=SimpleNamespace(weight=w, quant_method=UnquantizedLinearMethod(), bias=None,
                                                       gather_output=False),
                          act_fn=object.__new__(SiluAndMul), down_proj=down)
    x = torch.zeros(3, 16, dtype=torch.bfloat16)
    out = fwd(mlp, x)
    assert calls["fused"] == ((3, 16), (48, 16)) and out.shape == (3, 1) and float(out[0, 0]) == 24.0
    assert patching.get_usage_summary()["operators"]["GateUpSiluAndMul"]["hits"] == 1
    mlp.gate_up_proj.quant_method = object()
    assert fwd(mlp, x) == "vllm"


def test_fused_mlp_patch_is_opt_in(monkeypatch):
    """Configs written for the reference (no GateUpSiluAndMul key) leave LlamaMLP alone."""
    spec = next(s for s in patching._FUNCTION_PATCH_SPECS if s.patch_id == "GateUpSiluAndMul")
    config.reset_backend_config_cache()
    assert patching._function_patch_enabled(spec)  # all-b200.yaml names it
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/hybrid-default.yaml"))
    config.reset_backend_config_cache()
    try:
        assert not patching._function_patch_enabled(spec)
    finally:
        config.reset_backend_config_cache()


def test_flashinfer_hooks_decode_only_and_kv_store(monkeypatch):
    """FlashInferImpl hooks: pure-decode batches with a decode block table go to the
    kernels on the [blocks, 2, 16, H, D] cache (kv_dim 1); prefill stays on FlashInfer."""
    calls = {}
    monkeypatch.setattr(patching, "_attn_impl_reason", lambda *a: None)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))

    def fake_decode(out, q, kv, seq, table, n, scale, msl, kv_dim):
        calls["decode"] = (tuple(kv.shape), tuple(seq.shape), tuple(table.shape), n, msl, kv_dim)
        out[:n].fill_(1.0)

    def fake_store(key, value, kv, slots, kv_dim):
        calls["store"] = (tuple(kv.shape), kv_dim)

    monkeypatch.setattr(patching, "paged_attention_decode_flash", fake_decode)
    monkeypatch.setattr(patching, "store_kv_cache_flash", fake_store)
    orig = lambda *a, **k: "flashinfer"  # noqa: E731
    fwd = patching._build_flashinfer_forward(orig)
    upd = patching._build_flashinfer_kv_update(orig)
    impl = SimpleNamespace(num_heads=4, head_size=128, scale=0.1)
    kv = torch.zeros(6, 2, 16, 2, 128)
    q = torch.zeros(5, 4, 128)
    out = torch.zeros(5, 4 * 128)
    dec = SimpleNamespace(block_tables=torch.zeros(3, 3, dtype=torch.int32), seq_lens=torch.tensor([4, 9, 40]),
                          max_seq_len=40)
    meta = SimpleNamespace(num_actual_tokens=3, num_decodes=3, num_decode_tokens=3, num_prefills=0, decode=dec,
                           use_cascade=False)
    assert fwd(impl, None, q, q, q, kv, meta, out) is out
    assert calls["decode"] == ((6, 2, 16, 2, 128), (3,), (3, 3), 3, 40, 1)
    assert out[:3].eq(1).all() and out[3:].eq(0).all()
    mixed = SimpleNamespace(**{**vars(meta), "num_prefills": 1})
    assert fwd(impl, None, q, q, q, kv, mixed, out) == "flashinfer"
    planned = SimpleNamespace(**{**vars(meta), "decode": SimpleNamespace(wrapper=object())})
    assert fwd(impl, None, q, q, q, kv, planned, out) == "flashinfer"
    upd(impl, None, torch.zeros(5, 2, 128), torch.zeros(5, 2, 128), kv, torch.tensor([1, 2, 3]))
    assert calls["store"] == ((6, 2, 16, 2, 128), 1)


def test_sampler_hooks_patch_vllm_and_route(monkeypatch):
    """TopKTopP / RandomSample replace vLLM's topk_topp_sampler functions (the reference's
    patch targets); CPU or non-fp32 tensors go to vLLM's code uncounted, eligible calls to
    the kernels and are counted; RejectionSample only counts and runs vLLM's code."""
    from vllm.v1.sample.ops import topk_topp_sampler as tks

    vllm_nt.register()
    assert patching._is_function_patch(tks.apply_top_k_top_p, "TopKTopP")
    assert patching._is_function_patch(tks.random_sample, "RandomSample")

    calls = []
    monkeypatch.setattr(patching, "nt_apply_top_k_top_p", lambda lg, k, p: calls.append("mask") or lg)
    monkeypatch.setattr(patching, "nt_random_sample", lambda pr, gens: calls.append("sample") or "kernel")
    mask = patching._build_apply_top_k_top_p_patch(lambda lg, k, p: "vllm")
    sample = patching._build_random_sample_patch(lambda pr, gens: "vllm")
    logits = torch.randn(2, 8)
    k = torch.tensor([2, 3])
    assert mask(logits, k, None) == "vllm" and sample(logits, {}) == "vllm"  # CPU: vLLM's code
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    assert mask(logits, None, None) == "vllm"  # nothing to mask
    assert mask(logits.half(), k, None) == "vllm"  # not fp32
    assert mask(logits, k, None) is logits and sample(logits, {}) == "kernel"
    assert calls == ["mask", "sample"]
    ops = patching.get_usage_summary()["operators"]
    assert ops["TopKTopP"]["hits"] == 1 and ops["RandomSample"]["hits"] == 1

    reject = patching._build_rejection_sample_patch(lambda *a, **kw: "vllm")
    assert reject(None, [1], 1, None, None, torch.zeros(1, 8), None, None) == "vllm"
    assert reject(target_logits=torch.zeros(1, 8)) == "vllm"
    assert patching.get_usage_summary()["operators"]["RejectionSample"]["hits"] == 2


def test_sampler_patches_follow_the_config(monkeypatch):
    """The reference's default map sends TopKTopP / RandomSample to its kernel backend, so
    the patches apply; original-only.yaml keeps vLLM's sampler functions."""
    def enabled():
        config.reset_backend_config_cache()
        return {s.patch_id for s in patching._FUNCTION_PATCH_SPECS if patching._function_patch_enabled(s)}

    monkeypatch.delenv("VLLM_NT_BACKEND_CONFIG")
    assert {"TopKTopP", "RandomSample", "RejectionSample"} <= enabled()
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/original-only.yaml"))
    assert not {"TopKTopP", "RandomSample"} & enabled()


def test_fused_rope_kv_hook_is_opt_in_and_declines_what_it_cannot_fuse(monkeypatch):
    """RoPEKVCache (LlamaAttention.forward) applies only when the config names it; a module
    whose rotary embedding is not vLLM's base RotaryEmbedding runs vLLM's path (rotary_emb,
    then attn) and the call is counted as declined with its reason."""
    spec = next(s for s in patching._FUNCTION_PATCH_SPECS if s.patch_id == "RoPEKVCache")
    config.reset_backend_config_cache()
    assert patching._function_patch_enabled(spec)  # all-b200.yaml names it
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/hybrid-default.yaml"))
    config.reset_backend_config_cache()
    assert not patching._function_patch_enabled(spec)
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml"))
    config.reset_backend_config_cache()

    calls = []
    qkv = torch.zeros(3, 6)
    module = SimpleNamespace(
        qkv_proj=lambda h: (qkv, None), q_size=4, kv_size=1,
        rotary_emb=lambda p, q, k: (calls.append("rope"), (q, k))[1],
        attn=lambda q, k, v: (calls.append("attn"), q)[1],
        o_proj=lambda a: (a, None))
    fwd = patching._build_attention_rope_kv_forward(lambda *a: pytest.fail("the patch replaces forward"))
    out = fwd(module, torch.arange(3), None)
    assert calls == ["rope", "attn"] and out.shape == (3, 4)
    op = patching.get_usage_summary()["operators"]["RoPEKVCache"]
    assert op["hits"] == 0 and op["declined"] == {"not the base RotaryEmbedding": 1}


def test_norm_qkv_decoder_hook_is_opt_in_and_declines_what_it_cannot_fuse(monkeypatch, tmp_path):
    """RMSNormQKV (LlamaDecoderLayer.forward) applies only when a config names it (the
    shipped all-b200.yaml does); a call it cannot serve (here: CPU activations, then a batch
    above two tokens) runs vLLM's layer forward and is counted as declined with its reason."""
    spec = next(s for s in patching._FUNCTION_PATCH_SPECS if s.patch_id == "RMSNormQKV")
    config.reset_backend_config_cache()
    assert patching._function_patch_enabled(spec)  # all-b200.yaml names it
    cfg = tmp_path / "no-norm-qkv.yaml"
    cfg.write_text((ROOT / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml").read_text().replace("  RMSNormQKV: b200\n", ""))
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(cfg))
    config.reset_backend_config_cache()
    assert not patching._function_patch_enabled(spec)
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml"))
    config.reset_backend_config_cache()

    layer = _norm_qkv_layer()
    seen = []
    fwd = patching._build_decoder_norm_qkv_forward(lambda self, p, h, r: (seen.append(h.shape[0]), (h, r))[1])
    h = torch.zeros(1, 8)
    assert fwd(layer, torch.arange(1), h, None)[0] is h
    h3 = torch.zeros(3, 8)
    assert fwd(layer, torch.arange(3), h3, None)[0] is h3
    op = patching.get_usage_summary()["operators"]["RMSNormQKV"]
    assert seen == [1, 3] and op["hits"] == 0
    assert op["declined"] == {"activation / weight dtype or device": 1, "batch above 2 token(s)": 1}


def _norm_qkv_layer(**changes):
    """A decoder layer stand-in with vLLM's RMSNorm (built without its config-dependent
    constructor) and an unquantised qkv projection of a [12, 8] weight; ``changes`` sets
    attributes of the norm (``ln_*``) or of qkv_proj (``qkv_*``)."""
    from vllm.model_executor.layers.layernorm import RMSNorm

    ln = RMSNorm.__new__(RMSNorm)
    for name, value in (("weight", torch.ones(8)), ("variance_epsilon", 1e-6), ("has_weight", True),
                        ("variance_size_override", None)):
        object.__setattr__(ln, name, value)
    qkv_proj = SimpleNamespace(quant_method=patching.UnquantizedLinearMethod(), bias=None, gather_output=False,
                               weight=torch.zeros(12, 8))
    for key, value in changes.items():
        owner, attr = key.split("_", 1)
        if owner == "ln":
            object.__setattr__(ln, attr, value)
        else:
            setattr(qkv_proj, attr, value)
    return SimpleNamespace(input_layernorm=ln, self_attn=SimpleNamespace(qkv_proj=qkv_proj))


@pytest.mark.parametrize("changes,hidden_shape,reason", [
    ({"ln_has_weight": False}, (1, 8), "input_layernorm is not a plain RMSNorm"),
    ({"ln_variance_size_override": 4}, (1, 8), "input_layernorm is not a plain RMSNorm"),
    ({"qkv_quant_method": object()}, (1, 8), "quantised qkv_proj"),
    ({"qkv_bias": torch.zeros(12)}, (1, 8), "qkv_proj bias or gathered output"),
    ({"qkv_gather_output": True}, (1, 8), "qkv_proj bias or gathered output"),
    ({"qkv_weight": torch.zeros(12, 6)}, (1, 6), "qkv_proj weight layout"),
    ({"qkv_weight": torch.zeros(8, 12).t()}, (1, 8), "qkv_proj weight layout"),
    ({}, (1, 16), "hidden states are not [tokens, hidden]"),
    ({}, (1, 1, 8), "hidden states are not [tokens, hidden]"),
    ({}, (3, 8), "batch above 2 token(s)"),
    ({}, (2, 8), "activation / weight dtype or device"),  # eligible but for the CPU tensor
])
def test_norm_qkv_decline_reasons(changes, hidden_shape, reason):
    """Each reason the RMSNorm + qkv decoder hook gives for leaving a call to vLLM, checked
    in the order the hook tests them (the device check last but one, so every layer and
    shape reason shows on CPU tensors)."""
    layer = _norm_qkv_layer(**changes)
    assert patching._why_not_norm_qkv(layer, torch.zeros(hidden_shape), None) == reason

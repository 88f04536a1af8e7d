"""The plugin's hooks on a GPU: vLLM layer objects dispatch into the B200 kernels (hits are
counted under the b200 backend) and agree with the CPU oracle.  Uses vLLM's own classes
(RMSNorm, SiluAndMul, RotaryEmbedding, Unquantized{Linear,Embedding}Method) and the
FlashAttentionImpl hooks with a real paged KV cache."""

import math
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

import oracle
from _util import bits_equal, cuda_device, seeded

pytestmark = pytest.mark.gpu
pytest.importorskip("vllm")
ROOT = Path(__file__).resolve().parents[1]
TOL = dict(rtol=2e-2, atol=2e-2)


@pytest.fixture(autouse=True)
def _b200_config(monkeypatch):
    cuda_device()
    import vllm_nt
    from vllm_nt._ntops import patching

    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(ROOT / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml"))
    vllm_nt.register()
    patching._reset_usage_state()
    yield patching
    patching._reset_usage_state()


@pytest.fixture()
def vllm_ctx():
    from vllm.config import VllmConfig, set_current_vllm_config

    with set_current_vllm_config(VllmConfig()):
        yield


def _hits(patching, op):
    return patching.get_usage_summary()["operators"][op]["backends"].get("b200", {}).get("hits", 0)


def test_rmsnorm_layer_runs_the_fused_kernel(_b200_config, vllm_ctx):
    from vllm.model_executor.layers.layernorm import RMSNorm

    layer = RMSNorm(4096, eps=1e-5).to(device="cuda", dtype=torch.bfloat16)
    assert type(layer).__name__ == "NTRMSNorm"
    g = seeded(0)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    layer.weight.data.copy_(w)
    x = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    r = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    out, res = layer(x.cuda(), r.cuda())
    ref, ref_r = oracle.fused_add_rms_norm(x, r, w, 1e-5)
    torch.testing.assert_close(out.float().cpu(), ref.float(), **TOL)
    assert bits_equal(res.cpu(), ref_r)
    plain = layer(x.cuda())
    torch.testing.assert_close(plain.float().cpu(), oracle.rms_norm(x, w, 1e-5).float(), **TOL)
    assert _hits(_b200_config, "RMSNorm") == 2


def test_silu_and_mul_layer(_b200_config, vllm_ctx):
    from vllm.model_executor.layers.activation import SiluAndMul

    layer = SiluAndMul()
    x = torch.randn(16, 2 * 14336, generator=seeded(1)).to(torch.bfloat16)
    out = layer(x.cuda())
    torch.testing.assert_close(out.float().cpu(), oracle.silu_and_mul(x).float(), **TOL)
    assert _hits(_b200_config, "SiluAndMul") == 1


def test_rotary_embedding_layer_bit_exact(_b200_config, vllm_ctx):
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding

    rope = RotaryEmbedding(128, 128, 4096, 500000.0, True, torch.bfloat16).cuda()
    g = seeded(2)
    pos = torch.randint(0, 4096, (24,), generator=g)
    qkv = torch.randn(24, (32 + 16) * 128, generator=g).to(torch.bfloat16)
    q, k = qkv[:, : 32 * 128], qkv[:, 32 * 128 : 40 * 128]
    qd_all = qkv.cuda()
    qd, kd = qd_all[:, : 32 * 128], qd_all[:, 32 * 128 : 40 * 128]
    rope(pos.cuda(), qd, kd)
    cache = rope.cos_sin_cache.float().cpu()
    ref_q, ref_k = oracle.rope_neox(pos, q, k, cache, 128, 128)
    assert bits_equal(qd.cpu().contiguous(), ref_q.contiguous()) and bits_equal(kd.cpu().contiguous(), ref_k.contiguous())
    assert _hits(_b200_config, "RoPE") == 1


def test_linear_and_embedding_methods(_b200_config, vllm_ctx):
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod
    from vllm.model_executor.layers.vocab_parallel_embedding import UnquantizedEmbeddingMethod

    g = seeded(3)
    w = (0.02 * torch.randn(6144, 4096, generator=g)).to(torch.bfloat16)
    x = torch.randn(7, 4096, generator=g).to(torch.bfloat16)
    layer = SimpleNamespace(weight=torch.nn.Parameter(w.cuda(), requires_grad=False))
    out = UnquantizedLinearMethod().apply(layer, x.cuda())
    torch.testing.assert_close(out.float().cpu(), oracle.linear(x, w), **TOL)
    assert _hits(_b200_config, "MatMul") == 1
    table = torch.randn(1000, 4096, generator=g).to(torch.bfloat16)
    emb_layer = SimpleNamespace(weight=torch.nn.Parameter(table.cuda(), requires_grad=False))
    ids = torch.randint(0, 1000, (2, 5), generator=g)
    e = UnquantizedEmbeddingMethod().embedding(emb_layer, ids.cuda())
    assert torch.equal(e.cpu(), table[ids])
    head = UnquantizedEmbeddingMethod().apply(emb_layer, x[:, :4096].cuda())
    torch.testing.assert_close(head.float().cpu(), oracle.linear(x, table), **TOL)
    assert _hits(_b200_config, "Embedding") == 1 and _hits(_b200_config, "LMHead") == 1


def test_flash_attention_impl_hooks_store_and_decode(_b200_config):
    patching = _b200_config
    fwd = patching._build_flash_attn_forward(lambda *a, **k: pytest.fail("decode fell back to vLLM"))
    upd = patching._build_flash_attn_kv_update(lambda *a, **k: pytest.fail("store fell back to vLLM"))
    impl = SimpleNamespace(num_heads=32, num_kv_heads=8, head_size=128, scale=1 / math.sqrt(128), attn_type="decoder",
                           kv_cache_dtype="auto", alibi_slopes=None, logits_soft_cap=None, sinks=None,
                           sliding_window=None, dcp_world_size=1)
    g = seeded(4)
    nb = 64
    kv = torch.randn(2, nb, 16, 8, 128, generator=g).to(torch.bfloat16)
    ctx = [5, 40, 200]  # tokens already cached; this step appends one token each
    table = torch.randperm(nb, generator=g)[:3 * 16].view(3, 16).to(torch.int32)
    slots = torch.tensor([int(table[b, c // 16]) * 16 + c % 16 for b, c in enumerate(ctx)])
    key = torch.randn(4, 8, 128, generator=g).to(torch.bfloat16)  # 3 real rows + 1 padding row
    value = torch.randn(4, 8, 128, generator=g).to(torch.bfloat16)
    kvd = kv.cuda()
    upd(impl, None, key.cuda(), value.cuda(), kvd, slots.cuda())
    ref_kv = kv.clone()
    ref_kv[0][slots // 16, slots % 16] = key[:3]
    ref_kv[1][slots // 16, slots % 16] = value[:3]
    assert torch.equal(kvd.cpu(), ref_kv)
    q = torch.randn(4, 32, 128, generator=g).to(torch.bfloat16)
    out = torch.zeros(4, 32 * 128, dtype=torch.bfloat16, device="cuda")
    seq = torch.tensor([c + 1 for c in ctx], dtype=torch.int32)
    meta = SimpleNamespace(num_actual_tokens=3, max_query_len=1, use_cascade=False, max_seq_len=max(seq).item(),
                           query_start_loc=torch.arange(4, dtype=torch.int32).cuda(), seq_lens=seq.cuda(),
                           block_table=table.cuda())
    fwd(impl, None, q.cuda(), None, None, kvd, meta, out)
    ref = oracle.paged_decode(q[:3], ref_kv[0], ref_kv[1], seq, table, impl.scale)
    torch.testing.assert_close(out[:3].view(3, 32, 128).float().cpu(), ref, **TOL)
    assert not out[3].any()
    assert _hits(patching, "StoreKVCache") == 1 and _hits(patching, "PagedAttentionDecode") == 1


def test_flash_attention_impl_hook_mixed_prefill_batch(_b200_config):
    """A chunked-prefill step: one request prefills 150 new tokens after 100 cached ones, two
    decode; FlashAttentionImpl.forward runs on the B200 kernels (no fallback) and matches
    the oracle."""
    patching = _b200_config
    fwd = patching._build_flash_attn_forward(lambda *a, **k: pytest.fail("prefill fell back to vLLM"))
    impl = SimpleNamespace(num_heads=32, num_kv_heads=8, head_size=128, scale=1 / math.sqrt(128), attn_type="decoder",
                           kv_cache_dtype="auto", alibi_slopes=None, logits_soft_cap=None, sinks=None,
                           sliding_window=None, dcp_world_size=1)
    g = seeded(5)
    nb = 80
    kv = torch.randn(2, nb, 16, 8, 128, generator=g).to(torch.bfloat16)
    qlens, ctxs = [1, 150, 1], [37, 250, 400]
    table = torch.randperm(nb, generator=g)[: 3 * 25].view(3, 25).to(torch.int32)
    cu = torch.tensor([0, 1, 151, 152], dtype=torch.int32)
    q = torch.randn(160, 32, 128, generator=g).to(torch.bfloat16)  # 152 real rows + padding
    out = torch.zeros(160, 32 * 128, dtype=torch.bfloat16, device="cuda")
    seq = torch.tensor(ctxs, dtype=torch.int32)
    meta = SimpleNamespace(num_actual_tokens=152, max_query_len=150, use_cascade=False, max_seq_len=400, causal=True,
                           query_start_loc=cu.cuda(), seq_lens=seq.cuda(), block_table=table.cuda())
    fwd(impl, None, q.cuda(), None, None, kv.cuda(), meta, out)
    ref = oracle.paged_prefill(q[:152], kv[0], kv[1], cu, seq, table, impl.scale)
    torch.testing.assert_close(out[:152].view(152, 32, 128).float().cpu(), ref, **TOL)
    assert not out[152:].any()
    assert _hits(patching, "PagedAttentionPrefill") == 1


def test_fused_mlp_hook_on_a_llama_shaped_mlp(_b200_config, vllm_ctx):
    """The LlamaMLP.forward replacement: fused gate_up + SiluAndMul kernel, then the
    down projection through its own hook."""
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.linear import UnquantizedLinearMethod

    patching = _b200_config
    g = seeded(9)
    wgu = (0.02 * torch.randn(2 * 512, 1024, generator=g)).to(torch.bfloat16)
    wd = (0.02 * torch.randn(1024, 512, generator=g)).to(torch.bfloat16)
    x = torch.randn(24, 1024, generator=g).to(torch.bfloat16)
    down = SimpleNamespace(weight=torch.nn.Parameter(wd.cuda(), requires_grad=False))
    mlp = SimpleNamespace(
        gate_up_proj=SimpleNamespace(weight=wgu.cuda(), quant_method=UnquantizedLinearMethod(), bias=None,
                                     gather_output=False),
        act_fn=SiluAndMul(),
        down_proj=lambda h: (UnquantizedLinearMethod().apply(down, h), None),
    )
    fwd = patching._build_mlp_forward(lambda *a: pytest.fail("fused MLP fell back to vLLM"))
    out = fwd(mlp, x.cuda())
    h = oracle.silu_and_mul(oracle.linear(x, wgu).to(torch.bfloat16))
    ref = oracle.linear(h.to(torch.bfloat16), wd)
    torch.testing.assert_close(out.float().cpu(), ref.float(), **TOL)
    assert _hits(patching, "GateUpSiluAndMul") == 1 and _hits(patching, "MatMul") == 1


@pytest.mark.parametrize("layout", ["NHD", "HND"])
def test_flashinfer_impl_hooks_store_and_decode(_b200_config, layout):
    """FlashInferImpl hooks on FlashInfer's cache, logically [blocks, 2, 16, H, D] and
    stored NHD or HND (heads outside tokens): the kernels take the strides as they are."""
    patching = _b200_config
    fwd = patching._build_flashinfer_forward(lambda *a, **k: pytest.fail("decode fell back to FlashInfer"))
    upd = patching._build_flashinfer_kv_update(lambda *a, **k: pytest.fail("store fell back to FlashInfer"))
    impl = SimpleNamespace(num_heads=32, num_kv_heads=8, head_size=128, scale=1 / math.sqrt(128), attn_type="decoder",
                           kv_cache_dtype="auto", alibi_slopes=None, logits_soft_cap=None, sinks=None,
                           sliding_window=None, kv_sharing_target_layer_name=None)
    g = seeded(14)
    nb = 48
    kv = torch.randn(nb, 2, 16, 8, 128, generator=g).to(torch.bfloat16)
    if layout == "HND":
        kvd = kv.permute(0, 1, 3, 2, 4).contiguous().cuda().permute(0, 1, 3, 2, 4)
        assert kvd.stride(2) == 128 and kvd.stride(3) == 16 * 128
    else:
        kvd = kv.cuda()
    ctx = [0, 17, 200]
    table = torch.randperm(nb, generator=g)[:3 * 16].view(3, 16).to(torch.int32)
    slots = torch.tensor([int(table[b, c // 16]) * 16 + c % 16 for b, c in enumerate(ctx)])
    key = torch.randn(4, 8, 128, generator=g).to(torch.bfloat16)
    value = torch.randn(4, 8, 128, generator=g).to(torch.bfloat16)
    upd(impl, None, key.cuda(), value.cuda(), kvd, slots.cuda())
    ref_kv = kv.clone()
    ref_kv[slots // 16, 0, slots % 16] = key[:3]
    ref_kv[slots // 16, 1, slots % 16] = value[:3]
    assert torch.equal(kvd.cpu(), ref_kv)
    q = torch.randn(4, 32, 128, generator=g).to(torch.bfloat16)
    out = torch.zeros(4, 32 * 128, dtype=torch.bfloat16, device="cuda")
    seq = torch.tensor([c + 1 for c in ctx], dtype=torch.int32)
    dec = SimpleNamespace(block_tables=table.cuda(), seq_lens=seq.cuda(), max_seq_len=int(seq.max()))
    meta = SimpleNamespace(num_actual_tokens=3, num_decodes=3, num_decode_tokens=3, num_prefills=0, decode=dec,
                           use_cascade=False)
    fwd(impl, None, q.cuda(), None, None, kvd, meta, out)
    ref = oracle.paged_decode(q[:3], ref_kv[:, 0].contiguous(), ref_kv[:, 1].contiguous(), seq, table, impl.scale)
    torch.testing.assert_close(out[:3].view(3, 32, 128).float().cpu(), ref, **TOL)
    assert not out[3].any()
    assert _hits(patching, "StoreKVCache") == 1 and _hits(patching, "PagedAttentionDecode") == 1


def test_fused_rope_kv_store_attention_hook(_b200_config, vllm_ctx, monkeypatch):
    """The opt-in LlamaAttention.forward patch: RoPE of q/k and the KV store in one kernel
    (bit-identical to the RoPE hook followed by the KV-store hook), then the layer's own
    KV-store call finds its rows stored and returns without storing again."""
    from vllm.model_executor.layers.attention import attention as vattn
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding

    patching = _b200_config
    rope = RotaryEmbedding(128, 128, 4096, 500000.0, True, torch.bfloat16).cuda()
    g = seeded(41)
    t, hq, hk, nb = 6, 32, 8, 32
    qkv = torch.randn(t, (hq + 2 * hk) * 128, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 4096, (t,), generator=g)
    kv0 = torch.randn(2, nb, 16, hk, 128, generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * 16, generator=g)[:t - 1]  # the last row is vLLM padding
    kvd, slots_d = kv0.cuda(), slots.cuda()

    class FlashAttentionImpl:  # the impl class the hooks recognise, with a supported config
        num_heads, num_kv_heads, head_size, scale = hq, hk, 128, 1.0
        attn_type, kv_cache_dtype, alibi_slopes, logits_soft_cap, sinks = "decoder", "auto", None, None, None
        sliding_window, dcp_world_size = None, 1

    store = patching._build_flash_attn_kv_update(lambda *a, **k: pytest.fail("the KV store ran twice"))

    class Attn:
        layer_name = "model.layers.0.self_attn.attn"
        impl = FlashAttentionImpl()
        kv_sharing_target_layer_name = None
        attn_backend = SimpleNamespace(forward_includes_kv_cache_update=False)

        def __call__(self, q, k, v):
            store(self.impl, self, k.view(-1, hk, 128), v.view(-1, hk, 128), kvd, slots_d)
            return q

    attn = Attn()
    monkeypatch.setattr(vattn, "get_attention_context", lambda name: (None, attn, kvd, slots_d))
    qkvd = qkv.cuda()
    module = SimpleNamespace(qkv_proj=lambda h: (qkvd, None), q_size=hq * 128, kv_size=hk * 128, rotary_emb=rope,
                             attn=attn, o_proj=lambda a: (a, None))
    fwd = patching._build_attention_rope_kv_forward(lambda *a, **k: pytest.fail("fell back to vLLM"))
    out = fwd(module, pos.cuda(), None)
    torch.cuda.synchronize()
    cache = rope.cos_sin_cache.float().cpu()
    ref_q, ref_k = oracle.rope_neox(pos, qkv[:, : hq * 128], qkv[:, hq * 128 : (hq + hk) * 128], cache, 128, 128)
    assert bits_equal(out.cpu().contiguous(), ref_q.contiguous())
    ref_kv = kv0.clone()
    v = qkv[:, (hq + hk) * 128 :]
    ref_kv[0][slots // 16, slots % 16] = ref_k[: t - 1].reshape(t - 1, hk, 128)
    ref_kv[1][slots // 16, slots % 16] = v[: t - 1].reshape(t - 1, hk, 128)
    assert bits_equal(kvd.cpu(), ref_kv)
    assert not getattr(attn, "_ntb200_kv_stored", False)
    assert _hits(patching, "RoPEKVCache") == 1 and _hits(patching, "StoreKVCache") == 1


def test_norm_qkv_decoder_hook(_b200_config, vllm_ctx):
    """The LlamaDecoderLayer.forward patch of the shipped config on decode batches of one
    and two tokens: vLLM's (hooked) input RMSNorm with its residual add and the qkv
    projection as one kernel; the new residual bit for bit and the projection against the
    oracle's restatement of the fused kernel; the attention and the MLP run as the layer's
    own modules.  A five-token batch declines to vLLM's layer forward."""
    from vllm.model_executor.layers.layernorm import RMSNorm

    from vllm_nt._ntops import config

    patching = _b200_config
    config.reset_backend_config_cache()
    g = seeded(43)
    hidden, hq, hk = 4096, 32, 8
    x = torch.randn(5, hidden, generator=g).to(torch.bfloat16)
    r = torch.randn(5, hidden, generator=g).to(torch.bfloat16)
    gam = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    w = (0.02 * torch.randn((hq + 2 * hk) * 128, hidden, generator=g)).to(torch.bfloat16)
    ln = RMSNorm(hidden, eps=1e-5).to(device="cuda", dtype=torch.bfloat16)
    ln.weight.data.copy_(gam)
    qkv_proj = SimpleNamespace(quant_method=patching.UnquantizedLinearMethod(), bias=None, gather_output=False,
                               weight=w.cuda())
    self_attn = SimpleNamespace(qkv_proj=qkv_proj, q_size=hq * 128, kv_size=hk * 128,
                                rotary_emb=lambda p, q, k: (q, k), attn=lambda q, k, v: q,
                                o_proj=lambda a: (a, None))
    layer = SimpleNamespace(input_layernorm=ln, self_attn=self_attn,
                            post_attention_layernorm=lambda h, res: (h, res), mlp=lambda h: h)
    declined = []
    fwd = patching._build_decoder_norm_qkv_forward(lambda self, p, h, res: (declined.append(h.shape[0]), (h, res))[1])
    for t in (1, 2):
        h, res = fwd(layer, torch.arange(t).cuda(), x[:t].cuda(), r[:t].cuda())
        torch.cuda.synchronize()
        ref, res_ref = oracle.rms_norm_linear(x[:t], gam, 1e-5, w, r[:t])
        assert bits_equal(res.cpu(), res_ref)
        torch.testing.assert_close(h.float().cpu(), ref[:, : hq * 128], rtol=2e-2, atol=2e-2)
    assert _hits(patching, "RMSNormQKV") == 2 and declined == []
    fwd(layer, torch.arange(5).cuda(), x.cuda(), r.cuda())
    assert declined == [5] and _hits(patching, "RMSNormQKV") == 2

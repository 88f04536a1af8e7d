"""GPU parity of the memory-bound ops against the CPU oracle, called through the C ABI
(ctypes, include/ntb200.h) and through torch.ops.ntb200.  Sizes are the benchmark
configs plus edge cases.  Tolerances: fp32 1e-5, bf16 2e-2 (rtol = atol); RoPE, the KV
store and the embedding are checked bit for bit."""

import numpy as np
import pytest
import torch

import oracle
from _util import bits_equal, cuda_device, dtype_code, ptr, seeded, stream
from vllm_nt._ntops import capi

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


@pytest.fixture(autouse=True)
def _clean_device_error():
    dev = cuda_device()
    torch.cuda.synchronize(dev)
    capi.read_device_error(stream())
    yield
    torch.cuda.synchronize(dev)


def _close(got, ref, dtype):
    torch.testing.assert_close(got.float().cpu(), ref.float(), rtol=TOL[dtype], atol=TOL[dtype])


# ------------------------------------------------------------------------------ RMS norm


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_add_rms_norm_config_a_capi(dtype):
    """Config (a): x, residual [128, 4096] ~N(0,1), weight ~N(1, 0.1), eps 1e-6."""
    dev = cuda_device()
    g = seeded(0)
    x = torch.randn(128, 4096, generator=g).to(dtype)
    r = torch.randn(128, 4096, generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(4096, generator=g)).to(dtype)
    ref_y, ref_r = oracle.fused_add_rms_norm(x, r, w, 1e-6)
    xd, rd, wd = x.to(dev), r.to(dev), w.to(dev)
    out = torch.empty_like(xd)
    capi.call("ntb200_fused_add_rms_norm", ptr(out), ptr(rd), ptr(xd), ptr(wd), 128, 4096, 4096, 4096, 4096,
              1e-6, dtype_code(dtype), stream())
    torch.cuda.synchronize()
    _close(out, ref_y, dtype)
    assert bits_equal(rd.cpu(), ref_r)  # residual is x + r rounded once: exact
    assert capi.read_device_error(stream()) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(3, 40000), (7, 4095), (2, 16384), (4, 24), (1, 9000)])
def test_fused_add_rms_norm_long_and_ragged_rows(dtype, shape):
    """Rows past the register-resident window (second pass over L2), rows that need the
    scalar path, and a row that fills exactly the largest CTA."""
    dev = cuda_device()
    g = seeded(11)
    x = torch.randn(shape, generator=g).to(dtype)
    r = torch.randn(shape, generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
    ref_y, ref_r = oracle.fused_add_rms_norm(x, r, w, 1e-6)
    xd, rd, wd = x.to(dev), r.to(dev), w.to(dev)
    out = torch.empty_like(xd)
    rows, hidden = shape
    capi.call("ntb200_fused_add_rms_norm", ptr(out), ptr(rd), ptr(xd), ptr(wd), rows, hidden, hidden, hidden,
              hidden, 1e-6, dtype_code(dtype), stream())
    torch.cuda.synchronize()
    _close(out, ref_y, dtype)
    assert bits_equal(rd.cpu(), ref_r)
    assert capi.read_device_error(stream()) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 4096), (32, 4096), (7, 4095), (3, 40000), (5, 96)])
def test_rms_norm_shapes_torch_op(dtype, shape):
    dev = cuda_device()
    g = seeded(1)
    x = torch.randn(shape, generator=g).to(dtype)
    w = torch.randn(shape[-1], generator=g).to(dtype)
    from vllm_nt._ntops.torch.rms_norm import rms_norm

    out = rms_norm(x.to(dev), shape[-1], w.to(dev), 1e-6)
    _close(out, oracle.rms_norm(x, w, 1e-6), dtype)


def test_rms_norm_no_weight_and_strided_rows():
    dev = cuda_device()
    g = seeded(2)
    big = torch.randn(16, 1024 + 64, generator=g).to(torch.bfloat16)
    x = big[:, 32 : 32 + 1024]  # row stride 1088, 64-byte offset
    out = torch.empty(16, 1024, dtype=torch.bfloat16, device=dev)
    xd = big.to(dev)[:, 32 : 32 + 1024]
    capi.call("ntb200_rms_norm", ptr(out), ptr(xd), None, 16, 1024, 1088, 1024, 1e-5, 1, stream())
    torch.cuda.synchronize()
    _close(out, oracle.rms_norm(x, None, 1e-5), torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(128, 4096), (7, 4095), (3, 40000), (1, 2304)])
def test_gemma_rms_norm_capi(dtype, shape):
    """Gemma variant (vLLM's GemmaRMSNorm.forward_native rounding: (1 + w) in fp32, one
    rounding of the product) against the oracle; register-resident, second-pass and scalar
    rows.  The weight is the raw Gemma parameter, ~N(0, 0.3)."""
    dev = cuda_device()
    g = seeded(17)
    x = torch.randn(shape, generator=g).to(dtype)
    w = (0.3 * torch.randn(shape[-1], generator=g)).to(dtype)
    rows, hidden = shape
    xd, wd = x.to(dev), w.to(dev)
    out = torch.empty_like(xd)
    capi.call("ntb200_gemma_rms_norm", ptr(out), ptr(xd), ptr(wd), rows, hidden, hidden, hidden, 1e-6,
              dtype_code(dtype), stream())
    torch.cuda.synchronize()
    _close(out, oracle.gemma_rms_norm(x, w, 1e-6), dtype)
    assert capi.read_device_error(stream()) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(128, 4096), (7, 4095), (3, 40000)])
def test_gemma_fused_add_rms_norm_capi(dtype, shape):
    """Gemma with a residual: the sum is taken in the input dtype (bf16 rounds it before the
    statistics), written back bit-exact; fp16 is rejected (vLLM returns an fp32 residual)."""
    dev = cuda_device()
    g = seeded(18)
    x = torch.randn(shape, generator=g).to(dtype)
    r = torch.randn(shape, generator=g).to(dtype)
    w = (0.3 * torch.randn(shape[-1], generator=g)).to(dtype)
    ref_y, ref_r = oracle.gemma_rms_norm(x, w, 1e-6, r)
    rows, hidden = shape
    xd, rd, wd = x.to(dev), r.to(dev), w.to(dev)
    out = torch.empty_like(xd)
    capi.call("ntb200_gemma_fused_add_rms_norm", ptr(out), ptr(rd), ptr(xd), ptr(wd), rows, hidden, hidden, hidden,
              hidden, 1e-6, dtype_code(dtype), stream())
    torch.cuda.synchronize()
    _close(out, ref_y, dtype)
    assert bits_equal(rd.cpu(), ref_r)
    h = x.to(torch.float16).to(dev)
    with pytest.raises(capi.NtB200Error) as e:
        capi.call("ntb200_gemma_fused_add_rms_norm", ptr(h), ptr(h.clone()), ptr(h), ptr(h[0]), rows, hidden, hidden,
                  hidden, hidden, 1e-6, 2, stream())
    assert e.value.status == -2
    assert capi.read_device_error(stream()) == 0


def test_gemma_rms_norm_matches_vllm_forward_native_through_the_hook(monkeypatch):
    """The GemmaRMSNorm hook (all-b200 config) on a layer with vLLM's GemmaRMSNorm state
    (bf16, with and without a residual) against GemmaRMSNorm.forward_native; the inputs are
    left untouched, as vLLM's native code leaves them, and every call is a kernel hit."""
    from pathlib import Path
    from types import SimpleNamespace

    from vllm.model_executor.layers.layernorm import GemmaRMSNorm

    from vllm_nt._ntops import patching

    root = Path(__file__).resolve().parents[1]
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(root / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml"))
    monkeypatch.setenv("VLLM_NT_ENABLE_STATS", "1")
    patching._reset_usage_state()
    dev = cuda_device()
    g = seeded(19)
    layer = SimpleNamespace(weight=torch.nn.Parameter((0.3 * torch.randn(2048, generator=g)).to(torch.bfloat16).to(dev)),
                            variance_epsilon=1e-6)
    x = torch.randn(33, 2048, generator=g).to(torch.bfloat16).to(dev)
    r = torch.randn(33, 2048, generator=g).to(torch.bfloat16).to(dev)
    x0, r0 = x.clone(), r.clone()
    want = GemmaRMSNorm.forward_native(layer, x.clone())
    got = patching._nt_gemma_rms_norm_forward(layer, x)
    _close(got, want.cpu(), torch.bfloat16)
    want_y, want_r = GemmaRMSNorm.forward_native(layer, x.clone(), r.clone())
    got_y, got_r = patching._nt_gemma_rms_norm_forward(layer, x, r)
    _close(got_y, want_y.cpu(), torch.bfloat16)
    assert torch.equal(got_r, want_r)
    assert torch.equal(x, x0) and torch.equal(r, r0)
    op = patching.get_usage_summary()["operators"]["GemmaRMSNorm"]
    assert op["hits"] == 2 and op["fallbacks"] == 0
    patching._reset_usage_state()


def test_fused_add_rms_norm_in_place_output_aliases_input():
    dev = cuda_device()
    g = seeded(3)
    x = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    r = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    w = torch.randn(4096, generator=g).to(torch.bfloat16)
    ref_y, ref_r = oracle.fused_add_rms_norm(x, r, w, 1e-5)
    xd, rd, wd = x.to(dev), r.to(dev), w.to(dev)
    from vllm_nt._ntops.torch._ext import ops

    ops().fused_add_rms_norm(xd, rd, xd, wd, 1e-5)  # out == x, vLLM's in-place convention
    _close(xd, ref_y, torch.bfloat16)
    assert bits_equal(rd.cpu(), ref_r)


# ------------------------------------------------------------------------------ silu_and_mul


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_silu_and_mul_config_b_capi(dtype):
    """Config (b): input [128, 22016] ~N(0,1) -> [128, 11008]."""
    dev = cuda_device()
    x = torch.randn(128, 22016, generator=seeded(4)).to(dtype)
    xd = x.to(dev)
    out = torch.empty(128, 11008, dtype=dtype, device=dev)
    capi.call("ntb200_silu_and_mul", ptr(out), ptr(xd), 128, 11008, 22016, 11008, dtype_code(dtype), stream())
    torch.cuda.synchronize()
    _close(out, oracle.silu_and_mul(x), dtype)


@pytest.mark.parametrize("shape", [(1, 8192), (32, 8192), (1, 32, 8192), (3, 2002), (70000, 16)])
def test_silu_and_mul_shapes(shape):
    dev = cuda_device()
    x = torch.randn(shape, generator=seeded(5)).to(torch.bfloat16)
    from vllm_nt._ntops.torch.silu import silu_and_mul

    _close(silu_and_mul(x.to(dev)), oracle.silu_and_mul(x), torch.bfloat16)


def test_silu_and_mul_strided_input():
    dev = cuda_device()
    big = torch.randn(8, 3 * 512, generator=seeded(6)).to(torch.bfloat16)
    x = big[:, 256 : 256 + 1024]
    out = torch.empty(8, 512, dtype=torch.bfloat16, device=dev)
    xd = big.to(dev)[:, 256 : 256 + 1024]
    capi.call("ntb200_silu_and_mul", ptr(out), ptr(xd), 8, 512, 1536, 512, 1, stream())
    torch.cuda.synchronize()
    _close(out, oracle.silu_and_mul(x), torch.bfloat16)


# ------------------------------------------------------------------------------ RoPE


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_config_c_bit_exact(dtype):
    """Config (c): q [128, 32, 128], k [128, 8, 128] ~N(0,1), positions U[0, 4096),
    base 10000, rotary_dim 128.  Op-by-op rounding like the native path: bit-exact."""
    dev = cuda_device()
    g = seeded(7)
    q = torch.randn(128, 32 * 128, generator=g).to(dtype)
    k = torch.randn(128, 8 * 128, generator=g).to(dtype)
    pos = torch.randint(0, 4096, (128,), generator=g)
    cache = oracle.build_cos_sin_cache(128, 4096, 10000.0)
    ref_q, ref_k = oracle.rope_neox(pos, q, k, cache, 128, 128)
    qd, kd, posd, cd = q.to(dev), k.to(dev), pos.to(dev), cache.to(dtype).to(dev)
    capi.call("ntb200_rotary_embedding_neox", ptr(posd), 4, ptr(qd), ptr(kd), ptr(cd), 128, 32, 8, 128, 128,
              4096, 128, 1024, 128, 128, 4096, dtype_code(dtype), stream())
    torch.cuda.synchronize()
    assert bits_equal(qd.cpu(), ref_q)
    assert bits_equal(kd.cpu(), ref_k)


def test_rope_partial_rotary_strided_qkv_int32_positions():
    """q/k are views into a fused qkv buffer (vLLM layout), rotary_dim 64 < head 128."""
    dev = cuda_device()
    g = seeded(8)
    t, hq, hk, d = 33, 8, 2, 128
    qkv = torch.randn(t, (hq + 2 * hk) * d, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 2048, (t,), generator=g).to(torch.int32)
    cache = oracle.build_cos_sin_cache(64, 2048, 500000.0)
    q, k = qkv[:, : hq * d], qkv[:, hq * d : (hq + hk) * d]
    ref_q, ref_k = oracle.rope_neox(pos, q, k, cache, d, 64)
    qkvd = qkv.to(dev)
    from vllm_nt._ntops.torch.rotary_emb import rotary_embedding

    qd, kd = qkvd[:, : hq * d], qkvd[:, hq * d : (hq + hk) * d]
    rotary_embedding(pos.to(dev), qd, kd, d, cache.to(torch.bfloat16).to(dev), 64)
    assert bits_equal(qd.cpu().contiguous(), ref_q.contiguous())
    assert bits_equal(kd.cpu().contiguous(), ref_k.contiguous())
    assert torch.equal(qkvd[:, (hq + hk) * d :].cpu(), qkv[:, (hq + hk) * d :])  # v untouched


def test_rope_out_of_range_position_is_flagged_and_skipped():
    dev = cuda_device()
    q = torch.randn(4, 2 * 64, generator=seeded(9)).to(torch.bfloat16)
    cache = oracle.build_cos_sin_cache(64, 16, 10000.0).to(torch.bfloat16)
    pos = torch.tensor([0, 99, 3, 1])
    qd = q.to(dev)
    capi.call("ntb200_rotary_embedding_neox", ptr(pos.to(dev)), 4, ptr(qd), None, ptr(cache.to(dev)), 4, 2, 0,
              64, 64, 128, 64, 0, 0, 64, 16, 1, stream())
    torch.cuda.synchronize()
    assert capi.read_device_error(stream()) & capi.DEVERR_INDEX_RANGE
    assert torch.equal(qd[1].cpu(), q[1])
    ref, _ = oracle.rope_neox(pos[[0]], q[[0]], None, cache.float(), 64, 64)
    assert bits_equal(qd[0].cpu(), ref[0])


# ------------------------------------------------------------------------------ KV store


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_reshape_and_cache_config_bit_exact():
    """num_tokens 4096, 8 KV heads, head 128, block 16, 8192 blocks, distinct random
    slots, zero-filled caches: the whole cache must match the oracle bit for bit."""
    dev = cuda_device()
    g = seeded(10)
    key = torch.randn(4096, 8, 128, generator=g).to(torch.bfloat16)
    value = torch.randn(4096, 8, 128, generator=g).to(torch.bfloat16)
    slots = torch.randperm(8192 * 16, generator=g)[:4096]
    kc = torch.zeros(8192, 16, 8, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    kd, vd, sd = key.to(dev), value.to(dev), slots.to(dev)
    capi.call("ntb200_reshape_and_cache", ptr(kd), ptr(vd), ptr(kc), ptr(vc), ptr(sd), 4, 4096, 8, 128, 16,
              8192 * 16, 1024, 128, 1024, 128, 16 * 1024, 1024, 128, 2, stream())
    torch.cuda.synchronize()
    ek = np.zeros((8192, 16, 8, 128), np.uint16)
    ev = np.zeros_like(ek)
    oracle.reshape_and_cache(_u16(key), _u16(value), ek, ev, slots.numpy())
    assert np.array_equal(_u16(kc.cpu()), ek)
    assert np.array_equal(_u16(vc.cpu()), ev)
    assert capi.read_device_error(stream()) == 0


def test_reshape_and_cache_padding_slots_int32_and_padded_rows():
    """vLLM pads key/value but not the slot mapping; -1 slots are skipped."""
    dev = cuda_device()
    g = seeded(11)
    key = torch.randn(10, 2, 128, generator=g).to(torch.bfloat16)
    value = torch.randn(10, 2, 128, generator=g).to(torch.bfloat16)
    slots = torch.tensor([5, -1, 0, 63, -1, 17], dtype=torch.int32)  # 6 of 10 rows
    kc = torch.zeros(4, 16, 2, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    from vllm_nt._ntops.torch.kv_cache import store_kvcache

    store_kvcache(key.to(dev), value.to(dev), kc, vc, slots.to(dev))
    ek = np.zeros((4, 16, 2, 128), np.uint16)
    ev = np.zeros_like(ek)
    oracle.reshape_and_cache(_u16(key[:6]), _u16(value[:6]), ek, ev, slots.numpy())
    assert np.array_equal(_u16(kc.cpu()), ek) and np.array_equal(_u16(vc.cpu()), ev)


def test_reshape_and_cache_reference_flat_cache_and_narrow_heads():
    """vllm_nt/tests/test_kv_cache.py:26-45: key (3,2,4) into an (8,8) flat cache at
    slots [1,4,6]; 8-byte head rows take the narrow-unit path."""
    dev = cuda_device()
    for dtype in (torch.float16, torch.bfloat16):
        key = torch.randn(3, 2, 4, generator=seeded(12)).to(dtype).to(dev)
        value = torch.randn(3, 2, 4, generator=seeded(13)).to(dtype).to(dev)
        kc = torch.zeros(8, 8, dtype=dtype, device=dev)
        vc = torch.zeros(8, 8, dtype=dtype, device=dev)
        from vllm_nt._ntops.torch.kv_cache import store_kvcache

        store_kvcache(key, value, kc, vc, torch.tensor([1, 4, 6], dtype=torch.int32, device=dev))
        for t, s in enumerate([1, 4, 6]):
            assert torch.equal(kc[s], key[t].reshape(-1)) and torch.equal(vc[s], value[t].reshape(-1))
        assert not kc[[0, 2, 3, 5, 7]].any()


def test_reshape_and_cache_out_of_range_slot_flagged():
    dev = cuda_device()
    key = torch.randn(2, 1, 128, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(2, 16, 1, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([3, 32], device=dev)  # 32 == num_slots
    from vllm_nt._ntops.torch.kv_cache import store_kvcache

    store_kvcache(key, key, kc, vc, slots)
    torch.cuda.synchronize()
    assert capi.read_device_error(stream()) & capi.DEVERR_INDEX_RANGE
    assert torch.equal(kc[0, 3], key[0]) and kc.view(-1).count_nonzero() == 128


# ------------------------------------------------------------------------------ embedding


def test_embedding_gather_bit_exact():
    dev = cuda_device()
    g = seeded(14)
    w = torch.randn(32000, 4096, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 32000, (4096,), generator=g)
    out = torch.empty(4096, 4096, dtype=torch.bfloat16, device=dev)
    wd, idd = w.to(dev), ids.to(dev)
    capi.call("ntb200_embedding", ptr(out), ptr(idd), 4, ptr(wd), 4096, 32000, 4096, 4096, 4096, 2, stream())
    torch.cuda.synchronize()
    assert np.array_equal(_u16(out.cpu()), oracle.embedding(ids.numpy(), _u16(w)))


def test_embedding_reference_case_int32_and_out_of_range():
    """vllm_nt/tests/test_oot.py:135-146 table (32, 16) ids [[0,3,7],[4,1,2]]; plus an id
    past the table, which must give a zero row and the index-range flag."""
    dev = cuda_device()
    w = torch.randn(32, 16, generator=seeded(15)).to(torch.float16).to(dev)
    from vllm_nt._ntops.torch.embedding import embedding

    ids = torch.tensor([[0, 3, 7], [4, 1, 2]], dtype=torch.int32, device=dev)
    assert torch.equal(embedding(ids, w), torch.nn.functional.embedding(ids.long(), w))
    bad = torch.tensor([5, 32, -1], device=dev)
    out = embedding(bad, w)
    torch.cuda.synchronize()
    assert capi.read_device_error(stream()) & capi.DEVERR_INDEX_RANGE
    assert torch.equal(out[0], w[5]) and not out[1:].any()


# ------------------------------------------------------------------ any-rank row layouts


def test_torch_ops_take_any_rank_rows():
    """[batch, tokens, hidden] activations go into the ops without Python reshapes; the
    in-place fused norm (vLLM's CUDA convention) overwrites x and the residual."""
    from vllm_nt._ntops.torch.rms_norm import fused_add_rms_norm, rms_norm
    from vllm_nt._ntops.torch.silu import silu_and_mul

    dev = cuda_device()
    g = seeded(21)
    x = torch.randn(2, 3, 4096, generator=g).to(torch.bfloat16)
    r = torch.randn(2, 3, 4096, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    ref_y, ref_r = oracle.fused_add_rms_norm(x.view(6, 4096), r.view(6, 4096), w, 1e-6)
    xd, rd = x.to(dev), r.to(dev)
    y, res = fused_add_rms_norm(xd, rd, w.to(dev), 1e-6, inplace=True)
    assert y.data_ptr() == xd.data_ptr() and res.data_ptr() == rd.data_ptr() and y.shape == (2, 3, 4096)
    _close(y.view(6, 4096), ref_y, torch.bfloat16)
    assert bits_equal(res.view(6, 4096).cpu(), ref_r)
    _close(rms_norm(x.to(dev), 4096, w.to(dev), 1e-6).view(6, 4096), oracle.rms_norm(x.view(6, 4096), w, 1e-6),
           torch.bfloat16)
    a = torch.randn(2, 5, 2 * 512, generator=g).to(torch.bfloat16)
    out = silu_and_mul(a.to(dev))
    assert out.shape == (2, 5, 512)
    _close(out.view(10, 512), oracle.silu_and_mul(a.view(10, 1024)), torch.bfloat16)


def test_linear_realigns_an_unaligned_activation():
    """x whose base is 8 bytes off a 16-byte boundary and whose row stride is not a
    multiple of 8 elements is copied once into a TMA-legal tensor by the op."""
    from vllm_nt._ntops.torch.linear import linear

    dev = cuda_device()
    g = seeded(22)
    big = torch.randn(5, 44, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(24, 32, generator=g)).to(torch.bfloat16)
    x = big.to(dev)[:, 4:36]
    assert x.data_ptr() % 16 != 0 and x.stride(0) % 8 != 0
    out = linear(x, w.to(dev))
    _close(out, oracle.linear(big[:, 4:36], w), torch.bfloat16)

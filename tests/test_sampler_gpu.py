"""GPU parity of the sampler kernels against the CPU oracle (the reference's sort-based
torch sampler), through the C ABI and through the plugin's hooks on vLLM's own sampler
functions.

Bar: top-k masks are exact.  A top-p mask may differ from the oracle only at logits whose
running probability (fp64, from the smallest logit up) lies within TOP_P_TOL of 1 - p,
where the two fp32 summation orders can legitimately disagree; the row maximum always
survives.  Random samples are exact for the same exponential draws."""

from types import SimpleNamespace

import pytest
import torch

import oracle
from _util import bits_equal, cuda_device, golden, ptr, seeded, stream
from vllm_nt._ntops import capi
from vllm_nt._ntops.torch.sampler import apply_top_k_top_p, random_sample

pytestmark = pytest.mark.gpu

TOP_P_TOL = 2e-4
NEG_INF = float("-inf")
VOCAB = 128256  # Llama-3 vocabulary


def _check_mask(got, logits, k, p):
    """got (CPU) against the oracle's mask of logits under the bar above."""
    ref = oracle.apply_top_k_top_p(logits, k, p)
    if p is None:
        assert bits_equal(got, ref)
        return
    kept_got, kept_ref = got != NEG_INF, ref != NEG_INF
    # survivors keep their logit bit for bit
    assert bits_equal(got[kept_got], logits[kept_got])
    running = oracle.top_p_cumulative(logits, k)
    diff = kept_got ^ kept_ref
    if diff.any():
        gap = (running - (1 - p.double()).unsqueeze(1)).abs()[diff]
        assert float(gap.max()) < TOP_P_TOL, f"{int(diff.sum())} logits differ, max gap {float(gap.max())}"
    rows = torch.arange(logits.shape[0])
    assert kept_got[rows, logits.argmax(dim=-1)].all()


def test_golden_fixture_capi():
    """The reference's own outputs (tests/golden/sampler_f32.npz): top-k alone, top-p
    alone and both, through the C ABI with int64 k; ties at a top-k cut, -inf entries."""
    dev = cuda_device()
    g = golden("sampler_f32")
    logits, k, p = g["logits"], g["k"], g["p"]
    rows, vocab = logits.shape
    for kk, pp, key in ((k, None, "top_k_out"), (None, p, "top_p_out"), (k, p, "top_k_top_p_out")):
        x = logits.to(dev)
        kd = kk.to(dev) if kk is not None else None
        pd = pp.to(dev) if pp is not None else None
        capi.call("ntb200_top_k_top_p", ptr(x), rows, vocab, vocab, ptr(kd), 4, ptr(pd), stream())
        torch.cuda.synchronize()
        _check_mask(x.cpu(), logits, kk, pp)
        if pp is None:
            assert bits_equal(x.cpu(), g[key])


@pytest.mark.parametrize("k_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("b", [8, 64])
def test_llama_vocabulary_batch(k_dtype, b):
    """Rows of a 128256-token vocabulary (8: one cluster of CTAs per row; 64: one CTA per
    row), logit spreads 0.5 .. 8, k from 1 to V (V and V - 1 included), p from 0.3 to 1.0."""
    dev = cuda_device()
    g = seeded(31)
    spread = torch.tensor([0.5, 1.0, 2.0, 3.0, 5.0, 8.0, 1.5, 4.0]).repeat(b // 8).unsqueeze(1)
    logits = torch.randn(b, VOCAB, generator=g) * spread
    k = torch.randint(1, 2000, (b,), generator=g)
    k[::9] = VOCAB
    k[5] = VOCAB - 1
    k[6] = 1
    p = 0.3 + 0.7 * torch.rand(b, generator=g)
    p[::7] = 1.0
    x = logits.to(dev)
    apply_top_k_top_p(x, k.to(k_dtype).to(dev), p.to(dev))
    _check_mask(x.cpu(), logits, k, p)
    only_k = logits.to(dev)
    apply_top_k_top_p(only_k, k.to(k_dtype).to(dev), None)
    _check_mask(only_k.cpu(), logits, k, None)
    only_p = logits.to(dev)
    apply_top_k_top_p(only_p, None, p.to(dev))
    _check_mask(only_p.cpu(), logits, None, p)


def test_odd_vocabulary_strided_rows_and_masked_entries():
    """A 1001-token vocabulary in rows of a wider buffer (row stride 1003: the scalar
    path), rows with -inf entries, a row of -inf only (left as it is) and a row of one
    repeated value (every copy survives top-k)."""
    dev = cuda_device()
    g = seeded(32)
    rows, vocab = 6, 1001
    buf = torch.randn(rows, vocab + 2, generator=g) * 3.0
    buf[1, torch.randperm(vocab, generator=g)[:400]] = NEG_INF
    buf[2, :vocab] = NEG_INF
    buf[3, :vocab] = 0.25
    logits = buf[:, :vocab].clone()
    k = torch.tensor([3, 10, 5, 7, vocab, 1])
    p = torch.tensor([0.9, 0.8, 0.5, 0.9, 0.6, 0.95])
    bd = buf.to(dev)
    apply_top_k_top_p(bd[:, :vocab], k.to(dev), p.to(dev))
    got = bd[:, :vocab].cpu()
    assert bits_equal(bd[:, vocab:].cpu(), buf[:, vocab:])  # the padding columns are untouched
    assert bits_equal(got[2], logits[2])
    assert bits_equal(got[3], logits[3])  # all ties: top-k keeps all, top-p keeps all
    keep = [0, 1, 4, 5]
    _check_mask(got[keep], logits[keep], k[keep], p[keep])


def test_random_sample_golden_and_large_exact():
    """argmax(probs / q) for the fixture's draws (the reference's sample) and for a
    128256-token batch: exact indices."""
    dev = cuda_device()
    g = golden("sampler_f32")
    out = torch.empty(6, dtype=torch.int64, device=dev)
    pd, qd = g["probs"].to(dev), g["q"].to(dev)
    capi.call("ntb200_random_sample", ptr(out), ptr(pd), ptr(qd), 6, 1000, 1000, 1000, stream())
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), g["sample"])

    gen = seeded(33)
    b = 48
    probs = (torch.randn(b, VOCAB, generator=gen) * 3).softmax(dim=-1)
    q = torch.empty(b, VOCAB).exponential_(generator=gen)
    out = torch.empty(b, dtype=torch.int64, device=dev)
    from vllm_nt._ntops.torch._ext import ops

    ops().random_sample(out, probs.to(dev), q.to(dev))
    assert torch.equal(out.cpu(), oracle.random_sample_from_draws(probs, q))


def test_random_sample_ties_nan_and_scalar_path():
    """Equal quotients take the first index; a NaN quotient ranks above every number (the
    first NaN wins), as torch.argmax does; an odd vocabulary takes the scalar path."""
    dev = cuda_device()
    vocab = 1001
    probs = torch.full((3, vocab), 1.0 / vocab)
    q = torch.ones(3, vocab)
    q[0, [17, 500, 900]] = 0.5  # three equal maxima in row 0
    probs[1, 300] = float("nan")
    probs[1, 700] = float("nan")
    q[2, 999] = 0.25
    out = torch.empty(3, dtype=torch.int64, device=dev)
    pd, qd = probs.to(dev), q.to(dev)
    capi.call("ntb200_random_sample", ptr(out), ptr(pd), ptr(qd), 3, vocab, vocab, vocab, stream())
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [17, 300, 999]
    assert torch.equal(out.cpu(), oracle.random_sample_from_draws(probs, q))


def test_plugin_random_sample_draws_like_the_reference():
    """random_sample(probs, generators) with a generator for every row returns exactly the
    index the reference's torch code returns with the same generators on the device."""
    dev = cuda_device()
    gen = seeded(34)
    b = 8
    probs = (torch.randn(b, VOCAB, generator=gen) * 2).softmax(dim=-1).to(dev)

    def gens():
        return {i: torch.Generator(device=dev).manual_seed(70 + i) for i in range(b)}

    got = random_sample(probs, gens())
    q = torch.empty_like(probs)
    for i, generator in gens().items():
        q[i].exponential_(generator=generator)
    assert torch.equal(got.cpu(), oracle.random_sample_from_draws(probs.cpu(), q.cpu()))


def test_vllm_sampler_functions_run_the_kernels(monkeypatch):
    """After registration vLLM's topk_topp_sampler.apply_top_k_top_p / random_sample are the
    plugin's hooks: TopKTopPSampler.forward_native (the path vLLM takes with per-request
    generators) masks and samples on these kernels, with hits counted under b200."""
    from pathlib import Path

    pytest.importorskip("vllm")
    import vllm_nt
    from vllm_nt._ntops import patching

    root = Path(__file__).resolve().parents[1]
    monkeypatch.setenv("VLLM_NT_BACKEND_CONFIG", str(root / "vllm-nt_b200/vllm_nt/configs/all-b200.yaml"))
    vllm_nt.register()
    patching._reset_usage_state()
    from vllm.v1.sample.ops import topk_topp_sampler as tks

    dev = cuda_device()
    g = seeded(35)
    b = 16
    logits = torch.randn(b, VOCAB, generator=g) * 2
    k = torch.randint(1, 100, (b,), generator=g).to(torch.int32)
    p = torch.full((b,), 0.9)
    gens = {i: torch.Generator(device=dev).manual_seed(i) for i in range(b)}
    # forward_native reads only logprobs_mode from the sampler object
    ids, _ = tks.TopKTopPSampler.forward_native(SimpleNamespace(logprobs_mode="raw_logprobs"), logits.to(dev), gens,
                                                k.to(dev), p.to(dev))
    masked = logits.to(dev)
    tks.apply_top_k_top_p(masked, k.to(dev), p.to(dev))
    _check_mask(masked.cpu(), logits, k, p)
    probs = masked.softmax(dim=-1, dtype=torch.float32)
    q = torch.empty_like(probs)
    for i in range(b):
        q[i].exponential_(generator=torch.Generator(device=dev).manual_seed(i))
    assert torch.equal(ids.cpu(), oracle.random_sample_from_draws(probs.cpu(), q.cpu()))
    backends_hits = patching.get_usage_summary()["operators"]
    assert backends_hits["TopKTopP"]["backends"]["b200"]["hits"] == 2
    assert backends_hits["RandomSample"]["backends"]["b200"]["hits"] == 1
    patching._reset_usage_state()

"""GPU parity of the tcgen05 GEMM: out = x W^T (+ bias), bf16/f16 in, fp32 accumulate.

Small M is checked against the CPU oracle; for M >= 1024 the reference is a torch fp32
matmul on the GPU with TF32 disabled (a floating-point kernel's fp32 reference).
Tolerance 2e-2 (rtol = atol) on the 16-bit output."""

import math

import pytest
import torch

import oracle
from _util import cuda_device, dtype_code, ptr, seeded, stream
from vllm_nt._ntops import capi

pytestmark = pytest.mark.gpu
TOL = 2e-2
SHAPES = [(4096, 6144), (4096, 4096), (4096, 28672), (14336, 4096)]


@pytest.fixture(autouse=True)
def _setup():
    cuda_device()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    capi.read_device_error(stream())
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    assert capi.read_device_error(stream()) == 0


def _inputs(m, k, n, seed, dtype=torch.bfloat16, bias=False):
    g = seeded(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (0.02 * torch.randn(n, k, generator=g)).to(dtype)
    b = torch.randn(n, generator=g).to(dtype) if bias else None
    return x, w, b


def _ntb200_linear(x, w, b=None):
    from vllm_nt._ntops.torch.linear import linear

    return linear(x, w, b)


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 128, 256])
def test_linear_small_m_vs_oracle(m, k, n):
    x, w, _ = _inputs(m, k, n, seed=m + k + n)
    out = _ntb200_linear(x.cuda(), w.cuda())
    torch.testing.assert_close(out.float().cpu(), oracle.linear(x, w), rtol=TOL, atol=TOL)


@pytest.mark.parametrize("k,n", SHAPES)
def test_linear_m1024_vs_fp32(k, n):
    x, w, _ = _inputs(1024, k, n, seed=k + n)
    xd, wd = x.cuda(), w.cuda()
    ref = xd.float() @ wd.float().t()
    torch.testing.assert_close(_ntb200_linear(xd, wd).float(), ref, rtol=TOL, atol=TOL)


@pytest.mark.parametrize("k,n", SHAPES)
def test_linear_m2048_cta_pairs_vs_fp32(k, n):
    """M >= 2048 takes the CTA-pair kernel (256 x 256 tiles, tcgen05 cta_group::2)."""
    dev = cuda_device()
    gd = torch.Generator(device=dev).manual_seed(k + n + 1)
    x = torch.randn(2048, k, generator=gd, device=dev, dtype=torch.bfloat16)
    w = 0.02 * torch.randn(n, k, generator=gd, device=dev, dtype=torch.bfloat16)
    ref = x.float() @ w.float().t()
    torch.testing.assert_close(_ntb200_linear(x, w).float(), ref, rtol=TOL, atol=TOL)


@pytest.mark.parametrize("k,n", SHAPES)
def test_linear_m8192_row_subset(k, n):
    """The M = 8192 benchmark size of every projection (CTA-pair kernel, grouped
    rasterisation): 128 seeded rows, which land in many different 256-row tiles, against
    an fp32 reference of those rows."""
    dev = cuda_device()
    gd = torch.Generator(device=dev).manual_seed(3 + k + n)
    x = torch.randn(8192, k, generator=gd, device=dev, dtype=torch.bfloat16)
    w = 0.02 * torch.randn(n, k, generator=gd, device=dev, dtype=torch.bfloat16)
    out = _ntb200_linear(x, w)
    rows = torch.randperm(8192, generator=seeded(4 + n))[:128].to(dev)
    ref = x[rows].float() @ w.float().t()
    torch.testing.assert_close(out[rows].float(), ref, rtol=TOL, atol=TOL)


@pytest.mark.parametrize("m,k,n", [(200, 72, 300), (5, 32, 12), (129, 4096, 257), (1, 8, 8), (300, 136, 257), (1000, 4096, 640),
                                   (2100, 136, 520), (2048, 64, 256), (2304, 4096, 200), (4352, 6144, 520),
                                   # 256-row weight tiles (decode batches): K split over a cluster with
                                   # ragged N and K; one and two token tiles without a split
                                   (100, 4104, 6200), (3, 264, 6400), (200, 136, 37000), (129, 72, 36000)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_tails_and_bias_capi(m, k, n, dtype):
    x, w, b = _inputs(m, k, n, seed=m * 7 + n, dtype=dtype, bias=True)
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    out = torch.full((m, n), 3.0, dtype=dtype, device="cuda")
    capi.call("ntb200_linear", ptr(out), ptr(xd), ptr(wd), ptr(bd), m, n, k, k, k, n, None, 0,
              dtype_code(dtype), stream())
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), oracle.linear(x, w, b), rtol=TOL, atol=TOL)


def test_linear_strided_output_and_reference_cases():
    """vllm_nt/tests/test_oot.py:121-162: matmul (64x128)(128x32) and linear with bias on
    (2,3,16) x (8,16)."""
    from vllm_nt._ntops.oot_support import linear
    from vllm_nt._ntops.torch.linear import matmul

    for dtype in (torch.float16, torch.bfloat16):
        g = seeded(5)
        lhs = torch.randn(64, 128, generator=g).to(dtype)
        rhs = torch.randn(128, 32, generator=g).to(dtype)
        torch.testing.assert_close(matmul(lhs.cuda(), rhs.cuda()).float().cpu(), lhs.float() @ rhs.float(),
                                   rtol=5e-2, atol=5e-2)
        x = torch.randn(2, 3, 16, generator=g).to(dtype)
        w = torch.randn(8, 16, generator=g).to(dtype)
        b = torch.randn(8, generator=g).to(dtype)
        ref = torch.nn.functional.linear(x.float(), w.float(), b.float())
        torch.testing.assert_close(linear(x.cuda(), w.cuda(), b.cuda()).float().cpu(), ref, rtol=5e-2, atol=5e-2)


def test_linear_rejects_unaligned_and_fp32():
    x = torch.randn(4, 12, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(8, 12, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(4, 8, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(capi.NtB200Error) as e:  # row stride 12 elements = 24 bytes: not 16-aligned
        capi.call("ntb200_linear", ptr(out), ptr(x), ptr(w), None, 4, 8, 12, 12, 12, 8, None, 0, 1, stream())
    assert e.value.status == -3
    with pytest.raises(capi.NtB200Error) as e:
        capi.call("ntb200_linear", ptr(out), ptr(x), ptr(w), None, 4, 8, 12, 12, 12, 8, None, 0, 0, stream())
    assert e.value.status == -2


@pytest.mark.parametrize("m,k,i", [(1, 4096, 14336), (16, 4096, 14336), (256, 4096, 14336), (200, 72, 300),
                                   (1000, 4096, 1792), (2048, 4096, 14336), (2300, 136, 520), (100, 136, 14400)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_silu_and_mul_fused_capi(m, k, i, dtype):
    """Fused gate_up + SiluAndMul over every path (256-row gate/up tiles and swap-AB at
    M <= 256, single CTA, CTA pairs) against the oracle's unfused pair; I not a multiple of
    the tile covers the tail."""
    x, w, _ = _inputs(m, k, 2 * i, seed=m + k + i)
    xd, wd = x.to(dtype).cuda(), w.to(dtype).cuda()
    out = torch.full((m, i), 5.0, dtype=dtype, device="cuda")
    capi.call("ntb200_linear_silu_and_mul", ptr(out), ptr(xd), ptr(wd), m, i, k, k, k, i, dtype_code(dtype), stream())
    torch.cuda.synchronize()
    ref = oracle.silu_and_mul(oracle.linear(x.to(dtype), w.to(dtype)).to(dtype))
    torch.testing.assert_close(out.float().cpu(), ref.float(), rtol=TOL, atol=TOL)


def test_linear_silu_and_mul_decode_batch_matches_unfused_pair_exactly():
    """At a decode batch (M = 200, I = 14336) both the fused op and the unfused GEMM use
    256-row weight tiles without a K split, so each gate and up value is the same dot
    product in the same order: the two agree bit for bit."""
    from vllm_nt._ntops.torch.linear import linear, linear_silu_and_mul
    from vllm_nt._ntops.torch.silu import silu_and_mul

    dev = cuda_device()
    gd = torch.Generator(device=dev).manual_seed(78)
    x = torch.randn(200, 4096, generator=gd, device=dev, dtype=torch.bfloat16)
    w = 0.02 * torch.randn(2 * 14336, 4096, generator=gd, device=dev, dtype=torch.bfloat16)
    assert torch.equal(linear_silu_and_mul(x, w), silu_and_mul(linear(x, w)))


def test_linear_silu_and_mul_matches_unfused_pair_exactly():
    """The fused epilogue rounds where the unfused pair does: with the same GEMM
    decomposition (CTA pairs at M = 2048) the two agree bit for bit."""
    from vllm_nt._ntops.torch.linear import linear, linear_silu_and_mul
    from vllm_nt._ntops.torch.silu import silu_and_mul

    dev = cuda_device()
    gd = torch.Generator(device=dev).manual_seed(77)
    x = torch.randn(2048, 4096, generator=gd, device=dev, dtype=torch.bfloat16)
    w = 0.02 * torch.randn(2 * 1024, 4096, generator=gd, device=dev, dtype=torch.bfloat16)
    fused = linear_silu_and_mul(x, w)
    unfused = silu_and_mul(linear(x, w))
    assert torch.equal(fused, unfused)


@pytest.mark.parametrize("m,k,v", [(1, 4096, 32000), (7, 512, 32037), (256, 4096, 32000), (300, 512, 5000),
                                   (64, 136, 1000)])
def test_linear_argmax_matches_argmax_of_our_logits(m, k, v):
    """Fused LM head + greedy argmax == torch.argmax of the logits the unfused GEMM writes
    (same per-logit accumulation, logits compared at bf16, first index on ties)."""
    from vllm_nt._ntops.torch.linear import linear, linear_argmax

    dev = cuda_device()
    gd = torch.Generator(device=dev).manual_seed(m + k + v)
    x = torch.randn(m, k, generator=gd, device=dev, dtype=torch.bfloat16)
    w = 0.05 * torch.randn(v, k, generator=gd, device=dev, dtype=torch.bfloat16)
    got = linear_argmax(x, w)
    want = torch.argmax(linear(x, w), dim=-1)
    assert torch.equal(got, want)


def test_linear_argmax_ties_take_the_first_index():
    from vllm_nt._ntops.torch.linear import linear_argmax

    dev = cuda_device()
    x = torch.ones(3, 64, device=dev, dtype=torch.bfloat16)
    w = torch.zeros(40000, 64, device=dev, dtype=torch.bfloat16)
    w[[5, 17, 39999]] = 1.0       # three equal maxima for every row
    w[33000] = -2.0
    assert linear_argmax(x, w).tolist() == [5, 5, 5]
    w[39999] = 2.0
    assert linear_argmax(x, w).tolist() == [39999, 39999, 39999]


@pytest.fixture(scope="module")
def lm_head_case():
    """Llama-3 LM head: V = 128256, K = 4096, bf16, x ~N(0,1), W ~N(0,0.02); 256 token rows.
    Rows 100 and 128000 of W (different vocabulary tiles) are made equal and larger than
    every other logit of token row 3, a deliberate tie across two tiles.  The oracle's fp32
    logits of all 256 rows are computed once on the CPU."""
    g = seeded(2026)
    x = torch.randn(256, 4096, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(128256, 4096, generator=g)).to(torch.bfloat16)
    tie = (0.05 * torch.sign(x[3].float())).to(torch.bfloat16)
    w[100] = tie
    w[128000] = tie
    ids, logits = oracle.linear_argmax(x, w)
    return x, w, w.cuda(), ids, logits


@pytest.mark.parametrize("m", [1, 16, 128, 256])
def test_linear_argmax_lm_head_vs_oracle(lm_head_case, m):
    """ntb200_linear_argmax at the LM-head shape against the oracle's greedy token (first
    index of the largest bf16-rounded fp32 logit).  A different index is accepted only where
    the two candidates' oracle logits lie within one bf16 ulp of each other (the GEMM's own
    fp32 accumulation order can round such a pair apart), and such rows must be rare; the
    tie across tiles must resolve to the first index."""
    x, w, wd, ids, logits = lm_head_case
    from vllm_nt._ntops.torch.linear import linear_argmax

    got = linear_argmax(x[:m].cuda(), wd).cpu()
    want = ids[:m]
    diff = (got != want).nonzero().flatten().tolist()
    for r in diff:
        top = float(logits[r, want[r]])
        ulp = 2.0 ** (math.floor(math.log2(abs(top))) - 7)
        assert abs(float(logits[r, got[r]]) - top) <= ulp, (r, int(got[r]), int(want[r]))
    assert len(diff) <= max(1, m // 50)
    if m > 3:
        assert int(got[3]) == 100 and int(want[3]) == 100


def test_linear_small_m_is_deterministic_and_graph_replayable():
    """The split-K partials are summed in a fixed order, so repeated calls give the same
    bits; a CUDA graph of the torch op replays correctly several times in a row on new
    inputs."""
    from vllm_nt._ntops.torch.linear import linear

    x, w, _ = _inputs(256, 4096, 6144, seed=91)
    xd, wd = x.cuda(), w.cuda()
    first = linear(xd, wd)
    for _ in range(3):
        assert torch.equal(linear(xd, wd), first)
    torch.testing.assert_close(first.float().cpu(), oracle.linear(x, w), rtol=TOL, atol=TOL)
    out = torch.empty_like(first)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out.copy_(linear(xd, wd))
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out.copy_(linear(xd, wd))
    for i in range(4):
        out.zero_()
        xd.copy_((x * (i + 1)).cuda())
        graph.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), oracle.linear(x * (i + 1), w), rtol=TOL, atol=TOL * (i + 1))


@pytest.mark.parametrize("m", [1, 5, 16])
@pytest.mark.parametrize("k,n", [(4096, 6144), (4096, 28672), (14336, 4096), (1032, 700)])
@pytest.mark.parametrize("with_residual", [False, True])
def test_rms_norm_linear_vs_oracle(m, k, n, with_residual):
    """RMSNorm (after the residual add) formed as the decode GEMM's input: out against the
    oracle's restatement of the fused rounding points (split and unsplit K, ragged N and K),
    the new residual bit for bit against the oracle's, and out at least as close to the
    unrounded fp64 value as our two separate kernels (the reference's op order) are."""
    from vllm_nt._ntops.torch.linear import linear, rms_norm_linear
    from vllm_nt._ntops.torch.rms_norm import fused_add_rms_norm, rms_norm

    g = seeded(m * 31 + k + n + with_residual)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    res = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, generator=g)).to(torch.bfloat16)
    eps = 1e-5
    xd, rd, gd, wd = x.cuda(), res.cuda(), gamma.cuda(), w.cuda()
    ref, res_ref = oracle.rms_norm_linear(x, gamma, eps, w, res if with_residual else None)
    if with_residual:
        out, new_res = rms_norm_linear(xd, gd, eps, wd, rd)
        assert torch.equal(new_res.cpu(), res_ref)
        assert torch.equal(rd.cpu(), res)  # the input residual is left as it was
        h2, _ = fused_add_rms_norm(xd, rd, gd, eps)
    else:
        out = rms_norm_linear(xd, gd, eps, wd)
        h2 = rms_norm(xd, k, gd, eps)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=TOL, atol=TOL)
    exact = oracle.rms_norm_linear_exact(x, gamma, eps, w, res if with_residual else None)
    err = (out.cpu().double() - exact).pow(2).mean().sqrt()
    err_pair = (linear(h2, wd).cpu().double() - exact).pow(2).mean().sqrt()
    assert err <= 1.02 * err_pair, (err.item(), err_pair.item())


def test_rms_norm_linear_rejects_large_batches_and_aliasing():
    x = torch.randn(17, 256, device="cuda", dtype=torch.bfloat16)
    g = torch.ones(256, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(512, 256, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(17, 512, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(capi.NtB200Error) as e:  # more than 16 rows
        capi.call("ntb200_rms_norm_linear", ptr(out), None, ptr(x), None, ptr(g), 1e-5, ptr(w), 17, 512, 256,
                  256, 0, 0, 256, 512, 1, stream())
    assert e.value.status == -6
    r = torch.randn(4, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(capi.NtB200Error) as e:  # residual_out aliasing the residual
        capi.call("ntb200_rms_norm_linear", ptr(out), ptr(r), ptr(x), ptr(r), ptr(g), 1e-5, ptr(w), 4, 512, 256,
                  256, 256, 256, 256, 512, 1, stream())
    assert e.value.status == -1

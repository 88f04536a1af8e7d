"""The selection rule of the top-k/top-p kernel (csrc/sampler.cu), restated in numpy, gives
the reference's sort-based mask (oracle.apply_top_k_top_p).  CPU only: this checks the
design -- cuts found by three radix digits (11, 11 and 10 bits) over order-preserving
keys, top-k by counts from the top, top-p by probability mass from the bottom -- not the
CUDA code, whose parity the GPU tests check.

The restatement follows the kernel step for step: the top-k pass picks the bin holding the
k-th largest key; the top-p pass picks the smallest non-empty bin whose inclusive mass,
added to the mass below it, exceeds 1 - p (else the largest non-empty bin); survivors are
the logits >= t_k whose key is >= the top-p cut."""

import numpy as np
import pytest
import torch

import oracle
from _util import golden

SHIFT = (21, 10, 0)
DIGIT = (0x7FF, 0x7FF, 0x3FF)
PREFIX = (0x0, 0xFFE00000, 0xFFFFFC00)


def _keys(x: np.ndarray) -> np.ndarray:
    b = x.view(np.uint32)
    return np.where(b & 0x80000000, ~b, b ^ 0x80000000).astype(np.uint32)


def _value(u: int) -> np.float32:
    b = (u ^ 0x80000000) if (u & 0x80000000) else (~u & 0xFFFFFFFF)
    return np.array([b], np.uint32).view(np.float32)[0]


def _top_k_cut(u: np.ndarray, k: int) -> np.float32:
    remaining, prefix = k, 0
    for d in range(3):
        sel = (u & PREFIX[d]) == prefix
        count = np.bincount((u[sel] >> SHIFT[d]) & DIGIT[d], minlength=2048)
        above = count.sum() - np.cumsum(count)  # keys in bins above each bin
        b = int(np.nonzero((count > 0) & (above < remaining) & (remaining <= above + count))[0][0])
        remaining -= int(above[b])
        prefix |= b << SHIFT[d]
    return _value(prefix)


def _top_p_cut(x: np.ndarray, u: np.ndarray, t_k: np.float32, p: float) -> int:
    keep = x >= t_k
    e = np.exp((x - x.max()).astype(np.float32)).astype(np.float32)
    w = (e / np.float32(e[keep].astype(np.float64).sum())).astype(np.float32)
    target = float(np.float32(1.0) - np.float32(p))
    base, prefix = 0.0, 0
    for d in range(3):
        sel = keep & ((u & PREFIX[d]) == prefix)
        bins = (u[sel] >> SHIFT[d]) & DIGIT[d]
        count = np.bincount(bins, minlength=2048)
        mass = np.bincount(bins, weights=w[sel].astype(np.float64), minlength=2048)
        incl = np.cumsum(mass)
        hit = np.nonzero((count > 0) & (target < base + incl))[0]
        b = int(hit[0]) if hit.size else int(np.nonzero(count)[0].max())
        base += incl[b] - mass[b]
        prefix |= b << SHIFT[d]
    return prefix


def radix_mask(logits: torch.Tensor, k: torch.Tensor | None, p: torch.Tensor | None) -> torch.Tensor:
    out = []
    for r in range(logits.shape[0]):
        x = logits[r].numpy().astype(np.float32)
        u = _keys(x)
        vocab = x.size
        t_k = np.float32(-np.inf)
        if k is not None and min(max(int(k[r]), 1), vocab) < vocab:
            t_k = _top_k_cut(u, min(max(int(k[r]), 1), vocab))
        cut = 0
        if p is not None and x.max() != -np.inf:
            cut = _top_p_cut(x, u, t_k, float(p[r]))
        out.append(np.where((x >= t_k) & (u >= np.uint32(cut)), x, np.float32(-np.inf)))
    return torch.from_numpy(np.stack(out))


def test_rule_reproduces_the_reference_fixture():
    g = golden("sampler_f32")
    for k, p, key in ((g["k"], None, "top_k_out"), (None, g["p"], "top_p_out"), (g["k"], g["p"], "top_k_top_p_out")):
        assert torch.equal(radix_mask(g["logits"], k, p), g[key])


@pytest.mark.parametrize("seed", [0, 1])
def test_rule_matches_the_sort_based_mask_on_full_vocabulary_rows(seed):
    """Six rows of the Llama-3 vocabulary (128256) over spreads 0.5 .. 8 and cuts from
    k = 1 to a top-p set of tens of thousands of logits."""
    gen = torch.Generator().manual_seed(seed)
    vocab = 128256
    logits = torch.randn(6, vocab, generator=gen) * torch.tensor([0.5, 1.0, 2.0, 3.0, 5.0, 8.0]).unsqueeze(1)
    k = torch.tensor([1, 20, 1000, vocab, 5000, vocab - 1])
    p = torch.tensor([0.9, 0.95, 0.5, 0.8, 0.99, 1.0])
    got = radix_mask(logits, k, p)
    ref = oracle.apply_top_k_top_p(logits, k, p)
    diff = (got != float("-inf")) ^ (ref != float("-inf"))
    if diff.any():  # only at logits whose running mass is within summation error of 1 - p
        running = oracle.top_p_cumulative(logits, k)
        assert float((running - (1 - p.double()).unsqueeze(1)).abs()[diff].max()) < 2e-4
    assert torch.equal(radix_mask(logits, k, None), oracle.apply_top_k_top_p(logits, k, None))


def test_tie_run_straddling_the_top_p_cut_is_kept_whole():
    """The one designed difference from the reference: 100 equal logits whose running mass
    crosses 1 - p.  The reference keeps the part of the run its sort puts last; the radix
    rule, which compares values, keeps every member of the run (a superset: nothing the
    reference keeps is dropped)."""
    logits = torch.full((1, 200), -2.0)
    logits[0, 100:] = 0.5  # the run: 100 copies, holding nearly all of the mass
    p = torch.tensor([0.5])
    got = radix_mask(logits, None, p)
    ref = oracle.apply_top_k_top_p(logits, None, p)
    kept_got, kept_ref = got != float("-inf"), ref != float("-inf")
    assert int(kept_got.sum()) == 100 and bool(kept_got[0, 100:].all())
    assert 0 < int(kept_ref.sum()) < 100
    assert not (kept_ref & ~kept_got).any()

"""Generates tests/golden/*.npz: small seeded inputs and the outputs of the REAL reference
implementations, used to pin the CPU oracle (oracle/ops.py).

Run on a CPU machine with vLLM 0.22 importable and a checkout of the reference:
    python tests/golden/make_golden.py --reference <vllm-nt checkout> [--only main|f16|gemma|sampler]

Sources of truth per op:
  rms_norm / fused_add_rms_norm  vllm.ir.ops.rms_norm / fused_add_rms_norm (native)
  gemma_rms_norm                 vllm GemmaRMSNorm.forward_native (with and without a residual)
  silu_and_mul                   vllm SiluAndMul.forward_native
  rope (NeoX)                    vllm RotaryEmbedding.forward_static with the cache of
                                 RotaryEmbeddingBase._compute_cos_sin_cache
  kv store                       torch index_put at [slot // bs, slot % bs], slot < 0 skipped
                                 (the reference's torch store, vllm_nt/_ntops/patching.py:1752-1770)
  embedding                      torch.nn.functional.embedding
  paged decode                   gather + torch scaled_dot_product_attention per sequence
                                 (the reference's oracle, vllm_nt/tests/test_attention.py:41-102)
  linear                         torch.nn.functional.linear in fp32
  sampler (top-k / top-p, random the reference's own torch sampler, vllm_nt/_ntops/torch/sampler.py,
  sample)                        loaded by file path from the read-only reference checkout (it
                                 imports only torch), and vLLM's apply_top_k_top_p_pytorch
bf16 tensors are stored as their uint16 bit patterns (key suffix ``__bf16``).
``--only sampler`` / ``--only f16`` regenerate just the sampler / the fp16 fixtures.
"""

from __future__ import annotations

import itertools
import math
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn.functional as F

OUT = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> tuple[str, np.ndarray]:
    if t.dtype == torch.bfloat16:
        return "__bf16", t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return "", t.contiguous().numpy()


def save(name: str, **tensors: torch.Tensor) -> None:
    arrays = {}
    for key, t in tensors.items():
        suffix, arr = _np(t)
        arrays[key + suffix] = arr
    np.savez_compressed(OUT / f"{name}.npz", **arrays)


def main() -> None:
    from vllm import ir
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding, RotaryEmbeddingBase

    g = torch.Generator().manual_seed(20261201)

    for dtype, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        x = torch.randn(4, 512, generator=g).to(dtype)
        r = torch.randn(4, 512, generator=g).to(dtype)
        w = (1.0 + 0.1 * torch.randn(512, generator=g)).to(dtype)
        y, res = ir.ops.fused_add_rms_norm(x.clone(), r.clone(), w, 1e-6)
        y0 = ir.ops.rms_norm(x.clone(), w, 1e-6)
        save(f"rms_norm_{tag}", x=x, residual=r, weight=w, out=y, residual_out=res, out_plain=y0)

        xs = torch.randn(4, 2 * 256, generator=g).to(dtype)
        save(f"silu_and_mul_{tag}", x=xs, out=SiluAndMul.forward_native(xs.clone()))

        head, rot, max_pos, base = 64, 64, 128, 10000.0
        cache = RotaryEmbeddingBase._compute_cos_sin_cache(
            type("C", (), {"rotary_dim": rot, "base": base, "max_position_embeddings": max_pos,
                           "_compute_inv_freq": lambda self, b: RotaryEmbeddingBase._compute_inv_freq(self, b)})()
        )
        pos = torch.randint(0, max_pos, (6,), generator=g)
        q = torch.randn(6, 4 * head, generator=g).to(dtype)
        k = torch.randn(6, 2 * head, generator=g).to(dtype)
        qo, ko = RotaryEmbedding.forward_static(pos, q.clone(), k.clone(), head, rot, cache.to(dtype), True)
        # partial rotary (rotary_dim 32 < head_size 64): a 32-wide cos|sin table
        cache32 = torch.cat((cache[:, :16], cache[:, 32:48]), dim=-1)
        qp, kp = RotaryEmbedding.forward_static(pos, q.clone(), k.clone(), head, 32, cache32.to(dtype), True)
        save(f"rope_{tag}", positions=pos, query=q, key=k, cos_sin_cache=cache, query_out=qo, key_out=ko,
             cos_sin_cache_rot32=cache32, query_out_rot32=qp, key_out_rot32=kp)

        xl = torch.randn(5, 32, generator=g).to(dtype)
        wl = (0.02 * torch.randn(12, 32, generator=g)).to(dtype)
        bl = torch.randn(12, generator=g).to(dtype)
        save(f"linear_{tag}", x=xl, weight=wl, bias=bl,
             out=F.linear(xl.float(), wl.float(), bl.float()))

    # KV store (bf16, byte copy)
    key = torch.randn(5, 2, 16, generator=g).to(torch.bfloat16)
    value = torch.randn(5, 2, 16, generator=g).to(torch.bfloat16)
    kc = torch.zeros(8, 4, 2, 16, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([3, -1, 17, 30, 8], dtype=torch.int64)
    valid = slots >= 0
    s = slots[valid]
    kc2, vc2 = kc.clone(), vc.clone()
    kc2[s // 4, s % 4] = key[valid]
    vc2[s // 4, s % 4] = value[valid]
    save("kv_store_bf16", key=key, value=value, slot_mapping=slots, key_cache_out=kc2, value_cache_out=vc2)

    # embedding
    wt = torch.randn(32, 16, generator=g).to(torch.bfloat16)
    ids = torch.tensor([[0, 3, 7], [4, 1, 31]], dtype=torch.int64)
    save("embedding_bf16", weight=wt, ids=ids, out=F.embedding(ids, wt))

    # paged decode: B=3, Hq=4, Hkv=2, D=16, bs=4, ctx [1, 5, 9]
    hq, hkv, d, bs, nb = 4, 2, 16, 4, 12
    qd = torch.randn(3, hq, d, generator=g).to(torch.bfloat16)
    kcd = torch.randn(nb, bs, hkv, d, generator=g).to(torch.bfloat16)
    vcd = torch.randn(nb, bs, hkv, d, generator=g).to(torch.bfloat16)
    seq = torch.tensor([1, 5, 9], dtype=torch.int32)
    table = torch.randperm(nb, generator=g)[:9].reshape(3, 3).to(torch.int32)
    outs = []
    for b in range(3):
        n = int(seq[b])
        ks, vs, rem = [], [], n
        for blk in table[b].tolist():
            if rem <= 0:
                break
            take = min(bs, rem)
            ks.append(kcd[blk, :take])
            vs.append(vcd[blk, :take])
            rem -= take
        kk = torch.cat(ks).float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0).unsqueeze(0)
        vv = torch.cat(vs).float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0).unsqueeze(0)
        qq = qd[b].float().unsqueeze(0).unsqueeze(2)  # [1, Hq, 1, D]
        o = F.scaled_dot_product_attention(qq, kk, vv, scale=1.0 / math.sqrt(d))
        outs.append(o[0, :, 0, :])
    save("paged_decode_bf16", query=qd, key_cache=kcd, value_cache=vcd, seq_lens=seq, block_table=table,
         out=torch.stack(outs))

    # varlen prefill over a paged cache: Hq=4, Hkv=2, D=16, bs=4; (q_len, ctx) per sequence
    # (3, 3) a plain prompt, (2, 7) a prompt after a 5-token cached prefix, (1, 6) a decode
    # row, (0, 4) no queries; causal, aligned to the end of each context (an explicit mask,
    # since SDPA's is_causal aligns to the start)
    hq, hkv, d, bs, nb = 4, 2, 16, 4, 12
    qlens, ctxs = [3, 2, 1, 0], [3, 7, 6, 4]
    cu_q = torch.tensor([0] + list(itertools.accumulate(qlens)), dtype=torch.int32)
    qp = torch.randn(int(cu_q[-1]), hq, d, generator=g).to(torch.bfloat16)
    kcp = torch.randn(nb, bs, hkv, d, generator=g).to(torch.bfloat16)
    vcp = torch.randn(nb, bs, hkv, d, generator=g).to(torch.bfloat16)
    seqp = torch.tensor(ctxs, dtype=torch.int32)
    tablep = torch.randperm(nb, generator=g)[:8].reshape(4, 2).to(torch.int32)
    outp = torch.zeros(int(cu_q[-1]), hq, d)
    for b, (ql, n) in enumerate(zip(qlens, ctxs)):
        if ql == 0:
            continue
        ids = tablep[b].long()
        kk = kcp[ids].reshape(-1, hkv, d)[:n].float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)
        vv = vcp[ids].reshape(-1, hkv, d)[:n].float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)
        qq = qp[int(cu_q[b]) : int(cu_q[b + 1])].float().transpose(0, 1)  # [Hq, q_len, D]
        mask = torch.ones(ql, n, dtype=torch.bool).tril(diagonal=n - ql)
        o = F.scaled_dot_product_attention(qq[None], kk[None], vv[None], attn_mask=mask, scale=1.0 / math.sqrt(d))
        outp[int(cu_q[b]) : int(cu_q[b + 1])] = o[0].transpose(0, 1)
    save("paged_prefill_bf16", query=qp, key_cache=kcp, value_cache=vcp, query_start_loc=cu_q, seq_lens=seqp,
         block_table=tablep, out=outp)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


def half_fixtures() -> None:
    """fp16 counterparts of the RMS-norm, SiluAndMul and RoPE fixtures (vLLM's native code
    on fp16 inputs), from their own generator so the other fixtures stay as they are."""
    from vllm import ir
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding, RotaryEmbeddingBase

    g = torch.Generator().manual_seed(20261203)
    dtype = torch.float16
    x = torch.randn(4, 512, generator=g).to(dtype)
    r = torch.randn(4, 512, generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(512, generator=g)).to(dtype)
    y, res = ir.ops.fused_add_rms_norm(x.clone(), r.clone(), w, 1e-6)
    y0 = ir.ops.rms_norm(x.clone(), w, 1e-6)
    save("rms_norm_f16", x=x, residual=r, weight=w, out=y, residual_out=res, out_plain=y0)
    xs = torch.randn(4, 2 * 256, generator=g).to(dtype)
    save("silu_and_mul_f16", x=xs, out=SiluAndMul.forward_native(xs.clone()))
    head, rot, max_pos, base = 64, 64, 128, 10000.0
    cache = RotaryEmbeddingBase._compute_cos_sin_cache(
        type("C", (), {"rotary_dim": rot, "base": base, "max_position_embeddings": max_pos,
                       "_compute_inv_freq": lambda self, b: RotaryEmbeddingBase._compute_inv_freq(self, b)})()
    )
    pos = torch.randint(0, max_pos, (6,), generator=g)
    q = torch.randn(6, 4 * head, generator=g).to(dtype)
    k = torch.randn(6, 2 * head, generator=g).to(dtype)
    qo, ko = RotaryEmbedding.forward_static(pos, q.clone(), k.clone(), head, rot, cache.to(dtype), True)
    cache32 = torch.cat((cache[:, :16], cache[:, 32:48]), dim=-1)
    qp, kp = RotaryEmbedding.forward_static(pos, q.clone(), k.clone(), head, 32, cache32.to(dtype), True)
    save("rope_f16", positions=pos, query=q, key=k, cos_sin_cache=cache, query_out=qo, key_out=ko,
         cos_sin_cache_rot32=cache32, query_out_rot32=qp, key_out_rot32=kp)


def gemma_fixture() -> None:
    """GemmaRMSNorm.forward_native (vLLM) in fp32, bf16 and fp16, with and without a
    residual: (1 + w) in fp32, the product rounded once, the bf16 residual sum rounded to
    bf16 before the statistics, the fp16 residual sum kept in fp32."""
    from vllm.model_executor.layers.layernorm import GemmaRMSNorm

    g = torch.Generator().manual_seed(20261204)
    arrays = {}
    for dtype, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16"), (torch.float16, "f16")):
        # forward_native reads only weight and variance_epsilon off the layer (constructing
        # a CustomOp needs a vLLM config)
        layer = SimpleNamespace(weight=torch.nn.Parameter((0.3 * torch.randn(512, generator=g)).to(dtype)),
                                variance_epsilon=1e-6)
        x = torch.randn(5, 512, generator=g).to(dtype)
        r = torch.randn(5, 512, generator=g).to(dtype)
        out_plain = GemmaRMSNorm.forward_native(layer, x.clone())
        out, res = GemmaRMSNorm.forward_native(layer, x.clone(), r.clone())
        arrays.update({f"{tag}_x": x, f"{tag}_residual": r, f"{tag}_weight": layer.weight.data, f"{tag}_out_plain": out_plain,
                       f"{tag}_out": out, f"{tag}_residual_out": res})
    save("gemma_rms_norm", **arrays)


def _reference_sampler_path() -> Path:
    """The reference's torch sampler module: ``--reference DIR`` (a vllm-nt checkout) or
    the VLLM_NT_REFERENCE environment variable."""
    import os
    import sys

    root = None
    if "--reference" in sys.argv:
        root = sys.argv[sys.argv.index("--reference") + 1]
    root = root or os.environ.get("VLLM_NT_REFERENCE")
    if not root:
        raise SystemExit("the sampler fixture needs the reference checkout: --reference DIR or VLLM_NT_REFERENCE=DIR")
    return Path(root) / "vllm_nt" / "_ntops" / "torch" / "sampler.py"


def sampler_fixture() -> None:
    """Six rows over a 1000-token vocabulary: logits of spread 1, 2, 5 and 0.5, one row with
    a run of -inf entries (logits processors mask tokens that way), one with ties at the
    top-k cut; per-row k (1 .. V) and p (0.1 .. 1.0).  Outputs of the reference's
    apply_top_k_top_p for k alone, p alone and both, vLLM's own native function for both,
    and the reference's random_sample with a seeded generator for every row (so the
    exponential draws q are fixed and stored)."""
    import importlib.util

    from vllm.v1.sample.ops.topk_topp_sampler import apply_top_k_top_p_pytorch

    spec = importlib.util.spec_from_file_location("reference_sampler", _reference_sampler_path())
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)

    g = torch.Generator().manual_seed(20261202)
    rows, vocab = 6, 1000
    scale = torch.tensor([1.0, 2.0, 5.0, 0.5, 2.0, 3.0]).unsqueeze(1)
    logits = torch.randn(rows, vocab, generator=g) * scale
    logits[4, torch.randperm(vocab, generator=g)[:300]] = float("-inf")
    logits[5, :7] = logits[5].sort(descending=True).values[9]  # 7 copies of the 10th-largest value
    k = torch.tensor([1, 5, 50, vocab, 200, 10], dtype=torch.int64)
    p = torch.tensor([0.9, 0.5, 0.95, 0.8, 1.0, 0.1], dtype=torch.float32)
    topk = ref.apply_top_k_top_p(logits.clone(), k, None)
    topp = ref.apply_top_k_top_p(logits.clone(), None, p)
    both = ref.apply_top_k_top_p(logits.clone(), k, p)
    both_vllm = apply_top_k_top_p_pytorch(logits.clone(), k, p)
    probs = both.softmax(dim=-1, dtype=torch.float32)
    gens = {i: torch.Generator().manual_seed(900 + i) for i in range(rows)}
    sample = ref.random_sample(probs.clone(), gens)
    q = torch.stack([torch.empty(vocab).exponential_(generator=torch.Generator().manual_seed(900 + i))
                     for i in range(rows)])
    save("sampler_f32", logits=logits, k=k, p=p, top_k_out=topk, top_p_out=topp, top_k_top_p_out=both,
         top_k_top_p_out_vllm=both_vllm, probs=probs, q=q, sample=sample)


if __name__ == "__main__":
    import sys

    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    steps = {"main": main, "f16": half_fixtures, "gemma": gemma_fixture, "sampler": sampler_fixture}
    for name, step in steps.items():
        if only in (None, name):
            step()

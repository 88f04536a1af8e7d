"""oracle -- TEST INFRASTRUCTURE ONLY.

CPU restatements of the seven hooked decoder ops, used as the checker of the sm_100a
kernels: by tests/, by ``__graft_entry__.smoke()`` and by ``bench.py``'s cpu_baseline /
``--impl reference`` legs.  No product code imports this package; the plugin has no CPU
fallback.

What each function restates (citations: ``vllm:`` = vLLM 0.22 sources, the host framework
the plugin patches; other paths are inside the vllm_nt reference project):

* floating-point ops follow vLLM's torch-native implementations -- the oracle named for
  parity -- with the same fp32 intermediates and the same rounding points to the storage
  dtype (GemmaRMSNorm included: (1 + w) in fp32, one rounding of the product);
* the fused RMSNorm + projection restates its own rounding points (s * w rounded once,
  1 / rms applied to the fp32 products); its tests also compare it, and the reference's
  unfused pair, with the unrounded fp64 value;
* the LM head's greedy token is the first index of the largest bf16-rounded logit of the
  fp32 projection (F.linear, then torch.argmax, as vLLM's greedy sampler takes it);
* the KV-cache store and the embedding gather are byte copies (numpy on raw 16-bit views),
  exact; RoPE fused with the KV store is the two restatements composed in vLLM's order;
* paged decode follows the reference's own test oracle (gather the cached tokens through
  the block table, fp32 softmax attention per sequence, GQA by head grouping);
* top-k / top-p masking and the exponential-race sample restate the reference's torch
  sampler (sort, mask in sorted order, scatter back; argmax of probs / q);
* varlen prefill gathers the cached tokens the same way and applies fp32 softmax attention
  with the causal mask aligned to the end of each context (vLLM's rule; the reference's
  start-aligned mask is the same when a sequence has as many keys as queries).

Pinning: tests/golden/make_golden.py runs vLLM's real forward_native code (and torch's
scaled_dot_product_attention for decode and prefill) on seeded inputs and commits the outputs;
tests/test_oracle.py checks these functions against those fixtures and against the
known-answer cases of the reference's tests (tests/test_kv_cache.py:26-45,
tests/test_rope.py:26-46, tests/test_attention.py:57-104, tests/test_oot.py:33-177).
"""

from oracle.ops import (  # noqa: F401
    apply_top_k_top_p,
    build_cos_sin_cache,
    embedding,
    fused_add_rms_norm,
    gather_paged_kv,
    gemma_rms_norm,
    linear,
    linear_argmax,
    paged_decode,
    paged_prefill,
    random_sample_from_draws,
    reshape_and_cache,
    rms_norm,
    rms_norm_linear,
    rms_norm_linear_exact,
    rope_and_cache,
    rope_neox,
    silu_and_mul,
    top_p_cumulative,
    varlen_attention,
)

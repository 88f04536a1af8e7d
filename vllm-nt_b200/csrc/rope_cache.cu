// NeoX rotary embedding of q and k fused with the paged KV-cache store of k and v.
//
// In a decoder layer the RoPE hook and the KV-store hook run back to back on the same
// tokens: vLLM's attention layer rotates q/k in place (RotaryEmbedding.forward), then
// stores the rotated k and the untouched v into the paged cache
// (FlashAttentionImpl.do_kv_cache_update).  The reference reaches them as two kernels
// (vllm_nt/_ntops/kernels/rotary_emb.py:6-37 through oot_support.py:134-204, and
// vllm_nt/_ntops/kernels/kv_cache.py:4-45 through torch/kv_cache.py:7-21).  This kernel
// does both in one pass: one CTA per token, each thread owns one 16-byte vector item of
//
//   [ q rotation pairs | k rotation pairs | k dims past rotary_dim | v ]
//
// A q item is rotated and written back.  A k item is rotated, written back to k and the
// same rounded vector written to key_cache[slot / block_size, slot % block_size, head].
// The k tail (rotary_dim < head_size) and v items are copied bit for bit into the
// caches.  The rotation is the one of rope.cu (separately rounded products, no FMA
// contraction, 16-bit results rounded per torch op), so q, k and both caches are
// bit-identical to the RoPE kernel followed by the KV-store kernel.
//
// Slots: negative (vLLM padding) or past the slot mapping (padded rows) -> rotation only;
// >= num_slots -> rotation only and NTB200_DEVERR_INDEX_RANGE.  A position outside the
// cos/sin cache sets NTB200_DEVERR_INDEX_RANGE and leaves the token's q/k unrotated; its
// unrotated k and its v are still stored (what the two kernels in sequence do).
//
// Dispatch: the fused kernel keeps a token's dependent chain (position -> cos/sin row ->
// rotation -> stores) inside one CTA of ~450 threads at 64 registers, two CTAs per SM; at
// a decode step that costs less than a second launch (256 Llama-3-8B tokens: 3.7 us fused
// against 6.5 us for the pair on a B200), but from a few thousand tokens on the pair keeps
// more bytes in flight (16384 tokens: 141 us fused, 117 us for the pair).  The entry point
// therefore launches the pair from kPairFromTokens tokens on; the results are the same bits
// either way.
#include "common.cuh"

namespace ntb200 {
namespace {

template <typename T>
__device__ __forceinline__ void rotate_pair(float x1, float x2, float c, float s, float& o1,
                                            float& o2) {
  const float a = Elem<T>::round(__fmul_rn(x1, c));
  const float b = Elem<T>::round(__fmul_rn(x2, s));
  const float e = Elem<T>::round(__fmul_rn(x2, c));
  const float f = Elem<T>::round(__fmul_rn(x1, s));
  o1 = __fsub_rn(a, b);
  o2 = __fadd_rn(e, f);
}

struct Geometry {
  int hq, hk;               // query / kv heads
  int pairs;                // rotation vectors per head half (rotary_dim / 2 / VEC)
  int tail;                 // vectors per head past rotary_dim
  int vvec;                 // vectors per v head (head_size / VEC)
  int half;                 // rotary_dim / 2 (elements)
  int rot;                  // rotary_dim (elements)
  int64_t qt, qh, kt, kh, vt, vh;   // element strides
  int64_t cs_row, cs_rows;          // cos/sin cache row stride and row count
  int64_t store_tokens;             // tokens with a slot_mapping entry (a prefix)
  int64_t block_size, num_slots;
  int64_t cbs, cps, chs;            // cache block / page / head strides (both caches)
};

enum ItemKind { kQRot = 0, kKRot = 1, kKTail = 2, kVCopy = 3 };

struct Item {
  int kind, head, off;  // off: element offset inside the head
};

template <int VEC>
__device__ __forceinline__ Item decode_item(const Geometry& g, int item) {
  const int nq = g.hq * g.pairs, nk = g.hk * g.pairs, nt = g.hk * g.tail;
  Item it;
  if (item < nq) {
    it.kind = kQRot;
    it.head = item / g.pairs;
    it.off = (item - it.head * g.pairs) * VEC;
  } else if (item < nq + nk) {
    const int r = item - nq;
    it.kind = kKRot;
    it.head = r / g.pairs;
    it.off = (r - it.head * g.pairs) * VEC;
  } else if (item < nq + nk + nt) {
    const int r = item - nq - nk;
    it.kind = kKTail;
    it.head = r / g.tail;
    it.off = g.rot + (r - it.head * g.tail) * VEC;
  } else {
    const int r = item - nq - nk - nt;
    it.kind = kVCopy;
    it.head = r / g.vvec;
    it.off = (r - it.head * g.vvec) * VEC;
  }
  return it;
}

template <typename T, int VEC, typename P, typename S>
__global__ void __launch_bounds__(1024) rope_and_cache_kernel(
    const P* __restrict__ positions, const S* __restrict__ slots, T* __restrict__ q,
    T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ cos_sin,
    T* __restrict__ kc, T* __restrict__ vc, Geometry g, unsigned int* err) {
  using V = Vec<T, VEC>;
  const int64_t t = blockIdx.x;
  const int total = (g.hq + g.hk) * g.pairs + g.hk * (g.tail + g.vvec);
  pdl_trigger();
  pdl_wait();
  // The first item's data does not depend on the position or the slot: its loads are
  // issued together with the two index loads.
  const int item0 = threadIdx.x;
  V a0, b0;
  Item it0{0, 0, 0};
  if (item0 < total) {
    it0 = decode_item<VEC>(g, item0);
    const T* src = it0.kind == kQRot   ? q + t * g.qt + int64_t(it0.head) * g.qh
                   : it0.kind == kVCopy ? v + t * g.vt + int64_t(it0.head) * g.vh
                                        : k + t * g.kt + int64_t(it0.head) * g.kh;
    a0 = *reinterpret_cast<const V*>(src + it0.off);
    if (it0.kind <= kKRot) b0 = *reinterpret_cast<const V*>(src + g.half + it0.off);
  }
  const int64_t pos = static_cast<int64_t>(positions[t]);
  const int64_t slot = t < g.store_tokens ? static_cast<int64_t>(slots[t]) : -1;
  const bool pos_ok = pos >= 0 && pos < g.cs_rows;
  if (!pos_ok && threadIdx.x == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
  bool store = slot >= 0;
  if (slot >= g.num_slots) {
    if (threadIdx.x == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    store = false;
  }
  int64_t dst_row = 0;
  if (store) {
    const int64_t blk = slot / g.block_size;
    dst_row = blk * g.cbs + (slot - blk * g.block_size) * g.cps;
  }
  const T* cs = cos_sin + (pos_ok ? pos : 0) * g.cs_row;
  for (int item = item0; item < total; item += blockDim.x) {
    const Item it = item == item0 ? it0 : decode_item<VEC>(g, item);
    if (it.kind >= kKTail && !store) continue;
    if (!pos_ok && (it.kind == kQRot || !store)) continue;
    T* base = it.kind == kQRot   ? q + t * g.qt + int64_t(it.head) * g.qh
              : it.kind == kVCopy ? const_cast<T*>(v) + t * g.vt + int64_t(it.head) * g.vh
                                  : k + t * g.kt + int64_t(it.head) * g.kh;
    V a, b;
    if (item == item0) {
      a = a0;
      b = b0;
    } else {
      a = *reinterpret_cast<const V*>(base + it.off);
      if (it.kind <= kKRot) b = *reinterpret_cast<const V*>(base + g.half + it.off);
    }
    T* cache_head = (it.kind == kVCopy ? vc : kc) + dst_row + int64_t(it.head) * g.chs;
    if (it.kind >= kKTail) {  // bit copy into the cache
      *reinterpret_cast<V*>(cache_head + it.off) = a;
      continue;
    }
    if (!pos_ok) {  // unrotated key into the cache, as the KV store alone would leave it
      *reinterpret_cast<V*>(cache_head + it.off) = a;
      *reinterpret_cast<V*>(cache_head + g.half + it.off) = b;
      continue;
    }
    float c[VEC], s[VEC];
    load_f<T, VEC>(cs + it.off, c);
    load_f<T, VEC>(cs + g.half + it.off, s);
    V r1, r2;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      float o1, o2;
      rotate_pair<T>(Elem<T>::to_f(a.v[j]), Elem<T>::to_f(b.v[j]), c[j], s[j], o1, o2);
      r1.v[j] = Elem<T>::from_f(o1);
      r2.v[j] = Elem<T>::from_f(o2);
    }
    *reinterpret_cast<V*>(base + it.off) = r1;
    *reinterpret_cast<V*>(base + g.half + it.off) = r2;
    if (it.kind == kKRot && store) {
      *reinterpret_cast<V*>(cache_head + it.off) = r1;
      *reinterpret_cast<V*>(cache_head + g.half + it.off) = r2;
    }
  }
}

template <typename T, typename P, typename S>
int launch(const void* positions, const void* slots, void* q, void* k, const void* v,
           const void* cos_sin, void* kc, void* vc, int64_t tokens, int64_t head_size,
           Geometry g, cudaStream_t stream) {
  constexpr int kVec = 16 / sizeof(T);
  bool vec_ok = g.half % kVec == 0 && head_size % kVec == 0 && aligned16(q) && aligned16(k) &&
                aligned16(v) && aligned16(cos_sin) && aligned16(kc) && aligned16(vc);
  for (int64_t s : {g.qt, g.qh, g.kt, g.kh, g.vt, g.vh, g.cs_row, g.cbs, g.cps, g.chs})
    vec_ok = vec_ok && s % kVec == 0;
  const int vec = vec_ok ? kVec : 1;
  g.pairs = g.half / vec;
  g.tail = static_cast<int>((head_size - g.rot) / vec);
  g.vvec = static_cast<int>(head_size / vec);
  const int64_t items = int64_t(g.hq + g.hk) * g.pairs + int64_t(g.hk) * (g.tail + g.vvec);
  if (items > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rope_and_cache: too many heads");
  // one item per thread where possible: all of a token's loads are in flight at once
  const int threads = static_cast<int>(items >= 1024 ? 1024 : (items < 32 ? 32 : ceil_div(items, 32) * 32));
  unsigned int* err = device_error_word();
  const dim3 grid(static_cast<unsigned>(tokens));
  if (vec_ok)
    return launch_kernel("rope_and_cache", rope_and_cache_kernel<T, kVec, P, S>, grid, dim3(threads), 0,
                         stream, static_cast<const P*>(positions), static_cast<const S*>(slots),
                         static_cast<T*>(q), static_cast<T*>(k), static_cast<const T*>(v),
                         static_cast<const T*>(cos_sin), static_cast<T*>(kc), static_cast<T*>(vc), g, err);
  return launch_kernel("rope_and_cache", rope_and_cache_kernel<T, 1, P, S>, grid, dim3(threads), 0, stream,
                       static_cast<const P*>(positions), static_cast<const S*>(slots), static_cast<T*>(q),
                       static_cast<T*>(k), static_cast<const T*>(v), static_cast<const T*>(cos_sin),
                       static_cast<T*>(kc), static_cast<T*>(vc), g, err);
}

template <typename T, typename P>
int by_slot(const void* positions, const void* slots, int slot_dtype, void* q, void* k,
            const void* v, const void* cos_sin, void* kc, void* vc, int64_t tokens,
            int64_t head_size, const Geometry& g, cudaStream_t stream) {
  if (slot_dtype == NTB200_DTYPE_I64)
    return launch<T, P, int64_t>(positions, slots, q, k, v, cos_sin, kc, vc, tokens, head_size, g, stream);
  if (slot_dtype == NTB200_DTYPE_I32)
    return launch<T, P, int32_t>(positions, slots, q, k, v, cos_sin, kc, vc, tokens, head_size, g, stream);
  return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rope_and_cache: slot dtype %d", slot_dtype);
}

template <typename T>
int by_pos(const void* positions, int pos_dtype, const void* slots, int slot_dtype, void* q,
           void* k, const void* v, const void* cos_sin, void* kc, void* vc, int64_t tokens,
           int64_t head_size, const Geometry& g, cudaStream_t stream) {
  if (pos_dtype == NTB200_DTYPE_I64)
    return by_slot<T, int64_t>(positions, slots, slot_dtype, q, k, v, cos_sin, kc, vc, tokens, head_size, g,
                               stream);
  if (pos_dtype == NTB200_DTYPE_I32)
    return by_slot<T, int32_t>(positions, slots, slot_dtype, q, k, v, cos_sin, kc, vc, tokens, head_size, g,
                               stream);
  return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rope_and_cache: positions dtype %d", pos_dtype);
}

// token count from which the two-kernel form is launched (see the dispatch note above)
constexpr int64_t kPairFromTokens = 2048;

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_rope_and_cache(
    const void* positions, int positions_dtype, void* query, void* key, const void* value,
    const void* cos_sin_cache, void* key_cache, void* value_cache, const void* slot_mapping,
    int slot_dtype, int64_t num_tokens, int64_t num_store_tokens, int64_t num_q_heads,
    int64_t num_kv_heads,
    int64_t head_size, int64_t rotary_dim, int64_t q_token_stride, int64_t q_head_stride,
    int64_t k_token_stride, int64_t k_head_stride, int64_t v_token_stride,
    int64_t v_head_stride, int64_t cache_row_stride, int64_t num_cache_rows,
    int64_t block_size, int64_t num_slots, int64_t cache_block_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, int dtype, void* stream) {
  using namespace ntb200;
  if (num_tokens < 0 || num_store_tokens < 0 || num_store_tokens > num_tokens || num_q_heads < 0 ||
      num_kv_heads <= 0 || head_size <= 0 || block_size <= 0 || num_slots < 0 || num_cache_rows < 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope_and_cache: bad shape");
  if (rotary_dim <= 0 || rotary_dim > head_size || rotary_dim % 2 != 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope_and_cache: rotary_dim must be even and <= head_size");
  if (num_tokens == 0) return NTB200_OK;
  if (num_tokens > 0x7fffffff || num_q_heads > 0x7fffffff || num_kv_heads > 0x7fffffff)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rope_and_cache: too many tokens or heads");
  if (!positions || !query || !key || !value || !cos_sin_cache || !key_cache || !value_cache ||
      !slot_mapping)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope_and_cache: null pointer");
  if (cache_row_stride < rotary_dim)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope_and_cache: cache row stride < rotary_dim");
  if (num_tokens >= kPairFromTokens) {
    const int es = dtype_size(dtype);
    if (es == 0 || dtype == NTB200_DTYPE_I32 || dtype == NTB200_DTYPE_I64)
      return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rope_and_cache: dtype %d", dtype);
    const int rc = ntb200_rotary_embedding_neox(positions, positions_dtype, query, key, cos_sin_cache, num_tokens,
                                                num_q_heads, num_kv_heads, head_size, rotary_dim, q_token_stride,
                                                q_head_stride, k_token_stride, k_head_stride, cache_row_stride,
                                                num_cache_rows, dtype, stream);
    if (rc != NTB200_OK || num_store_tokens == 0) return rc;
    return ntb200_reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, slot_dtype, num_store_tokens,
                                    num_kv_heads, head_size, block_size, num_slots, k_token_stride, k_head_stride,
                                    v_token_stride, v_head_stride, cache_block_stride, cache_page_stride,
                                    cache_head_stride, es, stream);
  }
  Geometry g{};
  g.hq = static_cast<int>(num_q_heads);
  g.hk = static_cast<int>(num_kv_heads);
  g.half = static_cast<int>(rotary_dim / 2);
  g.rot = static_cast<int>(rotary_dim);
  g.qt = q_token_stride;
  g.qh = q_head_stride;
  g.kt = k_token_stride;
  g.kh = k_head_stride;
  g.vt = v_token_stride;
  g.vh = v_head_stride;
  g.cs_row = cache_row_stride;
  g.cs_rows = num_cache_rows;
  g.store_tokens = num_store_tokens;
  g.block_size = block_size;
  g.num_slots = num_slots;
  g.cbs = cache_block_stride;
  g.cps = cache_page_stride;
  g.chs = cache_head_stride;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NTB200_DTYPE_F32:
      return by_pos<float>(positions, positions_dtype, slot_mapping, slot_dtype, query, key, value,
                           cos_sin_cache, key_cache, value_cache, num_tokens, head_size, g, s);
    case NTB200_DTYPE_BF16:
      return by_pos<__nv_bfloat16>(positions, positions_dtype, slot_mapping, slot_dtype, query, key, value,
                                   cos_sin_cache, key_cache, value_cache, num_tokens, head_size, g, s);
    case NTB200_DTYPE_F16:
      return by_pos<__half>(positions, positions_dtype, slot_mapping, slot_dtype, query, key, value,
                            cos_sin_cache, key_cache, value_cache, num_tokens, head_size, g, s);
    default: return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rope_and_cache: dtype %d", dtype);
  }
}

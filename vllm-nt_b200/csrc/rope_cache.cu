// NeoX rotary embedding of q and k fused with the paged KV-cache store of k and v.
//
// In a decoder layer the RoPE hook and the KV-store hook run back to back on the same
// tokens: vLLM's attention layer rotates q/k in place (RotaryEmbedding.forward), then
// stores the rotated k and the untouched v into the paged cache
// (FlashAttentionImpl.do_kv_cache_update).  The reference reaches them as two kernels
// (vllm_nt/_ntops/kernels/rotary_emb.py:6-37 through oot_support.py:134-204, and
// vllm_nt/_ntops/kernels/kv_cache.py:4-45 through torch/kv_cache.py:7-21).  This kernel
// does both in one pass over the token's 16-byte vector items
//
//   [ q rotation pairs | k rotation pairs | k dims past rotary_dim | v ]
//
// A q item is rotated and written back.  A k item is rotated, written back to k and the
// same rounded vector written to key_cache[slot / block_size, slot % block_size, head].
// The k tail (rotary_dim < head_size) and v items are copied bit for bit into the
// caches.  The rotation is the one of rope.cu (rope_math.cuh: separately rounded products,
// no FMA contraction, 16-bit results rounded per torch op), so q, k and both caches are
// bit-identical to the RoPE kernel followed by the KV-store kernel.
//
// Slots: negative (vLLM padding) or past the slot mapping (padded rows) -> rotation only;
// >= num_slots -> rotation only and NTB200_DEVERR_INDEX_RANGE.  A position outside the
// cos/sin cache sets NTB200_DEVERR_INDEX_RANGE and leaves the token's q/k unrotated; its
// unrotated k and its v are still stored (what the two kernels in sequence do).
//
// Dispatch: warps take (token, chunk) work units (see the kernel), so a decode step spreads
// each token over several warps.  Measured against the RoPE kernel followed by the KV-store
// kernel (CUDA graph, Llama-3-8B qkv, B200): 1024 tokens 6.8 against 9.4 us, 2048 tokens 12.1
// against 11.9 us, 4096 tokens 20.6 against 18.5 us, 16384 tokens 85.5 against 78.9 us --
// the fused kernel's extra stores per work unit cost more than the second launch once a call
// fills the GPU.  The entry point therefore launches the pair from kPairFromTokens tokens on;
// the results are the same bits either way.
#include <algorithm>

#include "common.cuh"
#include "rope_math.cuh"

namespace ntb200 {
namespace {

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

// Work units as in rope.cu: a unit is (token, chunk of 32 x ITEMS items); one warp takes
// one unit at a time from a grid-stride sequence.  Its item loads (q/k halves, k tail, v)
// are issued together with the position and slot loads; the cos/sin loads follow the
// position; then each item is rotated and/or stored.  With SHARED_CS (rotation vectors per
// head half divide 32) a lane's rotation items share one cos/sin pair (ITEMS = 4, else 2);
// calls too small to give every SM 16 warps of such units take one item per lane.
constexpr int kThreads = 256;

template <typename T, int VEC, bool SHARED_CS, int ITEMS, typename P, typename S>
__global__ void __launch_bounds__(kThreads, ITEMS == 1 ? 4 : 2) rope_and_cache_kernel(
    const P* __restrict__ positions, const S* __restrict__ slots, T* __restrict__ q,
    T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ cos_sin,
    T* __restrict__ kc, T* __restrict__ vc, Geometry g, int64_t num_tokens, unsigned int* err) {
  using V = Vec<T, VEC>;
  constexpr int kItems = ITEMS;
  constexpr int kUnitItems = 32 * kItems;
  constexpr int kCs = SHARED_CS ? 1 : kItems;
  const int total = (g.hq + g.hk) * g.pairs + g.hk * (g.tail + g.vvec);
  const int chunks = (total + kUnitItems - 1) / kUnitItems;
  const int lane = threadIdx.x & 31;
  const int64_t units = num_tokens * chunks;
  const int64_t warps = int64_t(gridDim.x) * (kThreads / 32);
  pdl_trigger();
  pdl_wait();
  for (int64_t u = int64_t(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5); u < units; u += warps) {
    const int64_t t = u / chunks;
    const int first = int(u - t * chunks) * kUnitItems + lane;
    V a[kItems], b[kItems], c[kCs], s[kCs];
    Item it[kItems];
    T* base[kItems];
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int item = first + 32 * j;
      if (item < total) {
        it[j] = decode_item<VEC>(g, item);
        base[j] = it[j].kind == kQRot   ? q + t * g.qt + int64_t(it[j].head) * g.qh
                  : it[j].kind == kVCopy ? const_cast<T*>(v) + t * g.vt + int64_t(it[j].head) * g.vh
                                         : k + t * g.kt + int64_t(it[j].head) * g.kh;
        a[j] = *reinterpret_cast<const V*>(base[j] + it[j].off);
        if (it[j].kind <= kKRot) b[j] = *reinterpret_cast<const V*>(base[j] + g.half + it[j].off);
      }
    }
    const int64_t pos = static_cast<int64_t>(positions[t]);
    const int64_t slot = t < g.store_tokens ? static_cast<int64_t>(slots[t]) : -1;
    const bool pos_ok = pos >= 0 && pos < g.cs_rows;
    if (!pos_ok && first == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    bool store = slot >= 0;
    if (slot >= g.num_slots) {
      if (first == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
      store = false;
    }
    int64_t dst_row = 0;
    if (store) {
      const int64_t blk = slot / g.block_size;
      dst_row = blk * g.cbs + (slot - blk * g.block_size) * g.cps;
    }
    const T* cs = cos_sin + (pos_ok ? pos : 0) * g.cs_row;
    if (pos_ok) {
#pragma unroll
      for (int j = 0; j < kCs; ++j) {
        if (first + 32 * j < total && it[j].kind <= kKRot) {
          c[j] = *reinterpret_cast<const V*>(cs + it[j].off);
          s[j] = *reinterpret_cast<const V*>(cs + g.half + it[j].off);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      if (first + 32 * j >= total) continue;
      const Item& m = it[j];
      T* cache_head = (m.kind == kVCopy ? vc : kc) + dst_row + int64_t(m.head) * g.chs;
      if (m.kind >= kKTail) {  // bit copy into the cache
        if (store) *reinterpret_cast<V*>(cache_head + m.off) = a[j];
        continue;
      }
      if (!pos_ok) {  // unrotated key into the cache, as the KV store alone would leave it
        if (m.kind == kKRot && store) {
          *reinterpret_cast<V*>(cache_head + m.off) = a[j];
          *reinterpret_cast<V*>(cache_head + g.half + m.off) = b[j];
        }
        continue;
      }
      const V& cj = c[SHARED_CS ? 0 : j];
      const V& sj = s[SHARED_CS ? 0 : j];
      V r1, r2;
      rotate_vec<T, VEC>(a[j], b[j], cj, sj, r1, r2);
      *reinterpret_cast<V*>(base[j] + m.off) = r1;
      *reinterpret_cast<V*>(base[j] + g.half + m.off) = r2;
      if (m.kind == kKRot && store) {
        *reinterpret_cast<V*>(cache_head + m.off) = r1;
        *reinterpret_cast<V*>(cache_head + g.half + m.off) = r2;
      }
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
  const bool shared_cs = vec_ok && 32 % g.pairs == 0;
  const int big = shared_cs ? 4 : 2;
  const int sms = num_sms();
  // several items per lane once every SM has 16 warps of work at that size; else one
  const bool many = tokens * ceil_div(items, 32 * big) >= int64_t(sms) * 16;
  const int per_lane = many ? big : 1;
  const int64_t units = tokens * ceil_div(items, 32 * per_lane);  // as the kernel counts them
  // persistent CTAs: the resident count per SM the kernel's launch bound allows, or fewer
  const int64_t ctas = std::min<int64_t>(ceil_div(units, kThreads / 32), int64_t(sms) * (many ? 2 : 4));
  unsigned int* err = device_error_word();
  const dim3 grid(static_cast<unsigned>(ctas));
#define NTB200_RC_LAUNCH(V, SHARED, ITEMS)                                                                     \
  return launch_kernel("rope_and_cache", rope_and_cache_kernel<T, V, SHARED, ITEMS, P, S>, grid, dim3(kThreads), \
                       0, stream, static_cast<const P*>(positions), static_cast<const S*>(slots),             \
                       static_cast<T*>(q), static_cast<T*>(k), static_cast<const T*>(v),                      \
                       static_cast<const T*>(cos_sin), static_cast<T*>(kc), static_cast<T*>(vc), g, tokens, err)
  if (!vec_ok) NTB200_RC_LAUNCH(1, false, 1);
  if (shared_cs) {
    if (many) NTB200_RC_LAUNCH(kVec, true, 4);
    NTB200_RC_LAUNCH(kVec, true, 1);
  }
  if (many) NTB200_RC_LAUNCH(kVec, false, 2);
  NTB200_RC_LAUNCH(kVec, false, 1);
#undef NTB200_RC_LAUNCH
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
constexpr int64_t kPairFromTokens = 4096;

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

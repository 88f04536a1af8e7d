// In-place NeoX rotary embedding over query and key with the cos/sin gather fused in.
//
// The reference gathers cos/sin rows with a torch index_select and then launches one
// rotary kernel for q and one for k (vllm_nt/_ntops/oot_support.py:164-204,
// vllm_nt/_ntops/kernels/rotary_emb.py:6-37).  Here one launch covers both: warps take
// (token, chunk) work units and rotate 128-bit vectors of (x1, x2) pairs of the token's q
// and k heads, reading cos/sin straight from the cache row (L1/L2 resident).
//
// The rotation (rope_math.cuh) mirrors vLLM's torch-native arithmetic op by op, so the
// result is bit-identical to the torch-native path.
#include <algorithm>

#include "common.cuh"
#include "rope_math.cuh"

namespace ntb200 {
namespace {

// Work units: a unit is (token, chunk of 32 x ITEMS vector items of that token), where an
// item is one (head, 16-byte vector) of the token's x1 half with its x2 partner.  One warp
// takes one unit at a time from a grid-stride sequence (persistent CTAs): it issues the
// unit's x loads (independent of the position) and the position load together, then the
// cos/sin loads, then rotates and stores; the stores do not hold the warp, so the next
// unit's loads follow at once.  Small calls (a decode step) spread a token over several
// warps; large ones keep 16 units (64 KB of q/k) in flight per SM.  When the vectors per
// head half divide 32 (every power-of-two rotary width), lane l's items all sit at the same
// offset in their heads, so one cos/sin pair per lane serves the whole unit (SHARED_CS,
// ITEMS = 4); otherwise each item loads its own pair (ITEMS = 2, to stay in registers).
// Calls too small to give every SM 16 warps of such units take one item per lane.
constexpr int kRopeThreads = 256;

template <typename T, int VEC, bool SHARED_CS, int ITEMS, typename P>
__global__ void __launch_bounds__(kRopeThreads, ITEMS == 1 ? 4 : 2) rope_neox_kernel(
    const P* __restrict__ positions, T* __restrict__ q, T* __restrict__ k,
    const T* __restrict__ cache, int64_t num_tokens, int num_q_heads, int num_k_heads, int half,
    int64_t q_tok, int64_t q_head, int64_t k_tok, int64_t k_head, int64_t cache_row,
    int64_t cache_rows, unsigned int* err) {
  using V = Vec<T, VEC>;
  constexpr int kItems = ITEMS;
  constexpr int kUnitItems = 32 * kItems;
  constexpr int kCs = SHARED_CS ? 1 : kItems;
  const int vph = half / VEC;  // vectors per head half
  const int total = (num_q_heads + (k != nullptr ? num_k_heads : 0)) * vph;
  const int chunks = (total + kUnitItems - 1) / kUnitItems;
  const int lane = threadIdx.x & 31;
  const int64_t units = num_tokens * chunks;
  const int64_t warps = int64_t(gridDim.x) * (kRopeThreads / 32);
  pdl_trigger();
  pdl_wait();
  for (int64_t u = int64_t(blockIdx.x) * (kRopeThreads / 32) + (threadIdx.x >> 5); u < units; u += warps) {
    const int64_t t = u / chunks;
    const int first = int(u - t * chunks) * kUnitItems + lane;
    T* const qt = q + t * q_tok;
    T* const kt = k + t * k_tok;
    V x1[kItems], x2[kItems], c[kCs], s[kCs];
    int64_t at[kItems];  // element offset of the item's x1 vector from its token's q (>= 0) or k (< 0) base
    int off[kItems];
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int item = first + 32 * j;
      if (item < total) {
        const int h = item / vph;
        off[j] = (item - h * vph) * VEC;
        const T* src;
        if (h < num_q_heads) {
          at[j] = int64_t(h) * q_head + off[j];
          src = qt + at[j];
        } else {
          at[j] = -1 - (int64_t(h - num_q_heads) * k_head + off[j]);
          src = kt + (-1 - at[j]);
        }
        x1[j] = *reinterpret_cast<const V*>(src);
        x2[j] = *reinterpret_cast<const V*>(src + half);
      }
    }
    const int64_t pos = static_cast<int64_t>(positions[t]);
    if (pos < 0 || pos >= cache_rows) {  // the token stays untouched; flagged once
      if (first == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
      continue;
    }
    const T* cs = cache + pos * cache_row;
#pragma unroll
    for (int j = 0; j < kCs; ++j) {
      if (first + 32 * j < total) {
        c[j] = *reinterpret_cast<const V*>(cs + off[j]);
        s[j] = *reinterpret_cast<const V*>(cs + half + off[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      if (first + 32 * j >= total) continue;
      const V& cj = c[SHARED_CS ? 0 : j];
      const V& sj = s[SHARED_CS ? 0 : j];
      V o1, o2;
      rotate_vec<T, VEC>(x1[j], x2[j], cj, sj, o1, o2);
      T* dst = at[j] >= 0 ? qt + at[j] : kt + (-1 - at[j]);
      *reinterpret_cast<V*>(dst) = o1;
      *reinterpret_cast<V*>(dst + half) = o2;
    }
  }
}

template <typename T, typename P>
int launch(const void* positions, void* q, void* k, const void* cache, int64_t tokens,
           int64_t hq, int64_t hk, int64_t rot, int64_t qt, int64_t qh, int64_t kt, int64_t kh,
           int64_t cr, int64_t rows, cudaStream_t stream) {
  unsigned int* err = device_error_word();
  constexpr int kVec = 16 / sizeof(T);
  const int64_t half = rot / 2;
  bool vec_ok = half % kVec == 0 && qt % kVec == 0 && qh % kVec == 0 && cr % kVec == 0 &&
                aligned16(q) && aligned16(cache);
  if (k != nullptr) vec_ok = vec_ok && kt % kVec == 0 && kh % kVec == 0 && aligned16(k);
  const int64_t vec = vec_ok ? kVec : 1;
  const int64_t items = (hq + (k != nullptr ? hk : 0)) * (half / vec);
  const bool shared_cs = vec_ok && 32 % (half / vec) == 0;
  const int big = shared_cs ? 4 : 2;
  const int sms = num_sms();
  // several items per lane once every SM has 16 warps of work at that size; else one, to
  // spread a small call over as many warps as it has items
  const bool many = tokens * ceil_div(items, 32 * big) >= int64_t(sms) * 16;
  const int per_lane = many ? big : 1;
  const int64_t units = tokens * ceil_div(items, 32 * per_lane);  // as the kernel counts them
  // persistent CTAs: the resident count per SM the kernel's launch bound allows, or fewer
  const int64_t ctas = std::min<int64_t>(ceil_div(units, kRopeThreads / 32), int64_t(sms) * (many ? 2 : 4));
  const dim3 grid(static_cast<unsigned>(ctas));
#define NTB200_ROPE_LAUNCH(V, SHARED, ITEMS)                                                                   \
  return launch_kernel("rotary_embedding_neox", rope_neox_kernel<T, V, SHARED, ITEMS, P>, grid,               \
                       dim3(kRopeThreads), 0, stream, static_cast<const P*>(positions), static_cast<T*>(q),   \
                       static_cast<T*>(k), static_cast<const T*>(cache), tokens, int(hq), int(hk), int(half), \
                       qt, qh, kt, kh, cr, rows, err)
  if (!vec_ok) NTB200_ROPE_LAUNCH(1, false, 1);
  if (shared_cs) {
    if (many) NTB200_ROPE_LAUNCH(kVec, true, 4);
    NTB200_ROPE_LAUNCH(kVec, true, 1);
  }
  if (many) NTB200_ROPE_LAUNCH(kVec, false, 2);
  NTB200_ROPE_LAUNCH(kVec, false, 1);
#undef NTB200_ROPE_LAUNCH
}

template <typename T>
int by_pos(const void* positions, int pdtype, void* q, void* k, const void* cache,
           int64_t tokens, int64_t hq, int64_t hk, int64_t rot, int64_t qt, int64_t qh,
           int64_t kt, int64_t kh, int64_t cr, int64_t rows, cudaStream_t stream) {
  if (pdtype == NTB200_DTYPE_I64)
    return launch<T, int64_t>(positions, q, k, cache, tokens, hq, hk, rot, qt, qh, kt, kh, cr, rows, stream);
  if (pdtype == NTB200_DTYPE_I32)
    return launch<T, int32_t>(positions, q, k, cache, tokens, hq, hk, rot, qt, qh, kt, kh, cr, rows, stream);
  return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rope: positions dtype %d", pdtype);
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_rotary_embedding_neox(
    const void* positions, int positions_dtype, void* query, void* key,
    const void* cos_sin_cache, int64_t num_tokens, int64_t num_q_heads, int64_t num_k_heads,
    int64_t head_size, int64_t rotary_dim, int64_t q_token_stride, int64_t q_head_stride,
    int64_t k_token_stride, int64_t k_head_stride, int64_t cache_row_stride,
    int64_t num_cache_rows, int dtype, void* stream) {
  using namespace ntb200;
  if (num_tokens < 0 || num_q_heads < 0 || num_k_heads < 0 || head_size <= 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope: bad shape");
  if (rotary_dim <= 0 || rotary_dim > head_size || rotary_dim % 2 != 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope: rotary_dim must be even and <= head_size");
  if (num_tokens == 0) return NTB200_OK;
  if (num_tokens > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rope: too many tokens");
  if (positions == nullptr || query == nullptr || cos_sin_cache == nullptr)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope: null pointer");
  if (cache_row_stride < rotary_dim)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rope: cache row stride < rotary_dim");
  if (int64_t(num_q_heads + num_k_heads) * (rotary_dim / 2) > 0x7fffffff)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rope: too many heads");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NTB200_DTYPE_F32:
      return by_pos<float>(positions, positions_dtype, query, key, cos_sin_cache, num_tokens,
                           num_q_heads, num_k_heads, rotary_dim, q_token_stride, q_head_stride,
                           k_token_stride, k_head_stride, cache_row_stride, num_cache_rows, s);
    case NTB200_DTYPE_BF16:
      return by_pos<__nv_bfloat16>(positions, positions_dtype, query, key, cos_sin_cache,
                                   num_tokens, num_q_heads, num_k_heads, rotary_dim,
                                   q_token_stride, q_head_stride, k_token_stride, k_head_stride,
                                   cache_row_stride, num_cache_rows, s);
    case NTB200_DTYPE_F16:
      return by_pos<__half>(positions, positions_dtype, query, key, cos_sin_cache, num_tokens,
                            num_q_heads, num_k_heads, rotary_dim, q_token_stride, q_head_stride,
                            k_token_stride, k_head_stride, cache_row_stride, num_cache_rows, s);
    default: return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rope: dtype %d", dtype);
  }
}

// In-place NeoX rotary embedding over query and key with the cos/sin gather fused in.
//
// The reference gathers cos/sin rows with a torch index_select and then launches one
// rotary kernel for q and one for k (vllm_nt/_ntops/oot_support.py:164-204,
// vllm_nt/_ntops/kernels/rotary_emb.py:6-37).  Here one CTA owns one token: it reads the
// token's position, then every thread rotates 128-bit vectors of (x1, x2) pairs of the
// token's q and k heads, reading cos/sin straight from the cache row (L1/L2 resident).
//
// Arithmetic mirrors vLLM's ApplyRotaryEmb.forward_static
// (vllm/model_executor/layers/rotary_embedding/common.py:144-183) op by op: each product
// and the final sum/difference are separately rounded (no FMA contraction), and for
// 16-bit types each torch op's result is rounded to the storage type.  The result is
// therefore bit-identical to the torch-native path.
#include "common.cuh"

namespace ntb200 {
namespace {

template <typename T>
__device__ __forceinline__ void rotate(float x1, float x2, float c, float s, float& o1,
                                       float& o2) {
  const float a = Elem<T>::round(__fmul_rn(x1, c));
  const float b = Elem<T>::round(__fmul_rn(x2, s));
  const float e = Elem<T>::round(__fmul_rn(x2, c));
  const float f = Elem<T>::round(__fmul_rn(x1, s));
  o1 = __fsub_rn(a, b);
  o2 = __fadd_rn(e, f);
}

template <typename T, int VEC, typename P>
__global__ void __launch_bounds__(1024) rope_neox_kernel(
    const P* __restrict__ positions, T* __restrict__ q, T* __restrict__ k,
    const T* __restrict__ cache, int num_q_heads, int num_k_heads, int half,
    int64_t q_tok, int64_t q_head, int64_t k_tok, int64_t k_head, int64_t cache_row,
    int64_t cache_rows, unsigned int* err) {
  const int64_t t = blockIdx.x;
  const int vph = half / VEC;  // vectors per head
  const int total = (num_q_heads + (k != nullptr ? num_k_heads : 0)) * vph;
  auto head_base = [&](int h) -> T* {
    return h < num_q_heads ? q + t * q_tok + int64_t(h) * q_head
                           : k + t * k_tok + int64_t(h - num_q_heads) * k_head;
  };
  // The x loads of this thread's first item do not depend on the position: issue them
  // before the position read so the two latencies overlap.
  float x1[VEC], x2[VEC];
  const int item0 = threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (item0 < total) {
    const int h = item0 / vph;
    const int i = (item0 - h * vph) * VEC;
    load_f<T, VEC>(head_base(h) + i, x1);
    load_f<T, VEC>(head_base(h) + half + i, x2);
  }
  const int64_t pos = static_cast<int64_t>(positions[t]);
  if (pos < 0 || pos >= cache_rows) {
    if (threadIdx.x == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    return;
  }
  const T* cs = cache + pos * cache_row;
  for (int item = item0; item < total; item += blockDim.x) {
    const int h = item / vph;
    const int i = (item - h * vph) * VEC;
    T* base = head_base(h);
    float c[VEC], s[VEC], o1[VEC], o2[VEC];
    if (item != item0) {
      load_f<T, VEC>(base + i, x1);
      load_f<T, VEC>(base + half + i, x2);
    }
    load_f<T, VEC>(cs + i, c);
    load_f<T, VEC>(cs + half + i, s);
#pragma unroll
    for (int j = 0; j < VEC; ++j) rotate<T>(x1[j], x2[j], c[j], s[j], o1[j], o2[j]);
    store_f<T, VEC>(base + i, o1);
    store_f<T, VEC>(base + half + i, o2);
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
  const unsigned grid = static_cast<unsigned>(tokens);
  // one vector item per thread where possible: every load of the token is in flight at once
  auto threads_for = [&](int64_t vec) {
    const int64_t items = (hq + (k != nullptr ? hk : 0)) * (half / vec);
    return static_cast<int>(items >= 1024 ? 1024 : (items < 32 ? 32 : ceil_div(items, 32) * 32));
  };
  if (vec_ok)
    return launch_kernel("rotary_embedding_neox", rope_neox_kernel<T, kVec, P>, dim3(grid),
                         dim3(threads_for(kVec)), 0, stream, static_cast<const P*>(positions),
                         static_cast<T*>(q), static_cast<T*>(k), static_cast<const T*>(cache),
                         int(hq), int(hk), int(half), qt, qh, kt, kh, cr, rows, err);
  return launch_kernel("rotary_embedding_neox", rope_neox_kernel<T, 1, P>, dim3(grid),
                       dim3(threads_for(1)), 0, stream, static_cast<const P*>(positions),
                       static_cast<T*>(q), static_cast<T*>(k), static_cast<const T*>(cache),
                       int(hq), int(hk), int(half), qt, qh, kt, kh, cr, rows, err);
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

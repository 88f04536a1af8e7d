// Embedding gather: out[t, :] = weight[ids[t], :]  (bit-exact copy).
//
// One CTA per token row: the id is read once, then 16-byte units of the weight row are
// copied, each thread loading up to four units before storing them (8/4/2/1-byte units
// when a pointer or stride is not 16-byte aligned).  Ids out
// of range give a zero row and raise NTB200_DEVERR_INDEX_RANGE -- they never read outside
// the table.  The reference kernel (vllm_nt/_ntops/kernels/wpe.py:11-67) tiles 64x64 with
// num_tokens constexpr, i.e. one JIT compile per batch size; this kernel takes every size
// at run time.
#include "common.cuh"

namespace ntb200 {
namespace {

constexpr int kItems = 4;  // units per thread, all loaded before any is stored

template <typename U, typename I>
__global__ void __launch_bounds__(256) embedding_kernel(char* __restrict__ out,
                                                         const I* __restrict__ ids,
                                                         const char* __restrict__ weight,
                                                         int64_t num_embeddings, int64_t units,
                                                         int64_t w_stride, int64_t o_stride,
                                                         unsigned int* err) {
  const int64_t t = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  const int64_t id = static_cast<int64_t>(ids[t]);
  U* dst = reinterpret_cast<U*>(out + t * o_stride);
  if (id < 0 || id >= num_embeddings) {
    if (threadIdx.x == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    for (int64_t u = threadIdx.x; u < units; u += blockDim.x) dst[u] = U{};
    return;
  }
  const U* src = reinterpret_cast<const U*>(weight + id * w_stride);
  const int64_t step = blockDim.x;
  for (int64_t base = threadIdx.x; base < units; base += step * kItems) {
    U v[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i)
      if (base + i * step < units) v[i] = src[base + i * step];
#pragma unroll
    for (int i = 0; i < kItems; ++i)
      if (base + i * step < units) dst[base + i * step] = v[i];
  }
}

template <typename U, typename I>
int launch(void* out, const void* ids, const void* weight, int64_t tokens, int64_t num_emb,
           int64_t row_bytes, int64_t wsb, int64_t osb, cudaStream_t stream) {
  const int64_t units = row_bytes / static_cast<int64_t>(sizeof(U));
  const int64_t want = ceil_div(units, kItems);
  const int threads = want >= 256 ? 256 : static_cast<int>(ceil_div(want, 32) * 32);
  return launch_kernel("embedding", embedding_kernel<U, I>, dim3(static_cast<unsigned>(tokens)),
                       dim3(threads), 0, stream, static_cast<char*>(out), static_cast<const I*>(ids),
                       static_cast<const char*>(weight), num_emb, units, wsb, osb,
                       device_error_word());
}

template <typename I>
int by_unit(void* out, const void* ids, const void* weight, int64_t tokens, int64_t num_emb,
            int64_t row_bytes, int64_t wsb, int64_t osb, cudaStream_t stream) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(weight) |
                         static_cast<uintptr_t>(row_bytes) | static_cast<uintptr_t>(wsb) |
                         static_cast<uintptr_t>(osb);
  if ((bits & 15u) == 0) return launch<uint4, I>(out, ids, weight, tokens, num_emb, row_bytes, wsb, osb, stream);
  if ((bits & 7u) == 0) return launch<uint2, I>(out, ids, weight, tokens, num_emb, row_bytes, wsb, osb, stream);
  if ((bits & 3u) == 0) return launch<uint32_t, I>(out, ids, weight, tokens, num_emb, row_bytes, wsb, osb, stream);
  if ((bits & 1u) == 0) return launch<uint16_t, I>(out, ids, weight, tokens, num_emb, row_bytes, wsb, osb, stream);
  return launch<uint8_t, I>(out, ids, weight, tokens, num_emb, row_bytes, wsb, osb, stream);
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_embedding(void* out, const void* ids, int ids_dtype, const void* weight,
                                int64_t num_tokens, int64_t num_embeddings, int64_t embedding_dim,
                                int64_t weight_row_stride, int64_t out_row_stride, int elem_bytes,
                                void* stream) {
  using namespace ntb200;
  if (num_tokens < 0 || num_embeddings < 0 || embedding_dim <= 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "embedding: bad shape");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "embedding: elem_bytes %d", elem_bytes);
  if (num_tokens == 0) return NTB200_OK;
  if (num_tokens > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "embedding: too many tokens");
  if (!out || !ids || !weight) return fail(NTB200_ERR_INVALID_ARGUMENT, "embedding: null pointer");
  if (weight_row_stride < embedding_dim || out_row_stride < embedding_dim)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "embedding: row stride < embedding_dim");
  const int64_t eb = elem_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ids_dtype == NTB200_DTYPE_I64)
    return by_unit<int64_t>(out, ids, weight, num_tokens, num_embeddings, embedding_dim * eb,
                            weight_row_stride * eb, out_row_stride * eb, s);
  if (ids_dtype == NTB200_DTYPE_I32)
    return by_unit<int32_t>(out, ids, weight, num_tokens, num_embeddings, embedding_dim * eb,
                            weight_row_stride * eb, out_row_stride * eb, s);
  return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "embedding: ids dtype %d", ids_dtype);
}

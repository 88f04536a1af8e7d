// reshape_and_cache: slot-mapped scatter of one step's key/value rows into the paged cache.
//
// Pure data movement, bit-exact, no atomics.  One CTA per token: its threads load up to
// four 16-byte units each of the token's (K|V, head) rows while the slot is read, then
// store them to cache[slot / block_size, slot % block_size, head, :].  The unit shrinks to 8,
// 4, 2 or 1 bytes when a pointer or stride is not 16-byte aligned.  Loads are marked
// streaming (read once) and stores evict-first: the cache rows written here are read
// back only by a later decode step, from HBM.
//
// The reference kernel (vllm_nt/_ntops/kernels/kv_cache.py:4-45) writes
// k_cache[slot_mapping[t]] for every token with all shapes constexpr (a JIT recompile per
// token count) and does not skip vLLM's padding slot -1; this kernel takes the counts at run
// time and skips negative slots the way vLLM's reshape_and_cache_flash does.
#include "common.cuh"

namespace ntb200 {
namespace {

template <typename U>
__device__ __forceinline__ U ld_stream(const U* p) {
  return __ldcs(p);
}
template <>
__device__ __forceinline__ uint16_t ld_stream<uint16_t>(const uint16_t* p) {
  return *p;
}
template <>
__device__ __forceinline__ uint8_t ld_stream<uint8_t>(const uint8_t* p) {
  return *p;
}
template <typename U>
__device__ __forceinline__ void st_stream(U* p, U v) {
  __stcs(p, v);
}
template <>
__device__ __forceinline__ void st_stream<uint16_t>(uint16_t* p, uint16_t v) {
  *p = v;
}
template <>
__device__ __forceinline__ void st_stream<uint8_t>(uint8_t* p, uint8_t v) {
  *p = v;
}

// All strides in bytes.
constexpr int kItems = 4;  // units per thread, loaded together before any store

template <typename U>
struct RowSrc {
  const char* key;
  const char* value;
  int64_t kts, khs, vts, vhs;
  int per_tensor, units_per_head;
  __device__ __forceinline__ const U* unit(int64_t t, int item, int& h, int& u, bool& is_v) const {
    is_v = item >= per_tensor;
    const int rem = is_v ? item - per_tensor : item;
    h = rem / units_per_head;
    u = rem - h * units_per_head;
    const char* base = is_v ? value + t * vts + h * vhs : key + t * kts + h * khs;
    return reinterpret_cast<const U*>(base) + u;
  }
};

template <typename U, typename S>
__global__ void __launch_bounds__(1024) reshape_and_cache_kernel(
    const char* __restrict__ key, const char* __restrict__ value, char* __restrict__ kc,
    char* __restrict__ vc, const S* __restrict__ slots, int64_t num_slots, int64_t block_size,
    int num_heads, int units_per_head, int64_t kts, int64_t khs, int64_t vts, int64_t vhs,
    int64_t cbs, int64_t cps, int64_t chs, unsigned int* err) {
  const int64_t t = blockIdx.x;
  const RowSrc<U> src{key, value, kts, khs, vts, vhs, num_heads * units_per_head, units_per_head};
  const int total = 2 * src.per_tensor;
  const int step = blockDim.x;
  pdl_trigger();
  pdl_wait();
  // the first group of units is in flight before the slot is known
  U v[kItems];
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int item = threadIdx.x + i * step;
    int h, u;
    bool is_v;
    if (item < total) v[i] = ld_stream(src.unit(t, item, h, u, is_v));
  }
  const int64_t slot = static_cast<int64_t>(slots[t]);
  if (slot < 0) return;  // padding token
  if (slot >= num_slots) {
    if (threadIdx.x == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    return;
  }
  const int64_t blk = slot / block_size;
  const int64_t dst_row = blk * cbs + (slot - blk * block_size) * cps;
  for (int base = threadIdx.x; base < total; base += step * kItems) {
    if (base != threadIdx.x) {
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int item = base + i * step;
        int h, u;
        bool is_v;
        if (item < total) v[i] = ld_stream(src.unit(t, item, h, u, is_v));
      }
    }
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int item = base + i * step;
      if (item < total) {
        int h, u;
        bool is_v;
        src.unit(t, item, h, u, is_v);
        char* dst = (is_v ? vc : kc) + dst_row + h * chs;
        st_stream(reinterpret_cast<U*>(dst) + u, v[i]);
      }
    }
  }
}

template <typename U, typename S>
int launch(const void* key, const void* value, void* kc, void* vc, const void* slots,
           int64_t tokens, int64_t heads, int64_t head_bytes, int64_t block_size,
           int64_t num_slots, int64_t kts, int64_t khs, int64_t vts, int64_t vhs, int64_t cbs,
           int64_t cps, int64_t chs, cudaStream_t stream) {
  const int uph = static_cast<int>(head_bytes / sizeof(U));
  const int64_t items = 2 * heads * uph;
  // up to kItems units per thread (all loads of a token in flight at once)
  const int64_t want = ceil_div(items, kItems);
  const int threads = want >= 1024 ? 1024 : static_cast<int>(ceil_div(want, 32) * 32);
  return launch_kernel("reshape_and_cache", reshape_and_cache_kernel<U, S>,
                       dim3(static_cast<unsigned>(tokens)), dim3(threads), 0, stream,
                       static_cast<const char*>(key), static_cast<const char*>(value),
                       static_cast<char*>(kc), static_cast<char*>(vc), static_cast<const S*>(slots),
                       num_slots, block_size, static_cast<int>(heads), uph, kts, khs, vts, vhs, cbs,
                       cps, chs, device_error_word());
}

template <typename S>
int by_unit(const void* key, const void* value, void* kc, void* vc, const void* slots,
            int64_t tokens, int64_t heads, int64_t head_bytes, int64_t block_size,
            int64_t num_slots, int64_t kts, int64_t khs, int64_t vts, int64_t vhs, int64_t cbs,
            int64_t cps, int64_t chs, cudaStream_t stream) {
  uintptr_t bits = reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                   reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc);
  for (int64_t v : {head_bytes, kts, khs, vts, vhs, cbs, cps, chs}) bits |= static_cast<uintptr_t>(v);
#define NTB200_KV_LAUNCH(U) \
  launch<U, S>(key, value, kc, vc, slots, tokens, heads, head_bytes, block_size, num_slots, kts, khs, vts, vhs, cbs, cps, chs, stream)
  if ((bits & 15u) == 0) return NTB200_KV_LAUNCH(uint4);
  if ((bits & 7u) == 0) return NTB200_KV_LAUNCH(uint2);
  if ((bits & 3u) == 0) return NTB200_KV_LAUNCH(uint32_t);
  if ((bits & 1u) == 0) return NTB200_KV_LAUNCH(uint16_t);
  return NTB200_KV_LAUNCH(uint8_t);
#undef NTB200_KV_LAUNCH
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_reshape_and_cache(
    const void* key, const void* value, void* key_cache, void* value_cache,
    const void* slot_mapping, int slot_dtype, int64_t num_tokens, int64_t num_heads,
    int64_t head_size, int64_t block_size, int64_t num_slots, int64_t key_token_stride,
    int64_t key_head_stride, int64_t value_token_stride, int64_t value_head_stride,
    int64_t cache_block_stride, int64_t cache_page_stride, int64_t cache_head_stride,
    int elem_bytes, void* stream) {
  using namespace ntb200;
  if (num_tokens < 0 || num_heads <= 0 || head_size <= 0 || block_size <= 0 || num_slots < 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "reshape_and_cache: bad shape");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "reshape_and_cache: elem_bytes %d", elem_bytes);
  if (num_tokens == 0) return NTB200_OK;
  if (num_tokens > 0x7fffffff || num_heads * head_size * elem_bytes > (int64_t(1) << 30))
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "reshape_and_cache: too large");
  if (!key || !value || !key_cache || !value_cache || !slot_mapping)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "reshape_and_cache: null pointer");
  const int64_t eb = elem_bytes;
  const int64_t hb = head_size * eb;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (slot_dtype == NTB200_DTYPE_I64)
    return by_unit<int64_t>(key, value, key_cache, value_cache, slot_mapping, num_tokens,
                            num_heads, hb, block_size, num_slots, key_token_stride * eb,
                            key_head_stride * eb, value_token_stride * eb, value_head_stride * eb,
                            cache_block_stride * eb, cache_page_stride * eb,
                            cache_head_stride * eb, s);
  if (slot_dtype == NTB200_DTYPE_I32)
    return by_unit<int32_t>(key, value, key_cache, value_cache, slot_mapping, num_tokens,
                            num_heads, hb, block_size, num_slots, key_token_stride * eb,
                            key_head_stride * eb, value_token_stride * eb, value_head_stride * eb,
                            cache_block_stride * eb, cache_page_stride * eb,
                            cache_head_stride * eb, s);
  return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "reshape_and_cache: slot dtype %d", slot_dtype);
}

// reshape_and_cache: slot-mapped scatter of one step's key/value rows into the paged cache.
//
// Pure data movement, bit-exact, no atomics.  One CTA per token: it reads the token's slot
// once, then its threads move 16-byte units of every (K|V, head) row from the projection
// output to cache[slot / block_size, slot % block_size, head, :].  The unit shrinks to 8,
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
template <typename U, typename S>
__global__ void __launch_bounds__(1024) reshape_and_cache_kernel(
    const char* __restrict__ key, const char* __restrict__ value, char* __restrict__ kc,
    char* __restrict__ vc, const S* __restrict__ slots, int64_t num_slots, int64_t block_size,
    int num_heads, int units_per_head, int64_t kts, int64_t khs, int64_t vts, int64_t vhs,
    int64_t cbs, int64_t cps, int64_t chs, unsigned int* err) {
  const int64_t t = blockIdx.x;
  const int per_tensor = num_heads * units_per_head;
  // The first item's load does not depend on the slot: issue it together with the slot
  // read so the two memory latencies overlap instead of adding up.
  const int item0 = threadIdx.x;
  U first{};
  if (item0 < 2 * per_tensor) {
    const bool is_v = item0 >= per_tensor;
    const int rem = is_v ? item0 - per_tensor : item0;
    const int h = rem / units_per_head;
    const char* src = is_v ? value + t * vts + h * vhs : key + t * kts + h * khs;
    first = ld_stream(reinterpret_cast<const U*>(src) + (rem - h * units_per_head));
  }
  const int64_t slot = static_cast<int64_t>(slots[t]);
  if (slot < 0) return;  // padding token
  if (slot >= num_slots) {
    if (threadIdx.x == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    return;
  }
  const int64_t blk = slot / block_size;
  const int64_t dst_row = blk * cbs + (slot - blk * block_size) * cps;
  for (int item = item0; item < 2 * per_tensor; item += blockDim.x) {
    const bool is_v = item >= per_tensor;
    const int rem = is_v ? item - per_tensor : item;
    const int h = rem / units_per_head;
    const int u = rem - h * units_per_head;
    char* dst = (is_v ? vc : kc) + dst_row + h * chs;
    U v = first;
    if (item != item0) {
      const char* src = is_v ? value + t * vts + h * vhs : key + t * kts + h * khs;
      v = ld_stream(reinterpret_cast<const U*>(src) + u);
    }
    st_stream(reinterpret_cast<U*>(dst) + u, v);
  }
}

template <typename U, typename S>
int launch(const void* key, const void* value, void* kc, void* vc, const void* slots,
           int64_t tokens, int64_t heads, int64_t head_bytes, int64_t block_size,
           int64_t num_slots, int64_t kts, int64_t khs, int64_t vts, int64_t vhs, int64_t cbs,
           int64_t cps, int64_t chs, cudaStream_t stream) {
  const int uph = static_cast<int>(head_bytes / sizeof(U));
  const int64_t items = 2 * heads * uph;
  // one unit per thread where the row allows it (all loads of a token in flight at once)
  const int threads = items >= 1024 ? 1024 : static_cast<int>(ceil_div(items, 32) * 32);
  reshape_and_cache_kernel<U, S><<<static_cast<unsigned>(tokens), threads, 0, stream>>>(
      static_cast<const char*>(key), static_cast<const char*>(value), static_cast<char*>(kc),
      static_cast<char*>(vc), static_cast<const S*>(slots), num_slots, block_size,
      static_cast<int>(heads), uph, kts, khs, vts, vhs, cbs, cps, chs, device_error_word());
  return check_launch("reshape_and_cache");
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

// Paged-attention decode for callers that cannot allocate device memory.
//
// ntb200_paged_attention_decode keeps the per-chunk partial results of its split-K pass
// in a workspace the caller passes in.  Some callers cannot produce one at the point of
// the call:
//   * a serving loop that must not call cudaMalloc/cudaFree while decoding -- those calls
//     can synchronise the whole device and serialise on a process-wide lock, stalling
//     every stream of the process;
//   * code being recorded into a CUDA graph, where an allocation in the middle of the
//     recorded region is not allowed;
//   * hosts that bind only this C ABI and have no device allocator of their own (every
//     buffer they hold was handed to them by another runtime).
// For them, ntb200_paged_attention_decode_noalloc runs the same kernels with the partials
// kept in a fixed-size array compiled into this library (file scope, below).
//
// Properties a caller must know:
//   * The array is NTB200_DECODE_NOALLOC_SCRATCH_BYTES (64 MiB).  It is part of the
//     library's device image: every GPU on which this entry point is set up holds it until
//     the process exits.  A call whose split-K partials need more (about
//     num_seqs * num_q_heads * ceil(max_seq_len / split) * 516 bytes) is rejected with
//     NTB200_ERR_WORKSPACE and a message naming both sizes; nothing is launched.
//   * The first call on a device resolves the array's device address (one
//     cudaGetSymbolAddress with that device current).  Make that first call before
//     capturing a stream into a CUDA graph.  Only a successful lookup is kept: a lookup
//     that fails (for example because the module could not be loaded, or because it was
//     attempted during a capture) returns NTB200_ERR_CUDA, clears the CUDA error it left,
//     and the next call on that device tries again.
//   * Under CUDA's default lazy module loading, a GPU holds the array only once this
//     library's device code is loaded on it; with CUDA_MODULE_LOADING=EAGER every GPU whose
//     context loads the library holds it, whether or not this entry point is called.
//   * Every call on a device shares the one array and leaves its partials there.  No
//     part of it needs to start at zero: each partial the merge step reads was written by
//     the same call.  Two calls whose kernels overlap on the GPU (different streams, or
//     different host threads, without ordering between them) race on the array and give
//     wrong results; order them on one stream.
#include <mutex>

#include "common.cuh"

#define NTB200_DECODE_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)

// In host code this name is a host-side stand-in, not a device address: only the address
// returned by cudaGetSymbolAddress may be handed to a kernel.
static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[NTB200_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex[kMaxDevices];
void* g_scratch_addr[kMaxDevices];  // written once under the device's mutex, then only read

// The device address of the scratch array on `dev` (the current device), or nullptr with
// *err set when the lookup fails; a failed lookup is not remembered.
void* scratch_address(int dev, cudaError_t* err) {
  std::lock_guard<std::mutex> lock(g_setup_mutex[dev]);
  if (g_scratch_addr[dev] != nullptr) return g_scratch_addr[dev];
  void* p = nullptr;
  *err = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
  if (*err != cudaSuccess || p == nullptr) {
    cudaGetLastError();  // leave no sticky-looking error behind for the caller's next check
    return nullptr;
  }
  g_scratch_addr[dev] = p;
  return p;
}
}  // namespace

extern "C" int ntb200_paged_attention_decode_noalloc(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks_per_seq, int64_t block_table_stride,
    int64_t max_seq_len, float scale, int64_t q_seq_stride, int64_t q_head_stride,
    int64_t out_seq_stride, int64_t out_head_stride, int64_t cache_block_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, int dtype, void* stream) {
  using namespace ntb200;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "paged_decode_noalloc: no current CUDA device");
  }
  cudaError_t lookup = cudaSuccess;
  void* scratch = scratch_address(dev, &lookup);
  if (scratch == nullptr) {
    return fail(NTB200_ERR_CUDA, "paged_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(lookup));
  }
  // the split-K partials this call needs, for the same effective context bound the
  // decode entry point uses (max_seq_len clamped to the block table's capacity)
  const int64_t cap = max_blocks_per_seq * block_size;
  const int64_t msl = (max_seq_len <= 0 || max_seq_len > cap) ? cap : max_seq_len;
  if (num_seqs > 0 && msl > 0) {
    const size_t need = ntb200_paged_attention_decode_workspace_size(num_seqs, num_q_heads, num_kv_heads,
                                                                      head_size, block_size, msl);
    if (need > NTB200_DECODE_NOALLOC_SCRATCH_BYTES) {
      return fail(NTB200_ERR_WORKSPACE,
                  "paged_decode_noalloc: this call needs %zu bytes of split-K scratch; the static scratch holds %u "
                  "bytes -- use ntb200_paged_attention_decode with a caller workspace",
                  need, NTB200_DECODE_NOALLOC_SCRATCH_BYTES);
    }
  }
  return ntb200_paged_attention_decode(out, query, key_cache, value_cache, seq_lens, block_tables, num_seqs,
                                       num_q_heads, num_kv_heads, head_size, block_size, num_blocks,
                                       max_blocks_per_seq, block_table_stride, max_seq_len, scale, q_seq_stride,
                                       q_head_stride, out_seq_stride, out_head_stride, cache_block_stride,
                                       cache_page_stride, cache_head_stride, scratch,
                                       NTB200_DECODE_NOALLOC_SCRATCH_BYTES, dtype, stream);
}

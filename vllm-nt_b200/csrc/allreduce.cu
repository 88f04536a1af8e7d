// One-shot all-reduce over peer memory, for the row-parallel projections of tensor
// parallelism (o_proj, down).  Each rank's GEMM writes its partial [M, N] into ordinary
// local memory; this kernel pushes it over NVLink into a slot of every rank's peer-mapped
// buffer, meets the other ranks at one barrier, and sums the W partials that were pushed
// into its own buffer (local HBM reads) in fp32.  No NCCL on this path.
//
// Buffer layout (identical on every rank; the caller maps the peers' buffers), for W
// ranks and at most `capacity` elements, slot = capacity elements rounded to 256 bytes:
//   [0, kFlagBytes)                 flags: kMaxBlocks x kMaxRanks uint32, written by peers
//   [kFlagBytes, kDataOffset)       header: calls completed on this buffer, and a count of
//                                   the running call's finished CTAs
//   [kDataOffset, + 2 W slot)       partials, [parity][rank][slot]; call e uses parity e & 1
//
// Per CTA b (the grid never exceeds the SM count, so all CTAs of a rank are resident
// together, and every rank runs the same grid over the same units): push units
// u = b, b + grid, ... of the partial into slot [e & 1][rank] of every rank; store e into
// flag [b][rank] of every rank (release, system scope, after a CTA barrier); wait, bounded,
// until the own flags [b][r] reach e -- rank r's CTA b has pushed the same units here --
// and sum them.  A rank pushes into parity e & 1 again only in call e + 2, after the
// barrier of call e + 1, which it passes only once every rank has started call e + 1 and
// hence finished reading call e: two slots need no second barrier.  e is read from the
// header and advanced by the call's last CTA, so flags only grow (compared by signed
// distance), nothing is ever cleared, and a call can be captured in a CUDA graph and
// replayed.  A wait that runs out sets NTB200_DEVERR_WAIT_TIMEOUT and the CTA goes on (its
// output is then not the sum), so no kernel can hang on a missing peer.
#include <cstring>

#include "common.cuh"

namespace ntb200 {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
constexpr int64_t kFlagBytes = int64_t(kMaxRanks) * kMaxBlocks * 4;  // 8 KiB
constexpr int64_t kDataOffset = kFlagBytes + 256;
constexpr int kThreads = 512;

int64_t slot_bytes(int64_t numel, int elem_bytes) { return ceil_div(numel * elem_bytes, 256) * 256; }

struct Header {
  uint32_t calls;     // calls completed on this buffer
  uint32_t finished;  // CTAs of the running call that are done
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// epoch a - epoch b as a signed distance, so that the comparison survives wrap-around
__device__ __forceinline__ bool reached(uint32_t seen, uint32_t epoch) {
  return static_cast<int32_t>(seen - epoch) >= 0;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) allreduce_oneshot_kernel(T* __restrict__ out,
                                                                     const T* __restrict__ partial,
                                                                     const uint64_t* __restrict__ peers,
                                                                     int64_t numel, int64_t slot, int rank,
                                                                     int world, unsigned int* err) {
  const int b = blockIdx.x;
  __shared__ uint32_t s_call;
  pdl_trigger();
  pdl_wait();  // the partial (written by the kernel before) is complete
  char* own = reinterpret_cast<char*>(peers[rank]);
  Header* hdr = reinterpret_cast<Header*>(own + kFlagBytes);
  if (threadIdx.x == 0) s_call = *reinterpret_cast<volatile uint32_t*>(&hdr->calls) + 1u;
  __syncthreads();
  const uint32_t call = s_call;
  const int64_t parity_off = kDataOffset + int64_t(call & 1u) * world * slot;

  constexpr int kVec = 16 / sizeof(T);
  const int64_t units = numel / kVec;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t first = int64_t(b) * blockDim.x + threadIdx.x;

  // 1. push this rank's units into slot [parity][rank] of every rank
  for (int64_t u = first; u < units; u += stride) {
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(partial) + u);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world)
        reinterpret_cast<uint4*>(reinterpret_cast<char*>(peers[r]) + parity_off + int64_t(rank) * slot)[u] = v;
  }
  for (int64_t e = units * kVec + first; e < numel; e += stride) {
    const T v = partial[e];
    for (int r = 0; r < world; ++r)
      reinterpret_cast<T*>(reinterpret_cast<char*>(peers[r]) + parity_off + int64_t(rank) * slot)[e] = v;
  }
  __syncthreads();

  // 2. barrier with CTA b of every rank
  if (threadIdx.x < world) {
    st_release_sys(reinterpret_cast<uint32_t*>(peers[threadIdx.x]) + b * kMaxRanks + rank, call);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(own) + b * kMaxRanks + threadIdx.x;
    if (!reached(ld_acquire_sys(mine), call)) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t it = 1;; ++it) {
        if (reached(ld_acquire_sys(mine), call)) break;
        if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitTimeoutNs) {
          raise_device_error(err, NTB200_DEVERR_WAIT_TIMEOUT);
          break;
        }
      }
    }
  }
  __syncthreads();

  // 3. sum the W partials now in this rank's buffer (L2 loads: the same addresses held
  //    another call's data two calls ago)
  const char* mine_data = own + parity_off;
  for (int64_t u = first; u < units; u += stride) {
    uint4 raw[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) raw[r] = __ldcg(reinterpret_cast<const uint4*>(mine_data + int64_t(r) * slot) + u);
    float acc[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) acc[j] = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        const T* v = reinterpret_cast<const T*>(&raw[r]);
#pragma unroll
        for (int j = 0; j < kVec; ++j) acc[j] += Elem<T>::to_f(v[j]);
      }
    }
    store_f<T, kVec>(out + u * kVec, acc);
  }
  for (int64_t e = units * kVec + first; e < numel; e += stride) {
    float acc = 0.f;
    for (int r = 0; r < world; ++r) {
      const unsigned short bits = __ldcg(reinterpret_cast<const unsigned short*>(mine_data + int64_t(r) * slot) + e);
      T v;
      memcpy(&v, &bits, sizeof(v));
      acc += Elem<T>::to_f(v);
    }
    out[e] = Elem<T>::from_f(acc);
  }

  // 4. the call's last CTA advances the call count
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&hdr->finished, 1u) == gridDim.x - 1u) {
      hdr->finished = 0u;
      __threadfence();
      atomicExch(&hdr->calls, call);
    }
  }
}

}  // namespace
}  // namespace ntb200

extern "C" size_t ntb200_allreduce_buffer_size(int64_t capacity, int elem_bytes, int world_size) {
  if (capacity < 0 || elem_bytes <= 0 || world_size < 1 || world_size > ntb200::kMaxRanks) return 0;
  return static_cast<size_t>(ntb200::kDataOffset + 2 * world_size * ntb200::slot_bytes(capacity, elem_bytes));
}

extern "C" int ntb200_allreduce_oneshot(void* out, const void* partial, const uint64_t* peer_buffers,
                                        int64_t numel, int64_t capacity, int rank, int world_size, int dtype,
                                        void* stream) {
  using namespace ntb200;
  if (numel < 0 || numel > capacity)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce: numel outside [0, capacity]");
  if (world_size < 1 || world_size > kMaxRanks || rank < 0 || rank >= world_size)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce: rank %d of %d (at most %d ranks)", rank, world_size,
                kMaxRanks);
  if (numel == 0) return NTB200_OK;
  if (out == nullptr || partial == nullptr || peer_buffers == nullptr)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce: null pointer");
  if (!aligned16(out) || !aligned16(partial))
    return fail(NTB200_ERR_MISALIGNED, "allreduce: out and partial must be 16-byte aligned");
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "allreduce: dtype %d (bf16/f16 only)", dtype);
  const int64_t units = ceil_div(numel, 8);
  int64_t grid = ceil_div(units, kThreads);
  const int64_t cap = num_sms() < kMaxBlocks ? num_sms() : kMaxBlocks;
  if (grid > cap) grid = cap;
  const int64_t slot = slot_bytes(capacity, 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == NTB200_DTYPE_BF16)
    return launch_kernel("allreduce_oneshot", allreduce_oneshot_kernel<__nv_bfloat16>, dim3(unsigned(grid)),
                         dim3(kThreads), 0, s, static_cast<__nv_bfloat16*>(out),
                         static_cast<const __nv_bfloat16*>(partial), peer_buffers, numel, slot, rank, world_size,
                         device_error_word());
  return launch_kernel("allreduce_oneshot", allreduce_oneshot_kernel<__half>, dim3(unsigned(grid)), dim3(kThreads),
                       0, s, static_cast<__half*>(out), static_cast<const __half*>(partial), peer_buffers, numel,
                       slot, rank, world_size, device_error_word());
}

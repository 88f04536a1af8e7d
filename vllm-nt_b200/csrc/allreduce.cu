// One-shot all-reduce over peer memory, for the row-parallel projections of tensor
// parallelism (o_proj, down): every rank's GEMM writes its partial [M, N] into its own
// peer-mapped buffer, then each rank reads all W partials over NVLink, sums them in fp32
// and writes the result into local memory.  No NCCL on this path.
//
// Buffer layout (identical on every rank; the caller maps the peers' buffers):
//   [0, kFlagBytes)              flags: kMaxBlocks x kMaxRanks uint32, written by peers
//   [kFlagBytes, kDataOffset)    header: the number of calls completed on this buffer and
//                                a count of this call's finished CTAs
//   [kDataOffset, + capacity)    this rank's partial (the GEMM writes it there)
//
// Synchronisation, per CTA b (the grid never exceeds the SM count, so all CTAs of a rank
// are resident together): entry barrier -- CTA b of every rank stores 2e-1 into flag
// [b][rank] of every peer (release, system scope) and waits, bounded, until its own flags
// [b][r] reach 2e-1: every peer's partial is complete.  It then sums its share.  Exit
// barrier -- the same with 2e: no peer reads this rank's partial any more, so the next
// call's GEMM may overwrite it.  e is the call's number, read from the header; the last
// CTA to finish advances it.  Flags only grow and are compared by signed distance, so
// nothing is ever cleared, and everything lives on the device: a call can be captured in
// a CUDA graph and replayed.  A wait that runs out sets NTB200_DEVERR_WAIT_TIMEOUT and the
// CTA goes on (its output is then not the sum), so no kernel can hang on a missing peer.
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

// Peer partials are read with strong (relaxed, system-scope) loads: a weak or
// cache-volatile load may be served from a line this GPU cached in an earlier call, while
// a strong load observes the value the peer's GEMM wrote before its release of the flag.
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint16_t ld_relaxed_sys_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.relaxed.sys.global.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
  return v;
}

// epoch a - epoch b as a signed distance, so that the comparison survives wrap-around
__device__ __forceinline__ bool reached(uint32_t seen, uint32_t epoch) {
  return static_cast<int32_t>(seen - epoch) >= 0;
}

// CTA b's barrier with its counterparts on every rank: announce `value`, wait for theirs.
__device__ __forceinline__ void peer_barrier(const uint64_t* peers, int b, int rank, int world, uint32_t value,
                                             unsigned int* err) {
  if (threadIdx.x < world) {
    __threadfence_system();
    char* peer = reinterpret_cast<char*>(peers[threadIdx.x]);
    st_release_sys(reinterpret_cast<uint32_t*>(peer) + b * kMaxRanks + rank, value);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(peers[rank]) + b * kMaxRanks + threadIdx.x;
    if (!reached(ld_acquire_sys(mine), value)) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t it = 1;; ++it) {
        if (reached(ld_acquire_sys(mine), value)) break;
        if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitTimeoutNs) {
          raise_device_error(err, NTB200_DEVERR_WAIT_TIMEOUT);
          break;
        }
      }
    }
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kThreads) allreduce_oneshot_kernel(T* __restrict__ out,
                                                                     const uint64_t* __restrict__ peers,
                                                                     int64_t numel, int rank, int world,
                                                                     unsigned int* err) {
  const int b = blockIdx.x;
  __shared__ uint32_t s_call;
  pdl_trigger();
  pdl_wait();  // the partial of this rank (written by the kernel before) is complete
  Header* hdr = reinterpret_cast<Header*>(reinterpret_cast<char*>(peers[rank]) + kFlagBytes);
  if (threadIdx.x == 0) s_call = *reinterpret_cast<volatile uint32_t*>(&hdr->calls) + 1u;
  __syncthreads();
  const uint32_t call = s_call;
  peer_barrier(peers, b, rank, world, 2u * call - 1u, err);

  // sum: 16-byte units (8 bf16/f16), all W loads of a unit in flight before the adds
  constexpr int kVec = 16 / sizeof(T);
  const int64_t units = numel / kVec;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t u = int64_t(b) * blockDim.x + threadIdx.x; u < units; u += stride) {
    uint4 raw[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world)
        raw[r] = ld_relaxed_sys_v4(reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(peers[r]) + kDataOffset) + u);
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
  // ragged tail
  for (int64_t e = units * kVec + int64_t(b) * blockDim.x + threadIdx.x; e < numel; e += stride) {
    float acc = 0.f;
    for (int r = 0; r < world; ++r) {
      const uint16_t bits =
          ld_relaxed_sys_u16(reinterpret_cast<const T*>(reinterpret_cast<const char*>(peers[r]) + kDataOffset) + e);
      T v;
      memcpy(&v, &bits, sizeof(v));
      acc += Elem<T>::to_f(v);
    }
    out[e] = Elem<T>::from_f(acc);
  }
  __syncthreads();  // this CTA's reads of the peers' partials are done
  peer_barrier(peers, b, rank, world, 2u * call, err);
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&hdr->finished, 1u) == gridDim.x - 1u) {  // the call's last CTA
      hdr->finished = 0u;
      __threadfence();
      atomicExch(&hdr->calls, call);
    }
  }
}

}  // namespace
}  // namespace ntb200

extern "C" size_t ntb200_allreduce_buffer_size(int64_t capacity, int elem_bytes) {
  if (capacity < 0 || elem_bytes <= 0) return 0;
  return static_cast<size_t>(ntb200::kDataOffset + ntb200::slot_bytes(capacity, elem_bytes));
}

extern "C" int64_t ntb200_allreduce_data_offset(void) { return ntb200::kDataOffset; }

extern "C" int ntb200_allreduce_oneshot(void* out, const uint64_t* peer_buffers, int64_t numel, int rank,
                                        int world_size, int dtype, void* stream) {
  using namespace ntb200;
  if (numel < 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce: numel < 0");
  if (world_size < 1 || world_size > kMaxRanks || rank < 0 || rank >= world_size)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce: rank %d of %d (at most %d ranks)", rank, world_size,
                kMaxRanks);
  if (numel == 0) return NTB200_OK;
  if (out == nullptr || peer_buffers == nullptr) return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce: null pointer");
  if (!aligned16(out)) return fail(NTB200_ERR_MISALIGNED, "allreduce: out must be 16-byte aligned");
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "allreduce: dtype %d (bf16/f16 only)", dtype);
  const int64_t units = ceil_div(numel, 8);
  int64_t grid = ceil_div(units, kThreads);
  const int64_t cap = num_sms() < kMaxBlocks ? num_sms() : kMaxBlocks;
  if (grid > cap) grid = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == NTB200_DTYPE_BF16)
    return launch_kernel("allreduce_oneshot", allreduce_oneshot_kernel<__nv_bfloat16>, dim3(unsigned(grid)),
                         dim3(kThreads), 0, s, static_cast<__nv_bfloat16*>(out), peer_buffers, numel, rank,
                         world_size, device_error_word());
  return launch_kernel("allreduce_oneshot", allreduce_oneshot_kernel<__half>, dim3(unsigned(grid)), dim3(kThreads),
                       0, s, static_cast<__half*>(out), peer_buffers, numel, rank, world_size, device_error_word());
}

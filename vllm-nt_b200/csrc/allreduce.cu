// One-shot all-reduce over peer memory, for the row-parallel projections of tensor
// parallelism (o_proj, down).  Each rank's GEMM writes its partial [M, N] into ordinary
// local memory; this kernel pushes it over NVLink into a slot of every rank's peer-mapped
// buffer, meets the other ranks at one barrier, and sums the W partials that were pushed
// into its own buffer (local HBM reads) in fp32.  No NCCL on this path.
//
// Buffer layout (identical on every rank; the caller maps the peers' buffers), for W
// ranks and at most `capacity` elements, slot = capacity elements rounded to 256 bytes,
// chunk slot = ceil(capacity / W) elements (a multiple of 8) rounded to 256 bytes:
//   [0, 8 KiB)                      flag array 1: kMaxBlocks x kMaxRanks uint32, written by peers
//   [8 KiB, 16 KiB)                 flag array 2 (the two-shot kernel's second barrier)
//   [16 KiB, kDataOffset)           header: calls completed on this buffer, and a count of
//                                   the running call's finished CTAs
//   [kDataOffset, + 2 W slot)       one-shot partials, [parity][rank][slot]; call e uses parity e & 1
//   [.., + W chunk slot)            two-shot scatter slots [rank]
//   [.., + chunk slot)              two-shot reduced chunk of this rank
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
constexpr int64_t kFlagBytes = int64_t(kMaxRanks) * kMaxBlocks * 4;  // 8 KiB per flag array
constexpr int64_t kFlags2 = kFlagBytes;                               // second barrier (two-shot)
constexpr int64_t kHeaderOffset = 2 * kFlagBytes;
constexpr int64_t kDataOffset = kHeaderOffset + 256;
constexpr int kThreads = 512;

int64_t slot_bytes(int64_t numel, int elem_bytes) { return ceil_div(numel * elem_bytes, 256) * 256; }

// Two-shot chunking: the message is cut into `world` chunks of chunk_elems (a multiple of 8,
// so every chunk starts on 16 bytes); rank r reduces chunk r.
int64_t chunk_elems(int64_t numel, int world) { return ceil_div(ceil_div(numel, world), 8) * 8; }

// Offset of the two-shot area (after the one-shot parity slots): W scatter slots of one
// chunk each, then the reduced chunk.
int64_t twoshot_offset(int64_t capacity, int elem_bytes, int world) {
  return kDataOffset + 2 * world * slot_bytes(capacity, elem_bytes);
}

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
  Header* hdr = reinterpret_cast<Header*>(own + kHeaderOffset);
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

// Waits (bounded) until CTA b of every rank has stored `call` into flag array `flags` of
// this rank's buffer, after storing it into the same slot of every peer's array.  Thread t
// < world handles peer t.
__device__ __forceinline__ void rank_barrier(const uint64_t* peers, int64_t flags, const char* own, int b,
                                             int rank, int world, uint32_t call, unsigned int* err) {
  if (threadIdx.x < world) {
    st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(peers[threadIdx.x]) + flags) +
                       b * kMaxRanks + rank,
                   call);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(own + flags) + b * kMaxRanks + threadIdx.x;
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
}

__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Two-shot all-reduce (reduce-scatter, then all-gather) over the same peer-mapped buffers:
//   1. push chunk d of the partial into scatter slot [rank] of rank d (all d, own included);
//   2. barrier 1 (flag array 1) with CTA b of every rank;
//   3. sum the W slots of the own chunk in fp32 (rank order), round, write it to `out` and
//      to the own reduced-chunk area;
//   4. barrier 2 (flag array 2);
//   5. read every other rank's reduced chunk (system-scope loads over NVLink) into `out`.
// Each rank moves 2 (W - 1) / W of the message over NVLink instead of the one-shot push's
// (W - 1).  A 16-byte unit u of any chunk is handled by the same CTA (b = u / 512 mod grid)
// on every rank and in every step, so a rank writes a slot or its reduced area again (next
// call, step 1 or 3) only after the barrier at which every rank has finished reading it.
// Calls share the header's call count (and flag array 1) with the one-shot kernel, and the
// two-shot area lies past the one-shot slots, so the two kinds of call may alternate.
template <typename T>
__global__ void __launch_bounds__(kThreads) allreduce_twoshot_kernel(T* __restrict__ out, const T* __restrict__ partial,
                                                                     const uint64_t* __restrict__ peers,
                                                                     int64_t numel, int64_t chunk, int64_t cslot,
                                                                     int64_t area, int rank, int world,
                                                                     unsigned int* err) {
  const int b = blockIdx.x;
  __shared__ uint32_t s_call;
  pdl_trigger();
  pdl_wait();
  const char* own = reinterpret_cast<const char*>(peers[rank]);
  Header* hdr = reinterpret_cast<Header*>(const_cast<char*>(own) + kHeaderOffset);
  if (threadIdx.x == 0) s_call = *reinterpret_cast<volatile uint32_t*>(&hdr->calls) + 1u;
  __syncthreads();
  const uint32_t call = s_call;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t first = int64_t(b) * blockDim.x + threadIdx.x;
  auto chunk_units = [&](int d) -> int64_t {
    const int64_t lo = int64_t(d) * chunk;
    const int64_t hi = lo + chunk < numel ? lo + chunk : numel;
    return hi > lo ? (hi - lo) / 8 : 0;  // numel is a multiple of 8
  };

  // 1. scatter: chunk d of the partial -> rank d's slot [rank]; start with the next rank so
  //    that the ranks' first pushes go to different peers
  for (int i = 0; i < world; ++i) {
    const int d = (rank + 1 + i) % world;
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(peers[d]) + area + int64_t(rank) * cslot);
    const uint4* src = reinterpret_cast<const uint4*>(partial + int64_t(d) * chunk);
    const int64_t nu = chunk_units(d);
    for (int64_t u = first; u < nu; u += stride) dst[u] = __ldcs(src + u);
  }
  __syncthreads();
  rank_barrier(peers, 0, own, b, rank, world, call, err);

  // 3. reduce the own chunk
  {
    uint4* reduced = reinterpret_cast<uint4*>(const_cast<char*>(own) + area + int64_t(world) * cslot);
    uint4* dst = reinterpret_cast<uint4*>(out + int64_t(rank) * chunk);
    const int64_t nu = chunk_units(rank);
    for (int64_t u = first; u < nu; u += stride) {
      uint4 raw[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < world) raw[r] = __ldcg(reinterpret_cast<const uint4*>(own + area + int64_t(r) * cslot) + u);
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r < world) {
          const T* v = reinterpret_cast<const T*>(&raw[r]);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += Elem<T>::to_f(v[j]);
        }
      }
      const Vec<T, 8> packed = pack_f<T, 8>(acc);
      const uint4 bits = *reinterpret_cast<const uint4*>(&packed);
      dst[u] = bits;
      reduced[u] = bits;
    }
  }
  __syncthreads();
  rank_barrier(peers, kFlags2, own, b, rank, world, call, err);

  // 5. gather the other ranks' reduced chunks
  for (int i = 1; i < world; ++i) {
    const int d = (rank + i) % world;
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(peers[d]) + area +
                                                      int64_t(world) * cslot);
    uint4* dst = reinterpret_cast<uint4*>(out + int64_t(d) * chunk);
    const int64_t nu = chunk_units(d);
    for (int64_t u = first; u < nu; u += stride) dst[u] = ld_relaxed_sys_v4(src + u);
  }

  // 6. the call's last CTA advances the call count
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
  using namespace ntb200;
  if (capacity < 0 || elem_bytes <= 0 || world_size < 1 || world_size > kMaxRanks) return 0;
  const int64_t cslot = slot_bytes(chunk_elems(capacity, world_size), elem_bytes);
  return static_cast<size_t>(twoshot_offset(capacity, elem_bytes, world_size) + (world_size + 1) * cslot);
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

extern "C" int ntb200_allreduce_twoshot(void* out, const void* partial, const uint64_t* peer_buffers,
                                        int64_t numel, int64_t capacity, int rank, int world_size, int dtype,
                                        void* stream) {
  using namespace ntb200;
  if (numel < 0 || numel > capacity)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce_twoshot: numel outside [0, capacity]");
  if (numel % 8 != 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce_twoshot: numel must be a multiple of 8");
  if (world_size < 1 || world_size > kMaxRanks || rank < 0 || rank >= world_size)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce_twoshot: rank %d of %d (at most %d ranks)", rank, world_size,
                kMaxRanks);
  if (numel == 0) return NTB200_OK;
  if (out == nullptr || partial == nullptr || peer_buffers == nullptr)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "allreduce_twoshot: null pointer");
  if (!aligned16(out) || !aligned16(partial))
    return fail(NTB200_ERR_MISALIGNED, "allreduce_twoshot: out and partial must be 16-byte aligned");
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "allreduce_twoshot: dtype %d (bf16/f16 only)", dtype);
  const int64_t chunk = chunk_elems(numel, world_size);
  const int64_t cslot = slot_bytes(chunk_elems(capacity, world_size), 2);
  const int64_t area = twoshot_offset(capacity, 2, world_size);
  int64_t grid = ceil_div(chunk / 8, kThreads);
  const int64_t cap = num_sms() < kMaxBlocks ? num_sms() : kMaxBlocks;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == NTB200_DTYPE_BF16)
    return launch_kernel("allreduce_twoshot", allreduce_twoshot_kernel<__nv_bfloat16>, dim3(unsigned(grid)),
                         dim3(kThreads), 0, s, static_cast<__nv_bfloat16*>(out),
                         static_cast<const __nv_bfloat16*>(partial), peer_buffers, numel, chunk, cslot, area, rank,
                         world_size, device_error_word());
  return launch_kernel("allreduce_twoshot", allreduce_twoshot_kernel<__half>, dim3(unsigned(grid)), dim3(kThreads), 0,
                       s, static_cast<__half*>(out), static_cast<const __half*>(partial), peer_buffers, numel, chunk,
                       cslot, area, rank, world_size, device_error_word());
}

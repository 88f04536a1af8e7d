// Dense projection GEMM on the 5th-generation tensor cores:
//   out[M, N] = x[M, K] . W[N, K]^T (+ bias),  bf16/f16 in, fp32 accumulate in TMEM.
//
// 256 < M < 2048: persistent, warp-specialised, one CTA per SM (192 threads), tile 128 x BN
// with BN = 256, 192 or 128 picked per shape to fill whole waves of SMs:
//   warp 0      TMA producer: 128x64 x-tile + BNx64 W-tile per k-step (128-byte swizzle,
//               K-major) into a ~192-200 KB shared-memory ring;
//   warp 1      allocates TMEM for two 128xBN fp32 accumulators and its lane 0 issues
//               tcgen05.mma (M=128, N=BN, K=16; four per k-step), committing each stage
//               back to the producer and each finished tile to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM lanes
//               32*(w%4)..+31, i.e. output rows), add bias, round, store.
// The epilogue of tile i overlaps the MMAs of tile i+1 (double-buffered accumulator).
// M >= 2048: the same roles in CTA pairs with 256 x 256 tiles (tcgen05 cta_group::2).
// Tiles are walked with the M index fastest so a wave of CTAs shares W tiles through L2
// while x (M*K*2 bytes) stays L2-resident.  No TMA multicast is used anywhere.
//
// Every mbarrier wait is bounded (2 s); a timeout sets NTB200_DEVERR_WAIT_TIMEOUT, the
// roles leave their loops, in-flight copies and MMAs are drained (bounded), and TMEM is
// freed before the CTA exits.
//
// Replaces vllm_nt/_ntops/kernels/linear.py:9-85 (a Triton tl.dot tile loop).
#include <atomic>

#include "common.cuh"
#include "tcgen05.cuh"

namespace ntb200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kATileBytes = BM * BK * 2;

// Tile width BN (UMMA N) of the large-M kernel: 256, 192 or 128, chosen per shape so that
// the tiles fill whole waves of SMs.  The ring holds ~192-200 KB of stages either way.
template <int BN_>
struct GemmCfg {
  static constexpr int BN = BN_;
  static constexpr int kBTileBytes = BN * BK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kStages = BN == 256 ? 4 : (BN == 192 ? 5 : 6);
  static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;  // two accumulators, power of 2
  static constexpr int kRing = 0;
  static constexpr int kFull = kStages * kStageBytes;
  static constexpr int kEmpty = kFull + 8 * kStages;
  static constexpr int kTmemFull = kEmpty + 8 * kStages;
  static constexpr int kTmemEmpty = kTmemFull + 16;
  static constexpr int kMmaDone = kTmemEmpty + 16;
  static constexpr int kTmemBase = kMmaDone + 8;
  static constexpr int kEnd = kTmemBase + 8;
  static constexpr int kDynamicBytes = kEnd + 1024;
  static_assert(kDynamicBytes <= 227 * 1024, "ring exceeds shared memory");
};

struct GemmParams {
  void* out;
  const void* bias;
  int64_t M, N, K;
  int64_t out_stride;
  int num_m_blocks, num_n_blocks;
  int group_m;  // M blocks per raster group (num_m_blocks: plain M-fastest order)
  int64_t n_half;  // SwiGLU variants: output columns I; W rows [0, I) gate, [I, 2I) up
  unsigned int* err;
};

// silu(gate) * up for the fused gate_up epilogue, with the rounding points of vLLM's
// unfused pair (the GEMM rounds both halves to T, SiluAndMul rounds silu(gate) to T
// before the multiply, the store rounds the product) and the same silu expression as
// silu_and_mul.cu, so the fused and unfused results are identical.
template <typename T>
__device__ __forceinline__ float swiglu(float gate_acc, float up_acc) {
  const float g = Elem<T>::round(gate_acc), u = Elem<T>::round(up_acc);
  return Elem<T>::round(silu_f(g)) * u;
}

// Writes 32 consecutive output columns c0.. of one row (bias added when given; columns at
// or past ncols are dropped), with 16-byte stores when the segment is whole and aligned.
template <typename T>
__device__ __forceinline__ void store_row32(T* orow, int64_t c0, int64_t ncols, float (&v)[32], const T* bias) {
  if (bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c0 + i < ncols) v[i] += Elem<T>::to_f(bias[c0 + i]);
  }
  if (c0 + 32 <= ncols && ((reinterpret_cast<uintptr_t>(orow + c0) & 15u) == 0)) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = v[q * 8 + i];
      store_f<T, 8>(orow + c0 + q * 8, w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c0 + i < ncols) orow[c0 + i] = Elem<T>::from_f(v[i]);
  }
}

// Tile order: groups of `group_m` M blocks, M fastest inside a group, then N, then the next
// group.  With group_m = num_m_blocks this is plain M-fastest order (x stays L2-resident
// while each W tile is read once); a smaller group bounds the x rows a wave touches when x
// is larger than L2, so that neither operand is streamed from HBM once per wave.
__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& mb, int& nb) {
  const int per_group = p.group_m * p.num_n_blocks;
  const int g = tile / per_group;
  const int first_m = g * p.group_m;
  const int rows = p.num_m_blocks - first_m < p.group_m ? p.num_m_blocks - first_m : p.group_m;
  const int r = tile - g * per_group;
  mb = first_m + r % rows;
  nb = r / rows;
}

// SWIGLU: out[:, j] = silu(x.W[j]) * x.W[I + j] (W = vLLM's merged gate_up weight); a
// tile's B operand is BN/2 gate rows followed by the BN/2 matching up rows.
template <typename T, int BN_, bool SWIGLU = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_tcgen05_kernel(
    const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
    const GemmParams p) {
  using C = GemmCfg<BN_>;
  constexpr int BN = C::BN;
  constexpr int kStages = C::kStages;
  constexpr int kStageBytes = C::kStageBytes;
  constexpr int kTmemCols = C::kTmemCols;
  constexpr int kAccStride = BN == 192 ? 256 : BN;  // TMEM column offset of the 2nd accumulator
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + C::kEmpty);
  uint64_t* tmem_full = reinterpret_cast<uint64_t*>(smem + C::kTmemFull);
  uint64_t* tmem_empty = reinterpret_cast<uint64_t*>(smem + C::kTmemEmpty);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(smem + C::kMmaDone);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemBase);
  const uint32_t ring = smem_u32(smem + C::kRing);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int k_steps = static_cast<int>((p.K + BK - 1) / BK);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  // tensor memory is allocated only after the preceding kernel has finished: a CTA of it
  // that shares this SM may still be waiting to allocate its own
  pdl_wait();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a_map)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&b_map)) : "memory");
      uint32_t it = 0;  // global k-step counter of this CTA
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        for (int kb = 0; kb < k_steps; ++kb, ++it) {
          const uint32_t s = it % kStages;
          if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          const uint32_t a_dst = ring + s * kStageBytes;
          const uint32_t b_dst = a_dst + kATileBytes;
          tma_load_2d(a_dst, &a_map, kb * BK, mb * BM, smem_u32(&full[s]));
          if constexpr (SWIGLU) {
            tma_load_2d(b_dst, &b_map, kb * BK, nb * (BN / 2), smem_u32(&full[s]));
            tma_load_2d(b_dst + (BN / 2) * BK * 2, &b_map, kb * BK, static_cast<int>(p.n_half) + nb * (BN / 2),
                        smem_u32(&full[s]));
          } else {
            tma_load_2d(b_dst, &b_map, kb * BK, nb * BN, smem_u32(&full[s]));
          }
        }
      }
      // drain the copies still in flight
      const uint32_t first = it > kStages ? it - kStages : 0;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % kStages], (j / kStages) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc(sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value, BM, BN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const int use = local >> 1;
        if (use >= 1 && !mbar_wait(&tmem_empty[acc], (use - 1) & 1, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccStride;
        for (int kb = 0; kb < k_steps; ++kb, ++it) {
          const uint32_t s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = ring + s * kStageBytes;
          const uint32_t b_addr = a_addr + kATileBytes;
          const uint64_t adesc = sw128_kmajor_desc(a_addr);
          const uint64_t bdesc = sw128_kmajor_desc(b_addr);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 elements (32 bytes) along K inside the swizzled 128-byte rows
            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);  // accumulator complete
      }
      // all issued MMAs complete before TMEM may be released
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.err);
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    T* out = static_cast<T*>(p.out);
    const T* bias = static_cast<const T*>(p.bias);
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const int use = local >> 1;
      if (!mbar_wait(&tmem_full[acc], use & 1, p.err)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int64_t row = int64_t(mb) * BM + row_in_tile;
      T* orow = out + row * p.out_stride;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + acc * kAccStride;
      if constexpr (SWIGLU) {
        const int64_t col0 = int64_t(nb) * (BN / 2);
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 64; ++chunk) {
          uint32_t g[32], u[32];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it together
          tmem_ld_32(taddr + chunk * 32, g);
          tmem_ld_32(taddr + BN / 2 + chunk * 32, u);
          const int64_t c0 = col0 + chunk * 32;
          if (row < p.M && c0 < p.n_half) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = swiglu<T>(__uint_as_float(g[i]), __uint_as_float(u[i]));
            store_row32<T>(orow, c0, p.n_half, v, nullptr);
          }
        }
      } else {
        const int64_t col0 = int64_t(nb) * BN;
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          uint32_t r[32];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it together
          tmem_ld_32(taddr + chunk * 32, r);
          const int64_t c0 = col0 + chunk * 32;
          if (row < p.M && c0 < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            store_row32<T>(orow, c0, p.N, v, bias);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------------------------
// Large M (M >= kPairMinM): CTA pairs.  A cluster of two CTAs computes a 256 x 256 output
// tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  CTA r of the pair stages,
// per 64-wide k-step, x rows [256*mb + 128*r, +128) and W rows [256*nb + 128*r, +128) in
// its own shared memory; the MMA, issued by the even CTA, reads both CTAs' tiles and
// leaves each CTA's 128 output rows (all 256 columns) in that CTA's TMEM.  For the same
// tensor-core work per SM a k-step moves 32 KB into shared memory instead of the 48 KB of
// a 128 x 256 single-CTA tile.  Synchronisation across the pair:
//   full[s]       (even CTA) armed by its producer with both CTAs' bytes; both CTAs' TMA
//                 loads complete_tx on it (.cta_group::2 lets a load signal the peer);
//   empty[s]      (each CTA) the MMA issuer commits to both CTAs' barriers;
//   tmem_full[a]  (each CTA) committed to both CTAs when an accumulator is final;
//   tmem_empty[a] (even CTA) 8 arrivals: the 4 epilogue warps of each CTA.
// A cluster barrier after set-up and another before TMEM is freed keep each CTA's shared
// memory alive while its peer may still reach it.  No multicast is used.
// ------------------------------------------------------------------------------------
constexpr int64_t kPairMinM = 2048;

struct PairCfg {
  static constexpr int kHalf = 128;                  // x rows and W rows each CTA stages
  static constexpr int kTile = 256;                  // output tile of the pair (M and N)
  static constexpr int kHalfBytes = kHalf * BK * 2;  // 16 KB
  static constexpr int kStageBytes = 2 * kHalfBytes;
  static constexpr int kStages = 7;
  static constexpr int kTmemCols = 512;  // two 128 x 256 fp32 accumulators per CTA
  static constexpr int kRing = 0;
  static constexpr int kFull = kStages * kStageBytes;
  static constexpr int kEmpty = kFull + 8 * kStages;
  static constexpr int kTmemFull = kEmpty + 8 * kStages;
  static constexpr int kTmemEmpty = kTmemFull + 16;
  static constexpr int kMmaDone = kTmemEmpty + 16;
  static constexpr int kTmemBase = kMmaDone + 8;
  static constexpr int kEnd = kTmemBase + 8;
  static constexpr int kDynamicBytes = kEnd + 1024;
  static_assert(kDynamicBytes <= 227 * 1024, "ring exceeds shared memory");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}

// TMA tile load into this CTA's shared memory whose completion is counted on an mbarrier
// of either CTA of the pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` (a shared::cluster address in either CTA) once every tcgen05.mma this
// thread has issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void pair_cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// SWIGLU: the even CTA stages gate rows [128*nb, +128) and the odd CTA the matching up
// rows [I + 128*nb, +128), so accumulator columns [0, 128) hold x.gate and [128, 256)
// x.up for the same 128 output columns.
template <typename T, bool SWIGLU = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_pair_kernel(
    const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
    const GemmParams p) {
  using C = PairCfg;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + C::kEmpty);
  uint64_t* tmem_full = reinterpret_cast<uint64_t*>(smem + C::kTmemFull);
  uint64_t* tmem_empty = reinterpret_cast<uint64_t*>(smem + C::kTmemEmpty);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(smem + C::kMmaDone);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemBase);
  const uint32_t ring = smem_u32(smem + C::kRing);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: issues the MMAs; 1: its peer
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int k_steps = static_cast<int>((p.K + BK - 1) / BK);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  // tensor memory is allocated only after the preceding kernel has finished
  pdl_wait();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  pair_cluster_sync();  // both CTAs' barriers are initialised before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) ------------------------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a_map)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&b_map)) : "memory");
      const uint32_t full0 = peer_addr(smem_u32(&full[0]), 0);  // the even CTA's full[0]
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int arow = mb * C::kTile + static_cast<int>(rank) * C::kHalf;
        const int brow = SWIGLU ? (rank == 0 ? nb * C::kHalf : static_cast<int>(p.n_half) + nb * C::kHalf)
                                : nb * C::kTile + static_cast<int>(rank) * C::kHalf;
        for (int kb = 0; kb < k_steps; ++kb, ++it) {
          const uint32_t s = it % kStages;
          if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::kStageBytes);
          const uint32_t a_dst = ring + s * C::kStageBytes;
          tma_load_2d_pair(a_dst, &a_map, kb * BK, arow, full0 + 8 * s);
          tma_load_2d_pair(a_dst + C::kHalfBytes, &b_map, kb * BK, brow, full0 + 8 * s);
        }
      }
      // drain: every stage this CTA filled has been consumed (or the wait gives up)
      const uint32_t first = it > kStages ? it - kStages : 0;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&empty[j % kStages], (j / kStages) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (even CTA) ------------------------------
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc(std::is_same<T, __nv_bfloat16>::value, C::kTile, C::kTile);
      const uint32_t empty_peer = peer_addr(smem_u32(&empty[0]), 1);
      const uint32_t tfull_peer = peer_addr(smem_u32(&tmem_full[0]), 1);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++local) {
        const int acc = local & 1;
        const int use = local >> 1;
        if (use >= 1 && !mbar_wait(&tmem_empty[acc], (use - 1) & 1, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::kTile;
        for (int kb = 0; kb < k_steps; ++kb, ++it) {
          const uint32_t s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = ring + s * C::kStageBytes;
          const uint64_t adesc = sw128_kmajor_desc(a_addr);
          const uint64_t bdesc = sw128_kmajor_desc(a_addr + C::kHalfBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair(smem_u32(&empty[s]));  // frees the stage in both CTAs
          umma_commit_pair(empty_peer + 8 * s);
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tmem_full[acc]));  // accumulator complete in both CTAs
        umma_commit_pair(tfull_peer + 8 * acc);
      }
      umma_commit_pair(smem_u32(mma_done));
      mbar_wait(mma_done, 0, p.err);
    }
  } else {
    // ------------------------------ epilogue (both CTAs) ------------------------------
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = static_cast<int>(rank) * C::kHalf + quad * 32 + lane;
    const uint32_t tempty0 = peer_addr(smem_u32(&tmem_empty[0]), 0);
    T* out = static_cast<T*>(p.out);
    const T* bias = static_cast<const T*>(p.bias);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      const int acc = local & 1;
      const int use = local >> 1;
      if (!mbar_wait(&tmem_full[acc], use & 1, p.err)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int64_t row = int64_t(mb) * C::kTile + row_in_tile;
      T* orow = out + row * p.out_stride;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + acc * C::kTile;
      if constexpr (SWIGLU) {
        const int64_t col0 = int64_t(nb) * C::kHalf;
#pragma unroll 1
        for (int chunk = 0; chunk < C::kHalf / 32; ++chunk) {
          uint32_t g[32], u[32];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it together
          tmem_ld_32(taddr + chunk * 32, g);
          tmem_ld_32(taddr + C::kHalf + chunk * 32, u);
          const int64_t c0 = col0 + chunk * 32;
          if (row < p.M && c0 < p.n_half) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = swiglu<T>(__uint_as_float(g[i]), __uint_as_float(u[i]));
            store_row32<T>(orow, c0, p.n_half, v, nullptr);
          }
        }
      } else {
        const int64_t col0 = int64_t(nb) * C::kTile;
#pragma unroll 1
        for (int chunk = 0; chunk < C::kTile / 32; ++chunk) {
          uint32_t r[32];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it together
          tmem_ld_32(taddr + chunk * 32, r);
          const int64_t c0 = col0 + chunk * 32;
          if (row < p.M && c0 < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            store_row32<T>(orow, c0, p.N, v, bias);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty0 + 8 * acc);
    }
  }

  tc_fence_before();
  __syncthreads();
  pair_cluster_sync();  // the peer's MMAs, copies and arrivals that touch this CTA are done
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

// rows x K (K contiguous) operand, box = box_rows x 64, 128-byte swizzle
int make_kmajor_map(CUtensorMap* map, const void* base, bool bf16, int64_t rows, int64_t k,
                    int64_t row_stride, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(row_stride * 2)};
  const cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled (gemm) failed (%d)", int(r));
  return NTB200_OK;
}

// [2, I, K] view of a merged gate_up weight [2I, K] (K contiguous); box = 64 x 128 rows x
// both halves, 128-byte swizzle: one load brings 128 gate rows and the matching up rows.
int make_gate_up_map(CUtensorMap* map, const void* base, bool bf16, int64_t I, int64_t k, int64_t row_stride) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {cuuint64_t(k), cuuint64_t(I), 2};
  const cuuint64_t strides[2] = {cuuint64_t(row_stride * 2), cuuint64_t(I * row_stride * 2)};
  const cuuint32_t box[3] = {cuuint32_t(BK), 128, 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled (gate_up) failed (%d)", int(r));
  return NTB200_OK;
}

// ------------------------------------------------------------------------------------
// Small-M path (M <= 256: decode batches).  out^T = W . x^T ("swap AB"): weight rows fill
// the UMMA M=128 side, the few token rows are the UMMA N side (padded to MP = 16 .. 256;
// rows past M are TMA zero-fill and cost no HBM traffic).  A CTA owns NT adjacent 128-row
// weight tiles that share each k-step's token tile (NT = 2 for token tiles of 128 rows and
// more, halving the token operand's L2 re-reads; TMEM holds the NT accumulators).  With
// few weight tiles, K is split across the CTAs of a thread-block cluster (<= 8): each CTA
// parks one fp32 partial tile at a time in its shared memory and, after a cluster barrier,
// every CTA sums a share of the output rows across the cluster through distributed shared
// memory and writes them (bias added, rounded).  Without a split the epilogue stores
// straight from TMEM.  One launch, no global workspace.
// ------------------------------------------------------------------------------------

// BIG: the grid fits in one wave (one CTA per SM), so the ring takes ~192 KB and keeps
// twice the weight bytes in flight; otherwise ~96 KB so that two CTAs share an SM.
template <int MP, int NT, bool BIG>
struct SmallSmem {
  static constexpr int kXTile = MP * BK * 2;
  static constexpr int kStage = NT * kATileBytes + kXTile;  // NT weight tiles + token tile
  static constexpr int kRingTarget = BIG ? 192 * 1024 : 96 * 1024;
  static constexpr int kStages = kRingTarget / kStage < 3 ? 3 : kRingTarget / kStage;
  static constexpr int kRing = 0;
  static constexpr int kFull = kStages * kStage;
  static constexpr int kEmpty = kFull + 8 * kStages;
  static constexpr int kTmemFull = kEmpty + 8 * kStages;
  static constexpr int kTmemBase = kTmemFull + 8;
  static constexpr int kEnd = kTmemBase + 8;
  static constexpr int kDynamicBytes = kEnd + 1024;
  static constexpr int kTmemCols = NT * MP < 32 ? 32 : NT * MP;
  static_assert(NT * MP <= 512, "accumulators exceed TMEM");
  static_assert(MP * BM * 4 <= kStages * kStage, "partial tile must fit in the ring");
  static_assert(kDynamicBytes <= 227 * 1024, "ring exceeds shared memory");
};

struct SmallParams {
  void* out;
  const void* bias;
  int64_t M, N;
  int64_t out_stride;
  int n_tiles;  // 128-row weight tiles
  int splits;
  int k_steps_per_split;
  int k_steps_total;
  int64_t n_half;  // SwiGLU variant: output columns I (up rows start at row I of W)
  unsigned long long* argmax_keys;  // ARGMAX variant: one packed (value, index) per token
  unsigned int* err;
};

// Greedy-argmax key of one logit: the logit rounded to T (the dtype the unfused LM head
// writes and the sampler compares), mapped to an unsigned integer that orders like the
// float (NaN above +inf, as torch.argmax ranks it), in the high half; the complement of
// the vocabulary index in the low half, so that among equal logits the first index wins.
// The signed-integer image of the rounded logit: larger logit, larger integer; -0 is
// taken as +0 (they compare equal); a NaN rounds to the positive canonical NaN, which
// sorts above +inf.
template <typename T>
__device__ __forceinline__ int32_t argmax_ord(float logit) {
  uint32_t u = __float_as_uint(Elem<T>::round(logit));
  u = u == 0x80000000u ? 0u : u;
  return static_cast<int32_t>(u ^ ((static_cast<uint32_t>(static_cast<int32_t>(u) >> 31)) & 0x7FFFFFFFu));
}

__device__ __forceinline__ unsigned long long argmax_pack(int32_t ord, int64_t index) {
  return (static_cast<unsigned long long>(static_cast<uint32_t>(ord) ^ 0x80000000u) << 32) |
         (0xFFFFFFFFu - static_cast<uint32_t>(index));
}

template <typename T>
__device__ __forceinline__ unsigned long long argmax_key(float logit, int64_t index) {
  return argmax_pack(argmax_ord<T>(logit), index);
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int off) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v), off);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), off);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Remote shared-memory load of 4 floats.  Volatile keeps it after the (volatile) cluster
// barrier; no memory clobber, so that several of these can be in flight before their
// values are used.
__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  float4 v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote));
  return v;
}

// SWIGLU (NT = 2, no split): the CTA's two weight tiles are gate rows [128*g, +128) and
// the matching up rows [I + 128*g, +128), so each epilogue thread holds x.gate and x.up
// of the same output column.
// ARGMAX (no split): instead of writing logits, every warp reduces its 32 weight rows
// (vocabulary entries) per token to the best key and folds it into that token's key with
// one 64-bit atomicMax; the [M, N] logits are never written.
template <typename T, int MP, int NT, bool BIG, bool SWIGLU = false, bool ARGMAX = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_small_m_kernel(
    const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map,
    const SmallParams p) {
  using L = SmallSmem<MP, NT, BIG>;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L::kEmpty);
  uint64_t* tmem_full = reinterpret_cast<uint64_t*>(smem + L::kTmemFull);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemBase);
  const uint32_t ring = smem_u32(smem + L::kRing);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % p.splits;  // == rank in the cluster
  const int tile0 = (blockIdx.x / p.splits) * NT;
  const int kb0 = split * p.k_steps_per_split;
  const int kb1 = min(kb0 + p.k_steps_per_split, p.k_steps_total);
  const int nk = kb1 > kb0 ? kb1 - kb0 : 0;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
  }
  // tensor memory is allocated only after the preceding kernel has finished (see the
  // large-M kernel)
  pdl_wait();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base_slot)),
                 "r"(L::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&w_map)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&x_map)) : "memory");
      int issued = 0;
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&full[s], L::kStage);
        const uint32_t stage = ring + s * L::kStage;
        const int kx = (kb0 + it) * BK;
        // weight tiles past N (the last group of an odd tile count) are TMA zero-fill
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int wrow = SWIGLU ? (t == 0 ? 0 : static_cast<int>(p.n_half)) + (tile0 / NT) * BM : (tile0 + t) * BM;
          tma_load_2d(stage + t * kATileBytes, &w_map, kx, wrow, smem_u32(&full[s]));
        }
        tma_load_2d(stage + NT * kATileBytes, &x_map, kx, 0, smem_u32(&full[s]));
        issued = it + 1;
      }
      const int first = issued > kStages ? issued - kStages : 0;
      for (int j = first; j < issued; ++j) mbar_wait(&full[j % kStages], (j / kStages) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc(std::is_same<T, __nv_bfloat16>::value, BM, MP);
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1, p.err)) break;
        tc_fence_after();
        const uint32_t stage = ring + s * L::kStage;
        const uint64_t bdesc = sw128_kmajor_desc(stage + NT * kATileBytes);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint64_t adesc = sw128_kmajor_desc(stage + t * kATileBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(tmem_base + t * MP, adesc + 2 * k, bdesc + 2 * k, idesc, (it > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(tmem_full);  // also the "all MMAs done" point before TMEM is released
    }
  }

  T* out = static_cast<T*>(p.out);
  const T* bias = static_cast<const T*>(p.bias);
  const bool epilogue = warp >= 2;
  const int quad = warp & 3;
  const int n_local = quad * 32 + lane;  // TMEM lane = weight row within the tile
  bool acc_ok = false;
  if (epilogue) {
    acc_ok = mbar_wait(tmem_full, 0, p.err) && nk > 0;
    tc_fence_after();
  }

  if (ARGMAX) {
    // no split (the host plans none).  Per token, each thread keeps the best of its NT
    // weight rows as a signed ordinal (rows ascend with t, so a strict > keeps the first of
    // equal logits); the warp then takes the max ordinal and, among the lanes holding it,
    // the smallest (t, lane) -- the smallest vocabulary index -- with two redux.sync.
    if (epilogue) {
      const int64_t row0 = int64_t(tile0) * BM + quad * 32;  // vocabulary index of (t=0, lane 0)
#pragma unroll 1
      for (int c = 0; c < MP / 16; ++c) {
        int32_t bo[16];
        uint32_t bt[16];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          uint32_t r[16];
          __syncwarp();
          tmem_ld_16(tmem_base + (uint32_t(quad * 32) << 16) + t * MP + c * 16, r);
          const bool valid = acc_ok && row0 + t * BM + lane < p.N;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int32_t o = valid ? argmax_ord<T>(__uint_as_float(r[i])) : INT32_MIN;
            if (t == 0) {
              bo[i] = o;
              bt[i] = 0;
            } else if (o > bo[i]) {
              bo[i] = o;
              bt[i] = t;
            }
          }
        }
        unsigned long long mine = 0ull;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int32_t m = __reduce_max_sync(0xffffffffu, bo[i]);
          const uint32_t w = __reduce_min_sync(0xffffffffu, bo[i] == m ? bt[i] * 32u + uint32_t(lane) : 0xFFFFFFFFu);
          if (lane == i && m != INT32_MIN) mine = argmax_pack(m, row0 + int64_t(w >> 5) * BM + (w & 31u));
        }
        const int64_t m = c * 16 + lane;
        if (lane < 16 && m < p.M && mine != 0ull) atomicMax(p.argmax_keys + m, mine);
      }
      tc_fence_before();
    }
  } else if (SWIGLU) {
    // no split (the host plans none): silu(gate) * up straight from TMEM
    if (epilogue) {
      const int64_t n = int64_t(tile0 / NT) * BM + n_local;
#pragma unroll 1
      for (int c = 0; c < MP / 16; ++c) {
        uint32_t g[16], u[16];
        __syncwarp();
        tmem_ld_16(tmem_base + (uint32_t(quad * 32) << 16) + c * 16, g);
        tmem_ld_16(tmem_base + (uint32_t(quad * 32) << 16) + MP + c * 16, u);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int64_t m = c * 16 + i;
          if (m < p.M && n < p.n_half)
            out[m * p.out_stride + n] =
                Elem<T>::from_f(acc_ok ? swiglu<T>(__uint_as_float(g[i]), __uint_as_float(u[i])) : 0.f);
        }
      }
      tc_fence_before();
    }
  } else if (p.splits == 1) {
    // no split: TMEM -> registers -> global (lane = output column, column = token row)
    if (epilogue) {
#pragma unroll 1
      for (int t = 0; t < NT; ++t) {
        const int64_t n = int64_t(tile0 + t) * BM + n_local;
        const float b = (bias != nullptr && n < p.N) ? Elem<T>::to_f(bias[n]) : 0.f;
#pragma unroll 1
        for (int c = 0; c < MP / 16; ++c) {
          uint32_t r[16];
          __syncwarp();
          tmem_ld_16(tmem_base + (uint32_t(quad * 32) << 16) + t * MP + c * 16, r);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int64_t m = c * 16 + i;
            if (m < p.M && n < p.N)
              out[m * p.out_stride + n] = Elem<T>::from_f((acc_ok ? __uint_as_float(r[i]) : 0.f) + b);
          }
        }
      }
      tc_fence_before();
    }
  } else {
    // split-K: one weight tile at a time through shared memory and the cluster
    float* part = reinterpret_cast<float*>(smem + L::kRing);
    const uint32_t part_addr = smem_u32(smem + L::kRing);
    const int rows_per = static_cast<int>((p.M + p.splits - 1) / p.splits);
    const int r0 = split * rows_per;
    const int r1 = static_cast<int>(p.M < int64_t(r0) + rows_per ? p.M : int64_t(r0) + rows_per);
    const int q4 = threadIdx.x & 31;  // float4 column group: rows of the partial are 32 float4
#pragma unroll 1
    for (int t = 0; t < NT; ++t) {
      if (epilogue) {
#pragma unroll 1
        for (int c = 0; c < MP / 16; ++c) {
          uint32_t r[16];
          __syncwarp();
          tmem_ld_16(tmem_base + (uint32_t(quad * 32) << 16) + t * MP + c * 16, r);
#pragma unroll
          for (int i = 0; i < 16; ++i) part[(c * 16 + i) * BM + n_local] = acc_ok ? __uint_as_float(r[i]) : 0.f;
        }
      }
      // every CTA of the cluster has partial tile t in shared memory
      cluster_sync_all();
      const int64_t n0 = int64_t(tile0 + t) * BM + 4 * q4;
      float bvec[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) bvec[i] = (bias != nullptr && n0 + i < p.N) ? Elem<T>::to_f(bias[n0 + i]) : 0.f;
      // 192 threads cover 6 rows per pass; a pass has its splits x float4 remote loads in
      // flight before any is summed
      for (int m = r0 + (threadIdx.x >> 5); m < r1; m += kThreads / 32) {
        const uint32_t off = part_addr + uint32_t((m * BM + 4 * q4) * 4);
        float4 v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = r < p.splits ? ld_dsmem_f32x4(off, uint32_t(r)) : make_float4(0.f, 0.f, 0.f, 0.f);
        float acc[4] = {bvec[0], bvec[1], bvec[2], bvec[3]};
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[0] += v[r].x;
          acc[1] += v[r].y;
          acc[2] += v[r].z;
          acc[3] += v[r].w;
        }
        T* orow = out + int64_t(m) * p.out_stride;
        if (n0 + 4 <= p.N && ((reinterpret_cast<uintptr_t>(orow + n0) & 7u) == 0)) {
          store_f<T, 4>(orow + n0, acc);
        } else {
          for (int i = 0; i < 4; ++i)
            if (n0 + i < p.N) orow[n0 + i] = Elem<T>::from_f(acc[i]);
        }
      }
      // nobody overwrites (or frees) a partial tile while a partner still reads it
      cluster_sync_all();
    }
    if (epilogue) tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::kTmemCols)
                 : "memory");
  }
}

template <typename T, int MP, int NT, bool BIG, bool SWIGLU = false, bool ARGMAX = false>
int launch_small(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, cudaStream_t s,
                 int attr_slot) {
  using L = SmallSmem<MP, NT, BIG>;
  const void* fn = reinterpret_cast<const void*>(gemm_small_m_kernel<T, MP, NT, BIG, SWIGLU, ARGMAX>);
  int st = ensure_smem_attribute(fn, L::kDynamicBytes, attr_slot);
  if (st != NTB200_OK) return st;
  const int groups = (prm.n_tiles + NT - 1) / NT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(groups * prm.splits));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(prm.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  set_pdl_attribute(attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, gemm_small_m_kernel<T, MP, NT, BIG, SWIGLU, ARGMAX>, wmap, xmap, prm);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "linear (small M): launch failed: %s", cudaGetErrorString(e));
  }
  return NTB200_OK;
}

// How many clusters of `cluster` CTAs of `fn` (with `smem` bytes each) can be resident at
// once on the current device; cached per (device, variant slot, cluster size).
int resident_clusters(const void* fn, int smem, int cluster, int slot) {
  constexpr int kDevs = 16, kSlots = 128, kMaxCluster = 9;
  static std::atomic<int> cache[kDevs][kSlots][kMaxCluster];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kDevs || slot < 0 || slot >= kSlots || cluster < 1 || cluster >= kMaxCluster) return 0;
  const int hit = cache[dev][slot][cluster].load(std::memory_order_relaxed);
  if (hit != 0) return hit;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = -1;  // unknown: callers treat it as "does not fit"
  }
  cache[dev][slot][cluster].store(n, std::memory_order_relaxed);
  return n;
}

// The ~192 KB ring when every cluster of the grid is resident at once with one CTA per
// SM (clusters must fit inside a GPC, so this is asked of the runtime, not assumed);
// otherwise the ~96 KB ring, two CTAs per SM.
template <typename T, int MP, int NT>
int launch_small_ring(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& big_plan,
                      const SmallParams& small_plan, cudaStream_t s, int slot) {
  const int groups = (big_plan.n_tiles + NT - 1) / NT;
  {
    using LB = SmallSmem<MP, NT, true>;
    const void* fn = reinterpret_cast<const void*>(gemm_small_m_kernel<T, MP, NT, true>);
    int st = ensure_smem_attribute(fn, LB::kDynamicBytes, slot + 1);
    if (st != NTB200_OK) return st;
    if (resident_clusters(fn, LB::kDynamicBytes, big_plan.splits, slot + 1) >= groups)
      return launch_small<T, MP, NT, true>(wmap, xmap, big_plan, s, slot + 1);
  }
  using LS = SmallSmem<MP, NT, false>;
  const void* fn = reinterpret_cast<const void*>(gemm_small_m_kernel<T, MP, NT, false>);
  int st = ensure_smem_attribute(fn, LS::kDynamicBytes, slot);
  if (st != NTB200_OK) return st;
  if (resident_clusters(fn, LS::kDynamicBytes, small_plan.splits, slot) >= groups)
    return launch_small<T, MP, NT, false>(wmap, xmap, small_plan, s, slot);
  return launch_small<T, MP, NT, false>(wmap, xmap, big_plan, s, slot);
}

// token tile MP, weight tiles per CTA NT; two attribute slots (ring sizes) per (MP, NT)
template <typename T>
int dispatch_small(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& big_plan,
                   const SmallParams& small_plan, int mp, int nt, cudaStream_t s, int slot_base) {
  switch (mp) {
    case 16: return launch_small_ring<T, 16, 1>(wmap, xmap, big_plan, small_plan, s, slot_base + 0);
    case 32: return launch_small_ring<T, 32, 1>(wmap, xmap, big_plan, small_plan, s, slot_base + 2);
    case 64: return launch_small_ring<T, 64, 1>(wmap, xmap, big_plan, small_plan, s, slot_base + 4);
    case 128:
      return nt == 2 ? launch_small_ring<T, 128, 2>(wmap, xmap, big_plan, small_plan, s, slot_base + 6)
                     : launch_small_ring<T, 128, 1>(wmap, xmap, big_plan, small_plan, s, slot_base + 8);
    default:
      return nt == 2 ? launch_small_ring<T, 256, 2>(wmap, xmap, big_plan, small_plan, s, slot_base + 10)
                     : launch_small_ring<T, 256, 1>(wmap, xmap, big_plan, small_plan, s, slot_base + 12);
  }
}

// Two weight tiles per CTA (one token tile shared by both) only when the weight tiles alone
// fill the GPU, so that K is not split: halving the token re-reads does not pay for a
// second cluster-reduction round.
int small_tiles_per_cta(int mp, int64_t n_tiles, int sms) { return (mp >= 128 && n_tiles >= sms / 2) ? 2 : 1; }

// M blocks per raster group: all of them when x fits comfortably in L2, else 8.
int raster_group(int64_t M, int64_t K, int64_t mblocks) {
  constexpr int64_t kL2Budget = 48ll << 20;
  if (M * K * 2 <= kL2Budget || mblocks <= 8) return static_cast<int>(mblocks);
  return 8;
}

// Tile width for the large-M kernel: the widest of 256/192/128 whose tiles fill the SMs'
// waves (and cover N with little padding) to within 95% of the best candidate.
int pick_tile_width(int64_t M, int64_t N, int sms) {
  const int cands[3] = {256, 192, 128};
  double eff[3], best = 0.0;
  for (int i = 0; i < 3; ++i) {
    const int64_t nb = ceil_div(N, cands[i]);
    const int64_t tiles = ceil_div(M, BM) * nb;
    const int64_t waves = ceil_div(tiles, sms);
    eff[i] = (double(tiles) / double(waves * sms)) * (double(N) / double(nb * cands[i]));
    best = eff[i] > best ? eff[i] : best;
  }
  for (int i = 0; i < 3; ++i)
    if (eff[i] >= 0.95 * best) return cands[i];
  return 256;
}

// SWIGLU: `N` is the weight's row count 2I and out has I columns (see the kernel).
template <int BNV, bool SWIGLU = false>
int launch_large(void* out, const void* x, const void* weight, const void* bias, int64_t M, int64_t N,
                 int64_t K, int64_t xs, int64_t ws, int64_t os, bool bf16, cudaStream_t s) {
  using C = GemmCfg<BNV>;
  const int64_t n_out = SWIGLU ? N / 2 : N;
  const int64_t mblocks = ceil_div(M, BM), nblocks = ceil_div(n_out, SWIGLU ? BNV / 2 : BNV);
  if (mblocks * nblocks > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear: too many tiles");
  CUtensorMap amap, bmap;
  int st = make_kmajor_map(&amap, x, bf16, M, K, xs, BM);
  if (st != NTB200_OK) return st;
  st = make_kmajor_map(&bmap, weight, bf16, N, K, ws, SWIGLU ? BNV / 2 : BNV);
  if (st != NTB200_OK) return st;
  GemmParams prm;
  prm.out = out;
  prm.bias = bias;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.out_stride = os;
  prm.num_m_blocks = static_cast<int>(mblocks);
  prm.num_n_blocks = static_cast<int>(nblocks);
  prm.group_m = raster_group(M, K, mblocks);
  prm.n_half = n_out;
  prm.err = device_error_word();
  const int64_t tiles = mblocks * nblocks;
  const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  const int slot = (SWIGLU ? 42 : 32) + (BNV == 256 ? 0 : (BNV == 192 ? 2 : 4)) + (bf16 ? 0 : 1);
  if (bf16) {
    st = ensure_smem_attribute(reinterpret_cast<const void*>(gemm_tcgen05_kernel<__nv_bfloat16, BNV, SWIGLU>),
                               C::kDynamicBytes, slot);
    if (st != NTB200_OK) return st;
    return launch_kernel("linear", gemm_tcgen05_kernel<__nv_bfloat16, BNV, SWIGLU>, dim3(grid), dim3(kThreads),
                         C::kDynamicBytes, s, amap, bmap, prm);
  }
  st = ensure_smem_attribute(reinterpret_cast<const void*>(gemm_tcgen05_kernel<__half, BNV, SWIGLU>),
                             C::kDynamicBytes, slot);
  if (st != NTB200_OK) return st;
  return launch_kernel("linear", gemm_tcgen05_kernel<__half, BNV, SWIGLU>, dim3(grid), dim3(kThreads),
                       C::kDynamicBytes, s, amap, bmap, prm);
}

template <bool SWIGLU = false>
int launch_pair(void* out, const void* x, const void* weight, const void* bias, int64_t M, int64_t N,
                int64_t K, int64_t xs, int64_t ws, int64_t os, bool bf16, cudaStream_t s) {
  using C = PairCfg;
  const int64_t n_out = SWIGLU ? N / 2 : N;
  const int64_t mblocks = ceil_div(M, C::kTile), nblocks = ceil_div(n_out, SWIGLU ? C::kHalf : C::kTile);
  if (mblocks * nblocks > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear: too many tiles");
  CUtensorMap amap, bmap;
  int st = make_kmajor_map(&amap, x, bf16, M, K, xs, C::kHalf);
  if (st != NTB200_OK) return st;
  st = make_kmajor_map(&bmap, weight, bf16, N, K, ws, C::kHalf);
  if (st != NTB200_OK) return st;
  GemmParams prm;
  prm.out = out;
  prm.bias = bias;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.out_stride = os;
  prm.num_m_blocks = static_cast<int>(mblocks);
  prm.num_n_blocks = static_cast<int>(nblocks);
  prm.group_m = raster_group(M, K, mblocks);
  prm.n_half = n_out;
  prm.err = device_error_word();
  const int slot = (SWIGLU ? 48 : 40) + (bf16 ? 0 : 1);
  const void* fn = bf16 ? reinterpret_cast<const void*>(gemm_pair_kernel<__nv_bfloat16, SWIGLU>)
                        : reinterpret_cast<const void*>(gemm_pair_kernel<__half, SWIGLU>);
  st = ensure_smem_attribute(fn, C::kDynamicBytes, slot);
  if (st != NTB200_OK) return st;
  int pairs = resident_clusters(fn, C::kDynamicBytes, 2, slot);
  if (pairs <= 0) pairs = num_sms() / 2;
  const int64_t tiles = mblocks * nblocks;
  if (tiles < pairs) pairs = static_cast<int>(tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kDynamicBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  set_pdl_attribute(attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = bf16 ? cudaLaunchKernelEx(&cfg, gemm_pair_kernel<__nv_bfloat16, SWIGLU>, amap, bmap, prm)
                             : cudaLaunchKernelEx(&cfg, gemm_pair_kernel<__half, SWIGLU>, amap, bmap, prm);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "linear (CTA pairs): launch failed: %s", cudaGetErrorString(e));
  }
  return NTB200_OK;
}

// Fused gate_up + SiluAndMul for decode batches: one CTA per 128 output columns, both
// weight tiles (gate and up) in it, no K split.
template <typename T, int MP>
int launch_small_swiglu(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, cudaStream_t s,
                        int slot) {
  const int64_t groups = (prm.n_tiles + 1) / 2;
  if (groups <= num_sms()) return launch_small<T, MP, 2, true, true>(wmap, xmap, prm, s, slot + 1);
  return launch_small<T, MP, 2, false, true>(wmap, xmap, prm, s, slot);
}

template <typename T>
int dispatch_small_swiglu(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, int mp,
                          cudaStream_t s, int slot_base) {
  switch (mp) {
    case 16: return launch_small_swiglu<T, 16>(wmap, xmap, prm, s, slot_base + 0);
    case 32: return launch_small_swiglu<T, 32>(wmap, xmap, prm, s, slot_base + 2);
    case 64: return launch_small_swiglu<T, 64>(wmap, xmap, prm, s, slot_base + 4);
    case 128: return launch_small_swiglu<T, 128>(wmap, xmap, prm, s, slot_base + 6);
    default: return launch_small_swiglu<T, 256>(wmap, xmap, prm, s, slot_base + 8);
  }
}

// ------------------------------------------------------------------------------------
// Skinny-activation path of `ntb200_linear` (M <= 256: decode batches).  out = x . W^T with
// the weight rows on the UMMA N side (a 256-row weight tile per CTA) and the token rows on
// the M side (one token tile of MP <= 128 rows, or two of 128).  A kind::f16 tcgen05.mma
// (K = 16) occupies the tensor pipe for the same time whatever its N (16..256) or M (64,
// 128), so what one instruction consumes of the weights sets the weight streaming rate:
// 256 rows x 16 here, twice what a weight-rows-on-M tile consumes, which is the difference
// between falling short of and exceeding HBM bandwidth with a decode batch.
//   warp 0      TMA producer: per 64-wide k-step the token tile(s) (MP x 64; rows past M
//               are zero-fill and cost no memory traffic) and the 256 x 64 weight tile;
//   warp 1      allocates TMEM (TT x 256 fp32 columns) and issues the MMAs;
//   warps 2-5   epilogue: TMEM lane = token row, 256 output columns per row.
// With MP < 128 the MMA's A operand rows past MP read the rest of the stage (their
// accumulator rows are never stored).  When the weight tiles alone leave SMs idle, K is
// split across the CTAs of a cluster (<= 8 CTAs, sized so the clusters are resident at
// once): each CTA stages its fp32 partial rows in shared memory and, after a cluster
// barrier, sums a share of the (row, 4-column) units over the cluster through
// distributed shared memory, in split order, adds the bias and stores.  One launch, no
// global workspace, no TMA multicast.
// ------------------------------------------------------------------------------------
constexpr int kSkinnyBN = 256;
constexpr int kSkinnyWTile = kSkinnyBN * BK * 2;  // 32 KB

template <int MP, int TT>
struct SkinnySmem {
  static constexpr int kXTile = MP * BK * 2;  // one token tile
  static constexpr int kX = TT * kXTile;
  static constexpr int kRingOff = 0;
  static constexpr int kStage = kX + kSkinnyWTile;
  static constexpr int kStages = (225 * 1024) / kStage > 6 ? 6 : (225 * 1024) / kStage;
  static constexpr int kRing = kStages * kStage;
  static constexpr int kFull = kRing;
  static constexpr int kEmpty = kFull + 8 * kStages;
  static constexpr int kTmemFull = kEmpty + 8 * kStages;
  static constexpr int kTmemBase = kTmemFull + 8;
  static constexpr int kEnd = kTmemBase + 8;
  static constexpr int kDynamicBytes = kEnd + 1024;
  static constexpr int kTmemCols = TT * kSkinnyBN;
  static constexpr int kPartStride = kSkinnyBN + 4;  // floats per staged partial row (padded)
  static_assert(TT == 1 || MP == 128, "two token tiles are 128 rows each");
  static_assert(kStage >= BM * BK * 2, "an M = 128 A operand must lie inside its stage");
  static_assert(kStages >= 3, "ring too shallow");
  static_assert(128 * kPartStride * 4 <= kRing, "partial rows must fit in the ring");
  static_assert(kDynamicBytes <= 227 * 1024, "ring exceeds shared memory");
};

struct SkinnyParams {
  void* out;
  const void* bias;
  int64_t M, N;
  int64_t out_stride;
  int splits;
  int k_steps_per_split;
  int k_steps_total;
  int64_t n_half;  // SwiGLU variant: output columns I (up rows start at row I of W)
  unsigned int* err;
  // NORM variant: the GEMM input is RMSNorm(x [+ residual]) * norm_weight, formed here
  const void* nx;
  const void* nres;    // null: no residual add
  void* nres_out;      // the new residual (x + residual), written by the CTAs of weight tile 0
  const void* ngamma;
  float eps;
  int64_t K, x_stride, r_stride, ro_stride;
};

// Fused RMS norm (decode batches of at most kNormRows tokens): the normalised token rows of
// the CTA's whole K range stay in shared memory (16 rows x 64 columns = 2 KB per k-step,
// 128-byte swizzle, at most STEPS of them) ahead of a ring of weight tiles; the MMA reads
// its A operand from there, so only the weights stream through the ring.  The smaller A
// region (32 k-steps) leaves room for 5 ring stages, the larger (64) for 3.
constexpr int kNormRows = 16;
constexpr int kNormMaxSteps = 64;
constexpr int kNormThreads = 128;                  // the epilogue warps run the norm prologue
constexpr int kNormFirstThread = kThreads - kNormThreads;
constexpr int kNormGroupSteps = kNormThreads / 8;  // one 16-byte column vector per thread
template <int STEPS>
struct SkinnyNormSmem {
  static constexpr int kXTile = kNormRows * BK * 2;  // 2 KB: one k-step of normalised rows
  static constexpr int kX = 0;                       // a ring stage holds the weight tile only
  static constexpr int kA = STEPS * kXTile;
  static constexpr int kRingOff = kA;
  static constexpr int kStage = kSkinnyWTile;
  static constexpr int kStages = (225 * 1024 - kA) / kStage > 6 ? 6 : (225 * 1024 - kA) / kStage;
  static constexpr int kRing = kStages * kStage;
  static constexpr int kFull = kRingOff + kRing;
  static constexpr int kEmpty = kFull + 8 * kStages;
  static constexpr int kTmemFull = kEmpty + 8 * kStages;
  static constexpr int kTmemBase = kTmemFull + 8;
  static constexpr int kRowPart = kTmemBase + 8;  // float[16]: this CTA's row sums of squares
  static constexpr int kRstd = kRowPart + 64;     // float[16]: 1 / rms per row, then the
                                                  // [4 warps][16] partial sums of the prologue
  static constexpr int kAReady = kRstd + 64 + (kNormThreads / 32) * kNormRows * 4;  // per k-step group
  static constexpr int kEnd = kAReady + 8 * (STEPS / kNormGroupSteps);
  static constexpr int kDynamicBytes = kEnd + 1024;
  static constexpr int kTmemCols = kSkinnyBN;
  static constexpr int kPartStride = kSkinnyBN + 4;
  // the last k-step's M = 128 operand span (rows past 16 are never stored) stays inside
  static_assert(kA - kXTile + BM * BK * 2 <= kRingOff + kRing, "A span leaves shared memory");
  static_assert(128 * kPartStride * 4 <= kRingOff + kRing, "partial rows must fit");
  static_assert(kDynamicBytes <= 227 * 1024, "exceeds shared memory");
};

// Remote shared-memory load of one float (see ld_dsmem_f32x4).
__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote));
  return v;
}

// NORM prologue, run by the four epilogue warps while the producer streams the weights:
// the CTA's K range [64 kb0, +64 nk) of the M <= 16 token rows, s = x (+ residual) in fp32,
// this CTA's row sums of s^2 (into rowpart, summed in a fixed order), and round(s *
// norm_weight) into the resident A operand (16 rows x 64 columns per k-step, 128-byte
// swizzle; rows past M and columns past K hold zeros).  Thread e of the 128 writes column
// vector e of each group of kNormGroupSteps k-steps and then arrives on that group's
// a_ready barrier, so the MMAs of a group start as soon as its rows are in place.  The MMAs
// wait for no row statistics: RMSNorm scales each row by 1 / rms, which is linear in the
// product, so the epilogue applies it once the CTAs splitting K have their sums
// (out[m, n] = rstd[m] * sum_k round(s[m, k] w[k]) W[n, k]).  The CTAs of weight tile 0 also
// write the new residual.
template <typename T>
__device__ __forceinline__ void norm_prologue(const SkinnyParams& p, uint8_t* a, uint64_t* a_ready, uint8_t* rowpart_b,
                                              uint8_t* red_b, int kb0, int nk, bool write_residual) {
  float* rowpart = reinterpret_cast<float*>(rowpart_b);
  float* red = reinterpret_cast<float*>(red_b);  // [4 warps][kNormRows] warp partial sums
  const T* x = static_cast<const T*>(p.nx);
  const T* res = static_cast<const T*>(p.nres);
  T* res_out = static_cast<T*>(p.nres_out);
  const T* gamma = static_cast<const T*>(p.ngamma);
  const int M = static_cast<int>(p.M);
  const int64_t k0 = int64_t(kb0) * BK;
  const int64_t k1 = p.K < k0 + int64_t(nk) * BK ? p.K : k0 + int64_t(nk) * BK;
  const int nvec = k1 > k0 ? static_cast<int>((k1 - k0) / 8) : 0;  // 8-element vectors (K % 8 == 0)
  const int e = static_cast<int>(threadIdx.x) - kNormFirstThread;    // 0 .. kNormThreads - 1
  const int lane = threadIdx.x & 31;
  constexpr int kStepBytes = kNormRows * BK * 2;
  constexpr int kChunk = 8;  // rows whose loads are in flight together
  using V = Vec<T, 8>;
  float part[kNormRows];
#pragma unroll
  for (int m = 0; m < kNormRows; ++m) part[m] = 0.f;
  const int groups = (nk + kNormGroupSteps - 1) / kNormGroupSteps;
  for (int grp = 0; grp < groups; ++grp) {
    const int v = grp * kNormThreads + e;  // kNormThreads vectors = kNormGroupSteps k-steps
    if (v < nk * (BK / 8)) {
      const int step = v >> 3, chunk = v & 7;  // 8 vectors of 16 bytes per 128-byte row
      uint8_t* st = a + step * kStepBytes;
      if (v < nvec) {
        float g8[8];
        load_f<T, 8>(gamma + k0 + v * 8, g8);
#pragma unroll
        for (int m0 = 0; m0 < kNormRows; m0 += kChunk) {
          if (m0 >= M) break;
          V xr[kChunk], rr[kChunk];
#pragma unroll
          for (int i = 0; i < kChunk; ++i) {
            const int m = m0 + i;
            if (m < M) {
              xr[i] = *reinterpret_cast<const V*>(x + m * p.x_stride + k0 + v * 8);
              if (res != nullptr) rr[i] = *reinterpret_cast<const V*>(res + m * p.r_stride + k0 + v * 8);
            }
          }
#pragma unroll
          for (int i = 0; i < kChunk; ++i) {
            const int m = m0 + i;
            if (m < M) {
              float sv[8], y[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                sv[j] = Elem<T>::to_f(xr[i].v[j]);
                if (res != nullptr) sv[j] += Elem<T>::to_f(rr[i].v[j]);
                part[m0 + i] += sv[j] * sv[j];
                y[j] = sv[j] * g8[j];
              }
              if (res != nullptr && write_residual) store_f<T, 8>(res_out + m * p.ro_stride + k0 + v * 8, sv);
              *reinterpret_cast<V*>(st + m * 128 + ((chunk ^ (m & 7)) << 4)) = pack_f<T, 8>(y);
            }
          }
        }
      }
      // rows past M, and the whole column past K, are zeros
#pragma unroll
      for (int m = 0; m < kNormRows; ++m)
        if (m >= M || v >= nvec)
          *reinterpret_cast<uint4*>(st + m * 128 + ((chunk ^ (m & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core
    mbar_arrive(&a_ready[grp]);
  }
#pragma unroll
  for (int m = 0; m < kNormRows; ++m) {
    float t = part[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[(e >> 5) * kNormRows + m] = t;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kNormThreads) : "memory");
  if (e < M) {
    float t = 0.f;
    for (int w = 0; w < kNormThreads / 32; ++w) t += red[w * kNormRows + e];
    rowpart[e] = t;
  }
}

// 1 / rms of each token row into rstd[0, M), from the row sums of s^2 of the CTAs splitting
// K (read over DSMEM in rank order; the caller has passed a cluster barrier that follows
// every CTA's prologue), or from the CTA's own sums when K is not split.  Every thread of
// the CTA calls it.
__device__ __forceinline__ void norm_rstd(const SkinnyParams& p, float* rowpart, float* rstd) {
  __syncthreads();  // this CTA's rowpart is complete
  if (static_cast<int>(threadIdx.x) < p.M) {
    float total = 0.f;
    if (p.splits > 1) {
      for (int q = 0; q < p.splits; ++q) total += ld_dsmem_f32(smem_u32(rowpart + threadIdx.x), uint32_t(q));
    } else {
      total = rowpart[threadIdx.x];
    }
    rstd[threadIdx.x] = rsqrtf(total / static_cast<float>(p.K) + p.eps);
  }
  __syncthreads();
}

// SWIGLU (no K split): the weight tile is gate rows [128 nb, +128) then the matching up rows
// [I + 128 nb, +128) of vLLM's merged [2I, K] weight, fetched as one box of its [2, I, K]
// view (w_map), so accumulator columns [0, 128) hold x.gate and [128, 256) x.up of the same
// 128 output columns; the epilogue writes silu(gate) * up with the rounding points of the
// unfused pair.
template <typename T, int MP, int TT, bool SWIGLU = false, bool NORM = false, int NSTEPS = kNormMaxSteps>
__global__ void __launch_bounds__(kThreads, 1) gemm_skinny_kernel(
    const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map,
    const SkinnyParams p) {
  static_assert(!NORM || (MP == kNormRows && TT == 1 && !SWIGLU), "fused norm: one 16-row token tile");
  using L = std::conditional_t<NORM, SkinnyNormSmem<NSTEPS>, SkinnySmem<MP, TT>>;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L::kEmpty);
  uint64_t* tmem_full = reinterpret_cast<uint64_t*>(smem + L::kTmemFull);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemBase);
  // NORM: the normalised rows of k-step group g are in shared memory once a_ready[g] completes
  uint64_t* a_ready = nullptr;
  if constexpr (NORM) a_ready = reinterpret_cast<uint64_t*>(smem + L::kAReady);
  const uint32_t ring = smem_u32(smem + L::kRingOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % p.splits;  // == rank in the cluster
  const int nb = blockIdx.x / p.splits;     // weight rows [256 nb, +256)
  const int kb0 = split * p.k_steps_per_split;
  const int kb1 = min(kb0 + p.k_steps_per_split, p.k_steps_total);
  const int nk = kb1 > kb0 ? kb1 - kb0 : 0;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    if constexpr (NORM)
      for (int g = 0; g < NSTEPS / kNormGroupSteps; ++g) mbar_init(&a_ready[g], kNormThreads);
    fence_mbar_init();
  }
  // tensor memory is allocated only after the preceding kernel has finished
  pdl_wait();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base_slot)),
                 "r"(L::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&w_map)) : "memory");
      if (!NORM) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&x_map)) : "memory");
      int issued = 0;
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&full[s], L::kStage);
        const uint32_t stage = ring + s * L::kStage;
        const int kx = (kb0 + it) * BK;
        if (!NORM) {
#pragma unroll
          for (int t = 0; t < TT; ++t) tma_load_2d(stage + t * L::kXTile, &x_map, kx, t * BM, smem_u32(&full[s]));
        }
        if (SWIGLU) {
          // one box of the [2, I, K] view: gate rows then the matching up rows
          tma_load_3d(stage + L::kX, &w_map, kx, nb * (kSkinnyBN / 2), 0, smem_u32(&full[s]));
        } else {
          tma_load_2d(stage + L::kX, &w_map, kx, nb * kSkinnyBN, smem_u32(&full[s]));
        }
        issued = it + 1;
      }
      // no copy may still be landing when the CTA exits
      const int first = issued > kStages ? issued - kStages : 0;
      for (int j = first; j < issued; ++j) mbar_wait(&full[j % kStages], (j / kStages) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc(std::is_same<T, __nv_bfloat16>::value, BM, kSkinnyBN);
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        if (NORM && it % kNormGroupSteps == 0 && !mbar_wait(&a_ready[it / kNormGroupSteps], 0, p.err)) break;
        if (!mbar_wait(&full[s], (it / kStages) & 1, p.err)) break;
        tc_fence_after();
        const uint32_t stage = ring + s * L::kStage;
        const uint64_t bdesc = sw128_kmajor_desc(stage + L::kX);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            // NORM: the normalised rows of k-step `it`, resident ahead of the ring
            const uint32_t a = NORM ? smem_u32(smem) + it * L::kXTile : stage + t * L::kXTile;
            umma_f16(tmem_base + t * kSkinnyBN, sw128_kmajor_desc(a) + 2 * k, bdesc + 2 * k, idesc,
                     (it > 0 || k > 0) ? 1u : 0u);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(tmem_full);  // also the "all MMAs done" point before TMEM is released
    }
  } else if constexpr (NORM) {
    norm_prologue<T>(p, smem, a_ready, smem + L::kRowPart, smem + L::kRstd + 64, kb0, nk, nb == 0);
  }

  T* out = static_cast<T*>(p.out);
  const T* bias = static_cast<const T*>(p.bias);
  const bool epilogue = warp >= 2;
  const int quad = warp & 3;             // TMEM lane quadrant this warp may access
  const int row_in_tile = quad * 32 + lane;
  const int64_t n0 = int64_t(nb) * kSkinnyBN;
  bool acc_ok = false;
  if (epilogue) {
    acc_ok = mbar_wait(tmem_full, 0, p.err) && nk > 0;
    tc_fence_after();
  }

  if (SWIGLU) {
    // no split (the host plans none): silu(gate) * up straight from TMEM
    if (epilogue) {
#pragma unroll 1
      for (int t = 0; t < TT; ++t) {
        if (int64_t(t) * BM + quad * 32 >= p.M) continue;
        const int64_t m = int64_t(t) * BM + row_in_tile;
#pragma unroll 1
        for (int c = 0; c < kSkinnyBN / 64; ++c) {
          uint32_t g[32], u[32];
          __syncwarp();
          tmem_ld_32(tmem_base + (uint32_t(quad * 32) << 16) + t * kSkinnyBN + c * 32, g);
          tmem_ld_32(tmem_base + (uint32_t(quad * 32) << 16) + t * kSkinnyBN + kSkinnyBN / 2 + c * 32, u);
          if (m < p.M) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = acc_ok ? swiglu<T>(__uint_as_float(g[i]), __uint_as_float(u[i])) : 0.f;
            store_row32<T>(out + m * p.out_stride, int64_t(nb) * (kSkinnyBN / 2) + c * 32, p.n_half, v, nullptr);
          }
        }
      }
      tc_fence_before();
    }
  } else if (p.splits == 1) {
    // NORM: each row scaled by its 1 / rms
    float* rstd = nullptr;
    if constexpr (NORM) {
      rstd = reinterpret_cast<float*>(smem + L::kRstd);
      norm_rstd(p, reinterpret_cast<float*>(smem + L::kRowPart), rstd);
    }
    // TMEM -> registers -> global: a thread writes 32 consecutive columns of its row at a time
    if (epilogue) {
#pragma unroll 1
      for (int t = 0; t < TT; ++t) {
        if (int64_t(t) * BM + quad * 32 >= p.M) continue;  // the warp's rows are all past M
        const int64_t m = int64_t(t) * BM + row_in_tile;
        float scale = 1.f;
        if constexpr (NORM) scale = m < p.M ? rstd[m] : 0.f;
#pragma unroll 1
        for (int c = 0; c < kSkinnyBN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32(tmem_base + (uint32_t(quad * 32) << 16) + t * kSkinnyBN + c * 32, r);
          if (m < p.M) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = acc_ok ? __uint_as_float(r[i]) * scale : 0.f;
            store_row32<T>(out + m * p.out_stride, n0 + c * 32, p.N, v, bias);
          }
        }
      }
      tc_fence_before();
    }
  } else {
    float* part = reinterpret_cast<float*>(smem);
    const uint32_t part_addr = smem_u32(smem);
#pragma unroll 1
    for (int t = 0; t < TT; ++t) {
      const int rows = static_cast<int>(p.M - int64_t(t) * BM < BM ? p.M - int64_t(t) * BM : BM);
      if (epilogue && quad * 32 < rows) {
#pragma unroll 1
        for (int c = 0; c < kSkinnyBN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32(tmem_base + (uint32_t(quad * 32) << 16) + t * kSkinnyBN + c * 32, r);
          if (row_in_tile < rows) {
            float4* dst = reinterpret_cast<float4*>(part + row_in_tile * L::kPartStride + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              dst[q] = acc_ok ? make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                            __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      // every CTA of the cluster has its partial rows of token tile t in shared memory
      cluster_sync_all();
      float* rstd = nullptr;
      if constexpr (NORM) {
        rstd = reinterpret_cast<float*>(smem + L::kRstd);
        norm_rstd(p, reinterpret_cast<float*>(smem + L::kRowPart), rstd);
      }
      const int units = rows * (kSkinnyBN / 4);
      const int u0 = static_cast<int>(int64_t(units) * split / p.splits);
      const int u1 = static_cast<int>(int64_t(units) * (split + 1) / p.splits);
      for (int u = u0 + static_cast<int>(threadIdx.x); u < u1; u += kThreads) {
        const int row = u / (kSkinnyBN / 4);
        const int c4 = u - row * (kSkinnyBN / 4);
        const int64_t col = n0 + 4 * c4;
        if (col >= p.N) continue;
        const uint32_t off = part_addr + uint32_t((row * L::kPartStride + 4 * c4) * 4);
        float4 v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = r < p.splits ? ld_dsmem_f32x4(off, uint32_t(r)) : make_float4(0.f, 0.f, 0.f, 0.f);
        float acc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = (bias != nullptr && col + i < p.N) ? Elem<T>::to_f(bias[col + i]) : 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[0] += v[r].x;
          acc[1] += v[r].y;
          acc[2] += v[r].z;
          acc[3] += v[r].w;
        }
        if constexpr (NORM) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i] *= rstd[row];
        }
        T* orow = out + (int64_t(t) * BM + row) * p.out_stride;
        if (col + 4 <= p.N && ((reinterpret_cast<uintptr_t>(orow + col) & 7u) == 0)) {
          store_f<T, 4>(orow + col, acc);
        } else {
          for (int i = 0; i < 4; ++i)
            if (col + i < p.N) orow[col + i] = Elem<T>::from_f(acc[i]);
        }
      }
      // nobody overwrites (or frees) its partial rows while a partner still reads them
      cluster_sync_all();
    }
    if (epilogue) tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::kTmemCols)
                 : "memory");
  }
}

// Splits of K for `n_tiles` weight tiles: the most SMs busy (n_tiles x splits <= the SM
// count) whose clusters of `splits` CTAs are all resident at once.
// NORM: a CTA's K range must fit the resident A operand (at most kNormMaxSteps k-steps).
template <typename T, int MP, int TT, bool SWIGLU = false, bool NORM = false, int NSTEPS = kNormMaxSteps>
int launch_skinny(const CUtensorMap& wmap, const CUtensorMap& xmap, SkinnyParams prm, int n_tiles, cudaStream_t s,
                  int slot, int forced_splits = 0) {
  using L = std::conditional_t<NORM, SkinnyNormSmem<NSTEPS>, SkinnySmem<MP, TT>>;
  const void* fn = reinterpret_cast<const void*>(gemm_skinny_kernel<T, MP, TT, SWIGLU, NORM, NSTEPS>);
  int st = ensure_smem_attribute(fn, L::kDynamicBytes, slot);
  if (st != NTB200_OK) return st;
  const int sms = num_sms();
  int splits = forced_splits > 0 ? forced_splits : 1;
  for (int cand = (SWIGLU || forced_splits > 0) ? 1 : 8; cand >= 2; --cand) {
    if (cand > prm.k_steps_total || int64_t(n_tiles) * cand > sms) continue;
    const int per = static_cast<int>(ceil_div(prm.k_steps_total, cand));
    const int used = static_cast<int>(ceil_div(prm.k_steps_total, per));
    if (used != cand) continue;  // an uneven split that leaves a CTA without k-steps
    if (resident_clusters(fn, L::kDynamicBytes, cand, slot) < n_tiles) continue;
    splits = cand;
    break;
  }
  prm.splits = splits;
  prm.k_steps_per_split = static_cast<int>(ceil_div(prm.k_steps_total, splits));
  if (NORM && prm.k_steps_per_split > NSTEPS)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE,
                "rms_norm_linear: K = %d k-steps per CTA exceeds %d (too few weight tiles to split K)",
                prm.k_steps_per_split, NSTEPS);
  // a CTA range of at most 32 k-steps takes the layout with the deeper weight ring
  if constexpr (NORM && NSTEPS == kNormMaxSteps)
    if (prm.k_steps_per_split <= 32)
      return launch_skinny<T, MP, TT, SWIGLU, NORM, 32>(wmap, xmap, prm, n_tiles, s, slot + 2, splits);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * splits));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  set_pdl_attribute(attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_skinny_kernel<T, MP, TT, SWIGLU, NORM, NSTEPS>, wmap, xmap, prm);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "linear (M <= 256): launch failed: %s", cudaGetErrorString(e));
  }
  return NTB200_OK;
}

template <typename T, bool SWIGLU = false>
int dispatch_skinny(const CUtensorMap& wmap, const CUtensorMap& xmap, const SkinnyParams& prm, int mp, int n_tiles,
                    cudaStream_t s, int slot_base) {
  switch (mp) {
    case 16: return launch_skinny<T, 16, 1, SWIGLU>(wmap, xmap, prm, n_tiles, s, slot_base + 0);
    case 32: return launch_skinny<T, 32, 1, SWIGLU>(wmap, xmap, prm, n_tiles, s, slot_base + 1);
    case 64: return launch_skinny<T, 64, 1, SWIGLU>(wmap, xmap, prm, n_tiles, s, slot_base + 2);
    case 128: return launch_skinny<T, 128, 1, SWIGLU>(wmap, xmap, prm, n_tiles, s, slot_base + 3);
    default: return launch_skinny<T, 128, 2, SWIGLU>(wmap, xmap, prm, n_tiles, s, slot_base + 4);
  }
}

// Which decode-batch kernel `ntb200_linear` uses (M <= 256), from CUDA-graph timings with
// the weights beyond L2: the 256-row-tile kernel (gemm_skinny_kernel) wins where its tiles
// fill >= 70 % of the SMs without a K split (28672 x 4096: 46 vs 51 us at M = 128, 58 vs
// 68 us at M = 256), and with a split up to M = 128 once there are >= 24 tiles (6144 x 4096:
// 12.1 vs 13.5 us at M = 1, 16.7 vs 17.6 us at M = 128).  With fewer tiles, or 256 token
// rows, the fp32 partial rows its K split must sum (M x 256 per CTA) cost more than the
// halved MMA count saves, and the 128-row weight tiles of gemm_small_m_kernel are faster.
bool skinny_preferred(int64_t M, int64_t N, int sms) {
  const int64_t tiles = ceil_div(N, kSkinnyBN);
  if (tiles * 10 >= int64_t(sms) * 7) return true;
  return M <= 128 && tiles >= 24;
}

// ---- LM head + greedy argmax -------------------------------------------------------

template <typename T, int MP>
int launch_small_argmax(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, cudaStream_t s,
                        int slot) {
  const int64_t groups = (prm.n_tiles + 1) / 2;
  if (groups <= num_sms()) return launch_small<T, MP, 2, true, false, true>(wmap, xmap, prm, s, slot + 1);
  return launch_small<T, MP, 2, false, false, true>(wmap, xmap, prm, s, slot);
}

template <typename T>
int dispatch_small_argmax(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, int mp,
                          cudaStream_t s, int slot_base) {
  switch (mp) {
    case 16: return launch_small_argmax<T, 16>(wmap, xmap, prm, s, slot_base + 0);
    case 32: return launch_small_argmax<T, 32>(wmap, xmap, prm, s, slot_base + 2);
    case 64: return launch_small_argmax<T, 64>(wmap, xmap, prm, s, slot_base + 4);
    case 128: return launch_small_argmax<T, 128>(wmap, xmap, prm, s, slot_base + 6);
    default: return launch_small_argmax<T, 256>(wmap, xmap, prm, s, slot_base + 8);
  }
}

// token keys -> vocabulary indices
__global__ void __launch_bounds__(256) argmax_finalize_kernel(const unsigned long long* __restrict__ keys,
                                                              int64_t* __restrict__ out, int64_t M) {
  pdl_trigger();
  pdl_wait();
  const int64_t m = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (m < M) out[m] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(keys[m]));
}

// argmax of one row of logits already in memory (the path for M > 256): one CTA per row
template <typename T>
__global__ void __launch_bounds__(512) row_argmax_kernel(const T* __restrict__ logits, int64_t ld, int64_t V,
                                                          int64_t* __restrict__ out) {
  __shared__ unsigned long long red[16];
  pdl_trigger();
  pdl_wait();
  const T* row = logits + int64_t(blockIdx.x) * ld;
  unsigned long long best = 0ull;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
    const unsigned long long k = argmax_key<T>(Elem<T>::to_f(row[j]), j);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o2 = shfl_xor_u64(best, off);
    best = o2 > best ? o2 : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o2 = shfl_xor_u64(best, off);
      best = o2 > best ? o2 : best;
    }
    if (threadIdx.x == 0) out[blockIdx.x] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(best));
  }
}

}  // namespace
}  // namespace ntb200

extern "C" size_t ntb200_linear_argmax_workspace_size(int64_t M, int64_t V, int64_t K) {
  using ntb200::ceil_div;
  (void)K;
  if (M <= 0 || V <= 0) return 0;
  const size_t keys = static_cast<size_t>(ceil_div(M * 8, 256) * 256);
  if (M <= 256) return keys;
  return keys + static_cast<size_t>(ceil_div(M * V * 2, 256) * 256);
}

extern "C" int ntb200_linear_argmax(int64_t* out_index, const void* x, const void* weight, int64_t M, int64_t V,
                                    int64_t K, int64_t x_row_stride, int64_t weight_row_stride, void* workspace,
                                    size_t workspace_bytes, int dtype, void* stream) {
  using namespace ntb200;
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "linear_argmax: dtype %d (bf16/f16 only)", dtype);
  if (M < 0 || V <= 0 || K <= 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "linear_argmax: bad shape");
  if (M == 0) return NTB200_OK;
  if (V > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear_argmax: vocabulary too large");
  if (!out_index || !x || !weight) return fail(NTB200_ERR_INVALID_ARGUMENT, "linear_argmax: null pointer");
  if (x_row_stride < K || weight_row_stride < K)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "linear_argmax: row stride too small");
  if (!aligned16(x) || !aligned16(weight) || x_row_stride % 8 != 0 || weight_row_stride % 8 != 0)
    return fail(NTB200_ERR_MISALIGNED, "linear_argmax: x/weight must be 16-byte aligned with row strides %% 8 == 0");
  const size_t need = ntb200_linear_argmax_workspace_size(M, V, K);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(NTB200_ERR_WORKSPACE, "linear_argmax: workspace needs %zu bytes (256-aligned), got %zu", need,
                workspace_bytes);
  const bool bf16 = dtype == NTB200_DTYPE_BF16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long* keys = static_cast<unsigned long long*>(workspace);
  if (M > 256) {
    // logits through the ordinary GEMM, then one CTA per row
    void* logits = static_cast<char*>(workspace) + ceil_div(M * 8, 256) * 256;
    int st = ntb200_linear(logits, x, weight, nullptr, M, V, K, x_row_stride, weight_row_stride, V, nullptr, 0,
                           dtype, stream);
    if (st != NTB200_OK) return st;
    if (bf16)
      return launch_kernel("linear_argmax", row_argmax_kernel<__nv_bfloat16>, dim3(unsigned(M)), dim3(512), 0, s,
                           static_cast<const __nv_bfloat16*>(logits), V, V, out_index);
    return launch_kernel("linear_argmax", row_argmax_kernel<__half>, dim3(unsigned(M)), dim3(512), 0, s,
                         static_cast<const __half*>(logits), V, V, out_index);
  }
  if (cudaMemsetAsync(keys, 0, static_cast<size_t>(M) * 8, s) != cudaSuccess)
    return fail(NTB200_ERR_CUDA, "linear_argmax: clearing the keys: %s", cudaGetErrorString(cudaGetLastError()));
  const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  CUtensorMap wmap, xmap;
  int st = make_kmajor_map(&wmap, weight, bf16, V, K, weight_row_stride, BM);
  if (st != NTB200_OK) return st;
  st = make_kmajor_map(&xmap, x, bf16, M, K, x_row_stride, mp);
  if (st != NTB200_OK) return st;
  SmallParams sp;
  sp.out = nullptr;
  sp.bias = nullptr;
  sp.M = M;
  sp.N = V;
  sp.out_stride = 0;
  sp.n_tiles = static_cast<int>(ceil_div(V, BM));
  sp.splits = 1;
  sp.k_steps_total = static_cast<int>(ceil_div(K, BK));
  sp.k_steps_per_split = sp.k_steps_total;
  sp.n_half = 0;
  sp.argmax_keys = keys;
  sp.err = device_error_word();
  st = bf16 ? dispatch_small_argmax<__nv_bfloat16>(wmap, xmap, sp, mp, s, 70)
            : dispatch_small_argmax<__half>(wmap, xmap, sp, mp, s, 80);
  if (st != NTB200_OK) return st;
  return launch_kernel("linear_argmax", argmax_finalize_kernel, dim3(unsigned(ceil_div(M, 256))), dim3(256), 0, s,
                       static_cast<const unsigned long long*>(keys), out_index, M);
}

extern "C" int ntb200_linear_silu_and_mul(void* out, const void* x, const void* weight, int64_t M,
                                          int64_t I, int64_t K, int64_t x_row_stride,
                                          int64_t weight_row_stride, int64_t out_row_stride, int dtype,
                                          void* stream) {
  using namespace ntb200;
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "linear_silu_and_mul: dtype %d (bf16/f16 only)", dtype);
  if (M < 0 || I < 0 || K <= 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "linear_silu_and_mul: bad shape");
  if (M == 0 || I == 0) return NTB200_OK;
  if (!out || !x || !weight) return fail(NTB200_ERR_INVALID_ARGUMENT, "linear_silu_and_mul: null pointer");
  if (x_row_stride < K || weight_row_stride < K || out_row_stride < I)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "linear_silu_and_mul: row stride too small");
  if (!aligned16(x) || !aligned16(weight) || x_row_stride % 8 != 0 || weight_row_stride % 8 != 0)
    return fail(NTB200_ERR_MISALIGNED,
                "linear_silu_and_mul: x/weight must be 16-byte aligned with row strides %% 8 == 0");
  if (2 * I > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear_silu_and_mul: I too large");
  const bool bf16 = dtype == NTB200_DTYPE_BF16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M > 64 && M <= 256 && ceil_div(I, kSkinnyBN / 2) * 10 >= int64_t(num_sms()) * 7) {
    // 256-row weight tiles (128 gate + 128 up rows) filling the SMs without a K split; at
    // M <= 64 the 128-row tiles below measured faster (I = 14336, K = 4096: 38.5 against
    // 47.8 us at M = 1; 52.7 against 56.1 us at M = 128, 70.2 against 76.8 at M = 256)
    const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    CUtensorMap wmap, xmap;
    int st = make_gate_up_map(&wmap, weight, bf16, I, K, weight_row_stride);
    if (st != NTB200_OK) return st;
    st = make_kmajor_map(&xmap, x, bf16, M, K, x_row_stride, mp > BM ? BM : mp);
    if (st != NTB200_OK) return st;
    SkinnyParams sp;
    sp.out = out;
    sp.bias = nullptr;
    sp.M = M;
    sp.N = 2 * I;
    sp.out_stride = out_row_stride;
    sp.splits = 1;
    sp.k_steps_total = static_cast<int>(ceil_div(K, BK));
    sp.k_steps_per_split = sp.k_steps_total;
    sp.n_half = I;
    sp.err = device_error_word();
    const int tiles = static_cast<int>(ceil_div(I, kSkinnyBN / 2));
    return bf16 ? dispatch_skinny<__nv_bfloat16, true>(wmap, xmap, sp, mp, tiles, s, 106)
                : dispatch_skinny<__half, true>(wmap, xmap, sp, mp, tiles, s, 111);
  }
  if (M <= 256) {
    const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    CUtensorMap wmap, xmap;
    int st = make_kmajor_map(&wmap, weight, bf16, 2 * I, K, weight_row_stride, BM);
    if (st != NTB200_OK) return st;
    st = make_kmajor_map(&xmap, x, bf16, M, K, x_row_stride, mp);
    if (st != NTB200_OK) return st;
    SmallParams sp;
    sp.out = out;
    sp.bias = nullptr;
    sp.M = M;
    sp.N = 2 * I;
    sp.out_stride = out_row_stride;
    sp.n_tiles = static_cast<int>(2 * ceil_div(I, BM));
    sp.splits = 1;
    sp.k_steps_total = static_cast<int>(ceil_div(K, BK));
    sp.k_steps_per_split = sp.k_steps_total;
    sp.n_half = I;
    sp.argmax_keys = nullptr;
    sp.err = device_error_word();
    return bf16 ? dispatch_small_swiglu<__nv_bfloat16>(wmap, xmap, sp, mp, s, 50)
                : dispatch_small_swiglu<__half>(wmap, xmap, sp, mp, s, 60);
  }
  if (M >= kPairMinM)
    return launch_pair<true>(out, x, weight, nullptr, M, 2 * I, K, x_row_stride, weight_row_stride, out_row_stride,
                             bf16, s);
  switch (pick_tile_width(M, 2 * I, num_sms())) {
    case 128:
      return launch_large<128, true>(out, x, weight, nullptr, M, 2 * I, K, x_row_stride, weight_row_stride,
                                     out_row_stride, bf16, s);
    case 192:
      return launch_large<192, true>(out, x, weight, nullptr, M, 2 * I, K, x_row_stride, weight_row_stride,
                                     out_row_stride, bf16, s);
    default:
      return launch_large<256, true>(out, x, weight, nullptr, M, 2 * I, K, x_row_stride, weight_row_stride,
                                     out_row_stride, bf16, s);
  }
}

extern "C" size_t ntb200_linear_workspace_size(int64_t M, int64_t N, int64_t K) {
  (void)M;
  (void)N;
  (void)K;
  return 0;
}

extern "C" int ntb200_linear(void* out, const void* x, const void* weight, const void* bias,
                             int64_t M, int64_t N, int64_t K, int64_t x_row_stride,
                             int64_t weight_row_stride, int64_t out_row_stride, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream) {
  using namespace ntb200;
  (void)workspace;
  (void)workspace_bytes;
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "linear: dtype %d (bf16/f16 only)", dtype);
  if (M < 0 || N < 0 || K <= 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "linear: bad shape");
  if (M == 0 || N == 0) return NTB200_OK;
  if (!out || !x || !weight) return fail(NTB200_ERR_INVALID_ARGUMENT, "linear: null pointer");
  if (x_row_stride < K || weight_row_stride < K || out_row_stride < N)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "linear: row stride too small");
  if (!aligned16(x) || !aligned16(weight) || x_row_stride % 8 != 0 || weight_row_stride % 8 != 0)
    return fail(NTB200_ERR_MISALIGNED, "linear: x/weight must be 16-byte aligned with row strides %% 8 == 0");
  const bool bf16 = dtype == NTB200_DTYPE_BF16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M <= 256) {
    if (skinny_preferred(M, N, num_sms())) {
      // decode-sized batches: weight rows on the MMA's N side, K split over a cluster
      const int64_t n_tiles = ceil_div(N, kSkinnyBN);
      if (n_tiles > 0x7fffffff / 8) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear: too many tiles");
      const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
      CUtensorMap wmap, xmap;
      int st = make_kmajor_map(&wmap, weight, bf16, N, K, weight_row_stride, kSkinnyBN);
      if (st != NTB200_OK) return st;
      st = make_kmajor_map(&xmap, x, bf16, M, K, x_row_stride, mp > BM ? BM : mp);
      if (st != NTB200_OK) return st;
      SkinnyParams sp;
      sp.out = out;
      sp.bias = bias;
      sp.M = M;
      sp.N = N;
      sp.out_stride = out_row_stride;
      sp.splits = 1;
      sp.k_steps_total = static_cast<int>(ceil_div(K, BK));
      sp.k_steps_per_split = sp.k_steps_total;
      sp.n_half = 0;
      sp.err = device_error_word();
      return bf16 ? dispatch_skinny<__nv_bfloat16>(wmap, xmap, sp, mp, static_cast<int>(n_tiles), s, 96)
                  : dispatch_skinny<__half>(wmap, xmap, sp, mp, static_cast<int>(n_tiles), s, 101);
    }
    // swap-AB + cluster split-K path for decode-sized batches
    const int64_t n_tiles = ceil_div(N, BM);
    if (n_tiles > 0x7fffffff / 8) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear: too many tiles");
    const int ksteps = static_cast<int>(ceil_div(K, BK));
    const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    const int nt = small_tiles_per_cta(mp, n_tiles, num_sms());
    const int64_t groups = ceil_div(n_tiles, nt);
    // split K so that the grid has about `target` CTAs; clusters of 1, 2, 4 or 8 CTAs pack
    // into the GPCs without stranding SMs (a cluster must fit inside one GPC)
    auto plan = [&](int64_t target, int& splits, int& per) {
      const int64_t want = target / groups;
      splits = want >= 8 ? 8 : want >= 4 ? 4 : want >= 2 ? 2 : 1;
      if (splits > ksteps) splits = ksteps;
      per = static_cast<int>(ceil_div(ksteps, splits));
      splits = static_cast<int>(ceil_div(ksteps, per));
    };
    int splits_big, per_big, splits_small, per_small;
    plan(num_sms(), splits_big, per_big);          // one CTA per SM, ~192 KB rings
    plan(2 * num_sms(), splits_small, per_small);  // two CTAs per SM, ~96 KB rings
    CUtensorMap wmap, xmap;
    int st = make_kmajor_map(&wmap, weight, bf16, N, K, weight_row_stride, BM);
    if (st != NTB200_OK) return st;
    st = make_kmajor_map(&xmap, x, bf16, M, K, x_row_stride, mp);
    if (st != NTB200_OK) return st;
    SmallParams sp;
    sp.out = out;
    sp.bias = bias;
    sp.M = M;
    sp.N = N;
    sp.out_stride = out_row_stride;
    sp.n_tiles = static_cast<int>(n_tiles);
    sp.k_steps_total = ksteps;
    sp.n_half = 0;
    sp.argmax_keys = nullptr;
    sp.err = device_error_word();
    SmallParams sp_big = sp, sp_small = sp;
    sp_big.splits = splits_big;
    sp_big.k_steps_per_split = per_big;
    sp_small.splits = splits_small;
    sp_small.k_steps_per_split = per_small;
    return bf16 ? dispatch_small<__nv_bfloat16>(wmap, xmap, sp_big, sp_small, mp, nt, s, 4)
                : dispatch_small<__half>(wmap, xmap, sp_big, sp_small, mp, nt, s, 18);
  }
  if (M >= kPairMinM)
  if (M >= kPairMinM)
    return launch_pair(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
  const int bn = pick_tile_width(M, N, num_sms());
  switch (bn) {
    case 128: return launch_large<128>(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
    case 192: return launch_large<192>(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
    default: return launch_large<256>(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
  }
}

extern "C" int ntb200_rms_norm_linear(void* out, void* residual_out, const void* x, const void* residual,
                                      const void* norm_weight, float eps, const void* weight, int64_t M, int64_t N,
                                      int64_t K, int64_t x_row_stride, int64_t residual_row_stride,
                                      int64_t residual_out_row_stride, int64_t weight_row_stride,
                                      int64_t out_row_stride, int dtype, void* stream) {
  using namespace ntb200;
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rms_norm_linear: dtype %d (bf16/f16 only)", dtype);
  if (M < 0 || N < 0 || K <= 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm_linear: bad shape");
  if (M == 0 || N == 0) return NTB200_OK;
  if (M > kNormRows)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rms_norm_linear: decode batches of at most %d tokens (M = %lld)",
                kNormRows, static_cast<long long>(M));
  if (!out || !x || !norm_weight || !weight) return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm_linear: null pointer");
  if ((residual == nullptr) != (residual_out == nullptr))
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm_linear: residual and residual_out go together");
  if (residual_out != nullptr && (residual_out == residual || residual_out == x))
    return fail(NTB200_ERR_INVALID_ARGUMENT,
                "rms_norm_linear: residual_out must not alias residual or x (other CTAs still read them)");
  if (x_row_stride < K || weight_row_stride < K || out_row_stride < N ||
      (residual != nullptr && (residual_row_stride < K || residual_out_row_stride < K)))
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm_linear: row stride too small");
  const bool rows16 = x_row_stride % 8 == 0 && weight_row_stride % 8 == 0 &&
                      (residual == nullptr || (residual_row_stride % 8 == 0 && residual_out_row_stride % 8 == 0));
  if (K % 8 != 0 || !rows16 || !aligned16(x) || !aligned16(weight) || !aligned16(norm_weight) ||
      (residual != nullptr && (!aligned16(residual) || !aligned16(residual_out))))
    return fail(NTB200_ERR_MISALIGNED, "rms_norm_linear: 16-byte aligned rows and K %% 8 == 0 required");
  const bool bf16 = dtype == NTB200_DTYPE_BF16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n_tiles = ceil_div(N, kSkinnyBN);
  if (n_tiles > 0x7fffffff / 8) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rms_norm_linear: too many tiles");
  CUtensorMap wmap;
  int st = make_kmajor_map(&wmap, weight, bf16, N, K, weight_row_stride, kSkinnyBN);
  if (st != NTB200_OK) return st;
  SkinnyParams sp = {};
  sp.out = out;
  sp.bias = nullptr;
  sp.M = M;
  sp.N = N;
  sp.out_stride = out_row_stride;
  sp.splits = 1;
  sp.k_steps_total = static_cast<int>(ceil_div(K, BK));
  sp.k_steps_per_split = sp.k_steps_total;
  sp.n_half = 0;
  sp.err = device_error_word();
  sp.nx = x;
  sp.nres = residual;
  sp.nres_out = residual_out;
  sp.ngamma = norm_weight;
  sp.eps = eps;
  sp.K = K;
  sp.x_stride = x_row_stride;
  sp.r_stride = residual_row_stride;
  sp.ro_stride = residual_out_row_stride;
  // the token operand comes from shared memory: the second map argument is unused
  return bf16 ? launch_skinny<__nv_bfloat16, kNormRows, 1, false, true>(wmap, wmap, sp, static_cast<int>(n_tiles), s, 116)
              : launch_skinny<__half, kNormRows, 1, false, true>(wmap, wmap, sp, static_cast<int>(n_tiles), s, 117);
}

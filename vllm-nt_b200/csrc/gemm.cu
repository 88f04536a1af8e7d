// Dense projection GEMM on the 5th-generation tensor cores:
//   out[M, N] = x[M, K] . W[N, K]^T (+ bias),  bf16/f16 in, fp32 accumulate in TMEM.
//
// M > 256: persistent, warp-specialised, one CTA per SM (192 threads), tile 128 x BN with
// BN = 256, 192 or 128 picked per shape to fill whole waves of SMs:
//   warp 0      TMA producer: 128x64 x-tile + BNx64 W-tile per k-step (128-byte swizzle,
//               K-major) into a ~192-200 KB shared-memory ring;
//   warp 1      allocates TMEM for two 128xBN fp32 accumulators and its lane 0 issues
//               tcgen05.mma (M=128, N=BN, K=16; four per k-step), committing each stage
//               back to the producer and each finished tile to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM lanes
//               32*(w%4)..+31, i.e. output rows), add bias, round, store.
// The epilogue of tile i overlaps the MMAs of tile i+1 (double-buffered accumulator).
// Tiles are walked with the M index fastest so a wave of CTAs shares W tiles through L2
// while x (M*K*2 bytes) stays L2-resident.  No TMA multicast is used anywhere.
//
// Every mbarrier wait is bounded (2 s); a timeout sets NTB200_DEVERR_WAIT_TIMEOUT, the
// roles leave their loops, in-flight copies and MMAs are drained (bounded), and TMEM is
// freed before the CTA exits.
//
// Replaces vllm_nt/_ntops/kernels/linear.py:9-85 (a Triton tl.dot tile loop).
#include "common.cuh"

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

// K-major operand tile with 128-byte swizzle: 8-row atoms of 1024 bytes.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused here)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A/B both bf16 (or both f16),
// both K-major, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct GemmParams {
  void* out;
  const void* bias;
  int64_t M, N, K;
  int64_t out_stride;
  int num_m_blocks, num_n_blocks;
  unsigned int* err;
};

template <typename T, int BN_>
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
        const int mb = tile % p.num_m_blocks;
        const int nb = tile / p.num_m_blocks;
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
          tma_load_2d(b_dst, &b_map, kb * BK, nb * BN, smem_u32(&full[s]));
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
      const int mb = tile % p.num_m_blocks;
      const int nb = tile / p.num_m_blocks;
      const int64_t row = int64_t(mb) * BM + row_in_tile;
      const int64_t col0 = int64_t(nb) * BN;
      T* orow = out + row * p.out_stride;
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        uint32_t r[32];
        __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it together
        tmem_ld_32(tmem_base + (uint32_t(quad * 32) << 16) + acc * kAccStride + chunk * 32, r);
        const int64_t c0 = col0 + chunk * 32;
        if (row < p.M && c0 < p.N) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if (bias != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c0 + i < p.N) v[i] += Elem<T>::to_f(bias[c0 + i]);
        }
        if (c0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(orow + c0) & 15u) == 0)) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = v[q * 8 + i];
            store_f<T, 8>(orow + c0 + q * 8, w);
          }
        } else {
          for (int i = 0; i < 32 && c0 + i < p.N; ++i) orow[c0 + i] = Elem<T>::from_f(v[i]);
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

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
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

// ------------------------------------------------------------------------------------
// Small-M path (M <= 256: decode batches).  out^T = W . x^T ("swap AB"): the weight tile
// fills the UMMA M=128 side, the few token rows are the UMMA N side (padded to MP = 16 ..
// 256; rows past M are TMA zero-fill and cost no HBM traffic).  With only N/128 weight
// tiles, K is split across the CTAs of a thread-block cluster (<= 8); each CTA parks its
// fp32 partial tile in its own shared memory and, after a cluster barrier, every CTA sums
// a share of the output rows across the cluster through distributed shared memory and
// writes them (bias added, rounded).  One launch, no global workspace.
// ------------------------------------------------------------------------------------

// ring depth per token tile: about 96 KB of stages, so two CTAs fit on an SM
template <int MP>
constexpr int small_stages() {
  return (96 * 1024) / (kATileBytes + MP * BK * 2) < 3 ? 3 : (96 * 1024) / (kATileBytes + MP * BK * 2);
}

template <int MP>
struct SmallSmem {
  static constexpr int kSmallStages = small_stages<MP>();
  static constexpr int kXTile = MP * BK * 2;
  static constexpr int kStage = kATileBytes + kXTile;  // 128 weight rows + MP x rows
  static constexpr int kRing = 0;
  static constexpr int kFull = kSmallStages * kStage;
  static constexpr int kEmpty = kFull + 8 * kSmallStages;
  static constexpr int kTmemFull = kEmpty + 8 * kSmallStages;
  static constexpr int kTmemBase = kTmemFull + 8;
  static constexpr int kEnd = kTmemBase + 8;
  static constexpr int kDynamicBytes = kEnd + 1024;
  static constexpr int kTmemCols = MP < 32 ? 32 : MP;
  static_assert(MP * BM * 4 <= kSmallStages * kStage, "partial tile must fit in the ring");
};

struct SmallParams {
  void* out;
  const void* bias;
  int64_t M, N;
  int64_t out_stride;
  int splits;
  int k_steps_per_split;
  int k_steps_total;
  unsigned int* err;
};

__device__ __forceinline__ void tmem_ld_16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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

template <typename T, int MP>
__global__ void __launch_bounds__(kThreads, 1) gemm_small_m_kernel(
    const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map,
    const SmallParams p) {
  using L = SmallSmem<MP>;
  constexpr int kSmallStages = L::kSmallStages;
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
  const int ntile = blockIdx.x / p.splits;
  const int kb0 = split * p.k_steps_per_split;
  const int kb1 = min(kb0 + p.k_steps_per_split, p.k_steps_total);
  const int nk = kb1 > kb0 ? kb1 - kb0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmallStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
  }
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
        const int s = it % kSmallStages;
        if (it >= kSmallStages && !mbar_wait(&empty[s], ((it / kSmallStages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&full[s], L::kStage);
        const uint32_t w_dst = ring + s * L::kStage;
        const uint32_t x_dst = w_dst + kATileBytes;
        tma_load_2d(w_dst, &w_map, (kb0 + it) * BK, ntile * BM, smem_u32(&full[s]));
        tma_load_2d(x_dst, &x_map, (kb0 + it) * BK, 0, smem_u32(&full[s]));
        issued = it + 1;
      }
      const int first = issued > kSmallStages ? issued - kSmallStages : 0;
      for (int j = first; j < issued; ++j) mbar_wait(&full[j % kSmallStages], (j / kSmallStages) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc(std::is_same<T, __nv_bfloat16>::value, BM, MP);
      for (int it = 0; it < nk; ++it) {
        const int s = it % kSmallStages;
        if (!mbar_wait(&full[s], (it / kSmallStages) & 1, p.err)) break;
        tc_fence_after();
        const uint32_t w_addr = ring + s * L::kStage;
        const uint64_t adesc = sw128_kmajor_desc(w_addr);
        const uint64_t bdesc = sw128_kmajor_desc(w_addr + kATileBytes);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_f16(tmem_base, adesc + 2 * k, bdesc + 2 * k, idesc, (it > 0 || k > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(tmem_full);  // also the "all MMAs done" point before TMEM is released
    }
  } else {
    // epilogue warps: TMEM (lane = weight row n, column = token m) -> smem partial [MP][128]
    const int quad = warp & 3;
    const int n_local = quad * 32 + lane;
    float* part = reinterpret_cast<float*>(smem + L::kRing);
    const bool ok = mbar_wait(tmem_full, 0, p.err);
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < MP / 16; ++c) {
      uint32_t r[16];
      __syncwarp();
      tmem_ld_16(tmem_base + (uint32_t(quad * 32) << 16) + c * 16, r);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        part[(c * 16 + i) * BM + n_local] = (ok && nk > 0) ? __uint_as_float(r[i]) : 0.f;
    }
    tc_fence_before();
  }

  // every CTA of the cluster has its partial tile in shared memory
  cluster_sync_all();
  {
    // this CTA owns output rows [r0, r1); a row is 128 partial floats = 32 float4, so the
    // 192 threads cover 6 rows per pass, and each pass has its splits x float4 remote loads
    // in flight before any is summed
    const int rows_per = static_cast<int>((p.M + p.splits - 1) / p.splits);
    const int r0 = split * rows_per;
    const int r1 = static_cast<int>(p.M < int64_t(r0) + rows_per ? p.M : int64_t(r0) + rows_per);
    const int q4 = threadIdx.x & 31;  // float4 column group: n_local = 4 * q4 .. +3
    const uint32_t part_addr = smem_u32(smem + L::kRing);
    T* out = static_cast<T*>(p.out);
    const T* bias = static_cast<const T*>(p.bias);
    const int64_t n0 = int64_t(ntile) * BM + 4 * q4;
    float bvec[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) bvec[i] = (bias != nullptr && n0 + i < p.N) ? Elem<T>::to_f(bias[n0 + i]) : 0.f;
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
  }
  // no CTA may leave (or free its shared memory) while its partner still reads it
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::kTmemCols)
                 : "memory");
  }
}

template <typename T, int MP>
int launch_small(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, int n_tiles,
                 cudaStream_t s, int attr_slot) {
  using L = SmallSmem<MP>;
  const void* fn = reinterpret_cast<const void*>(gemm_small_m_kernel<T, MP>);
  int st = ensure_smem_attribute(fn, L::kDynamicBytes, attr_slot);
  if (st != NTB200_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * prm.splits));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(prm.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_small_m_kernel<T, MP>, wmap, xmap, prm);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "linear (small M): launch failed: %s", cudaGetErrorString(e));
  }
  return NTB200_OK;
}

template <typename T>
int dispatch_small(const CUtensorMap& wmap, const CUtensorMap& xmap, const SmallParams& prm, int n_tiles,
                   int mp, cudaStream_t s, int slot_base) {
  switch (mp) {
    case 16: return launch_small<T, 16>(wmap, xmap, prm, n_tiles, s, slot_base + 0);
    case 32: return launch_small<T, 32>(wmap, xmap, prm, n_tiles, s, slot_base + 1);
    case 64: return launch_small<T, 64>(wmap, xmap, prm, n_tiles, s, slot_base + 2);
    case 128: return launch_small<T, 128>(wmap, xmap, prm, n_tiles, s, slot_base + 3);
    default: return launch_small<T, 256>(wmap, xmap, prm, n_tiles, s, slot_base + 4);
  }
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

template <int BNV>
int launch_large(void* out, const void* x, const void* weight, const void* bias, int64_t M, int64_t N,
                 int64_t K, int64_t xs, int64_t ws, int64_t os, bool bf16, cudaStream_t s) {
  using C = GemmCfg<BNV>;
  const int64_t mblocks = ceil_div(M, BM), nblocks = ceil_div(N, BNV);
  if (mblocks * nblocks > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear: too many tiles");
  CUtensorMap amap, bmap;
  int st = make_kmajor_map(&amap, x, bf16, M, K, xs, BM);
  if (st != NTB200_OK) return st;
  st = make_kmajor_map(&bmap, weight, bf16, N, K, ws, BNV);
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
  prm.err = device_error_word();
  const int64_t tiles = mblocks * nblocks;
  const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  const int slot = 16 + (BNV == 256 ? 0 : (BNV == 192 ? 2 : 4)) + (bf16 ? 0 : 1);
  if (bf16) {
    st = ensure_smem_attribute(reinterpret_cast<const void*>(gemm_tcgen05_kernel<__nv_bfloat16, BNV>), C::kDynamicBytes, slot);
    if (st != NTB200_OK) return st;
    gemm_tcgen05_kernel<__nv_bfloat16, BNV><<<grid, kThreads, C::kDynamicBytes, s>>>(amap, bmap, prm);
  } else {
    st = ensure_smem_attribute(reinterpret_cast<const void*>(gemm_tcgen05_kernel<__half, BNV>), C::kDynamicBytes, slot);
    if (st != NTB200_OK) return st;
    gemm_tcgen05_kernel<__half, BNV><<<grid, kThreads, C::kDynamicBytes, s>>>(amap, bmap, prm);
  }
  return check_launch("linear");
}

}  // namespace
}  // namespace ntb200

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
    // swap-AB + cluster split-K path for decode-sized batches
    const int64_t n_tiles = ceil_div(N, BM);
    if (n_tiles > 0x7fffffff / 8) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "linear: too many tiles");
    const int ksteps = static_cast<int>(ceil_div(K, BK));
    int splits = static_cast<int>(num_sms() / n_tiles);
    splits = splits < 1 ? 1 : (splits > 8 ? 8 : splits);
    if (splits > ksteps) splits = ksteps;
    const int per = static_cast<int>(ceil_div(ksteps, splits));
    splits = static_cast<int>(ceil_div(ksteps, per));  // no empty split
    const int mp = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
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
    sp.splits = splits;
    sp.k_steps_per_split = per;
    sp.k_steps_total = ksteps;
    sp.err = device_error_word();
    return bf16 ? dispatch_small<__nv_bfloat16>(wmap, xmap, sp, static_cast<int>(n_tiles), mp, s, 4)
                : dispatch_small<__half>(wmap, xmap, sp, static_cast<int>(n_tiles), mp, s, 9);
  }
  const int bn = pick_tile_width(M, N, num_sms());
  switch (bn) {
    case 128: return launch_large<128>(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
    case 192: return launch_large<192>(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
    default: return launch_large<256>(out, x, weight, bias, M, N, K, x_row_stride, weight_row_stride, out_row_stride, bf16, s);
  }
}

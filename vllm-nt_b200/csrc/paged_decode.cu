// Paged-attention decode: split-K (flash-decoding) over KV blocks, GQA heads packed,
// K/V tiles staged by TMA through an mbarrier ring.
//
// Work unit = (sequence b, KV head h, chunk c of `chunk_tokens` cached tokens); one CTA
// per unit (grid x = chunk, y = KV head, z = sequence; CTAs past a sequence's last chunk
// exit at once).  Warp 4 is the producer: it stages the chunk's block ids in shared
// memory, then lane 0 issues, per 16-token KV block, two 4-D TMA boxes for K and two for V
// (64 dims x 16 tokens each, 128-byte swizzled) into an 8-slot ring guarded by full/empty
// mbarriers.  Warps 0-3 are consumers: warp w takes blocks w, w+4, ... of the chunk and
// keeps its own online-softmax state.
//
// Per block a consumer computes S^T = K . q^T with mma.m16n8k16 (16 tokens x 8 heads x 128
// dims: the GQA group's query heads sit in the n dimension, so one K tile is read once for
// all of them), applies the running max in fp32 (exp2 domain), turns the S^T accumulator
// into the P^T operand with movmatrix (no shared-memory round trip), and accumulates
// O^T += V^T . P^T with ldmatrix.trans-fed MMAs.  At the end the four warps merge their
// states through shared memory and the CTA writes the chunk's normalised partial output
// and log-sum-exp; `paged_decode_combine_kernel` merges the chunks of each (b, head).
//
// HBM traffic is one read of every cached K/V row of the sequence (the roofline term),
// plus q, the block table and the small partials.  The reference (vllm_nt/_ntops/kernels/
// attention.py:97-197, vllm_nt/_ntops/torch/attention.py:51-77) instead replicates the
// whole cache per GQA group with a torch copy and walks every block-table entry serially.
#include <cstring>

#include "common.cuh"

namespace ntb200 {
namespace {

constexpr int kHeadDim = 128;
constexpr int kBlockTokens = 16;
constexpr int kStages = 8;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHalfTileBytes = kBlockTokens * 64 * 2;  // 16 tokens x 64 dims x 2 B
constexpr int kTileBytes = 2 * kHalfTileBytes;         // one K (or V) block of one head
constexpr int kSlotBytes = 2 * kTileBytes;             // K + V
constexpr int kMaxChunkBlocks = 128;                   // block ids staged per unit
constexpr float kLog2e = 1.4426950408889634f;

struct SmemLayout {
  // offsets from a 1024-aligned base
  static constexpr int kSlots = 0;
  static constexpr int kFull = kStages * kSlotBytes;
  static constexpr int kEmpty = kFull + kStages * 8;
  static constexpr int kIds = kEmpty + kStages * 8;
  static constexpr int kEnd = kIds + kMaxChunkBlocks * 4;
  static constexpr int kDynamicBytes = kEnd + 1024;  // slack for aligning the base
};
// the cross-warp merge reuses the slot ring: o[4 warps][8 heads][128] + m,l[4][8]
static_assert(kConsumerWarps * 8 * kHeadDim * 4 + 2 * kConsumerWarps * 8 * 4 <= kStages * kSlotBytes,
              "merge scratch must fit in the slot ring");

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, int w, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Address of the 16-byte chunk `chunk` (0..7) of row `row` of a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + row * 128 + ((chunk ^ (row & 7)) << 4);
}

struct DecodeParams {
  const void* query;
  // varlen batches: sequence b's query row is query_start_loc[b], and sequences with more
  // (or fewer) than one query are skipped (a prefill kernel serves them); null: row b
  const int32_t* query_start_loc;
  const int32_t* seq_lens;
  const int32_t* block_tables;
  float* part_o;    // [B][Hkv][max_chunks][G][128]
  float* part_lse;  // [B][Hkv][max_chunks][G]
  // one chunk covers every sequence: the split kernel writes the output rows itself and
  // no partials or combine kernel are needed
  void* out;
  int64_t o_seq_stride, o_head_stride;
  int direct;
  int64_t q_seq_stride, q_head_stride;
  int64_t bt_stride;
  int64_t max_blocks_per_seq;
  int64_t num_blocks;
  int num_kv_heads;
  int group;  // q heads per kv head, 1..8
  int chunk_blocks;
  int max_chunks;
  float scale_log2;
  unsigned int* err;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) paged_decode_split_kernel(
    const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
    const DecodeParams p) {
  const int chunk = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  int64_t row = b;  // query / output row of sequence b
  if (p.query_start_loc != nullptr) {
    row = p.query_start_loc[b];
    if (p.query_start_loc[b + 1] - row != 1) return;  // uniform across the CTA
  }

  int ctx = p.seq_lens[b];
  if (ctx < 0) ctx = 0;
  int64_t total_blocks = (int64_t(ctx) + kBlockTokens - 1) / kBlockTokens;
  if (total_blocks > p.max_blocks_per_seq) total_blocks = p.max_blocks_per_seq;
  // a sequence longer than the max_seq_len the call was sized for would be cut to the
  // chunks that exist: flag it (the merge step flags the same in split mode)
  if (chunk == 0 && threadIdx.x == 0 && total_blocks > int64_t(p.max_chunks) * p.chunk_blocks)
    raise_device_error(p.err, NTB200_DEVERR_INDEX_RANGE);
  const int64_t blk_begin = int64_t(chunk) * p.chunk_blocks;
  if (blk_begin >= total_blocks) {  // uniform across the CTA
    if (p.direct) {  // an empty sequence attends to nothing: zero rows, as the combine writes
      T* ob = static_cast<T*>(p.out) + row * p.o_seq_stride;
      for (int idx = threadIdx.x; idx < p.group * kHeadDim; idx += kThreads) {
        const int hh = idx / kHeadDim;
        ob[int64_t(kvh * p.group + hh) * p.o_head_stride + (idx - hh * kHeadDim)] = Elem<T>::from_f(0.f);
      }
    }
    return;
  }
  const int nblk = static_cast<int>(
      total_blocks - blk_begin < p.chunk_blocks ? total_blocks - blk_begin : p.chunk_blocks);
  const int64_t tok_begin = blk_begin * kBlockTokens;
  const int64_t tok_end = ctx < total_blocks * kBlockTokens ? ctx : total_blocks * kBlockTokens;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SmemLayout::kFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + SmemLayout::kEmpty);
  int32_t* ids = reinterpret_cast<int32_t*>(smem + SmemLayout::kIds);
  const uint32_t slots_u32 = smem_u32(smem + SmemLayout::kSlots);

  // stage block ids (all threads), init barriers (one thread)
  const int32_t* bt_row = p.block_tables + int64_t(b) * p.bt_stride + blk_begin;
  for (int i = threadIdx.x; i < nblk; i += kThreads) {
    int32_t id = bt_row[i];
    if (id < 0 || id >= p.num_blocks) {
      raise_device_error(p.err, NTB200_DEVERR_INDEX_RANGE);
      id = -1;  // TMA fills the out-of-range box with zeros; never faults
    }
    ids[i] = id;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&k_map)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&v_map)) : "memory");
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&empty[s], ((j / kStages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&full[s], kSlotBytes);
        const uint32_t kdst = slots_u32 + s * kSlotBytes;
        const uint32_t vdst = kdst + kTileBytes;
        const uint32_t bar = smem_u32(&full[s]);
        const int id = ids[j];
        tma_load_4d(kdst, &k_map, 0, kvh, 0, id, bar);
        tma_load_4d(kdst + kHalfTileBytes, &k_map, 64, kvh, 0, id, bar);
        tma_load_4d(vdst, &v_map, 0, kvh, 0, id, bar);
        tma_load_4d(vdst + kHalfTileBytes, &v_map, 64, kvh, 0, id, bar);
        issued = j + 1;
      }
      // drain: never leave the CTA while a copy into the ring may still land
      for (int j = issued - kStages < 0 ? 0 : issued - kStages; j < issued; ++j) {
        mbar_wait(&full[j % kStages], (j / kStages) & 1, p.err);
      }
    }
    // the producer warp takes no part in the merge below
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g = lane >> 2;  // mma group id: token row (S^T) / head column (B operand)
  const int c = lane & 3;
  const int G = p.group;

  // q^T as the B operand of S^T = K q^T: b0 = q[g][16kk+2c..+1], b1 = q[g][16kk+8+2c..+1]
  uint32_t qf[8][2];
  {
    const T* qrow = static_cast<const T*>(p.query) + row * p.q_seq_stride +
                    int64_t(kvh * G + (g < G ? g : 0)) * p.q_head_stride;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      if (g < G) {
        qf[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * c);
        qf[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 8 + 2 * c);
      } else {
        qf[kk][0] = 0u;
        qf[kk][1] = 0u;
      }
    }
  }

  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY;  // running max (log2 units) of heads 2c, 2c+1
  float l0 = 0.f, l1 = 0.f;              // this thread's share of the running sums

  // ldmatrix lane geometry
  const int mi = lane >> 3, ri = lane & 7;

  for (int j = warp; j < nblk; j += kConsumerWarps) {
    const int s = j % kStages;
    if (!mbar_wait(&full[s], (j / kStages) & 1, p.err)) break;
    const uint32_t kbase = slots_u32 + s * kSlotBytes;
    const uint32_t vbase = kbase + kTileBytes;

    // ---- S^T[16 tok x 8 heads] = K[16 x 128] . q^T ----
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int dh = kk >> 2;
      const int ch = (kk & 3) * 2 + (mi >> 1);
      const int tok = ri + 8 * (mi & 1);
      uint32_t a[4];
      ldsm_x4(swz(kbase + dh * kHalfTileBytes, tok, ch), a);
      mma16816<T>(sacc, a, qf[kk][0], qf[kk][1]);
    }

    // ---- online softmax (exp2 domain) ----
    const int64_t t0 = tok_begin + int64_t(j) * kBlockTokens;
    const bool v_lo = t0 + g < tok_end;
    const bool v_hi = t0 + g + 8 < tok_end;
    float s0 = v_lo ? sacc[0] * p.scale_log2 : -INFINITY;  // tok g,   head 2c
    float s1 = v_lo ? sacc[1] * p.scale_log2 : -INFINITY;  // tok g,   head 2c+1
    float s2 = v_hi ? sacc[2] * p.scale_log2 : -INFINITY;  // tok g+8, head 2c
    float s3 = v_hi ? sacc[3] * p.scale_log2 : -INFINITY;  // tok g+8, head 2c+1
    float bm0 = fmaxf(s0, s2), bm1 = fmaxf(s1, s3);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float nm0 = fmaxf(m0, bm0), nm1 = fmaxf(m1, bm1);
    const float a0 = exp2f(m0 - nm0), a1 = exp2f(m1 - nm1);
    m0 = nm0;
    m1 = nm1;
    const float p0 = exp2f(s0 - nm0), p1 = exp2f(s1 - nm1);
    const float p2 = exp2f(s2 - nm0), p3 = exp2f(s3 - nm1);
    l0 = l0 * a0 + p0 + p2;
    l1 = l1 * a1 + p1 + p3;
    if (!__all_sync(0xffffffffu, a0 == 1.f && a1 == 1.f)) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= a0;
        o[mt][1] *= a1;
        o[mt][2] *= a0;
        o[mt][3] *= a1;
      }
    }
    // P^T as the B operand (k = token, n = head): transpose the two 8x8 halves of S^T
    const uint32_t pb0 = movmatrix_t(pack2<T>(p0, p1));
    const uint32_t pb1 = movmatrix_t(pack2<T>(p2, p3));

    // ---- O^T[128 x 8] += V^T[128 x 16] . P^T[16 x 8] ----
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int dh = mt >> 2;
      const int ch = (mt & 3) * 2 + (mi & 1);
      const int tok = ri + 8 * (mi >> 1);
      uint32_t a[4];
      ldsm_x4_t(swz(vbase + dh * kHalfTileBytes, tok, ch), a);
      mma16816<T>(o[mt], a, pb0, pb1);
    }

    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- merge the four warps' states, write the chunk partial ----
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  // all consumers are past the ring: reuse it as merge scratch
  named_barrier_sync(1, kConsumerWarps * 32);
  float* sm_o = reinterpret_cast<float*>(smem + SmemLayout::kSlots);  // [w][8][128]
  float* sm_m = sm_o + kConsumerWarps * 8 * kHeadDim;                 // [w][8]
  float* sm_l = sm_m + kConsumerWarps * 8;                            // [w][8]
  {
    float* ow = sm_o + warp * 8 * kHeadDim;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = 16 * mt + g;
      ow[(2 * c) * kHeadDim + d] = o[mt][0];
      ow[(2 * c + 1) * kHeadDim + d] = o[mt][1];
      ow[(2 * c) * kHeadDim + d + 8] = o[mt][2];
      ow[(2 * c + 1) * kHeadDim + d + 8] = o[mt][3];
    }
    if (g == 0) {
      sm_m[warp * 8 + 2 * c] = m0;
      sm_m[warp * 8 + 2 * c + 1] = m1;
      sm_l[warp * 8 + 2 * c] = l0;
      sm_l[warp * 8 + 2 * c + 1] = l1;
    }
  }
  named_barrier_sync(1, kConsumerWarps * 32);
  if (p.direct) {
    T* ob = static_cast<T*>(p.out) + row * p.o_seq_stride;
    for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kConsumerWarps * 32) {
      const int hh = idx / kHeadDim;
      const int d = idx - hh * kHeadDim;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm_m[w * 8 + hh]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = sm_m[w * 8 + hh];
        const float sc = mw == -INFINITY ? 0.f : exp2f(mw - M);
        L += sm_l[w * 8 + hh] * sc;
        O += sm_o[(w * 8 + hh) * kHeadDim + d] * sc;
      }
      ob[int64_t(kvh * G + hh) * p.o_head_stride + d] = Elem<T>::from_f(L > 0.f ? O / L : 0.f);
    }
    return;
  }
  const int64_t unit = (int64_t(b) * p.num_kv_heads + kvh) * p.max_chunks + chunk;
  float* po = p.part_o + unit * G * kHeadDim;
  float* pl = p.part_lse + unit * G;
  for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kConsumerWarps * 32) {
    const int hh = idx / kHeadDim;
    const int d = idx - hh * kHeadDim;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm_m[w * 8 + hh]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float mw = sm_m[w * 8 + hh];
      const float sc = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L += sm_l[w * 8 + hh] * sc;
      O += sm_o[(w * 8 + hh) * kHeadDim + d] * sc;
    }
    po[hh * kHeadDim + d] = L > 0.f ? O / L : 0.f;
    if (d == 0) pl[hh] = L > 0.f ? M + log2f(L) : -INFINITY;
  }
}

// One warp per (sequence, query head): merges the chunk partials with their log-sum-exp
// weights and writes the output row (4 dims per lane).
template <typename T>
__global__ void __launch_bounds__(128) paged_decode_combine_kernel(
    T* __restrict__ out, const float* __restrict__ part_o, const float* __restrict__ part_lse,
    const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ query_start_loc, int num_seqs,
    int num_q_heads, int group, int chunk_tokens, int max_chunks, int64_t max_blocks_per_seq,
    int64_t o_seq_stride, int64_t o_head_stride, unsigned int* err) {
  const int64_t wid = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (wid >= int64_t(num_seqs) * num_q_heads) return;
  const int b = static_cast<int>(wid / num_q_heads);
  const int qh = static_cast<int>(wid - int64_t(b) * num_q_heads);
  const int kvh = qh / group, hh = qh - kvh * group;
  const int num_kv = num_q_heads / group;
  int64_t row = b;
  if (query_start_loc != nullptr) {
    row = query_start_loc[b];
    if (query_start_loc[b + 1] - row != 1) return;  // not a decode row (warp-uniform)
  }
  int64_t ctx = seq_lens[b] < 0 ? 0 : seq_lens[b];
  if (ctx > max_blocks_per_seq * kBlockTokens) ctx = max_blocks_per_seq * kBlockTokens;
  int64_t nch = (ctx + chunk_tokens - 1) / chunk_tokens;
  if (nch > max_chunks) {
    if (lane == 0) raise_device_error(err, NTB200_DEVERR_INDEX_RANGE);
    nch = max_chunks;
  }
  T* orow = out + row * o_seq_stride + int64_t(qh) * o_head_stride;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (nch > 0) {
    const int64_t unit0 = (int64_t(b) * num_kv + kvh) * max_chunks;
    // lane c holds the log-sum-exp of chunks c, c+32, ...: one round trip for all of them
    float M = -INFINITY;
    for (int64_t ch = lane; ch < nch; ch += 32) M = fmaxf(M, part_lse[(unit0 + ch) * group + hh]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float wsum = 0.f;
    for (int64_t base = 0; base < nch; base += 32) {
      const int64_t mine = base + lane;
      float w_lane = 0.f;
      if (mine < nch) {
        const float lse = part_lse[(unit0 + mine) * group + hh];
        w_lane = lse == -INFINITY ? 0.f : exp2f(lse - M);
      }
      const int n = static_cast<int>(nch - base < 32 ? nch - base : 32);
      // the partial rows of this group of chunks are independent loads: issue them all
      for (int j = 0; j < n; ++j) {
        const float w = __shfl_sync(0xffffffffu, w_lane, j);
        const float4 v = *reinterpret_cast<const float4*>(
            part_o + ((unit0 + base + j) * group + hh) * kHeadDim + lane * 4);
        wsum += w;
        acc[0] += w * v.x;
        acc[1] += w * v.y;
        acc[2] += w * v.z;
        acc[3] += w * v.w;
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] *= inv;
  }
  store_f<T, 4>(orow + lane * 4, acc);
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

// 4-D view (d 128, kv head, token-in-block 16, block) of one cache; box = 64 dims x 16 tokens.
int make_cache_map(CUtensorMap* map, const void* base, int dtype, int64_t num_kv_heads,
                   int64_t num_blocks, int64_t block_stride, int64_t page_stride,
                   int64_t head_stride) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {cuuint64_t(kHeadDim), cuuint64_t(num_kv_heads),
                              cuuint64_t(kBlockTokens), cuuint64_t(num_blocks)};
  const cuuint64_t strides[3] = {cuuint64_t(head_stride * 2), cuuint64_t(page_stride * 2),
                                 cuuint64_t(block_stride * 2)};
  const cuuint32_t box[4] = {64, 1, cuuint32_t(kBlockTokens), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == NTB200_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return NTB200_OK;
}

// Tokens per split: large enough that the merge traffic stays small, small enough to give
// several CTAs per SM when the batch is small.
int choose_chunk_tokens(int64_t num_seqs, int64_t num_kv_heads, int64_t max_seq_len) {
  int chunk = 1024;
  const int64_t target_units = 4 * 148;
  while (chunk > 256 &&
         num_seqs * num_kv_heads * ceil_div(max_seq_len, chunk) < target_units) {
    chunk /= 2;
  }
  return chunk;
}

int64_t effective_max_seq_len(int64_t max_seq_len, int64_t max_blocks_per_seq,
                              int64_t block_size) {
  const int64_t cap = max_blocks_per_seq * block_size;
  if (max_seq_len <= 0 || max_seq_len > cap) return cap;
  return max_seq_len;
}

size_t workspace_bytes_for(int64_t num_seqs, int64_t num_q_heads, int64_t max_seq_len,
                           int chunk_tokens) {
  const int64_t max_chunks = ceil_div(max_seq_len, chunk_tokens);
  if (max_chunks == 1) return 0;  // the split kernel writes the output directly
  const int64_t units = num_seqs * num_q_heads * max_chunks;  // per query head
  const int64_t o_bytes = units * kHeadDim * 4;
  const int64_t l_bytes = units * 4;
  return static_cast<size_t>(((o_bytes + 255) / 256) * 256 + ((l_bytes + 255) / 256) * 256);
}

}  // namespace
}  // namespace ntb200

extern "C" size_t ntb200_paged_attention_decode_workspace_size(
    int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
    int64_t block_size, int64_t max_seq_len) {
  using namespace ntb200;
  if (num_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_seq_len <= 0 ||
      head_size != kHeadDim || block_size != kBlockTokens)
    return 0;
  const int chunk = choose_chunk_tokens(num_seqs, num_kv_heads, max_seq_len);
  return workspace_bytes_for(num_seqs, num_q_heads, max_seq_len, chunk);
}

namespace ntb200 {
namespace {

int decode_impl(void* out, const void* query, const void* key_cache, const void* value_cache,
                const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_tables,
                int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size,
                int64_t num_blocks, int64_t max_blocks_per_seq, int64_t block_table_stride, int64_t max_seq_len,
                float scale, int64_t q_seq_stride, int64_t q_head_stride, int64_t out_seq_stride,
                int64_t out_head_stride, int64_t cache_block_stride, int64_t cache_page_stride,
                int64_t cache_head_stride, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "paged_decode: dtype %d (bf16/f16 only)", dtype);
  if (head_size != kHeadDim || block_size != kBlockTokens)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "paged_decode: head_size must be 128 and block_size 16");
  if (num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "paged_decode: bad head counts");
  const int64_t group = num_q_heads / num_kv_heads;
  if (group > 8) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "paged_decode: GQA group > 8");
  if (num_seqs == 0) return NTB200_OK;
  if (num_seqs > 65535 || num_kv_heads > 65535)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "paged_decode: too many sequences/heads");
  if (!out || !query || !key_cache || !value_cache || !seq_lens || !block_tables)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "paged_decode: null pointer");
  if (num_blocks <= 0 || max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "paged_decode: bad block table geometry");
  if (!aligned16(key_cache) || !aligned16(value_cache) || cache_head_stride % 8 != 0 ||
      cache_page_stride % 8 != 0 || cache_block_stride % 8 != 0)
    return fail(NTB200_ERR_MISALIGNED, "paged_decode: cache must be 16-byte aligned with strides % 8 == 0");
  if ((reinterpret_cast<uintptr_t>(query) & 3u) != 0 || q_head_stride % 2 != 0 ||
      q_seq_stride % 2 != 0)
    return fail(NTB200_ERR_MISALIGNED, "paged_decode: query must be 4-byte aligned, even strides");
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0 || out_head_stride % 4 != 0 ||
      out_seq_stride % 4 != 0)
    return fail(NTB200_ERR_MISALIGNED, "paged_decode: out must be 8-byte aligned, strides % 4 == 0");

  const int64_t msl = effective_max_seq_len(max_seq_len, max_blocks_per_seq, block_size);
  const int chunk_tokens = choose_chunk_tokens(num_seqs, num_kv_heads, msl);
  const int64_t max_chunks = ceil_div(msl, chunk_tokens);
  const size_t need = workspace_bytes_for(num_seqs, num_q_heads, msl, chunk_tokens);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need ||
                   (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0))
    return fail(NTB200_ERR_WORKSPACE, "paged_decode: workspace needs %zu bytes (256-aligned), got %zu",
                need, workspace_bytes);
  if (max_chunks > 65535) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "paged_decode: context too long");

  CUtensorMap kmap, vmap;
  int st = make_cache_map(&kmap, key_cache, dtype, num_kv_heads, num_blocks, cache_block_stride,
                          cache_page_stride, cache_head_stride);
  if (st != NTB200_OK) return st;
  st = make_cache_map(&vmap, value_cache, dtype, num_kv_heads, num_blocks, cache_block_stride,
                      cache_page_stride, cache_head_stride);
  if (st != NTB200_OK) return st;

  DecodeParams prm;
  prm.query = query;
  prm.query_start_loc = query_start_loc;
  prm.seq_lens = seq_lens;
  prm.block_tables = block_tables;
  const int64_t units = num_seqs * num_q_heads * max_chunks;
  prm.part_o = static_cast<float*>(workspace);
  prm.part_lse = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                          ((units * kHeadDim * 4 + 255) / 256) * 256);
  prm.q_seq_stride = q_seq_stride;
  prm.q_head_stride = q_head_stride;
  prm.bt_stride = block_table_stride;
  prm.max_blocks_per_seq = max_blocks_per_seq;
  prm.num_blocks = num_blocks;
  prm.num_kv_heads = static_cast<int>(num_kv_heads);
  prm.group = static_cast<int>(group);
  prm.chunk_blocks = chunk_tokens / kBlockTokens;
  prm.max_chunks = static_cast<int>(max_chunks);
  prm.scale_log2 = scale * kLog2e;
  prm.err = device_error_word();
  prm.out = out;
  prm.o_seq_stride = out_seq_stride;
  prm.o_head_stride = out_head_stride;
  prm.direct = max_chunks == 1 ? 1 : 0;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int smem = SmemLayout::kDynamicBytes;
  dim3 grid(static_cast<unsigned>(max_chunks), static_cast<unsigned>(num_kv_heads),
            static_cast<unsigned>(num_seqs));
  if (dtype == NTB200_DTYPE_BF16) {
    st = ensure_smem_attribute(reinterpret_cast<const void*>(paged_decode_split_kernel<__nv_bfloat16>), smem, 0);
    if (st != NTB200_OK) return st;
    st = launch_kernel("paged_decode_split", paged_decode_split_kernel<__nv_bfloat16>, grid,
                       dim3(kThreads), smem, s, kmap, vmap, prm);
  } else {
    st = ensure_smem_attribute(reinterpret_cast<const void*>(paged_decode_split_kernel<__half>), smem, 1);
    if (st != NTB200_OK) return st;
    st = launch_kernel("paged_decode_split", paged_decode_split_kernel<__half>, grid,
                       dim3(kThreads), smem, s, kmap, vmap, prm);
  }
  if (st != NTB200_OK || prm.direct) return st;

  const int64_t warps = num_seqs * num_q_heads;
  const dim3 cgrid(static_cast<unsigned>(ceil_div(warps, 4)));
  if (dtype == NTB200_DTYPE_BF16)
    return launch_kernel("paged_decode_combine", paged_decode_combine_kernel<__nv_bfloat16>, cgrid,
                         dim3(128), 0, s, static_cast<__nv_bfloat16*>(out), prm.part_o,
                         prm.part_lse, seq_lens, query_start_loc, int(num_seqs), int(num_q_heads),
                         int(group), chunk_tokens, int(max_chunks), max_blocks_per_seq, out_seq_stride,
                         out_head_stride, prm.err);
  return launch_kernel("paged_decode_combine", paged_decode_combine_kernel<__half>, cgrid,
                       dim3(128), 0, s, static_cast<__half*>(out), prm.part_o, prm.part_lse,
                       seq_lens, query_start_loc, int(num_seqs), int(num_q_heads), int(group),
                       chunk_tokens, int(max_chunks), max_blocks_per_seq, out_seq_stride,
                       out_head_stride, prm.err);
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_paged_attention_decode(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks_per_seq, int64_t block_table_stride,
    int64_t max_seq_len, float scale, int64_t q_seq_stride, int64_t q_head_stride,
    int64_t out_seq_stride, int64_t out_head_stride, int64_t cache_block_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, void* workspace,
    size_t workspace_bytes, int dtype, void* stream) {
  return ntb200::decode_impl(out, query, key_cache, value_cache, nullptr, seq_lens, block_tables, num_seqs,
                             num_q_heads, num_kv_heads, head_size, block_size, num_blocks, max_blocks_per_seq,
                             block_table_stride, max_seq_len, scale, q_seq_stride, q_head_stride, out_seq_stride,
                             out_head_stride, cache_block_stride, cache_page_stride, cache_head_stride, workspace,
                             workspace_bytes, dtype, stream);
}

extern "C" int ntb200_paged_attention_decode_varlen(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size, int64_t num_blocks,
    int64_t max_blocks_per_seq, int64_t block_table_stride, int64_t max_seq_len, float scale,
    int64_t q_token_stride, int64_t q_head_stride, int64_t out_token_stride, int64_t out_head_stride,
    int64_t cache_block_stride, int64_t cache_page_stride, int64_t cache_head_stride, void* workspace,
    size_t workspace_bytes, int dtype, void* stream) {
  if (query_start_loc == nullptr)
    return ntb200::fail(NTB200_ERR_INVALID_ARGUMENT, "paged_decode_varlen: query_start_loc is null");
  return ntb200::decode_impl(out, query, key_cache, value_cache, query_start_loc, seq_lens, block_tables, num_seqs,
                             num_q_heads, num_kv_heads, head_size, block_size, num_blocks, max_blocks_per_seq,
                             block_table_stride, max_seq_len, scale, q_token_stride, q_head_stride,
                             out_token_stride, out_head_stride, cache_block_stride, cache_page_stride,
                             cache_head_stride, workspace, workspace_bytes, dtype, stream);
}

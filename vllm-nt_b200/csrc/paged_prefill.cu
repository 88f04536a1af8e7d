// Varlen paged prefill attention on the 5th-generation tensor cores: a flash-attention
// forward that reads K/V straight from vLLM's paged cache.
//   out[t, h] = softmax(scale * q[t, h] . K_b^T + mask) . V_b
// for every query token t of sequence b, K_b / V_b = the seq_lens[b] tokens cached for b
// (pages of 16 tokens found through block_table), K/V head h / (Hq / Hkv).  With causal
// masking the queries are aligned to the END of the context: query i of a sequence with
// q_len queries and ctx cached tokens sits at position ctx - q_len + i and sees keys
// 0 .. that position (vLLM's rule, which also covers a cached prefix and chunked prefill).
//
// Persistent: one CTA per SM walks the work items -- (128-query tile, q head) pairs of all
// sequences, a sequence's last tile first -- found from a prefix sum of the query tiles
// per sequence that every CTA builds in shared memory.  704 threads:
//   warp 0     TMA: the Q tile (two 64-column halves, 128-byte swizzle; double-buffered
//              across items) and half of each K tile's pages; three more producer warps
//              (warps 18-20, after the softmax warps) issue the other half of K's and V's
//              pages, so four threads issue copies at once (the issue rate of small copies
//              limits).  Per tile the 8 K pages and the 8 V pages (16 tokens x 64 columns
//              per copy) into 2-stage rings; page ids come from the block table (ids out of
//              range are reported and read as zeros: the copy lands outside the tensor map).
//   warp 1     TMEM (two S buffers and O: 384 of 512 columns); lane 0 issues
//              S_j = Q K_j^T (M = N = 128, eight K = 16 steps; both operands K-major) as
//              far ahead as the two S buffers allow: S_{j+2} reuses a buffer once
//              O += P_j V_j has read P_j.
//   warp 21    lane 0 issues O += P_j V_j (A = P_j in TMEM, written over S_j; B = V as
//              cached, MN-major) once the softmax has released P_j.  Two issuing threads
//              keep the tensor pipe about twice as busy as one.
//   warps 2-17 softmax, four threads per query row (warp w owns TMEM lanes 32*(w%4)..+31
//              and 32 of the 128 key columns; the four parts of a row meet at an mbarrier
//              to combine their maxima and sums): the S row from TMEM, scale and mask, the
//              running max and sum in fp32 in the exp2 domain, P = exp2(s - m) rounded to
//              the input type and stored back into TMEM over the S columns (packed in
//              pairs).  The running max is refreshed lazily:
//              only when a row's max grows by more than 2^8 is O (in TMEM) rescaled, so
//              P <= 256 and O / l is the same either way.  Epilogue: O / l, rounded, stored.
//
// Every mbarrier wait is bounded (2 s); a timeout sets NTB200_DEVERR_WAIT_TIMEOUT, the
// roles leave their loops, copies and MMAs in flight are drained, and TMEM is freed.
//
// Replaces vllm_nt/_ntops/kernels/attention.py:10-94 (_VarLen, reached from
// vllm_nt/_ntops/patching.py:639-671), which first copies every sequence's K/V out of the
// cache (vllm_nt/_ntops/torch/kv_cache.py:24-63) and masks from the upper left
// (attention.py:61-63); here no copy is made and the mask follows vLLM.
#include "common.cuh"
#include "tcgen05.cuh"

namespace ntb200 {
namespace {

constexpr int kD = 128;                       // head size
constexpr int kBQ = 128;                      // query rows per CTA
constexpr int kBKV = 128;                     // keys per tile
constexpr int kPage = 16;                     // tokens per cache block
constexpr int kPagesPerTile = kBKV / kPage;   // 8
constexpr int kSoftmaxThreads = 512;           // warps 2-17: four per query row
// Copy issue: four threads (warp 0 and the three warps after the softmax warps), each
// issuing half of a tile's pages of K or of V (and warp 0 also the Q tiles).
constexpr int kParts = 2;                           // issuing threads per operand
constexpr int kExtraWarp = 2 + kSoftmaxThreads / 32;  // first producer warp after the softmax warps
// The MMAs are issued by two threads: warp 1 issues S = Q K^T, this warp O += P V.  A thread
// issues one tcgen05.mma at a time, and one issuer for both products kept the tensor pipe
// about a third busy.
constexpr int kPvWarp = kExtraWarp + 2 * kParts - 1;
constexpr int kThreads = 64 + kSoftmaxThreads + 32 * (2 * kParts - 1) + 32;
constexpr int kRowParts = kSoftmaxThreads / kBQ;  // threads (warps per lane quadrant) per query row
constexpr int kPartCols = kBKV / kRowParts;        // S / O columns a softmax thread owns
static_assert(kPartCols == 32, "a softmax thread moves its columns with one 32-column TMEM access");
constexpr int kHalf = 128 * 64 * 2;           // 128 rows x 64 columns: 16 KB
constexpr int kTile = 2 * kHalf;              // 128 x 128: 32 KB
constexpr int kPageBytes = kPage * 128;       // one page of one half: 16 rows x 128 B
constexpr int kStages = 2;
constexpr float kRescaleLog2 = 8.0f;          // refresh a row's max when it grows by > 2^8
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;              // S buffers at columns 0 and 128, O at 256

struct Smem {
  static constexpr int kQ = 0;                    // two Q tiles: the next item's loads early
  static constexpr int kK = kQ + 2 * kTile;
  static constexpr int kV = kK + kStages * kTile;
  static constexpr int kQFull = kV + kStages * kTile;
  static constexpr int kQEmpty = kQFull + 16;
  static constexpr int kKFull = kQEmpty + 16;
  static constexpr int kKEmpty = kKFull + 8 * kStages;
  static constexpr int kVFull = kKEmpty + 8 * kStages;
  static constexpr int kVEmpty = kVFull + 8 * kStages;
  static constexpr int kSFull = kVEmpty + 8 * kStages;
  static constexpr int kPFull = kSFull + 16;
  static constexpr int kPEmpty = kPFull + 16;
  static constexpr int kPvDone = kPEmpty + 8;     // [2]: O += P V done, per S buffer
  static constexpr int kOFree = kPvDone + 16;
  static constexpr int kMmaDone = kOFree + 8;
  static constexpr int kPair = kMmaDone + 8;       // 4 mbarriers: the two warps of each row quadrant
  static constexpr int kRed = kPair + 32;          // [2][kRowParts][128] floats: row-max / row-sum exchange
  static constexpr int kTmemBase = kRed + 2 * kRowParts * 128 * 4;
  static constexpr int kPrefix = kTmemBase + 16;   // [num_seqs + 1] ints: the work list
  static constexpr int kMaxBytes = 227 * 1024;
  static constexpr int bytes_for(int64_t num_seqs) { return kPrefix + int(num_seqs + 1) * 4 + 1024; }
  static constexpr int64_t kMaxSeqs = (kMaxBytes - kPrefix - 1024) / 4 - 1;
};
static_assert(Smem::bytes_for(1024) <= Smem::kMaxBytes, "shared memory");

struct PrefillParams {
  void* out;
  const int32_t* query_start_loc;  // [num_seqs + 1]
  const int32_t* seq_lens;         // [num_seqs] (paged K/V)
  const int32_t* block_table;      // [num_seqs, bt_stride] (paged K/V)
  const int32_t* key_start_loc;    // [num_seqs + 1] (contiguous K/V)
  int num_keys;                    // rows of the contiguous K/V
  int64_t bt_stride;
  int64_t o_tok_stride, o_head_stride;
  int num_tokens;
  int max_blocks;
  int num_blocks;
  int num_seqs;
  int num_q_heads;
  int skip_single_query;  // sequences with one query token are left to the decode kernel
  int group;             // q heads per kv head
  int causal;
  int heads_outer;       // cache memory order [block, head, token, d] (else [block, token, head, d])
  float scale_log2;      // softmax scale * log2(e)
  unsigned int* err;
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
      : "memory");
}

// D (TMEM) (+)= A (TMEM, M rows on the lanes, K packed two per 32-bit column) . B (smem)
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// the hardware base-2 exponential (ex2.approx; exp2(-inf) = +0)
__device__ __forceinline__ float hw_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// One work item = (128-query tile, q head) of a sequence; the CTA's roles walk the same
// items in the same order and derive the same parameters from the metadata.
struct Item {
  int b, qh, kvh, q0, rows, q_begin, ctx, k_begin, shift, n_tiles;
};

// the largest b in [0, n) with prefix[b] <= t
__device__ __forceinline__ int find_sequence(const int* prefix, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <bool PAGED>
__device__ __forceinline__ Item make_item(const PrefillParams& p, const int* prefix, int w) {
  Item it;
  const int tl = w / p.num_q_heads;
  it.qh = w - tl * p.num_q_heads;
  it.kvh = it.qh / p.group;
  it.b = find_sequence(prefix, p.num_seqs, tl);
  const int t = tl - prefix[it.b];
  const int ntq = prefix[it.b + 1] - prefix[it.b];
  const int qt = ntq - 1 - t;  // a sequence's last (longest, when causal) tile first
  it.q_begin = p.query_start_loc[it.b];
  const int q_len = p.query_start_loc[it.b + 1] - it.q_begin;
  it.q0 = qt * kBQ;
  it.rows = q_len - it.q0 < kBQ ? q_len - it.q0 : kBQ;
  it.k_begin = 0;
  if constexpr (PAGED) {
    it.ctx = p.seq_lens[it.b] < 0 ? 0 : p.seq_lens[it.b];
    if (it.ctx > p.max_blocks * kPage) {
      raise_device_error(p.err, NTB200_DEVERR_INDEX_RANGE);
      it.ctx = p.max_blocks * kPage;
    }
  } else {
    it.k_begin = p.key_start_loc[it.b];
    it.ctx = p.key_start_loc[it.b + 1] - it.k_begin;  // validated by the scan
  }
  it.shift = it.ctx - q_len;  // position of the sequence's first query
  int kv_end = p.causal ? it.shift + it.q0 + it.rows : it.ctx;  // keys [0, kv_end) are visible to some row
  if (kv_end > it.ctx) kv_end = it.ctx;
  it.n_tiles = kv_end > 0 ? (kv_end + kBKV - 1) / kBKV : 0;
  return it;
}

// query tiles of sequence b (0 for a sequence skipped or with inconsistent metadata)
template <bool PAGED>
__device__ __forceinline__ int query_tiles(const PrefillParams& p, int b) {
  const int qb = p.query_start_loc[b];
  const int ql = p.query_start_loc[b + 1] - qb;
  if (qb < 0 || ql < 0 || qb + ql > p.num_tokens) {
    raise_device_error(p.err, NTB200_DEVERR_INDEX_RANGE);
    return 0;
  }
  if constexpr (!PAGED) {
    const int kb = p.key_start_loc[b];
    const int kl = p.key_start_loc[b + 1] - kb;
    if (kb < 0 || kl < 0 || kb + kl > p.num_keys) {
      raise_device_error(p.err, NTB200_DEVERR_INDEX_RANGE);
      return 0;
    }
  }
  if (p.skip_single_query && ql == 1) return 0;
  return (ql + kBQ - 1) / kBQ;
}

// PAGED: K/V pages of the cache through the block table; else contiguous [keys, kv_heads,
// 128] K/V, sequence b's keys at rows key_start_loc[b] .. key_start_loc[b + 1].
// Persistent: CTA i takes work items i, i + gridDim.x, ...; the K/V ring, the S buffers,
// P and O carry on from one item to the next (phases counted over the CTA's whole run).
template <typename T, bool PAGED>
__global__ void __launch_bounds__(kThreads, 1) paged_prefill_kernel(
    const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
    const __grid_constant__ CUtensorMap v_map, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int warp_sums[kThreads / 32];
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + Smem::kQFull);
  uint64_t* q_empty = reinterpret_cast<uint64_t*>(smem + Smem::kQEmpty);
  uint64_t* k_full = reinterpret_cast<uint64_t*>(smem + Smem::kKFull);
  uint64_t* k_empty = reinterpret_cast<uint64_t*>(smem + Smem::kKEmpty);
  uint64_t* v_full = reinterpret_cast<uint64_t*>(smem + Smem::kVFull);
  uint64_t* v_empty = reinterpret_cast<uint64_t*>(smem + Smem::kVEmpty);
  uint64_t* s_full = reinterpret_cast<uint64_t*>(smem + Smem::kSFull);
  uint64_t* p_full = reinterpret_cast<uint64_t*>(smem + Smem::kPFull);
  uint64_t* p_empty = reinterpret_cast<uint64_t*>(smem + Smem::kPEmpty);
  uint64_t* pv_done = reinterpret_cast<uint64_t*>(smem + Smem::kPvDone);
  uint64_t* o_free = reinterpret_cast<uint64_t*>(smem + Smem::kOFree);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(smem + Smem::kMmaDone);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Smem::kTmemBase);
  int* prefix = reinterpret_cast<int*>(smem + Smem::kPrefix);  // [num_seqs + 1] query tiles
  const uint32_t sm = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();  // queries, cache and metadata come from the kernels before

  // ---- work list: prefix sums of the query tiles per sequence (block scan) ----
  int carry = 0;
  if (threadIdx.x == 0) prefix[0] = 0;
  for (int base = 0; base < p.num_seqs; base += kThreads) {
    const int bb = base + threadIdx.x;
    const int c = bb < p.num_seqs ? query_tiles<PAGED>(p, bb) : 0;
    int v = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      before += w < warp ? warp_sums[w] : 0;
      total += warp_sums[w];
    }
    if (bb < p.num_seqs) prefix[bb + 1] = carry + before + v;
    carry += total;
    __syncthreads();
  }
  const int num_items = carry * p.num_q_heads;
  if (static_cast<int>(blockIdx.x) >= num_items) return;
  T* out = static_cast<T*>(p.out);

  if (threadIdx.x == 0) {
    for (int a = 0; a < 2; ++a) {
      mbar_init(&q_full[a], 1);
      mbar_init(&q_empty[a], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], kParts);  // one arrive (with its bytes) per issuing thread
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], kParts);
      mbar_init(&v_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&s_full[a], 1);
      mbar_init(&p_full[a], kSoftmaxThreads / 32);  // one arrive per softmax warp
      mbar_init(&pv_done[a], 1);
    }
    mbar_init(p_empty, 1);
    mbar_init(o_free, kSoftmaxThreads / 32);
    mbar_init(mma_done, 2);  // a commit from each issuer
    for (int q = 0; q < 4; ++q) mbar_init(reinterpret_cast<uint64_t*>(smem + Smem::kPair) + q, 32 * kRowParts);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || (warp >= kExtraWarp && warp < kPvWarp)) {
    // ------------------------------ TMA producers ------------------------------
    // role 0 (warp 0): Q and the first half of K's pages; role 1: the rest of K; roles 2
    // and 3: V.  Contiguous K/V: each role copies one 64-column half of its operand.
    const int role = warp == 0 ? 0 : warp - kExtraWarp + 1;
    const bool v_role = role >= kParts;
    const int part = role % kParts;
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(v_role ? &v_map : &q_map)) : "memory");
      if (!v_role) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&k_map)) : "memory");
      uint32_t g = 0, nq = 0;    // K/V tiles and Q tiles loaded so far
      uint32_t k_done = 0, v_done = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        const Item it = make_item<PAGED>(p, prefix, w);
        if (it.n_tiles == 0) continue;
        if (role == 0) {
          // the S products of the item two back have read this Q buffer
          const int qb = nq & 1;
          if (nq >= 2 && !mbar_wait(&q_empty[qb], ((nq / 2) - 1) & 1, p.err)) break;
          mbar_arrive_expect_tx(&q_full[qb], kTile);
          tma_load_3d(sm + Smem::kQ + qb * kTile, &q_map, 0, it.qh, it.q_begin + it.q0, smem_u32(&q_full[qb]));
          tma_load_3d(sm + Smem::kQ + qb * kTile + kHalf, &q_map, 64, it.qh, it.q_begin + it.q0,
                      smem_u32(&q_full[qb]));
          ++nq;
        }
        const int32_t* bt = p.block_table + int64_t(it.b) * p.bt_stride;
        const int n_pages = (it.ctx + kPage - 1) / kPage;
        const int hy = p.heads_outer ? 0 : it.kvh, hz = p.heads_outer ? it.kvh : 0;
        // page ids of tile j (-1: past the context, read as zeros and masked anyway); the
        // next tile's are fetched while this tile's copies are issued, so the block-table
        // round trip is off the copy path
        auto fetch_ids = [&](int j, int32_t (&ids)[kPagesPerTile]) {
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) {
            const int lb = j * kPagesPerTile + pg;
            ids[pg] = PAGED && lb < n_pages ? __ldg(bt + lb) : -1;
          }
        };
        int32_t next_ids[kPagesPerTile];
        fetch_ids(0, next_ids);
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
          const int s = g & 1;
          int32_t ids[kPagesPerTile];
#pragma unroll
          for (int pg = 0; pg < kPagesPerTile; ++pg) {
            ids[pg] = next_ids[pg];
            if (ids[pg] >= p.num_blocks || ids[pg] < -1 ||
                (ids[pg] == -1 && PAGED && j * kPagesPerTile + pg < n_pages)) {
              raise_device_error(p.err, NTB200_DEVERR_INDEX_RANGE);
              ids[pg] = -1;
            }
          }
          if (j + 1 < it.n_tiles) fetch_ids(j + 1, next_ids);
          if (v_role) {
            if (g >= kStages && !mbar_wait(&v_empty[s], ((g / kStages) - 1) & 1, p.err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&v_full[s], kTile / kParts);
            const uint32_t vdst = sm + Smem::kV + s * kTile;
            if constexpr (PAGED) {
#pragma unroll
              for (int pg = part * (kPagesPerTile / kParts); pg < (part + 1) * (kPagesPerTile / kParts); ++pg) {
                tma_load_4d(vdst + pg * kPageBytes, &v_map, 0, hy, hz, ids[pg], smem_u32(&v_full[s]));
                tma_load_4d(vdst + kHalf + pg * kPageBytes, &v_map, 64, hy, hz, ids[pg], smem_u32(&v_full[s]));
              }
            } else {
              tma_load_3d(vdst + part * kHalf, &v_map, part * 64, it.kvh, it.k_begin + j * kBKV, smem_u32(&v_full[s]));
            }
            v_done = g + 1;
            continue;
          }
          if (g >= kStages && !mbar_wait(&k_empty[s], ((g / kStages) - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[s], kTile / kParts);
          const uint32_t kdst = sm + Smem::kK + s * kTile;
          if constexpr (PAGED) {
#pragma unroll
            for (int pg = part * (kPagesPerTile / kParts); pg < (part + 1) * (kPagesPerTile / kParts); ++pg) {
              tma_load_4d(kdst + pg * kPageBytes, &k_map, 0, hy, hz, ids[pg], smem_u32(&k_full[s]));
              tma_load_4d(kdst + kHalf + pg * kPageBytes, &k_map, 64, hy, hz, ids[pg], smem_u32(&k_full[s]));
            }
          } else {
            tma_load_3d(kdst + part * kHalf, &k_map, part * 64, it.kvh, it.k_begin + j * kBKV, smem_u32(&k_full[s]));
          }
          k_done = g + 1;
        }
      }
      // drain the copies that may still be in flight
      for (uint32_t j = nq > 2 ? nq - 2 : 0; j < nq; ++j) mbar_wait(&q_full[j & 1], (j / 2) & 1, p.err);
      for (uint32_t j = k_done > kStages ? k_done - kStages : 0; j < k_done; ++j)
        mbar_wait(&k_full[j & 1], (j / kStages) & 1, p.err);
      for (uint32_t j = v_done > kStages ? v_done - kStages : 0; j < v_done; ++j)
        mbar_wait(&v_full[j & 1], (j / kStages) & 1, p.err);
    }
  } else if (warp == 1) {
    // -------------------------- MMA issuer: S = Q K^T --------------------------
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t idesc_s = make_idesc(kBf16, kBQ, kBKV);
      uint32_t g = 0, nq = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        const Item it = make_item<PAGED>(p, prefix, w);
        if (it.n_tiles == 0) continue;
        const int qb = nq & 1;
        if (!mbar_wait(&q_full[qb], (nq / 2) & 1, p.err)) break;
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
          // S_g = Q K_g^T into S[g & 1]; the buffer holds P_{g-2} until O += P_{g-2} V_{g-2}
          // has read it (pv_done[s] completes once per product on this buffer)
          const int s = g & 1;
          if (!mbar_wait(&k_full[s], (g / kStages) & 1, p.err) ||
              (g >= 2 && !mbar_wait(&pv_done[s], ((g / 2) - 1) & 1, p.err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kb = sm + Smem::kK + s * kTile;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const uint64_t adesc = sw128_kmajor_desc(sm + Smem::kQ + qb * kTile + hf * kHalf);
            const uint64_t bdesc = sw128_kmajor_desc(kb + hf * kHalf);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(tmem + s * kBKV, adesc + 2 * k, bdesc + 2 * k, idesc_s, (hf | k) ? 1u : 0u);
          }
          umma_commit(&k_empty[s]);
          umma_commit(&s_full[s]);
          if (j + 1 == it.n_tiles) umma_commit(&q_empty[qb]);  // the item's last S product is issued
        }
        ++nq;
      }
      // every issued MMA completes before TMEM may be released
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.err);
    }
  } else if (warp == kPvWarp) {
    // -------------------------- MMA issuer: O += P V --------------------------
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t idesc_o = make_idesc(kBf16, kBQ, kD) | (1u << 16);  // B (V) MN-major
      uint32_t g = 0, nq = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        const Item it = make_item<PAGED>(p, prefix, w);
        if (it.n_tiles == 0) continue;
        for (int j = 0; j < it.n_tiles; ++j, ++g) {
          const int s = g & 1;
          if (!mbar_wait(&p_full[s], (g / 2) & 1, p.err) || !mbar_wait(&v_full[s], (g / kStages) & 1, p.err)) {
            ok = false;
            break;
          }
          // O is overwritten by the item's first product only after the previous item's
          // epilogue has read it
          if (j == 0 && nq >= 1 && !mbar_wait(o_free, (nq - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vb = sm + Smem::kV + s * kTile;
#pragma unroll
          for (int kk = 0; kk < kBKV / 16; ++kk) {
            // A: P_g in TMEM over S[s], keys [16 kk, +16) = 8 packed columns (keys 0-63 at
            // columns 0-31, keys 64-127 at 64-95); B: V rows [16 kk, +16) (2 KB apart),
            // both 64-column halves of the head dimension
            const uint32_t a_tmem = tmem + s * kBKV + (kk >> 2) * 64 + (kk & 3) * 8;
            const uint64_t bdesc = sw128_mnmajor_desc(vb + kk * 2048, kHalf);
            umma_f16_tmem_a(tmem + kTmemO, a_tmem, bdesc, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&v_empty[s]);
          umma_commit(&pv_done[s]);
          umma_commit(p_empty);
        }
        ++nq;
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.err);
    }
  } else {
    // ------------------------------ softmax + epilogue ------------------------------
    // kRowParts warps per query row: warp w (2..17) reads TMEM lanes 32*(w%4)..+31 and owns
    // key columns [kPartCols*part, +kPartCols) of S, the same columns of O, and the
    // matching part of P.  The row max and sum are exchanged through shared memory at a
    // per-quadrant mbarrier.
    const int quad = warp & 3;
    const int part = (warp - 2) >> 2;
    const int col0 = part * kPartCols;
    const int r = quad * 32 + lane;  // query row within the tile (= TMEM lane)
    const uint32_t lanes = uint32_t(quad * 32) << 16;
    // P of keys [col0, +kPartCols), two per 32-bit column: keys 0-63 are packed into
    // columns 0-31 and keys 64-127 into columns 64-95 of the S buffer
    const int pcol = (col0 >> 6) * 64 + (col0 & 63) / 2;
    float* red = reinterpret_cast<float*>(smem + Smem::kRed);  // [2 buffers][kRowParts][128 rows]
    uint64_t* pair = reinterpret_cast<uint64_t*>(smem + Smem::kPair) + quad;
    uint32_t pair_uses = 0;
    // publish one float per row and read the row's kRowParts values (in part order);
    // false if a partner never came
    // (the tensor-memory fences order this part's S reads before another part's P writes
    // over the same columns)
    auto exchange = [&](float mine, float (&all)[kRowParts]) -> bool {
      float* buf = red + (pair_uses & 1) * (kRowParts * 128);
      buf[part * 128 + r] = mine;
      tc_fence_before();
      mbar_arrive(pair);
      const bool got = mbar_wait(pair, pair_uses & 1, p.err);
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < kRowParts; ++q) all[q] = buf[q * 128 + r];
      ++pair_uses;
      return got;
    };
    uint32_t g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
      const Item it = make_item<PAGED>(p, prefix, w);
      const int qi = it.q0 + r;
      T* orow = out + int64_t(it.q_begin + qi) * p.o_tok_stride + int64_t(it.qh) * p.o_head_stride + col0;
      if (it.n_tiles == 0) {
        // no visible key (empty context): zero rows, as for an empty softmax
        if (r < it.rows)
#pragma unroll
          for (int c = 0; c < kPartCols / 8; ++c) reinterpret_cast<uint4*>(orow)[c] = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      int limit = p.causal ? it.shift + qi + 1 : it.ctx;  // this row sees keys [0, limit)
      if (limit > it.ctx) limit = it.ctx;
      float m_run = -INFINITY;  // running max of scale*s*log2(e), the same in every part of a row
      float l_run = 0.f;        // this part's share of the running sum
      for (int j = 0; j < it.n_tiles; ++j, ++g) {
        const int s = g & 1;
        if (!mbar_wait(&s_full[s], (g / 2) & 1, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float x[kPartCols];
        {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32(tmem + lanes + s * kBKV + col0, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(v[i]);
        }
        const int nvalid = limit - j * kBKV - col0;  // columns col0 + i are visible iff i < nvalid
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
        if (nvalid >= kPartCols) {
#pragma unroll
          for (int i = 0; i < kPartCols; ++i) {
            x[i] *= p.scale_log2;
            m4[i & 3] = fmaxf(m4[i & 3], x[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < kPartCols; ++i) {
            x[i] = i < nvalid ? x[i] * p.scale_log2 : -INFINITY;
            m4[i & 3] = fmaxf(m4[i & 3], x[i]);
          }
        }
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        {
          float all[kRowParts];
          if (!exchange(mx, all)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int q = 0; q < kRowParts; ++q) mx = fmaxf(mx, all[q]);
        }
        // lazy max refresh, identical in every part of a row (same rows, same combined max);
        // warp-uniform, since O is rescaled with warp-wide TMEM accesses
        const float m_new = fmaxf(m_run, mx);
        const bool grow = m_new > m_run + kRescaleLog2;  // also true for the first finite max
        float alpha = 1.f;
        const bool any = __any_sync(0xffffffffu, grow);
        if (any) {
          alpha = m_run == -INFINITY ? 0.f : hw_exp2(m_run - m_new);
          if (m_new != -INFINITY) {
            l_run *= alpha;
            m_run = m_new;
          } else {
            alpha = 1.f;
          }
        }
        const float m_use = m_run == -INFINITY ? 0.f : m_run;
        uint32_t pk[kPartCols / 2];
        float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < kPartCols / 2; ++i) {
          const float p0 = hw_exp2(x[2 * i] - m_use);
          const float p1 = hw_exp2(x[2 * i + 1] - m_use);
          l4[i & 3] += p0 + p1;
          pk[i] = pack2<T>(p0, p1);
        }
        l_run += (l4[0] + l4[1]) + (l4[2] + l4[3]);

        // O is rescaled only once O += P_{g-1} V_{g-1} is complete (and before P_g is
        // released, so the next product sees the new scale)
        if (j > 0 && any) {
          if (!mbar_wait(p_empty, (g - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32(tmem + lanes + kTmemO + col0, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st_32(tmem + lanes + kTmemO + col0, v);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        if (it.ctx > j * kBKV && it.ctx < (j + 1) * kBKV && (!PAGED || (it.ctx & (kPage - 1)) != 0)) {
          // V rows past the context that were copied in hold whatever memory held there
          // (the rest of the last page, or the rows after the sequence): zero them, so
          // that P = 0 never meets a non-finite value.  (Pages wholly past the context
          // read as zeros.)
          if (!mbar_wait(&v_full[s], (g / kStages) & 1, p.err)) {
            ok = false;
            break;
          }
          const int t0 = it.ctx - j * kBKV;
          const int t1 = PAGED ? ((it.ctx + kPage - 1) / kPage) * kPage - j * kBKV : kBKV;  // <= kBKV
          uint8_t* vb = smem + Smem::kV + s * kTile;
          for (int i = threadIdx.x - 64; i < (t1 - t0) * 16; i += kSoftmaxThreads) {
            const int row = t0 + (i >> 4), hf = (i >> 3) & 1, c = i & 7;
            *reinterpret_cast<uint4*>(vb + hf * kHalf + row * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core
        }
        // P_g (this part's keys, packed in pairs); every part of the row has read its S
        // columns before the exchange above, so the packed columns may overwrite them
        __syncwarp();
        tmem_st_16(tmem + lanes + s * kBKV + pcol, pk);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
      }
      if (!ok) break;
      // the item's last product is complete: O is final
      ok = mbar_wait(p_empty, (g - 1) & 1, p.err);
      float l = 0.f;
      if (ok) {
        float all[kRowParts];
        ok = exchange(l_run, all);
#pragma unroll
        for (int q = 0; q < kRowParts; ++q) l += all[q];
      }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint32_t o[32];
      __syncwarp();
      tmem_ld_32(tmem + lanes + kTmemO + col0, o);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);  // the next item may overwrite O
      if (ok && r < it.rows) {
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          uint4 w4;
          w4.x = pack2<T>(__uint_as_float(o[g8 * 8 + 0]) * inv, __uint_as_float(o[g8 * 8 + 1]) * inv);
          w4.y = pack2<T>(__uint_as_float(o[g8 * 8 + 2]) * inv, __uint_as_float(o[g8 * 8 + 3]) * inv);
          w4.z = pack2<T>(__uint_as_float(o[g8 * 8 + 4]) * inv, __uint_as_float(o[g8 * 8 + 5]) * inv);
          w4.w = pack2<T>(__uint_as_float(o[g8 * 8 + 6]) * inv, __uint_as_float(o[g8 * 8 + 7]) * inv);
          reinterpret_cast<uint4*>(orow)[g8] = w4;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// [tokens, heads, 128] queries: box = 128 tokens x one head x 64 columns
int make_query_map(CUtensorMap* map, const void* base, bool bf16, int64_t tokens, int64_t heads,
                   int64_t tok_stride, int64_t head_stride) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {cuuint64_t(kD), cuuint64_t(heads), cuuint64_t(tokens)};
  const cuuint64_t strides[2] = {cuuint64_t(head_stride * 2), cuuint64_t(tok_stride * 2)};
  const cuuint32_t box[3] = {64, 1, cuuint32_t(kBQ)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled (prefill q) failed (%d)", int(r));
  return NTB200_OK;
}

// one of K/V of the paged cache: box = one 16-token page of one head x 64 columns, with the
// head and token dimensions ordered as they are in memory
int make_cache_map(CUtensorMap* map, const void* base, bool bf16, int64_t blocks, int64_t heads,
                   int64_t block_stride, int64_t page_stride, int64_t head_stride) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const bool heads_outer = head_stride > page_stride;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4];
  dims[0] = kD;
  box[0] = 64;
  if (heads_outer) {
    dims[1] = kPage, strides[0] = cuuint64_t(page_stride * 2), box[1] = kPage;
    dims[2] = cuuint64_t(heads), strides[1] = cuuint64_t(head_stride * 2), box[2] = 1;
  } else {
    dims[1] = cuuint64_t(heads), strides[0] = cuuint64_t(head_stride * 2), box[1] = 1;
    dims[2] = kPage, strides[1] = cuuint64_t(page_stride * 2), box[2] = kPage;
  }
  dims[3] = cuuint64_t(blocks), strides[2] = cuuint64_t(block_stride * 2), box[3] = 1;
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NTB200_ERR_CUDA, "cuTensorMapEncodeTiled (prefill cache) failed (%d)", int(r));
  return NTB200_OK;
}

// Persistent grid: at most one CTA per SM, and no more CTAs than the work items can be
// (sum over sequences of ceil(q_len / 128), times the q heads, bounded from the host's view).
template <typename T, bool PAGED>
int launch_prefill(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const PrefillParams& prm,
                   int64_t max_query_len, cudaStream_t s, int slot) {
  const void* fn = reinterpret_cast<const void*>(paged_prefill_kernel<T, PAGED>);
  const int bytes = Smem::bytes_for(prm.num_seqs);
  int st = ensure_smem_attribute(fn, bytes, slot);
  if (st != NTB200_OK) return st;
  const int64_t by_len = ceil_div(max_query_len, kBQ) * prm.num_seqs;
  const int64_t by_tokens = ceil_div(int64_t(prm.num_tokens), kBQ) + prm.num_seqs;
  const int64_t items = (by_len < by_tokens ? by_len : by_tokens) * prm.num_q_heads;
  const int64_t grid = items < num_sms() ? items : num_sms();
  return launch_kernel(PAGED ? "paged_attention_prefill" : "flash_attn_varlen", paged_prefill_kernel<T, PAGED>,
                       dim3(static_cast<unsigned>(grid)), dim3(kThreads), bytes, s, qm, km, vm, prm);
}

PrefillParams base_params(void* out, const int32_t* query_start_loc, int64_t num_tokens, int64_t num_q_heads,
                          int64_t num_kv_heads, float scale, int causal, int64_t out_token_stride,
                          int64_t out_head_stride) {
  PrefillParams prm = {};
  prm.out = out;
  prm.query_start_loc = query_start_loc;
  prm.o_tok_stride = out_token_stride;
  prm.o_head_stride = out_head_stride;
  prm.num_tokens = static_cast<int>(num_tokens);
  prm.num_q_heads = static_cast<int>(num_q_heads);
  prm.group = static_cast<int>(num_q_heads / num_kv_heads);
  prm.causal = causal ? 1 : 0;
  prm.scale_log2 = scale * 1.4426950408889634f;  // softmax in the exp2 domain
  prm.err = device_error_word();
  return prm;
}

}  // namespace
}  // namespace ntb200

namespace ntb200 {
namespace {

int prefill_paged(void* out, const void* query, const void* key_cache, const void* value_cache,
                  const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_tables,
                  int64_t num_seqs, int64_t num_tokens, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                  int64_t block_size, int64_t num_blocks, int64_t max_blocks_per_seq, int64_t block_table_stride,
                  int64_t max_query_len, float scale, int causal, int64_t q_token_stride, int64_t q_head_stride,
                  int64_t out_token_stride, int64_t out_head_stride, int64_t cache_block_stride,
                  int64_t cache_page_stride, int64_t cache_head_stride, int dtype, void* stream,
                  bool skip_single_query) {
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "paged_attention_prefill: dtype %d (bf16/f16 only)", dtype);
  if (head_size != kD || block_size != kPage)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "paged_attention_prefill: head_size %lld / block_size %lld (128 / 16 only)",
                (long long)head_size, (long long)block_size);
  if (num_seqs < 0 || num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 ||
      num_blocks <= 0 || max_blocks_per_seq < 0 || block_table_stride < max_blocks_per_seq)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "paged_attention_prefill: bad sizes");
  if (num_seqs == 0 || num_tokens == 0 || max_query_len <= 0) return NTB200_OK;
  if (num_seqs > Smem::kMaxSeqs || num_q_heads > 65535 || num_tokens > 0x7fffffff || num_blocks > 0x7fffffff ||
      max_blocks_per_seq * kPage > 0x7fffffff)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "paged_attention_prefill: sizes beyond the launch limits");
  if (!out || !query || !key_cache || !value_cache || !query_start_loc || !seq_lens || !block_tables)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "paged_attention_prefill: null pointer");
  if (!aligned16(out) || !aligned16(query) || !aligned16(key_cache) || !aligned16(value_cache) ||
      q_token_stride % 8 || q_head_stride % 8 || out_token_stride % 8 || out_head_stride % 8 ||
      cache_block_stride % 8 || cache_page_stride % 8 || cache_head_stride % 8)
    return fail(NTB200_ERR_MISALIGNED, "paged_attention_prefill: pointers 16-byte aligned, strides multiples of 8");
  const bool bf16 = dtype == NTB200_DTYPE_BF16;
  CUtensorMap qm, km, vm;
  int st = make_query_map(&qm, query, bf16, num_tokens, num_q_heads, q_token_stride, q_head_stride);
  if (st != NTB200_OK) return st;
  st = make_cache_map(&km, key_cache, bf16, num_blocks, num_kv_heads, cache_block_stride, cache_page_stride,
                      cache_head_stride);
  if (st != NTB200_OK) return st;
  st = make_cache_map(&vm, value_cache, bf16, num_blocks, num_kv_heads, cache_block_stride, cache_page_stride,
                      cache_head_stride);
  if (st != NTB200_OK) return st;
  PrefillParams prm = base_params(out, query_start_loc, num_tokens, num_q_heads, num_kv_heads, scale, causal,
                                  out_token_stride, out_head_stride);
  prm.seq_lens = seq_lens;
  prm.block_table = block_tables;
  prm.bt_stride = block_table_stride;
  prm.max_blocks = static_cast<int>(max_blocks_per_seq);
  prm.num_blocks = static_cast<int>(num_blocks);
  prm.heads_outer = cache_head_stride > cache_page_stride ? 1 : 0;
  prm.num_seqs = static_cast<int>(num_seqs);
  prm.skip_single_query = skip_single_query ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return bf16 ? launch_prefill<__nv_bfloat16, true>(qm, km, vm, prm, max_query_len, s, 90)
              : launch_prefill<__half, true>(qm, km, vm, prm, max_query_len, s, 91);
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_paged_attention_prefill(
    void* out, const void* query, const void* key_cache, const void* value_cache, const int32_t* query_start_loc,
    const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs, int64_t num_tokens,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size, int64_t num_blocks,
    int64_t max_blocks_per_seq, int64_t block_table_stride, int64_t max_query_len, float scale, int causal,
    int64_t q_token_stride, int64_t q_head_stride, int64_t out_token_stride, int64_t out_head_stride,
    int64_t cache_block_stride, int64_t cache_page_stride, int64_t cache_head_stride, int dtype, void* stream) {
  return ntb200::prefill_paged(out, query, key_cache, value_cache, query_start_loc, seq_lens, block_tables, num_seqs,
                               num_tokens, num_q_heads, num_kv_heads, head_size, block_size, num_blocks,
                               max_blocks_per_seq, block_table_stride, max_query_len, scale, causal, q_token_stride,
                               q_head_stride, out_token_stride, out_head_stride, cache_block_stride,
                               cache_page_stride, cache_head_stride, dtype, stream, false);
}

extern "C" int ntb200_flash_attn_varlen(void* out, const void* query, const void* key, const void* value,
                                        const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int64_t num_seqs,
                                        int64_t num_q_tokens, int64_t num_k_tokens, int64_t num_q_heads,
                                        int64_t num_kv_heads, int64_t head_size, int64_t max_query_len, float scale,
                                        int causal, int64_t q_token_stride, int64_t q_head_stride,
                                        int64_t k_token_stride, int64_t k_head_stride, int64_t v_token_stride,
                                        int64_t v_head_stride, int64_t out_token_stride, int64_t out_head_stride,
                                        int dtype, void* stream) {
  using namespace ntb200;
  if (dtype != NTB200_DTYPE_BF16 && dtype != NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "flash_attn_varlen: dtype %d (bf16/f16 only)", dtype);
  if (head_size != kD)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "flash_attn_varlen: head_size %lld (128 only)", (long long)head_size);
  if (num_seqs < 0 || num_q_tokens < 0 || num_k_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      num_q_heads % num_kv_heads != 0)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "flash_attn_varlen: bad sizes");
  if (num_seqs == 0 || num_q_tokens == 0 || max_query_len <= 0) return NTB200_OK;
  if (num_seqs > Smem::kMaxSeqs || num_q_heads > 65535 || num_q_tokens > 0x7fffffff || num_k_tokens > 0x7fffffff)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "flash_attn_varlen: sizes beyond the launch limits");
  if (!out || !query || !key || !value || !cu_seqlens_q || !cu_seqlens_k)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "flash_attn_varlen: null pointer");
  if (!aligned16(out) || !aligned16(query) || !aligned16(key) || !aligned16(value) || q_token_stride % 8 ||
      q_head_stride % 8 || k_token_stride % 8 || k_head_stride % 8 || v_token_stride % 8 || v_head_stride % 8 ||
      out_token_stride % 8 || out_head_stride % 8)
    return fail(NTB200_ERR_MISALIGNED, "flash_attn_varlen: pointers 16-byte aligned, strides multiples of 8");
  const bool bf16 = dtype == NTB200_DTYPE_BF16;
  CUtensorMap qm, km, vm;
  int st = make_query_map(&qm, query, bf16, num_q_tokens, num_q_heads, q_token_stride, q_head_stride);
  if (st != NTB200_OK) return st;
  if (num_k_tokens > 0) {
    st = make_query_map(&km, key, bf16, num_k_tokens, num_kv_heads, k_token_stride, k_head_stride);
    if (st != NTB200_OK) return st;
    st = make_query_map(&vm, value, bf16, num_k_tokens, num_kv_heads, v_token_stride, v_head_stride);
    if (st != NTB200_OK) return st;
  } else {
    km = qm;  // never read: every sequence has an empty context
    vm = qm;
  }
  PrefillParams prm = base_params(out, cu_seqlens_q, num_q_tokens, num_q_heads, num_kv_heads, scale, causal,
                                  out_token_stride, out_head_stride);
  prm.key_start_loc = cu_seqlens_k;
  prm.num_keys = static_cast<int>(num_k_tokens);
  prm.num_seqs = static_cast<int>(num_seqs);
  prm.skip_single_query = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return bf16 ? launch_prefill<__nv_bfloat16, false>(qm, km, vm, prm, max_query_len, s, 92)
              : launch_prefill<__half, false>(qm, km, vm, prm, max_query_len, s, 93);
}

// A vLLM batch of any mix: sequences with one query token go to the split-K decode kernel
// (reading and writing their rows through query_start_loc), the others to the persistent
// prefill kernel, which skips the single-token ones.  One launch of each (the decode one
// is left out when every sequence has max_query_len > 1 queries).
extern "C" int ntb200_paged_attention_varlen(
    void* out, const void* query, const void* key_cache, const void* value_cache, const int32_t* query_start_loc,
    const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs, int64_t num_tokens,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size, int64_t num_blocks,
    int64_t max_blocks_per_seq, int64_t block_table_stride, int64_t max_query_len, int64_t max_seq_len, float scale,
    int64_t q_token_stride, int64_t q_head_stride, int64_t out_token_stride, int64_t out_head_stride,
    int64_t cache_block_stride, int64_t cache_page_stride, int64_t cache_head_stride, void* workspace,
    size_t workspace_bytes, int dtype, void* stream) {
  using namespace ntb200;
  if (num_seqs == 0 || num_tokens == 0 || max_query_len <= 0) return NTB200_OK;
  const bool uniform_prefill = max_query_len > 1 && num_tokens == max_query_len * num_seqs;
  if (!uniform_prefill) {
    const int st = ntb200_paged_attention_decode_varlen(
        out, query, key_cache, value_cache, query_start_loc, seq_lens, block_tables, num_seqs, num_q_heads,
        num_kv_heads, head_size, block_size, num_blocks, max_blocks_per_seq, block_table_stride, max_seq_len, scale,
        q_token_stride, q_head_stride, out_token_stride, out_head_stride, cache_block_stride, cache_page_stride,
        cache_head_stride, workspace, workspace_bytes, dtype, stream);
    if (st != NTB200_OK || max_query_len == 1) return st;
  }
  return prefill_paged(out, query, key_cache, value_cache, query_start_loc, seq_lens, block_tables, num_seqs,
                       num_tokens, num_q_heads, num_kv_heads, head_size, block_size, num_blocks, max_blocks_per_seq,
                       block_table_stride, max_query_len, scale, 1, q_token_stride, q_head_stride, out_token_stride,
                       out_head_stride, cache_block_stride, cache_page_stride, cache_head_stride, dtype, stream,
                       /*skip_single_query=*/true);
}

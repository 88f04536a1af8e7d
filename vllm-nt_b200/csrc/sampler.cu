// Sampler kernels: the top-k / top-p logits mask and the exponential-race random sample.
//
// Top-k / top-p (the reference's apply_top_k_top_p, vllm_nt/_ntops/torch/sampler.py:4-31,
// which sorts every row of the [B, V] logits, masks in sorted order and scatters back).
// Here nothing is sorted.  One CTA owns one row and finds the two cut values by radix
// select over the row's fp32 logits, mapped to order-preserving 32-bit keys, one 11-, 11-
// and 10-bit digit per pass, with the digit histogram in shared memory:
//
//   top-k:  t_k = the k-th largest logit (counts from the top; every logit >= t_k kept,
//           ties included, as the reference's `logits_sort < threshold` mask does);
//   top-p:  over the logits kept by top-k, with probabilities pi = exp(x - max) / Z,
//           the cut c = the smallest logit whose inclusive cumulative probability from the
//           bottom exceeds 1 - p (the reference's `cumsum <= 1 - p` mask); logits >= c are
//           kept, the largest logit always.
//
// Passes over the row (each from L2 or HBM): max + first top-k digit, two more top-k
// digits, the softmax normaliser Z, three weighted top-p digits (probability sums per bin
// in shared memory, the bin search in fp64), then the masking write.  Histogram updates
// are run-length accumulated per thread (one shared atomic per run of equal bins).  A row
// with neither filter is left untouched.
//
// Random sample (the reference's random_sample, sampler.py:34-42): out[b] =
// argmax_i probs[b, i] / q[b, i] for the caller's exponential draws q, in one pass over
// probs and q: the quotient is IEEE-rounded as torch's division, NaN ranks above every
// number, and the first index wins ties, as torch.argmax does.  The [B, V] quotient the
// reference materialises is never written.
#include "common.cuh"

namespace ntb200 {
namespace {

constexpr int kThreads = 1024;
constexpr int kBins = 2048;  // 11-bit digits
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t ordered_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return b ^ ((b & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u ^ 0x80000000u) : ~u);
}

// digit d of a key: bits [shift, shift + width) with shifts 21, 10, 0 and widths 11, 11, 10
__device__ __forceinline__ int digit_shift(int d) { return d == 0 ? 21 : (d == 1 ? 10 : 0); }
__device__ __forceinline__ uint32_t digit_mask(int d) { return d == 2 ? 0x3FFu : 0x7FFu; }
// the key bits fixed before digit d
__device__ __forceinline__ uint32_t prefix_mask(int d) {
  return d == 0 ? 0u : (d == 1 ? 0xFFE00000u : 0xFFFFFC00u);
}

struct SamplerSmem {
  uint32_t count[kBins];
  float weight[kBins];
  double warp_d[kWarps];
  uint32_t warp_u[kWarps];
  float warp_f[kWarps];
  uint32_t chosen;     // bin picked by the last selection (or kBins if none)
  uint32_t fallback;   // largest non-empty bin of the last weighted pass
};

// Block-wide inclusive prefix sum of one value per thread, in thread order.  `total`
// receives the block sum.  Every thread of the block must call it.
template <typename T>
__device__ __forceinline__ T block_inclusive_scan(T v, T* warp_tot, T& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T n = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = lane < kWarps ? warp_tot[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T n = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += n;
    }
    warp_tot[lane] = w;  // inclusive scan of warp totals (kWarps == 32)
  }
  __syncthreads();
  const T before = warp == 0 ? T(0) : warp_tot[warp - 1];
  total = warp_tot[kWarps - 1];
  __syncthreads();  // warp_tot may be reused right after
  return v + before;
}

__device__ __forceinline__ float block_max(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll 1
  for (int w = 1; w < kWarps; ++w) r = fmaxf(r, scratch[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_sum(double v, double* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = 0.0;
#pragma unroll 1
  for (int w = 0; w < kWarps; ++w) r += scratch[w];
  __syncthreads();
  return r;
}

// Loads each thread keeps in flight per pass: a single CTA streams a whole row, so at small
// batches a pass is latency-bound and its speed grows with the bytes in flight.
constexpr int kInFlight = 4;

// Calls f(x) for every logit of the row, VEC at a time when the row allows it; each thread
// issues kInFlight loads before it consumes any of them.
template <int VEC, typename F>
__device__ __forceinline__ void for_row(const float* row, int64_t vocab, F&& f) {
  if constexpr (VEC == 4) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int64_t n4 = vocab / 4;
    for (int64_t i = threadIdx.x; i < n4; i += kInFlight * kThreads) {
      float4 v[kInFlight];
#pragma unroll
      for (int j = 0; j < kInFlight; ++j)
        if (i + j * kThreads < n4) v[j] = r4[i + j * kThreads];
#pragma unroll
      for (int j = 0; j < kInFlight; ++j) {
        if (i + j * kThreads < n4) {
          f(v[j].x);
          f(v[j].y);
          f(v[j].z);
          f(v[j].w);
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < vocab; i += kInFlight * kThreads) {
      float v[kInFlight];
#pragma unroll
      for (int j = 0; j < kInFlight; ++j)
        if (i + j * kThreads < vocab) v[j] = row[i + j * kThreads];
#pragma unroll
      for (int j = 0; j < kInFlight; ++j)
        if (i + j * kThreads < vocab) f(v[j]);
    }
  }
}

// Per-thread run-length accumulation into the shared histograms: consecutive keys of a
// thread that fall into the same bin cost one shared atomic per run instead of one per
// key.  Rows whose logits are mostly one value (a vocabulary masked to -inf by a logits
// processor, as guided decoding does) would otherwise serialise every thread of the CTA
// on a single shared-memory address.
struct BinRun {
  uint32_t bin = 0xFFFFFFFFu, n = 0;
  float w = 0.f;
  __device__ __forceinline__ void add(SamplerSmem& s, uint32_t b) {
    if (b != bin) {
      flush(s, false);
      bin = b;
    }
    ++n;
  }
  __device__ __forceinline__ void add(SamplerSmem& s, uint32_t b, float weight) {
    if (b != bin) {
      flush(s, true);
      bin = b;
    }
    ++n;
    w += weight;
  }
  __device__ __forceinline__ void flush(SamplerSmem& s, bool weighted) {
    if (n > 0) {
      atomicAdd(&s.count[bin], n);
      if (weighted) atomicAdd(&s.weight[bin], w);
    }
    n = 0;
    w = 0.f;
  }
};

// Top-k selection over s.count: the bin holding the `remaining`-th largest key among the
// keys that match the prefix.  Updates remaining (keys ranked above that bin removed).
__device__ __forceinline__ uint32_t select_from_top(SamplerSmem& s, uint32_t& remaining) {
  const int b0 = 2 * threadIdx.x, b1 = b0 + 1;
  const uint32_t c0 = s.count[b0], c1 = s.count[b1];
  uint32_t total;
  const uint32_t incl = block_inclusive_scan<uint32_t>(c0 + c1, s.warp_u, total);
  // keys in bins above b1 / above b0
  const uint32_t above1 = total - incl, above0 = above1 + c1;
  if (c1 > 0 && above1 < remaining && remaining <= above1 + c1) {
    s.chosen = b1;
    s.fallback = above1;
  }
  if (c0 > 0 && above0 < remaining && remaining <= above0 + c0) {
    s.chosen = b0;
    s.fallback = above0;
  }
  __syncthreads();
  const uint32_t bin = s.chosen;
  remaining -= s.fallback;
  __syncthreads();
  return bin;
}

// Top-p selection over s.weight/s.count: the smallest non-empty bin whose inclusive
// cumulative weight, added to `base`, exceeds target; if rounding leaves none, the
// largest non-empty bin.  Updates base with the weight of the bins below the choice.
__device__ __forceinline__ uint32_t select_from_bottom(SamplerSmem& s, double& base, double target) {
  const int b0 = 2 * threadIdx.x, b1 = b0 + 1;
  const double w0 = s.weight[b0], w1 = s.weight[b1];
  const uint32_t c0 = s.count[b0], c1 = s.count[b1];
  if (threadIdx.x == 0) {
    s.chosen = kBins;
    s.fallback = 0;
  }
  double total;
  const double incl1 = block_inclusive_scan<double>(w0 + w1, s.warp_d, total);  // syncs
  const double excl0 = incl1 - (w0 + w1), incl0 = excl0 + w0;
  // the inclusive sums grow with the bin index, so the smallest non-empty bin whose
  // inclusive sum exceeds the target is the crossing bin (no lower-bound test, which could
  // leave an ulp-sized gap between neighbouring threads' sums)
  if (c0 > 0 && target < base + incl0) atomicMin(&s.chosen, uint32_t(b0));
  if (c1 > 0 && target < base + incl1) atomicMin(&s.chosen, uint32_t(b1));
  if (c1 > 0) atomicMax(&s.fallback, uint32_t(b1));
  else if (c0 > 0) atomicMax(&s.fallback, uint32_t(b0));
  __syncthreads();
  const uint32_t bin = s.chosen < kBins ? s.chosen : s.fallback;
  // weight below the chosen bin: the owner of the bin publishes it
  if (bin == uint32_t(b0)) s.warp_d[0] = excl0;
  if (bin == uint32_t(b1)) s.warp_d[0] = incl0;
  __syncthreads();
  base += s.warp_d[0];
  __syncthreads();
  return bin;
}

template <int VEC, typename KT>
__global__ void __launch_bounds__(kThreads, 1) top_k_top_p_kernel(
    float* __restrict__ logits, int64_t vocab, int64_t row_stride, const KT* __restrict__ top_k,
    const float* __restrict__ top_p) {
  __shared__ SamplerSmem s;
  float* row = logits + static_cast<int64_t>(blockIdx.x) * row_stride;
  pdl_trigger();
  pdl_wait();
  const bool use_k = top_k != nullptr, use_p = top_p != nullptr;
  int64_t k = vocab;
  if (use_k) {
    k = static_cast<int64_t>(top_k[blockIdx.x]);
    k = k < 1 ? 1 : (k > vocab ? vocab : k);
  }
  const bool filter_k = use_k && k < vocab;
  for (int b = threadIdx.x; b < kBins; b += kThreads) s.count[b] = 0;
  __syncthreads();

  // pass 1: row max (always) and the first top-k digit
  float m = -INFINITY;
  {
    BinRun run;
    for_row<VEC>(row, vocab, [&](float x) {
      m = fmaxf(m, x);
      if (filter_k) run.add(s, ordered_key(x) >> 21);
    });
    run.flush(s, false);
  }
  m = block_max(m, s.warp_f);

  // top-k: three digits; every logit >= t_k survives
  float t_k = -INFINITY;
  if (filter_k) {
    uint32_t remaining = static_cast<uint32_t>(k), prefix = 0;
    for (int d = 0; d < 3; ++d) {
      if (d > 0) {
        for (int b = threadIdx.x; b < kBins; b += kThreads) s.count[b] = 0;
        __syncthreads();
        const uint32_t pm = prefix_mask(d), dm = digit_mask(d);
        const int sh = digit_shift(d);
        BinRun run;
        for_row<VEC>(row, vocab, [&](float x) {
          const uint32_t u = ordered_key(x);
          if ((u & pm) == prefix) run.add(s, (u >> sh) & dm);
        });
        run.flush(s, false);
        __syncthreads();
      } else {
        __syncthreads();
      }
      prefix |= select_from_top(s, remaining) << digit_shift(d);
    }
    t_k = key_value(prefix);
  }

  // top-p over the survivors of top-k
  uint32_t cut = 0;  // keys >= cut survive (0: everything)
  // A row of -inf logits has no probabilities (the reference's softmax gives NaN there and
  // masks nothing): it is left as it is.
  const bool filter_p = use_p && m != -INFINITY;
  if (filter_p) {
    double z = 0.0;
    {
      float zt = 0.f;
      for_row<VEC>(row, vocab, [&](float x) {
        if (x >= t_k) zt += expf(x - m);
      });
      z = block_sum(zt, s.warp_d);
    }
    const float zf = static_cast<float>(z);
    const double target = static_cast<double>(__fsub_rn(1.0f, top_p[blockIdx.x]));
    double base = 0.0;
    uint32_t prefix = 0;
    for (int d = 0; d < 3; ++d) {
      for (int b = threadIdx.x; b < kBins; b += kThreads) {
        s.count[b] = 0;
        s.weight[b] = 0.f;
      }
      __syncthreads();
      const uint32_t pm = prefix_mask(d), dm = digit_mask(d);
      const int sh = digit_shift(d);
      BinRun run;
      for_row<VEC>(row, vocab, [&](float x) {
        const uint32_t u = ordered_key(x);
        if (x >= t_k && (u & pm) == prefix) run.add(s, (u >> sh) & dm, __fdiv_rn(expf(x - m), zf));
      });
      run.flush(s, true);
      __syncthreads();
      prefix |= select_from_bottom(s, base, target) << sh;
    }
    cut = prefix;
  }

  if (!filter_k && !filter_p) return;
  // masking write, in place
  if constexpr (VEC == 4) {
    float4* r4 = reinterpret_cast<float4*>(row);
    const int64_t n4 = vocab / 4;
    auto keep = [&](float x) { return x >= t_k && ordered_key(x) >= cut ? x : -INFINITY; };
    for (int64_t i = threadIdx.x; i < n4; i += kInFlight * kThreads) {
      float4 v[kInFlight];
#pragma unroll
      for (int j = 0; j < kInFlight; ++j)
        if (i + j * kThreads < n4) v[j] = r4[i + j * kThreads];
#pragma unroll
      for (int j = 0; j < kInFlight; ++j) {
        if (i + j * kThreads < n4) {
          v[j].x = keep(v[j].x);
          v[j].y = keep(v[j].y);
          v[j].z = keep(v[j].z);
          v[j].w = keep(v[j].w);
          r4[i + j * kThreads] = v[j];
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < vocab; i += kThreads) {
      const float x = row[i];
      row[i] = x >= t_k && ordered_key(x) >= cut ? x : -INFINITY;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Small batches: one row per cluster of kCluster CTAs.  A single CTA streams its row about
// eight times (one pass per digit), so with few rows the GPU is mostly idle and each pass
// is latency-bound.  Here CTA r of the cluster loads slice r of the row into shared
// memory once; every pass then scans shared memory, and the digit histograms are merged
// through distributed shared memory: CTA r sums bins [256 r, +256) over the cluster and
// publishes its range total, every CTA finds the range that holds the cut, and the owner
// of that range finds the bin and publishes it.  The selection rules are those of the
// one-CTA kernel; the fp64 weight sums are associated by range first.
// ---------------------------------------------------------------------------------------

constexpr int kCluster = 8;
constexpr int kCThreads = 512;
constexpr int kCWarps = kCThreads / 32;
constexpr int kRange = kBins / kCluster;  // 256 bins per CTA of the cluster
constexpr int64_t kMaxSlice = 32768;      // floats of the row per CTA (128 KB)

struct ClusterState {
  uint32_t count[kBins];  // this CTA's histogram
  float weight[kBins];
  uint32_t mcount[kRange];  // merged histogram of this CTA's bin range
  double mweight[kRange];
  // written by every CTA of the cluster into every CTA (slot = the writer's rank)
  float peer_max[kCluster];
  double peer_sum[kCluster];
  uint32_t range_count[kCluster];
  double range_weight[kCluster];
  // written by the CTA that owns the chosen range
  uint32_t chosen_bin;
  uint32_t chosen_above;
  double chosen_below;
  uint32_t pick, pick_last;  // the owner's search within its range
  // block-reduction scratch
  uint32_t warp_u[kCWarps];
  double warp_d[kCWarps];
  float warp_f[kCWarps];
};

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem(const void* local, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
  return a;
}
__device__ __forceinline__ uint32_t ld_dsmem_u32(const void* local, uint32_t rank) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(dsmem(local, rank)) : "memory");
  return v;
}
__device__ __forceinline__ float ld_dsmem_f32(const void* local, uint32_t rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(dsmem(local, rank)) : "memory");
  return v;
}
// stores v into the same variable of every CTA of the cluster (this one included)
__device__ __forceinline__ void publish_u32(uint32_t* local, uint32_t v) {
  for (uint32_t c = 0; c < kCluster; ++c)
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(dsmem(local, c)), "r"(v) : "memory");
}
__device__ __forceinline__ void publish_f32(float* local, float v) {
  for (uint32_t c = 0; c < kCluster; ++c)
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem(local, c)), "f"(v) : "memory");
}
__device__ __forceinline__ void publish_f64(double* local, double v) {
  for (uint32_t c = 0; c < kCluster; ++c)
    asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(dsmem(local, c)), "d"(v) : "memory");
}

// Block-wide inclusive prefix sum (thread order) for kCThreads threads.
template <typename T>
__device__ __forceinline__ T cblock_scan(T v, T* warp_tot, T& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T n = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  T before = T(0), tot = T(0);
#pragma unroll
  for (int w = 0; w < kCWarps; ++w) {
    before += w < warp ? warp_tot[w] : T(0);
    tot += warp_tot[w];
  }
  total = tot;
  __syncthreads();
  return v + before;
}

// Top-k selection over the cluster's histograms: the bin holding the `remaining`-th
// largest key among the keys that match the prefix; `remaining` loses the keys ranked
// above that bin.  Every CTA of the cluster calls it.
__device__ __forceinline__ uint32_t cluster_select_top(ClusterState& st, uint32_t& remaining, uint32_t rank) {
  cluster_barrier();  // every CTA's histogram is complete
  const int t = threadIdx.x;
  // thread t < kRange holds bin kRange - 1 - t of this CTA's range (largest first)
  uint32_t c = 0;
  if (t < kRange) {
    const int b = static_cast<int>(rank) * kRange + (kRange - 1 - t);
#pragma unroll
    for (uint32_t q = 0; q < kCluster; ++q) c += ld_dsmem_u32(&st.count[b], q);
  }
  uint32_t total;
  const uint32_t incl = cblock_scan<uint32_t>(c, st.warp_u, total);  // keys at or above the bin
  if (t == 0) publish_u32(&st.range_count[rank], total);
  cluster_barrier();
  // the range holding the cut, from the top
  uint32_t above = 0;
  int q = 0;
  for (int r = kCluster - 1; r >= 0; --r) {
    if (remaining <= above + st.range_count[r]) {
      q = r;
      break;
    }
    above += st.range_count[r];
  }
  if (static_cast<int>(rank) == q && t < kRange && c > 0 && above + incl - c < remaining && remaining <= above + incl) {
    publish_u32(&st.chosen_bin, static_cast<uint32_t>(q * kRange + (kRange - 1 - t)));
    publish_u32(&st.chosen_above, above + incl - c);
  }
  cluster_barrier();
  remaining -= st.chosen_above;
  return st.chosen_bin;
}

// Top-p selection over the cluster's weighted histograms: the smallest non-empty bin whose
// inclusive cumulative weight, added to `base`, exceeds target; if rounding leaves none,
// the largest non-empty bin.  `base` gains the weight of the bins below the choice.
__device__ __forceinline__ uint32_t cluster_select_bottom(ClusterState& st, double& base, double target,
                                                          uint32_t rank) {
  cluster_barrier();
  const int t = threadIdx.x;
  // thread t < kRange holds bin t of this CTA's range (smallest first)
  uint32_t c = 0;
  double w = 0.0;
  if (t < kRange) {
    const int b = static_cast<int>(rank) * kRange + t;
#pragma unroll
    for (uint32_t q = 0; q < kCluster; ++q) {
      c += ld_dsmem_u32(&st.count[b], q);
      w += static_cast<double>(ld_dsmem_f32(&st.weight[b], q));
    }
  }
  double wtot;
  const double incl = cblock_scan<double>(w, st.warp_d, wtot);
  uint32_t ctot;
  cblock_scan<uint32_t>(c, st.warp_u, ctot);
  if (t == 0) {
    publish_u32(&st.range_count[rank], ctot);
    publish_f64(&st.range_weight[rank], wtot);
  }
  cluster_barrier();
  // the first non-empty range whose inclusive weight crosses the target, else the last
  // non-empty range (identical in every CTA)
  double cum = 0.0, cum_q = 0.0, cum_last = 0.0;
  int q = -1, last = 0;
  for (int r = 0; r < kCluster; ++r) {
    if (st.range_count[r] > 0) {
      last = r;
      cum_last = cum;
      if (q < 0 && target < base + cum + st.range_weight[r]) {
        q = r;
        cum_q = cum;
      }
    }
    cum += st.range_weight[r];
  }
  const bool fallback = q < 0;
  if (fallback) {
    q = last;
    cum_q = cum_last;
  }
  if (static_cast<int>(rank) == q) {  // CTA-uniform
    if (t == 0) {
      st.pick = kRange;
      st.pick_last = 0;
    }
    __syncthreads();
    if (t < kRange && c > 0) {
      if (!fallback && target < base + cum_q + incl) atomicMin(&st.pick, static_cast<uint32_t>(t));
      atomicMax(&st.pick_last, static_cast<uint32_t>(t) + 1u);
    }
    __syncthreads();
    const uint32_t b = st.pick < kRange ? st.pick : st.pick_last - 1u;
    if (static_cast<uint32_t>(t) == b) {
      publish_u32(&st.chosen_bin, static_cast<uint32_t>(q * kRange) + b);
      publish_f64(&st.chosen_below, cum_q + (incl - w));
    }
  }
  cluster_barrier();
  base += st.chosen_below;
  return st.chosen_bin;
}

template <int VEC, typename KT>
__global__ void __launch_bounds__(kCThreads, 1) top_k_top_p_cluster_kernel(
    float* __restrict__ logits, int64_t vocab, int64_t row_stride, const KT* __restrict__ top_k,
    const float* __restrict__ top_p, int slice_len) {
  __shared__ ClusterState st;
  extern __shared__ __align__(16) float slice[];
  const uint32_t rank = cta_rank();
  const int64_t row_id = static_cast<int64_t>(blockIdx.x) / kCluster;
  float* row = logits + row_id * row_stride;
  const int64_t c0 = int64_t(rank) * slice_len;
  const int n = static_cast<int>(c0 >= vocab ? 0 : (vocab - c0 < slice_len ? vocab - c0 : slice_len));
  pdl_trigger();
  pdl_wait();
  const bool use_k = top_k != nullptr, use_p = top_p != nullptr;
  int64_t k = vocab;
  if (use_k) {
    k = static_cast<int64_t>(top_k[row_id]);
    k = k < 1 ? 1 : (k > vocab ? vocab : k);
  }
  const bool filter_k = use_k && k < vocab;
  // this CTA's slice of the row into shared memory (read from memory once)
  if constexpr (VEC == 4) {
    const float4* src = reinterpret_cast<const float4*>(row + c0);
    float4* dst = reinterpret_cast<float4*>(slice);
    for (int i = threadIdx.x; i < n / 4; i += kCThreads) dst[i] = src[i];
  } else {
    for (int i = threadIdx.x; i < n; i += kCThreads) slice[i] = row[c0 + i];
  }
  for (int b = threadIdx.x; b < kBins; b += kCThreads) st.count[b] = 0;
  __syncthreads();
  cluster_barrier();  // every CTA of the cluster is running before any writes into another

  // pass 1: row max and the first top-k digit
  float m = -INFINITY;
  {
    uint32_t bin = 0xFFFFFFFFu, run = 0;
    for (int i = threadIdx.x; i < n; i += kCThreads) {
      const float x = slice[i];
      m = fmaxf(m, x);
      if (filter_k) {
        const uint32_t b = ordered_key(x) >> 21;
        if (b != bin) {
          if (run) atomicAdd(&st.count[bin], run);
          bin = b;
          run = 0;
        }
        ++run;
      }
    }
    if (run) atomicAdd(&st.count[bin], run);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((threadIdx.x & 31) == 0) st.warp_f[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = st.warp_f[0];
    for (int w = 1; w < kCWarps; ++w) mm = fmaxf(mm, st.warp_f[w]);
    publish_f32(&st.peer_max[rank], mm);
  }
  // the first selection's barrier (or this one) makes every CTA's max visible
  if (!filter_k) cluster_barrier();

  // top-k: three digits; every logit >= t_k survives
  float t_k = -INFINITY;
  if (filter_k) {
    uint32_t remaining = static_cast<uint32_t>(k), prefix = 0;
    for (int d = 0; d < 3; ++d) {
      if (d > 0) {
        // the previous selection's last barrier: no CTA reads this histogram any more
        for (int b = threadIdx.x; b < kBins; b += kCThreads) st.count[b] = 0;
        __syncthreads();
        const uint32_t pm = prefix_mask(d), dm = digit_mask(d);
        const int sh = digit_shift(d);
        uint32_t bin = 0xFFFFFFFFu, run = 0;
        for (int i = threadIdx.x; i < n; i += kCThreads) {
          const uint32_t u = ordered_key(slice[i]);
          if ((u & pm) != prefix) continue;
          const uint32_t b = (u >> sh) & dm;
          if (b != bin) {
            if (run) atomicAdd(&st.count[bin], run);
            bin = b;
            run = 0;
          }
          ++run;
        }
        if (run) atomicAdd(&st.count[bin], run);
      }
      __syncthreads();
      prefix |= cluster_select_top(st, remaining, rank) << digit_shift(d);
    }
    t_k = key_value(prefix);
  }
  m = st.peer_max[0];
#pragma unroll
  for (int c = 1; c < kCluster; ++c) m = fmaxf(m, st.peer_max[c]);

  // top-p over the survivors of top-k (a row of -inf logits is left as it is)
  uint32_t cut = 0;  // keys >= cut survive (0: everything)
  const bool filter_p = use_p && m != -INFINITY;
  if (filter_p) {
    float zt = 0.f;
    for (int i = threadIdx.x; i < n; i += kCThreads) {
      const float x = slice[i];
      if (x >= t_k) zt += expf(x - m);
    }
    double zd = zt;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zd += __shfl_xor_sync(0xFFFFFFFFu, zd, o);
    if ((threadIdx.x & 31) == 0) st.warp_d[threadIdx.x >> 5] = zd;
    __syncthreads();
    if (threadIdx.x == 0) {
      double zs = 0.0;
      for (int w = 0; w < kCWarps; ++w) zs += st.warp_d[w];
      publish_f64(&st.peer_sum[rank], zs);
    }
    cluster_barrier();
    double z = 0.0;
#pragma unroll
    for (int c = 0; c < kCluster; ++c) z += st.peer_sum[c];
    const float zf = static_cast<float>(z);
    const double target = static_cast<double>(__fsub_rn(1.0f, top_p[row_id]));
    double base = 0.0;
    uint32_t prefix = 0;
    for (int d = 0; d < 3; ++d) {
      // the last barrier passed: no CTA reads this CTA's histograms any more
      for (int b = threadIdx.x; b < kBins; b += kCThreads) {
        st.count[b] = 0;
        st.weight[b] = 0.f;
      }
      __syncthreads();
      const uint32_t pm = prefix_mask(d), dm = digit_mask(d);
      const int sh = digit_shift(d);
      uint32_t bin = 0xFFFFFFFFu, run = 0;
      float wrun = 0.f;
      for (int i = threadIdx.x; i < n; i += kCThreads) {
        const float x = slice[i];
        const uint32_t u = ordered_key(x);
        if (!(x >= t_k) || (u & pm) != prefix) continue;
        const uint32_t b = (u >> sh) & dm;
        if (b != bin) {
          if (run) {
            atomicAdd(&st.count[bin], run);
            atomicAdd(&st.weight[bin], wrun);
          }
          bin = b;
          run = 0;
          wrun = 0.f;
        }
        ++run;
        wrun += __fdiv_rn(expf(x - m), zf);
      }
      if (run) {
        atomicAdd(&st.count[bin], run);
        atomicAdd(&st.weight[bin], wrun);
      }
      __syncthreads();
      prefix |= cluster_select_bottom(st, base, target, rank) << sh;
    }
    cut = prefix;
  }

  if (!filter_k && !filter_p) return;
  // masking write of this CTA's slice, in place
  auto keep = [&](float x) { return x >= t_k && ordered_key(x) >= cut ? x : -INFINITY; };
  if constexpr (VEC == 4) {
    float4* dst = reinterpret_cast<float4*>(row + c0);
    const float4* src = reinterpret_cast<const float4*>(slice);
    for (int i = threadIdx.x; i < n / 4; i += kCThreads) {
      float4 v = src[i];
      v.x = keep(v.x);
      v.y = keep(v.y);
      v.z = keep(v.z);
      v.w = keep(v.w);
      dst[i] = v;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += kCThreads) row[c0 + i] = keep(slice[i]);
  }
}

// ---------------------------------------------------------------------------------------
// random sample: argmax_i probs[i] / q[i]
// ---------------------------------------------------------------------------------------

constexpr int kSampleThreads = 512;

// (quotient, index) packed so that the larger key is the larger quotient, NaN above every
// number, and on equal quotients the smaller index
__device__ __forceinline__ uint64_t sample_key(float v, int64_t i) {
  const uint32_t ord = isnan(v) ? 0xFFFFFFFFu : ordered_key(v);
  return (static_cast<uint64_t>(ord) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - static_cast<uint32_t>(i));
}

template <int VEC>
__global__ void __launch_bounds__(kSampleThreads) random_sample_kernel(
    int64_t* __restrict__ out, const float* __restrict__ probs, const float* __restrict__ q,
    int64_t vocab, int64_t probs_stride, int64_t q_stride) {
  __shared__ uint64_t warp_best[kSampleThreads / 32];
  const float* pr = probs + static_cast<int64_t>(blockIdx.x) * probs_stride;
  const float* qr = q + static_cast<int64_t>(blockIdx.x) * q_stride;
  pdl_trigger();
  pdl_wait();
  uint64_t best = 0;
  if constexpr (VEC == 4) {
    const int64_t n4 = vocab / 4;
    const float4* p4 = reinterpret_cast<const float4*>(pr);
    const float4* q4 = reinterpret_cast<const float4*>(qr);
    // two float4 of probs and two of q in flight per thread before any is consumed
    for (int64_t i = threadIdx.x; i < n4; i += 2 * kSampleThreads) {
      const int64_t i1 = i + kSampleThreads;
      const float4 a0 = __ldcs(p4 + i), b0 = __ldcs(q4 + i);
      float4 a1 = a0, b1 = b0;
      if (i1 < n4) {
        a1 = __ldcs(p4 + i1);
        b1 = __ldcs(q4 + i1);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (j == 1 && i1 >= n4) break;
        const float4 a = j == 0 ? a0 : a1, b = j == 0 ? b0 : b1;
        const int64_t e = 4 * (j == 0 ? i : i1);
        uint64_t k0 = sample_key(__fdiv_rn(a.x, b.x), e), k1 = sample_key(__fdiv_rn(a.y, b.y), e + 1);
        uint64_t k2 = sample_key(__fdiv_rn(a.z, b.z), e + 2), k3 = sample_key(__fdiv_rn(a.w, b.w), e + 3);
        k0 = k0 > k1 ? k0 : k1;
        k2 = k2 > k3 ? k2 : k3;
        k0 = k0 > k2 ? k0 : k2;
        best = best > k0 ? best : k0;
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < vocab; i += kSampleThreads) {
      const uint64_t k = sample_key(__fdiv_rn(pr[i], qr[i]), i);
      best = best > k ? best : k;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t n = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    best = best > n ? best : n;
  }
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t r = warp_best[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) r = r > warp_best[w] ? r : warp_best[w];
    out[blockIdx.x] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(r & 0xFFFFFFFFu));
  }
}

// Rows up to which one cluster per row beats one CTA per row, measured with a 128256-token
// vocabulary, k = 50 and p = 0.9: 1 row 36 against 88 us, 16 rows 69 against 89, 24 rows 73
// against 90, 32 rows 107 against 91 (top-p alone: 49 against 252 us at 1 row).
constexpr int64_t kClusterRowsMax = 24;

template <int VEC, typename KT>
int launch_top_k_top_p_cluster(float* logits, int64_t rows, int64_t vocab, int64_t stride, const KT* k,
                               const float* p, int slice, cudaStream_t stream, int slot) {
  const void* fn = reinterpret_cast<const void*>(top_k_top_p_cluster_kernel<VEC, KT>);
  const int smem = slice * static_cast<int>(sizeof(float));
  int st = ensure_smem_attribute(fn, smem, slot);
  if (st != NTB200_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows * kCluster));
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  set_pdl_attribute(attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, top_k_top_p_cluster_kernel<VEC, KT>, logits, vocab, stride, k, p, slice);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "top_k_top_p (clusters): launch failed: %s", cudaGetErrorString(e));
  }
  return NTB200_OK;
}

template <typename KT>
int launch_top_k_top_p(float* logits, int64_t rows, int64_t vocab, int64_t stride, const KT* k,
                       const float* p, cudaStream_t stream) {
  const bool vec = vocab % 4 == 0 && stride % 4 == 0 && aligned16(logits);
  const int64_t slice = (ceil_div(vocab, kCluster) + 3) / 4 * 4;  // floats per CTA, a multiple of 4
  if (rows <= kClusterRowsMax && slice <= kMaxSlice) {
    const int slot = 120 + (vec ? 0 : 1) + (sizeof(KT) == 8 ? 0 : 2);
    return vec ? launch_top_k_top_p_cluster<4, KT>(logits, rows, vocab, stride, k, p, static_cast<int>(slice), stream, slot)
               : launch_top_k_top_p_cluster<1, KT>(logits, rows, vocab, stride, k, p, static_cast<int>(slice), stream, slot);
  }
  if (vec)
    return launch_kernel("top_k_top_p", top_k_top_p_kernel<4, KT>, dim3(static_cast<unsigned>(rows)),
                         dim3(kThreads), 0, stream, logits, vocab, stride, k, p);
  return launch_kernel("top_k_top_p", top_k_top_p_kernel<1, KT>, dim3(static_cast<unsigned>(rows)),
                       dim3(kThreads), 0, stream, logits, vocab, stride, k, p);
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_top_k_top_p(float* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                                  const void* top_k, int top_k_dtype, const float* top_p, void* stream) {
  using namespace ntb200;
  if (num_rows < 0 || vocab < 0 || row_stride < vocab)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "top_k_top_p: bad shape");
  if (num_rows == 0 || vocab == 0 || (top_k == nullptr && top_p == nullptr)) return NTB200_OK;
  if (logits == nullptr) return fail(NTB200_ERR_INVALID_ARGUMENT, "top_k_top_p: null logits");
  if (num_rows > 0x7fffffff || vocab > 0x7fffffff)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "top_k_top_p: too many rows or a vocabulary >= 2^31");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (top_k == nullptr)
    return launch_top_k_top_p<int64_t>(logits, num_rows, vocab, row_stride, nullptr, top_p, s);
  if (top_k_dtype == NTB200_DTYPE_I64)
    return launch_top_k_top_p(logits, num_rows, vocab, row_stride, static_cast<const int64_t*>(top_k), top_p, s);
  if (top_k_dtype == NTB200_DTYPE_I32)
    return launch_top_k_top_p(logits, num_rows, vocab, row_stride, static_cast<const int32_t*>(top_k), top_p, s);
  return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "top_k_top_p: top_k dtype %d", top_k_dtype);
}

extern "C" int ntb200_random_sample(int64_t* out, const float* probs, const float* q, int64_t num_rows,
                                   int64_t vocab, int64_t probs_row_stride, int64_t q_row_stride,
                                   void* stream) {
  using namespace ntb200;
  if (num_rows < 0 || vocab <= 0 || probs_row_stride < vocab || q_row_stride < vocab)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "random_sample: bad shape");
  if (num_rows == 0) return NTB200_OK;
  if (out == nullptr || probs == nullptr || q == nullptr)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "random_sample: null pointer");
  if (num_rows > 0x7fffffff || vocab > 0x7fffffff)
    return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "random_sample: too many rows or a vocabulary >= 2^31");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = vocab % 4 == 0 && probs_row_stride % 4 == 0 && q_row_stride % 4 == 0 && aligned16(probs) &&
                   aligned16(q);
  const dim3 grid(static_cast<unsigned>(num_rows));
  if (vec)
    return launch_kernel("random_sample", random_sample_kernel<4>, grid, dim3(kSampleThreads), 0, s, out, probs,
                         q, vocab, probs_row_stride, q_row_stride);
  return launch_kernel("random_sample", random_sample_kernel<1>, grid, dim3(kSampleThreads), 0, s, out, probs, q,
                       vocab, probs_row_stride, q_row_stride);
}

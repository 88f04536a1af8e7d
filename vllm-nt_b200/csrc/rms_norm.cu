// RMS norm and fused residual-add RMS norm.
//
// One CTA per row, two 16-byte vectors per thread.  Every thread issues all of its loads
// of the row up front (x, the residual when fused, the weight), keeps the fp32 sum in
// registers, writes the new residual, reduces sum(s^2) with warp shuffles + one
// shared-memory step, then streams weight*normalised values out.  HBM traffic is the algorithmic minimum: x (+residual)
// read once, out (+residual) written once, weight read from L2 after the first rows.
//
// out may alias x (vLLM's in-place convention): each thread reads its own vectors of x
// before it writes the same vectors of out, so no pointer here is marked __restrict__
// except the residual and the weight.
//
// Rounding follows vLLM's torch-native path (vllm/ir/ops/layernorm.py:10-62, which the
// vllm_nt RMSNorm hook replaces): the add and the statistics are fp32, the normalised
// value is rounded to the weight dtype before the weight multiply, and that product is
// rounded again.
//
// The Gemma variant follows GemmaRMSNorm.forward_native
// (vllm/model_executor/layers/layernorm.py:153-170): the weight term is (1 + w) formed in
// fp32, the normalised value is not rounded before it multiplies that term (one rounding,
// of the product), and with a residual the sum is taken in the input dtype (a bf16 sum is
// rounded to bf16 before the statistics are formed from it; fp32 stays fp32).
#include "common.cuh"

namespace ntb200 {
namespace {

constexpr int kMaxItems = 2;  // vectors per thread kept in registers

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  constexpr int kWarps = THREADS / 32;
  if constexpr (kWarps == 1) {
    return v;
  } else {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < kWarps ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
  }
}

// T: storage type; VEC: elements per vector access; THREADS: CTA size; HAS_W: a weight
// is given; GEMMA: Gemma's (1 + w) weight and rounding points.  Rows with more than
// THREADS*kMaxItems vectors take a second pass (re-reading x and residual from L2) -- the
// register-resident path covers hidden <= 16384 bf16.
template <typename T, int VEC, int THREADS, bool FUSED, bool HAS_W, bool GEMMA>
__global__ void __launch_bounds__(THREADS) rms_norm_kernel(
    T* out, T* __restrict__ residual, const T* x, const T* __restrict__ weight, int64_t hidden,
    int64_t x_stride, int64_t r_stride, int64_t o_stride, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * x_stride;
  T* rr = FUSED ? residual + row * r_stride : nullptr;
  T* orow = out + row * o_stride;
  const int64_t nvec = hidden / VEC;
  pdl_trigger();
  pdl_wait();

  // Every load of the register-resident window (x, residual, weight) is issued before the
  // first store: a residual store between them would keep the compiler from hoisting the
  // later loads (x is not __restrict__), leaving one round trip to HBM per vector.
  using V = Vec<T, VEC>;
  V xraw[kMaxItems];
  V rraw[FUSED ? kMaxItems : 1];
  V wraw[HAS_W ? kMaxItems : 1];
#pragma unroll
  for (int it = 0; it < kMaxItems; ++it) {
    const int64_t vi = threadIdx.x + int64_t(it) * THREADS;
    if (vi < nvec) {
      xraw[it] = *reinterpret_cast<const V*>(xr + vi * VEC);
      if constexpr (FUSED) rraw[it] = *reinterpret_cast<const V*>(rr + vi * VEC);
      if constexpr (HAS_W) wraw[it] = *reinterpret_cast<const V*>(weight + vi * VEC);
    }
  }
  float s[kMaxItems][VEC];
  float sumsq = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxItems; ++it) {
    const int64_t vi = threadIdx.x + int64_t(it) * THREADS;
    if (vi < nvec) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        s[it][j] = Elem<T>::to_f(xraw[it].v[j]);
        if constexpr (FUSED) s[it][j] += Elem<T>::to_f(rraw[it].v[j]);
        if constexpr (FUSED && GEMMA) s[it][j] = Elem<T>::round(s[it][j]);
      }
      if constexpr (FUSED) store_f<T, VEC>(rr + vi * VEC, s[it]);
#pragma unroll
      for (int j = 0; j < VEC; ++j) sumsq += s[it][j] * s[it][j];
    }
  }
  // rows longer than the register-resident window
  for (int64_t vi = threadIdx.x + int64_t(kMaxItems) * THREADS; vi < nvec; vi += THREADS) {
    float t[VEC];
    load_f<T, VEC>(xr + vi * VEC, t);
    if constexpr (FUSED) {
      float r[VEC];
      load_f<T, VEC>(rr + vi * VEC, r);
#pragma unroll
      for (int j = 0; j < VEC; ++j) t[j] = GEMMA ? Elem<T>::round(t[j] + r[j]) : t[j] + r[j];
      store_f<T, VEC>(rr + vi * VEC, t);
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) sumsq += t[j] * t[j];
  }

  const float total = block_sum<THREADS>(sumsq, red);
  const float rstd = rsqrtf(total / static_cast<float>(hidden) + eps);

  auto emit = [&](int64_t vi, const float (&v)[VEC], const V& w) {
    float y[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      if constexpr (GEMMA) {
        y[j] = (v[j] * rstd) * (1.f + Elem<T>::to_f(w.v[j]));
      } else {
        const float wj = HAS_W ? Elem<T>::to_f(w.v[j]) : 1.f;
        y[j] = Elem<T>::round(v[j] * rstd) * wj;
      }
    }
    store_f<T, VEC>(orow + vi * VEC, y);
  };
#pragma unroll
  for (int it = 0; it < kMaxItems; ++it) {
    const int64_t vi = threadIdx.x + int64_t(it) * THREADS;
    if (vi < nvec) emit(vi, s[it], wraw[HAS_W ? it : 0]);
  }
  for (int64_t vi = threadIdx.x + int64_t(kMaxItems) * THREADS; vi < nvec; vi += THREADS) {
    float t[VEC];
    // the fused path already wrote the summed row into residual
    if constexpr (FUSED) {
      load_f<T, VEC>(rr + vi * VEC, t);
    } else {
      load_f<T, VEC>(xr + vi * VEC, t);
    }
    V w{};
    if constexpr (HAS_W) w = *reinterpret_cast<const V*>(weight + vi * VEC);
    emit(vi, t, w);
  }
}

template <typename T, int VEC, bool FUSED, bool HAS_W, bool GEMMA>
int launch_rows(T* out, T* residual, const T* x, const T* w, int64_t rows, int64_t hidden,
                int64_t xs, int64_t rs, int64_t os, float eps, cudaStream_t stream) {
  const int64_t nvec = hidden / VEC;
  const int64_t want = ceil_div(nvec, kMaxItems);
#define NTB200_RMS_LAUNCH(TH)                                                                 \
  return launch_kernel("rms_norm", rms_norm_kernel<T, VEC, TH, FUSED, HAS_W, GEMMA>,         \
                       dim3(static_cast<unsigned>(rows)), dim3(TH), 0, stream, out, residual, x, w, \
                       hidden, xs, rs, os, eps)
  if (want <= 64) NTB200_RMS_LAUNCH(64);
  if (want <= 128) NTB200_RMS_LAUNCH(128);
  if (want <= 256) NTB200_RMS_LAUNCH(256);
  if (want <= 512) NTB200_RMS_LAUNCH(512);
  NTB200_RMS_LAUNCH(1024);
#undef NTB200_RMS_LAUNCH
}

template <typename T, int VEC, bool FUSED>
int launch_weighted(T* out, T* residual, const T* x, const T* w, int64_t rows, int64_t hidden,
                    int64_t xs, int64_t rs, int64_t os, float eps, bool gemma, cudaStream_t stream) {
  if (gemma)
    return launch_rows<T, VEC, FUSED, true, true>(out, residual, x, w, rows, hidden, xs, rs, os, eps, stream);
  if (w != nullptr)
    return launch_rows<T, VEC, FUSED, true, false>(out, residual, x, w, rows, hidden, xs, rs, os, eps, stream);
  return launch_rows<T, VEC, FUSED, false, false>(out, residual, x, w, rows, hidden, xs, rs, os, eps, stream);
}

template <typename T, bool FUSED>
int dispatch_vec(void* out, void* residual, const void* x, const void* w, int64_t rows,
                 int64_t hidden, int64_t xs, int64_t rs, int64_t os, float eps, bool gemma,
                 cudaStream_t stream) {
  constexpr int kVec = 16 / sizeof(T);
  const bool vec_ok = hidden % kVec == 0 && xs % kVec == 0 && os % kVec == 0 &&
                      (!FUSED || rs % kVec == 0) && aligned16(x) && aligned16(out) &&
                      (!FUSED || aligned16(residual)) && (w == nullptr || aligned16(w));
  T* o = static_cast<T*>(out);
  T* r = static_cast<T*>(residual);
  const T* xi = static_cast<const T*>(x);
  const T* wi = static_cast<const T*>(w);
  if (vec_ok) return launch_weighted<T, kVec, FUSED>(o, r, xi, wi, rows, hidden, xs, rs, os, eps, gemma, stream);
  return launch_weighted<T, 1, FUSED>(o, r, xi, wi, rows, hidden, xs, rs, os, eps, gemma, stream);
}

template <bool FUSED>
int rms_entry(void* out, void* residual, const void* x, const void* w, int64_t rows,
              int64_t hidden, int64_t xs, int64_t rs, int64_t os, float eps, int dtype,
              void* stream, bool gemma = false) {
  if (rows < 0 || hidden <= 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm: bad shape");
  if (gemma && w == nullptr) return fail(NTB200_ERR_INVALID_ARGUMENT, "gemma_rms_norm: weight is required");
  // vLLM's Gemma norm sums an fp16 residual in fp32 and hands back an fp32 residual, which
  // an in-place fp16 residual buffer cannot hold
  if (gemma && FUSED && dtype == NTB200_DTYPE_F16)
    return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "gemma_fused_add_rms_norm: fp16 (the residual would be fp32)");
  if (rows == 0) return NTB200_OK;
  if (rows > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rms_norm: too many rows");
  if (out == nullptr || x == nullptr || (FUSED && residual == nullptr))
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm: null pointer");
  if (xs < hidden || os < hidden || (FUSED && rs < hidden))
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm: row stride smaller than hidden");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NTB200_DTYPE_F32:
      return dispatch_vec<float, FUSED>(out, residual, x, w, rows, hidden, xs, rs, os, eps, gemma, s);
    case NTB200_DTYPE_BF16:
      return dispatch_vec<__nv_bfloat16, FUSED>(out, residual, x, w, rows, hidden, xs, rs, os,
                                                eps, gemma, s);
    case NTB200_DTYPE_F16:
      return dispatch_vec<__half, FUSED>(out, residual, x, w, rows, hidden, xs, rs, os, eps, gemma, s);
    default:
      return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "rms_norm: dtype %d", dtype);
  }
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_rms_norm(void* out, const void* x, const void* weight, int64_t num_rows,
                               int64_t hidden, int64_t x_row_stride, int64_t out_row_stride,
                               float eps, int dtype, void* stream) {
  return ntb200::rms_entry<false>(out, nullptr, x, weight, num_rows, hidden, x_row_stride,
                                  hidden, out_row_stride, eps, dtype, stream);
}

extern "C" int ntb200_fused_add_rms_norm(void* out, void* residual, const void* x,
                                         const void* weight, int64_t num_rows, int64_t hidden,
                                         int64_t x_row_stride, int64_t residual_row_stride,
                                         int64_t out_row_stride, float eps, int dtype,
                                         void* stream) {
  return ntb200::rms_entry<true>(out, residual, x, weight, num_rows, hidden, x_row_stride,
                                 residual_row_stride, out_row_stride, eps, dtype, stream);
}

extern "C" int ntb200_gemma_rms_norm(void* out, const void* x, const void* weight, int64_t num_rows,
                                     int64_t hidden, int64_t x_row_stride, int64_t out_row_stride,
                                     float eps, int dtype, void* stream) {
  return ntb200::rms_entry<false>(out, nullptr, x, weight, num_rows, hidden, x_row_stride, hidden,
                                  out_row_stride, eps, dtype, stream, true);
}

extern "C" int ntb200_gemma_fused_add_rms_norm(void* out, void* residual, const void* x,
                                               const void* weight, int64_t num_rows, int64_t hidden,
                                               int64_t x_row_stride, int64_t residual_row_stride,
                                               int64_t out_row_stride, float eps, int dtype,
                                               void* stream) {
  return ntb200::rms_entry<true>(out, residual, x, weight, num_rows, hidden, x_row_stride,
                                 residual_row_stride, out_row_stride, eps, dtype, stream, true);
}

// RMS norm and fused residual-add RMS norm.
//
// One CTA per row.  Every thread issues all of its 128-bit loads of the row up front
// (x, and the residual when fused), keeps the fp32 sum in registers, writes the new
// residual, reduces sum(s^2) with warp shuffles + one shared-memory step, then streams
// weight*normalised values out.  HBM traffic is the algorithmic minimum: x (+residual)
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
#include "common.cuh"

namespace ntb200 {
namespace {

constexpr int kMaxItems = 4;  // vectors per thread kept in registers

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

// T: storage type; VEC: elements per vector access; THREADS: CTA size.
// Rows with more than THREADS*kMaxItems vectors take a second pass (re-reading x and
// residual from L2) -- the register-resident path covers hidden <= 32768 bf16.
template <typename T, int VEC, int THREADS, bool FUSED>
__global__ void __launch_bounds__(THREADS) rms_norm_kernel(
    T* out, T* __restrict__ residual, const T* x, const T* __restrict__ weight, int64_t hidden, int64_t x_stride, int64_t r_stride,
    int64_t o_stride, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * x_stride;
  T* rr = FUSED ? residual + row * r_stride : nullptr;
  T* orow = out + row * o_stride;
  const int64_t nvec = hidden / VEC;

  float s[kMaxItems][VEC];
  float sumsq = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxItems; ++it) {
    const int64_t vi = threadIdx.x + int64_t(it) * THREADS;
    if (vi < nvec) {
      load_f<T, VEC>(xr + vi * VEC, s[it]);
      if constexpr (FUSED) {
        float r[VEC];
        load_f<T, VEC>(rr + vi * VEC, r);
#pragma unroll
        for (int j = 0; j < VEC; ++j) s[it][j] += r[j];
        store_f<T, VEC>(rr + vi * VEC, s[it]);
      }
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
      for (int j = 0; j < VEC; ++j) t[j] += r[j];
      store_f<T, VEC>(rr + vi * VEC, t);
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) sumsq += t[j] * t[j];
  }

  // weight of the register-resident vectors, fetched before the reduction so that its
  // latency overlaps the block-wide sum
  Vec<T, VEC> wraw[kMaxItems];
#pragma unroll
  for (int it = 0; it < kMaxItems; ++it) {
    const int64_t vi = threadIdx.x + int64_t(it) * THREADS;
    if (weight != nullptr && vi < nvec) wraw[it] = *reinterpret_cast<const Vec<T, VEC>*>(weight + vi * VEC);
  }

  const float total = block_sum<THREADS>(sumsq, red);
  const float rstd = rsqrtf(total / static_cast<float>(hidden) + eps);

  auto emit_w = [&](int64_t vi, const float (&v)[VEC], const Vec<T, VEC>* w) {
    float y[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float wj = w != nullptr ? Elem<T>::to_f(w->v[j]) : 1.f;
      y[j] = Elem<T>::round(v[j] * rstd) * wj;
    }
    store_f<T, VEC>(orow + vi * VEC, y);
  };
  auto emit = [&](int64_t vi, const float (&v)[VEC]) {
    if (weight != nullptr) {
      const Vec<T, VEC> w = *reinterpret_cast<const Vec<T, VEC>*>(weight + vi * VEC);
      emit_w(vi, v, &w);
    } else {
      emit_w(vi, v, nullptr);
    }
  };
#pragma unroll
  for (int it = 0; it < kMaxItems; ++it) {
    const int64_t vi = threadIdx.x + int64_t(it) * THREADS;
    if (vi < nvec) emit_w(vi, s[it], weight != nullptr ? &wraw[it] : nullptr);
  }
  for (int64_t vi = threadIdx.x + int64_t(kMaxItems) * THREADS; vi < nvec; vi += THREADS) {
    float t[VEC];
    // the fused path already wrote the summed row into residual
    if constexpr (FUSED) {
      load_f<T, VEC>(rr + vi * VEC, t);
    } else {
      load_f<T, VEC>(xr + vi * VEC, t);
    }
    emit(vi, t);
  }
}

template <typename T, int VEC, bool FUSED>
int launch_rows(T* out, T* residual, const T* x, const T* w, int64_t rows, int64_t hidden,
                int64_t xs, int64_t rs, int64_t os, float eps, cudaStream_t stream) {
  const int64_t nvec = hidden / VEC;
  const int64_t want = ceil_div(nvec, kMaxItems);
#define NTB200_RMS_LAUNCH(TH)                                                            \
  rms_norm_kernel<T, VEC, TH, FUSED><<<static_cast<unsigned>(rows), TH, 0, stream>>>( \
      out, residual, x, w, hidden, xs, rs, os, eps)
  if (want <= 32) {
    NTB200_RMS_LAUNCH(32);
  } else if (want <= 64) {
    NTB200_RMS_LAUNCH(64);
  } else if (want <= 128) {
    NTB200_RMS_LAUNCH(128);
  } else if (want <= 256) {
    NTB200_RMS_LAUNCH(256);
  } else {
    // 512 threads keep 4 vectors each in registers without spilling; longer rows take
    // the second (L2) pass
    NTB200_RMS_LAUNCH(512);
  }
#undef NTB200_RMS_LAUNCH
  return check_launch("rms_norm");
}

template <typename T, bool FUSED>
int dispatch_vec(void* out, void* residual, const void* x, const void* w, int64_t rows,
                 int64_t hidden, int64_t xs, int64_t rs, int64_t os, float eps,
                 cudaStream_t stream) {
  constexpr int kVec = 16 / sizeof(T);
  const bool vec_ok = hidden % kVec == 0 && xs % kVec == 0 && os % kVec == 0 &&
                      (!FUSED || rs % kVec == 0) && aligned16(x) && aligned16(out) &&
                      (!FUSED || aligned16(residual)) && (w == nullptr || aligned16(w));
  T* o = static_cast<T*>(out);
  T* r = static_cast<T*>(residual);
  const T* xi = static_cast<const T*>(x);
  const T* wi = static_cast<const T*>(w);
  if (vec_ok) return launch_rows<T, kVec, FUSED>(o, r, xi, wi, rows, hidden, xs, rs, os, eps, stream);
  return launch_rows<T, 1, FUSED>(o, r, xi, wi, rows, hidden, xs, rs, os, eps, stream);
}

template <bool FUSED>
int rms_entry(void* out, void* residual, const void* x, const void* w, int64_t rows,
              int64_t hidden, int64_t xs, int64_t rs, int64_t os, float eps, int dtype,
              void* stream) {
  if (rows < 0 || hidden <= 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm: bad shape");
  if (rows == 0) return NTB200_OK;
  if (rows > 0x7fffffff) return fail(NTB200_ERR_UNSUPPORTED_SHAPE, "rms_norm: too many rows");
  if (out == nullptr || x == nullptr || (FUSED && residual == nullptr))
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm: null pointer");
  if (xs < hidden || os < hidden || (FUSED && rs < hidden))
    return fail(NTB200_ERR_INVALID_ARGUMENT, "rms_norm: row stride smaller than hidden");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NTB200_DTYPE_F32:
      return dispatch_vec<float, FUSED>(out, residual, x, w, rows, hidden, xs, rs, os, eps, s);
    case NTB200_DTYPE_BF16:
      return dispatch_vec<__nv_bfloat16, FUSED>(out, residual, x, w, rows, hidden, xs, rs, os,
                                                eps, s);
    case NTB200_DTYPE_F16:
      return dispatch_vec<__half, FUSED>(out, residual, x, w, rows, hidden, xs, rs, os, eps, s);
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

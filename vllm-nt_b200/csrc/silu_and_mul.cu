// silu_and_mul: out[r, i] = silu(x[r, i]) * x[r, d + i] in one pass (read 2d, write d).
//
// The reference runs a silu kernel on the strided left half into a temporary and then a
// torch multiply (vllm_nt/_ntops/oot_support.py:51-56): three passes over HBM.  Here each
// thread loads one 128-bit vector of the gate half and the matching vector of the up
// half, and writes one vector of the output.
//
// Rounding follows vLLM's torch-native SiluAndMul.forward_native
// (vllm/model_executor/layers/activation.py:137-141): silu is evaluated in fp32 and
// rounded to the storage type, then multiplied by the up value and rounded again.  silu
// uses the fast exponential / division intrinsics (silu_f in common.cuh): with exact expf
// and IEEE division the kernel issued ~80% of its cycles and stopped short of HBM speed.
#include "common.cuh"

namespace ntb200 {
namespace {

template <typename T, int VEC>
__global__ void __launch_bounds__(256) silu_and_mul_kernel(T* __restrict__ out,
                                                            const T* __restrict__ x,
                                                            int64_t d, int64_t x_stride,
                                                            int64_t o_stride) {
  const int64_t row = blockIdx.y;
  const int64_t vi = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_trigger();
  if (vi * VEC >= d) return;
  const T* xr = x + row * x_stride;
  pdl_wait();
  float g[VEC], u[VEC], y[VEC];
  load_f<T, VEC>(xr + vi * VEC, g);
  load_f<T, VEC>(xr + d + vi * VEC, u);
#pragma unroll
  for (int j = 0; j < VEC; ++j) y[j] = Elem<T>::round(silu_f(g[j])) * u[j];
  store_f<T, VEC>(out + row * o_stride + vi * VEC, y);
}

template <typename T>
int launch(void* out, const void* x, int64_t rows, int64_t d, int64_t xs, int64_t os,
           cudaStream_t stream) {
  constexpr int kVec = 16 / sizeof(T);
  const bool vec_ok = d % kVec == 0 && xs % kVec == 0 && os % kVec == 0 && aligned16(x) &&
                      aligned16(out);
  const int threads = 256;
  if (vec_ok) {
    dim3 grid(static_cast<unsigned>(ceil_div(d / kVec, threads)), static_cast<unsigned>(rows));
    return launch_kernel("silu_and_mul", silu_and_mul_kernel<T, kVec>, grid, dim3(threads), 0,
                         stream, static_cast<T*>(out), static_cast<const T*>(x), d, xs, os);
  }
  dim3 grid(static_cast<unsigned>(ceil_div(d, threads)), static_cast<unsigned>(rows));
  return launch_kernel("silu_and_mul", silu_and_mul_kernel<T, 1>, grid, dim3(threads), 0, stream,
                       static_cast<T*>(out), static_cast<const T*>(x), d, xs, os);
}

}  // namespace
}  // namespace ntb200

extern "C" int ntb200_silu_and_mul(void* out, const void* x, int64_t num_rows, int64_t d,
                                   int64_t x_row_stride, int64_t out_row_stride, int dtype,
                                   void* stream) {
  using namespace ntb200;
  if (num_rows < 0 || d < 0) return fail(NTB200_ERR_INVALID_ARGUMENT, "silu_and_mul: bad shape");
  if (num_rows == 0 || d == 0) return NTB200_OK;
  if (num_rows > 65535) {
    // grid.y limit: split the rows into chunks of 65535
    const int sz = dtype_size(dtype);
    if (sz == 0) return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "silu_and_mul: dtype %d", dtype);
    for (int64_t r0 = 0; r0 < num_rows; r0 += 65535) {
      const int64_t n = num_rows - r0 < 65535 ? num_rows - r0 : 65535;
      const int st = ntb200_silu_and_mul(
          static_cast<char*>(out) + r0 * out_row_stride * sz,
          static_cast<const char*>(x) + r0 * x_row_stride * sz, n, d, x_row_stride,
          out_row_stride, dtype, stream);
      if (st != NTB200_OK) return st;
    }
    return NTB200_OK;
  }
  if (out == nullptr || x == nullptr) return fail(NTB200_ERR_INVALID_ARGUMENT, "silu_and_mul: null pointer");
  if (x_row_stride < 2 * d || out_row_stride < d)
    return fail(NTB200_ERR_INVALID_ARGUMENT, "silu_and_mul: row stride too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NTB200_DTYPE_F32: return launch<float>(out, x, num_rows, d, x_row_stride, out_row_stride, s);
    case NTB200_DTYPE_BF16:
      return launch<__nv_bfloat16>(out, x, num_rows, d, x_row_stride, out_row_stride, s);
    case NTB200_DTYPE_F16: return launch<__half>(out, x, num_rows, d, x_row_stride, out_row_stride, s);
    default: return fail(NTB200_ERR_UNSUPPORTED_DTYPE, "silu_and_mul: dtype %d", dtype);
  }
}

// Shared host/device helpers of libntb200 (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <utility>

#include "ntb200.h"

namespace ntb200 {

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------

// Records a printf-style detail for ntb200_last_error() on this thread; returns status.
int fail(int status, const char* fmt, ...);
// Converts a pending launch error into NTB200_ERR_CUDA (with the CUDA error string).
int check_launch(const char* what);
// Device address of the current device's error word (resolved once per device).
unsigned int* device_error_word();
// Number of SMs of the current device (cached per device).
int num_sms();

// Raises `func`'s dynamic shared-memory limit to `bytes` once per device (so that calls
// made later, e.g. inside CUDA-graph capture, never touch the attribute again).
// `slot` identifies the kernel instantiation (a small per-file constant).
int ensure_smem_attribute(const void* func, int bytes, int slot);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int dtype_size(int dtype) {
  switch (dtype) {
    case NTB200_DTYPE_F32: return 4;
    case NTB200_DTYPE_BF16: return 2;
    case NTB200_DTYPE_F16: return 2;
    case NTB200_DTYPE_I32: return 4;
    case NTB200_DTYPE_I64: return 8;
    default: return 0;
  }
}
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Programmatic dependent launch.  Every kernel of the library is launched with
// programmatic stream serialization allowed, so that its launch and its prologue (index
// math, shared-memory and mbarrier set-up) overlap the tail of the kernel before it on the
// stream.  Each kernel calls pdl_wait() before its first global-memory access (read or
// write) and before it allocates tensor memory; pdl_wait() returns once the preceding
// kernel has completed and its writes are visible, so results are those of plain stream
// order.  NTB200_PDL=0 in the environment (read once per process) launches without it.
bool pdl_enabled();

inline void set_pdl_attribute(cudaLaunchAttribute& a) {
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
}

// Launches `kernel` on `stream` with the programmatic-serialization attribute; returns
// NTB200_OK or NTB200_ERR_CUDA (with `what` in the detail).
template <typename... KArgs, typename... Args>
int launch_kernel(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                  size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_pdl_attribute(attr[0]);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return NTB200_OK;
}

// ------------------------------------------------------------------------------------
// device side: element conversion
// ------------------------------------------------------------------------------------

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  // rounds an fp32 intermediate to the storage precision (identity for fp32)
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

// Two fp32 values to the storage type with one paired conversion (cvt.rn.{bf16x2,f16x2}.f32:
// round to nearest even, the same bits as two scalar conversions).  round() rounds in place
// (identity for fp32); store() writes the pair to two adjacent elements (4-byte aligned).
template <typename T> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ void round(float&, float&) {}
  static __device__ __forceinline__ void store(float* dst, float a, float b) {
    dst[0] = a;
    dst[1] = b;
  }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ void round(float& a, float& b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    a = __low2float(h);
    b = __high2float(h);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* dst, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a, b);
  }
};
template <> struct Pair<__half> {
  static __device__ __forceinline__ void round(float& a, float& b) {
    const __half2 h = __floats2half2_rn(a, b);
    a = __low2float(h);
    b = __high2float(h);
  }
  static __device__ __forceinline__ void store(__half* dst, float a, float b) {
    *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(a, b);
  }
};

// A 16-byte (or narrower) vector of N elements of T, loaded/stored as one transaction.
template <typename T, int N>
struct __align__(sizeof(T) * N) Vec {
  T v[N];
};

template <typename T, int N>
__device__ __forceinline__ void load_f(const T* p, float (&out)[N]) {
  Vec<T, N> raw = *reinterpret_cast<const Vec<T, N>*>(p);
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = Elem<T>::to_f(raw.v[i]);
}
// Converts N fp32 values to a vector of T, two at a time with the paired conversion where
// N is even (the same bits as N scalar conversions).
template <typename T, int N>
__device__ __forceinline__ Vec<T, N> pack_f(const float (&in)[N]) {
  Vec<T, N> raw;
  if constexpr (N % 2 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 2) Pair<T>::store(&raw.v[i], in[i], in[i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) raw.v[i] = Elem<T>::from_f(in[i]);
  }
  return raw;
}

template <typename T, int N>
__device__ __forceinline__ void store_f(T* p, const float (&in)[N]) {
  Vec<T, N> raw;
#pragma unroll
  for (int i = 0; i < N; ++i) raw.v[i] = Elem<T>::from_f(in[i]);
  *reinterpret_cast<Vec<T, N>*>(p) = raw;
}

// silu(g) = g / (1 + e^-g) in fp32 with the fast exponential and division intrinsics (a
// few ulp, far inside the bf16/fp16 rounding that follows and the 1e-5 fp32 tolerance);
// shared by silu_and_mul and the fused gate_up GEMM epilogue so that the two agree bit for bit.
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Waits until the kernel before this one on the stream has completed (no-op when the
// launch did not allow programmatic serialization).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allows the next kernel on the stream to launch once every CTA of this grid has called
// it (or exited); that kernel still waits for this one's completion in its pdl_wait().
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void raise_device_error(unsigned int* word, unsigned int bit) {
  if (word != nullptr) atomicOr(word, bit);
}

// ------------------------------------------------------------------------------------
// device side: mbarrier / async-proxy helpers with bounded waits
// ------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` for at most ~timeout_ns.  Returns false (and raises
// NTB200_DEVERR_WAIT_TIMEOUT) when the wait gave up, so that no kernel can spin forever.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitTimeoutNs) {
      raise_device_error(err, NTB200_DEVERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

}  // namespace ntb200

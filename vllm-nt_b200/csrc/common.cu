// Host-side plumbing of libntb200: status strings, the per-thread error detail, the
// per-device error word that bounded device waits and range checks report into.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace ntb200 {

namespace {
thread_local char g_last_error[512] = "";

// One word per device; a device-side check sets bits with atomicOr, the host reads and
// clears it through ntb200_read_device_error().
__device__ unsigned int g_device_error_word;

constexpr int kMaxDevices = 64;
std::once_flag g_resolve_once[kMaxDevices];
unsigned int* g_error_word_addr[kMaxDevices];
int g_sm_count[kMaxDevices];
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(NTB200_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return NTB200_OK;
}

static void resolve_device(int dev) {
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_device_error_word) != cudaSuccess) {
    cudaGetLastError();
    addr = nullptr;
  }
  g_error_word_addr[dev] = static_cast<unsigned int*>(addr);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;
  }
  g_sm_count[dev] = sms;
}

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return 0;
  }
  return dev;
}

unsigned int* device_error_word() {
  const int dev = current_device();
  std::call_once(g_resolve_once[dev], resolve_device, dev);
  return g_error_word_addr[dev];
}

int num_sms() {
  const int dev = current_device();
  std::call_once(g_resolve_once[dev], resolve_device, dev);
  return g_sm_count[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("NTB200_PDL");
    return !(v != nullptr && v[0] == '0' && v[1] == 0);
  }();
  return on;
}

namespace {
constexpr int kAttrSlots = 128;
std::atomic<int> g_attr_done[kMaxDevices][kAttrSlots];
}  // namespace

int ensure_smem_attribute(const void* func, int bytes, int slot) {
  const int dev = current_device();
  if (slot < 0 || slot >= kAttrSlots) return fail(NTB200_ERR_INVALID_ARGUMENT, "attribute slot %d", slot);
  if (g_attr_done[dev][slot].load(std::memory_order_acquire) >= bytes) return NTB200_OK;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NTB200_ERR_CUDA, "cudaFuncSetAttribute(%d bytes): %s", bytes, cudaGetErrorString(e));
  }
  g_attr_done[dev][slot].store(bytes, std::memory_order_release);
  return NTB200_OK;
}

}  // namespace ntb200

extern "C" {

int ntb200_version(void) { return 1; }

const char* ntb200_status_string(int status) {
  switch (status) {
    case NTB200_OK: return "ok";
    case NTB200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NTB200_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case NTB200_ERR_MISALIGNED: return "misaligned pointer or stride";
    case NTB200_ERR_WORKSPACE: return "workspace missing or too small";
    case NTB200_ERR_CUDA: return "CUDA error";
    case NTB200_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case NTB200_ERR_DEVICE: return "device-side error";
    default: return "unknown status";
  }
}

const char* ntb200_last_error(void) { return ntb200::g_last_error; }

int ntb200_read_device_error(int* word, void* stream) {
  if (word == nullptr) return ntb200::fail(NTB200_ERR_INVALID_ARGUMENT, "word is null");
  unsigned int* addr = ntb200::device_error_word();
  if (addr == nullptr) return ntb200::fail(NTB200_ERR_CUDA, "device error word unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int host = 0;
  if (cudaMemcpyAsync(&host, addr, sizeof(host), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemsetAsync(addr, 0, sizeof(unsigned int), s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    return ntb200::fail(NTB200_ERR_CUDA, "reading device error word: %s",
                        cudaGetErrorString(cudaGetLastError()));
  }
  *word = static_cast<int>(host);
  return NTB200_OK;
}

}  // extern "C"

// Error reporting, device queries and the library-wide entry points of the C ABI.
#include <mutex>

#include "fw_host.h"

namespace fw {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

cudaError_t ensure_smem_raw(const void* kernel, int bytes) {
  struct Entry {
    const void* kernel;
    int device;
    int bytes;
  };
  static std::mutex mu;
  static Entry table[256];
  static int used = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].kernel == kernel && table[i].device == dev && table[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  for (int i = 0; i < used; ++i)
    if (table[i].kernel == kernel && table[i].device == dev) {
      table[i].bytes = bytes;
      return cudaSuccess;
    }
  if (used < 256) table[used++] = Entry{kernel, dev, bytes};
  return cudaSuccess;
}

bool device_is_sm100() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

EncodeTiledFn tensor_map_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace fw

extern "C" {

const char* fw_last_error_string(void) { return fw::g_last_error.c_str(); }

int fw_version(void) { return 1; }

int fw_device_error(unsigned int* bits, int clear) {
  FW_REQUIRE(bits != nullptr, FW_ERR_NULL, "fw_device_error: bits is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fw::set_error(FW_ERR_LAUNCH, "fw_device_error: %s", cudaGetErrorString(e));
  *bits = fw::read_decode_errors(clear != 0) | fw::read_logmel_errors(clear != 0) |
          fw::read_encoder_errors(clear != 0);
  return FW_OK;
}

}  // extern "C"

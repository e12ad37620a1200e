// Host-side helpers shared by the C-ABI entry points: error strings, argument checks, device
// properties and the per-kernel shared-memory opt-in.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/flash_whisper.h"

namespace fw {

// Records a message for fw_last_error_string() and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

// Number of SMs of the current device (cached per device).
int num_sms();
// True when the current device is compute capability 10.x.
bool device_is_sm100();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Turns the status of a just-issued launch into an FW status.
inline int launch_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FW_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return FW_OK;
}

// Raises the dynamic shared-memory limit of `kernel` to at least `bytes` (once per kernel, device
// and size; later calls are a table lookup).
cudaError_t ensure_smem_raw(const void* kernel, int bytes);
template <typename K>
inline cudaError_t ensure_smem(K kernel, int bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  return ensure_smem_raw(reinterpret_cast<const void*>(kernel), bytes);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr if unavailable).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encode_fn();

// Device error words of each translation unit (defined next to the kernels).
unsigned int read_decode_errors(bool clear);
unsigned int read_logmel_errors(bool clear);
unsigned int read_encoder_errors(bool clear);

}  // namespace fw

#define FW_REQUIRE(cond, code, ...)                 \
  do {                                              \
    if (!(cond)) return fw::set_error(code, __VA_ARGS__); \
  } while (0)

// Internal declarations shared by the engine's translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/sf_engine.h"

namespace sf {

// Record `msg` as the calling thread's last error and return `code`.
int32_t fail(int32_t code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Translate a CUDA runtime error into SF_ERR_CUDA (with context) or SF_OK.
int32_t cuda_status(cudaError_t e, const char* what);

#define SF_CUDA_TRY(expr)                                  \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return ::sf::cuda_status(_e, #expr); \
  } while (0)

struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t smem_optin = 0;
  int* err_word = nullptr;  // device-side error word (cudaMalloc'd once per device)
};

// Lazily initialised per-device facts for the CURRENT device.
int32_t current_device_info(DeviceInfo** out, int* device);

// Error word of the no-alloc entry point on the CURRENT device (a static
// device array, so that entry point never allocates): read into *value and
// reset to zero when `clear`.  Reported by sf_device_error_status together
// with the per-device word above.
int32_t noalloc_error_word(int* value, bool clear);

// Releases the fused attention's stream-K tail workspace held for `stream`
// (called by sf_stream_destroy before the stream goes away).
void attention_release_stream(void* stream);

// Global knobs.
int fp32_mode();
int kernel_override();

}  // namespace sf

// common.cuh — helpers shared by the source files of libaugur_kv.so (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace augur_kv_dev {

constexpr int kMaxDevices = 64;

// Text of the last error on this host thread (augur_kv_last_error).
extern thread_local char g_last_error[512];
// Guards the per-device launch-configuration caches (recursive: cached
// queries such as sm_count may run while a caller holds it).
extern std::recursive_mutex g_cache_mutex;

// Record an error message and return `code`.
int fail(int code, const char* fmt, ...);
// AUGUR_KV_ECUDA with the runtime's message if the last launch failed.
int check_launch(const char* what);
// Bytes per element of an AUGUR_KV_* dtype (0 if unknown).
int elem_size(int32_t dtype);
// SM count of the current device (cached).
int sm_count();

// First device-side error wins.
__device__ __forceinline__ void record_status(int32_t* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

}  // namespace augur_kv_dev

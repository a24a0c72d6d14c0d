// Small host helpers shared by the translation units of the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "../../include/flashspec_b200.h"

namespace fsb {

// What lies behind the last FS_ERR_CUDA this thread returned (fs_last_error_detail).
inline thread_local char g_error_detail[256] = "";

inline int fail_cuda(const char* where, cudaError_t e) {
  snprintf(g_error_detail, sizeof(g_error_detail), "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
  return FS_ERR_CUDA;
}

inline int fail_cuda(const char* where, CUresult r) {
  snprintf(g_error_detail, sizeof(g_error_detail), "%s: CUresult %d", where, (int)r);
  return FS_ERR_CUDA;
}

inline int fail_cuda(const char* what) {
  snprintf(g_error_detail, sizeof(g_error_detail), "%s", what);
  return FS_ERR_CUDA;
}

// Status of a launch just issued: FS_OK, or FS_ERR_CUDA with the launch error recorded.
inline int launch_status(const char* kernel) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FS_OK : fail_cuda(kernel, e);
}

constexpr int kMaxDevices = 64;

inline int device_sm_count(int device) {
  static int cached[kMaxDevices] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= kMaxDevices) return 1;
  if (cached[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 1;
    cached[device] = n;
  }
  return cached[device];
}

}  // namespace fsb

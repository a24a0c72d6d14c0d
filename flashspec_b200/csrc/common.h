// Small host helpers shared by the translation units of the library.
#pragma once

#include <cuda_runtime.h>

#include <mutex>

namespace fsb {

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

// fs_read_bandwidth_probe: a read-only HBM stream, the denominator of the decode
// kernels' roofline beside the copy bandwidth.  The decode kernels only read their KV
// bytes (writes are a few MB of outputs), so a copy (read + write) peak understates
// what a pure read stream reaches; this kernel measures the latter on the same GPU in
// the same run.
//
// One persistent grid (resident CTAs of 512 threads); each thread streams 16-byte
// loads with eight in flight, bypassing L1 and marked evict-first in L2, and folds them
// into a 32-bit XOR that the first thread of each CTA stores to sink[blockIdx.x] (so the
// loads cannot be dropped).
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/flashspec_b200.h"
#include "common.h"

namespace fsb {

constexpr int kProbeThreads = 512;
constexpr int kProbeUnroll = 8;

__device__ __forceinline__ uint4 ld_stream(const uint4* p, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

__global__ void __launch_bounds__(kProbeThreads) read_probe_kernel(const uint4* __restrict__ buf, size_t n16,
                                                                     uint32_t* __restrict__ sink) {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  const size_t stride = (size_t)gridDim.x * kProbeThreads;
  size_t i = (size_t)blockIdx.x * kProbeThreads + threadIdx.x;
  uint32_t acc = 0;
  for (; i + (kProbeUnroll - 1) * stride < n16; i += kProbeUnroll * stride) {
    uint4 v[kProbeUnroll];
#pragma unroll
    for (int u = 0; u < kProbeUnroll; ++u) v[u] = ld_stream(buf + i + u * stride, policy);
#pragma unroll
    for (int u = 0; u < kProbeUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  for (; i < n16; i += stride) {
    const uint4 v = ld_stream(buf + i, policy);
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ uint32_t part[kProbeThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t x = 0;
    for (int w = 0; w < kProbeThreads / 32; ++w) x ^= part[w];
    sink[blockIdx.x] = x;
  }
}

}  // namespace fsb

extern "C" int fs_read_bandwidth_probe(const void* buf, size_t bytes, uint32_t* sink, int32_t sink_count,
                                       int32_t* ctas_used, void* stream) {
  using namespace fsb;
  if (buf == nullptr || sink == nullptr || bytes < 16 || (bytes & 15) || sink_count <= 0) return FS_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(buf) & 15) return FS_ERR_ALIGNMENT;
  int device = 0;
  if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
  int per_sm = 0;
  if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, read_probe_kernel, kProbeThreads, 0);
      e != cudaSuccess)
    return fail_cuda("occupancy of the read probe", e);
  int ctas = (per_sm > 0 ? per_sm : 1) * device_sm_count(device);
  if (ctas > sink_count) ctas = sink_count;
  if (ctas_used != nullptr) *ctas_used = ctas;
  read_probe_kernel<<<ctas, kProbeThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(buf), bytes / 16, sink);
  return launch_status("read probe kernel launch");
}

// Peer-memory exchange and merge of per-rank partial (O, LSE) rows, for decode steps
// whose KV pages are split across the GPUs of one node (sequence sharding).
//
// It replaces the collective of that step -- in the reference the combine of split
// partials (_combine_splits_kernel, src/flashspec/triton_fused.py:446-503) runs within one
// GPU; across GPUs the same log-sum-exp rule is applied to one partial per rank.  Each
// rank owns one exchange buffer (cudaMalloc'd here and shared by CUDA IPC handle); every
// rank maps every peer's buffer.  One kernel per step: CTA c takes a slice of rows,
// stores them (plain peer stores over NVLink, no multicast) into every rank's buffer,
// raises its flag there, waits with a time limit for the same slice's flags from all
// ranks, and merges the slice locally.
//
// Buffer layout (bytes): [0, 256) control words (epoch = calls completed, done = CTAs
// finished in the current call); [256, 256 + 4 * kXMaxRanks * kXMaxCtas) flags
// [sender][cta] = epoch the sender's slice belongs to; then the data, two epoch
// parities x kXMaxRanks slots of slot_floats floats (O [rows][D], then LSE [rows]).
// Parity: a peer may begin its next call as soon as it has this rank's flags, so its next
// rows land in the other parity while this rank still reads the current one; it cannot
// get two calls ahead, as that needs this rank's flags of the next call.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/flashspec_b200.h"
#include "common.h"
#include "ptx.cuh"

namespace fsb {

constexpr int kXMaxRanks = FS_EXCHANGE_MAX_RANKS;
constexpr int kXMaxCtas = 64;
constexpr int kXThreads = 256;
constexpr size_t kXCtrlBytes = 256;
constexpr size_t kXFlagBytes = 4ull * kXMaxRanks * kXMaxCtas;
constexpr size_t kXDataOffset = kXCtrlBytes + kXFlagBytes;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kXThreads) exchange_merge_kernel(const FsExchangeArgs a, int rows_per_cta) {
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x, c = blockIdx.x;
  const int D = a.head_dim;
  const int64_t r0 = (int64_t)c * rows_per_cta;
  const int64_t r1 = r0 + rows_per_cta < a.rows ? r0 + rows_per_cta : a.rows;
  uint8_t* own = static_cast<uint8_t*>(a.bufs[a.rank]);
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(own);
  if (tid == 0) s_epoch = ld_acquire_sys(ctrl) + 1u;  // the call this launch is
  __syncthreads();
  const uint32_t e = s_epoch;
  const size_t parity_off = kXDataOffset + (size_t)(e & 1u) * kXMaxRanks * a.slot_floats * 4;

  // 1. this rank's rows of the slice into slot [rank] of every rank's buffer
  const int64_t nO = (r1 - r0) * D;
  for (int p = 0; p < a.world; ++p) {
    float* dst = reinterpret_cast<float*>(static_cast<uint8_t*>(a.bufs[p]) + parity_off) + (size_t)a.rank * a.slot_floats;
    for (int64_t i = tid; i < nO / 4; i += kXThreads)
      reinterpret_cast<float4*>(dst + r0 * D)[i] = reinterpret_cast<const float4*>(a.o_mine + r0 * D)[i];
    for (int64_t r = r0 + tid; r < r1; r += kXThreads) dst[a.rows * D + r] = a.lse_mine[r];
  }
  __threadfence_system();  // this thread's stores are visible system-wide before the flags
  __syncthreads();
  // 2. raise this slice's flag in every rank's buffer
  if (tid < a.world) {
    uint32_t* fl = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a.bufs[tid]) + kXCtrlBytes);
    st_release_sys(fl + a.rank * kXMaxCtas + c, e);
  }
  // 3. wait (bounded) for the slice's flags of every rank
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (tid < a.world) {
    const uint32_t* fl = reinterpret_cast<const uint32_t*>(own + kXCtrlBytes) + tid * kXMaxCtas + c;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(fl) - e) < 0) {  // a peer may already be one call ahead
      if (globaltimer_ns() - t0 > (uint64_t)a.timeout_ns) {
        s_ok = 0;
        if (a.device_status != nullptr) atomicOr(a.device_status, FS_DEV_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  // 4. merge the slice from the local buffer: out = sum_r w_r O_r / sum_r w_r,
  //    w_r = exp(lse_r - max lse) (triton_fused.py:446-503 on one partial per rank)
  if (s_ok) {
    const float* data = reinterpret_cast<const float*>(own + parity_off);
    for (int64_t i = r0 * D + tid; i < r1 * D; i += kXThreads) {
      const int64_t row = i / D;
      float M = -INFINITY;
      for (int p = 0; p < a.world; ++p) M = fmaxf(M, data[(size_t)p * a.slot_floats + a.rows * D + row]);
      float W = 0.f, O = 0.f;
      if (M != -INFINITY)
        for (int p = 0; p < a.world; ++p) {
          const float l = data[(size_t)p * a.slot_floats + a.rows * D + row];
          const float w = l == -INFINITY ? 0.f : expf(l - M);
          W += w;
          O += w * data[(size_t)p * a.slot_floats + i];
        }
      const float o = W > 0.f ? O / W : 0.f;
      if (a.out_dtype == FS_F16)
        static_cast<__half*>(a.out)[i] = __float2half_rn(o);
      else
        static_cast<float*>(a.out)[i] = o;
    }
  }
  // 5. the last CTA out records the completed call
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(ctrl + 1, 1u) == gridDim.x - 1) {
      ctrl[1] = 0u;
      __threadfence();
      st_release_sys(ctrl, e);
    }
  }
}

size_t exchange_bytes(int64_t slot_floats) { return kXDataOffset + 2ull * kXMaxRanks * (size_t)slot_floats * 4; }

}  // namespace fsb

extern "C" {

int fs_exchange_create(int64_t slot_floats, void** buf, void* ipc_handle) {
  using namespace fsb;
  if (buf == nullptr || ipc_handle == nullptr || slot_floats <= 0 || slot_floats % 64) return FS_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  const size_t bytes = exchange_bytes(slot_floats);
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail_cuda("cudaMalloc of the exchange buffer", e);
  if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess) {
    cudaFree(p);
    return fail_cuda("cudaMemset of the exchange buffer", e);
  }
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
    cudaFree(p);
    return fail_cuda("cudaIpcGetMemHandle of the exchange buffer", e);
  }
  static_assert(sizeof(h) == FS_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return FS_OK;
}

int fs_exchange_open(const void* ipc_handle, void** peer_buf) {
  if (ipc_handle == nullptr || peer_buf == nullptr) return FS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? FS_OK : fsb::fail_cuda("cudaIpcOpenMemHandle of a peer exchange buffer", e);
}

int fs_exchange_close(void* peer_buf) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
  return e == cudaSuccess ? FS_OK : fsb::fail_cuda("cudaIpcCloseMemHandle", e);
}

int fs_exchange_destroy(void* buf) {
  const cudaError_t e = cudaFree(buf);
  return e == cudaSuccess ? FS_OK : fsb::fail_cuda("cudaFree of the exchange buffer", e);
}

int fs_exchange_merge(const FsExchangeArgs* a, void* stream) {
  using namespace fsb;
  if (a == nullptr || a->world < 1 || a->world > kXMaxRanks || a->rank < 0 || a->rank >= a->world || a->rows <= 0 ||
      a->head_dim <= 0 || a->head_dim % 4 || a->o_mine == nullptr || a->lse_mine == nullptr || a->out == nullptr ||
      a->slot_floats < a->rows * (a->head_dim + 1) || a->slot_floats % 64 || a->timeout_ns <= 0)
    return FS_ERR_INVALID_ARGUMENT;
  if (a->out_dtype != FS_F16 && a->out_dtype != FS_F32) return FS_ERR_UNSUPPORTED;
  for (int p = 0; p < a->world; ++p)
    if (a->bufs[p] == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(a->o_mine) & 15) return FS_ERR_ALIGNMENT;
  // slices of whole rows whose O part is a multiple of 4 floats
  int rows_per_cta = (int)((a->rows + kXMaxCtas - 1) / kXMaxCtas);
  const int ctas = (int)((a->rows + rows_per_cta - 1) / rows_per_cta);
  exchange_merge_kernel<<<ctas, kXThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a, rows_per_cta);
  return launch_status("exchange merge kernel launch");
}

}  // extern "C"

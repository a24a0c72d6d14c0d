// Peer-memory exchange and merge of per-rank partial (O, LSE) rows, for decode steps
// whose KV pages are split across the GPUs of one node (sequence sharding).
//
// It replaces the collective of that step -- in the reference the combine of split
// partials (_combine_splits_kernel, src/flashspec/triton_fused.py:446-503) runs within one
// GPU; across GPUs the same log-sum-exp rule is applied to one partial per rank.  Each
// rank owns one exchange buffer (cudaMalloc'd here and shared by CUDA IPC handle); every
// rank maps every peer's buffer.  One kernel per step: CTA c takes a slice of rows,
// stores them (plain peer stores over NVLink, no multicast) into every rank's buffer,
// and merges the slice locally as every rank's words for it arrive, waiting at most
// timeout_ns.
//
// Protocol and buffer layout: xwords.cuh.  Parity: a peer may begin its next call as
// soon as it has this rank's words, so its next words land in the other parity while
// this rank still reads the current one; it cannot get two calls ahead, as that needs
// this rank's words of the next call.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <unordered_map>

#include "../../include/flashspec_b200.h"
#include "common.h"
#include "ptx.cuh"
#include "xwords.cuh"

namespace fsb {

constexpr int kXThreads = 256;

// Slot size of every exchange buffer this process created or mapped, by address.
static std::mutex g_xbuf_mu;
static std::unordered_map<const void*, int64_t> g_xbuf_slots;

static void remember_buffer(const void* p, int64_t slot_floats) {
  std::lock_guard<std::mutex> lock(g_xbuf_mu);
  g_xbuf_slots[p] = slot_floats;
}

static void forget_buffer(const void* p) {
  std::lock_guard<std::mutex> lock(g_xbuf_mu);
  g_xbuf_slots.erase(p);
}

bool exchange_buffers_match(const FsExchangeArgs* a) {
  std::lock_guard<std::mutex> lock(g_xbuf_mu);
  for (int p = 0; p < a->world; ++p) {
    const auto it = g_xbuf_slots.find(a->bufs[p]);
    if (it == g_xbuf_slots.end() || it->second != a->slot_floats) return false;
  }
  return true;
}

__global__ void __launch_bounds__(kXThreads) exchange_merge_kernel(const FsExchangeArgs a, int rows_per_cta) {
  const int tid = threadIdx.x, c = blockIdx.x;
  const int D = a.head_dim;
  const int64_t r0 = (int64_t)c * rows_per_cta;
  const int64_t r1 = r0 + rows_per_cta < a.rows ? r0 + rows_per_cta : a.rows;
  uint8_t* own = static_cast<uint8_t*>(a.bufs[a.rank]);
  uint32_t* calls = reinterpret_cast<uint32_t*>(own);
  const uint32_t e = calls[c] + 1u;  // written by this CTA's previous call on this GPU
  const size_t parity_off = exchange_parity_offset(e, a.slot_floats);
  const int64_t lse_at = a.rows * D;
  const uint64_t deadline = globaltimer_ns() + (uint64_t)a.timeout_ns;

  // 1. this rank's rows of the slice, tagged, into slot [rank] of every rank's buffer
  for (int p = 0; p < a.world; ++p) {
    uint64_t* dst = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(a.bufs[p]) + parity_off) +
                    (size_t)a.rank * a.slot_floats;
    for (int64_t i = r0 * D + tid; i < r1 * D; i += kXThreads) st_word(dst + i, a.o_mine[i], e);
    for (int64_t r = r0 + tid; r < r1; r += kXThreads) st_word(dst + lse_at + r, a.lse_mine[r], e);
  }
  __syncthreads();
  // 2. merge the slice as the words arrive: out = sum_p w_p O_p / sum_p w_p,
  //    w_p = exp(lse_p - max lse) (triton_fused.py:446-503 on one partial per rank).
  //    Once a wait has run out, this thread waits no more and writes NaN for the rest
  //    of its elements, so a timed-out call never leaves plausible-looking output.
  const uint64_t* data = reinterpret_cast<const uint64_t*>(own + parity_off);
  bool ok = true;
  for (int64_t i = r0 * D + tid; i < r1 * D; i += kXThreads) {
    const int64_t row = i / D;
    float lse[kXMaxRanks], o[kXMaxRanks];
    float M = -INFINITY;
#pragma unroll
    for (int p = 0; p < kXMaxRanks; ++p) {
      lse[p] = -INFINITY;
      o[p] = 0.f;
      if (p < a.world && ok) {
        ok = wait_word(data + (size_t)p * a.slot_floats + lse_at + row, e, deadline, lse[p]) &&
             wait_word(data + (size_t)p * a.slot_floats + i, e, deadline, o[p]);
        M = fmaxf(M, lse[p]);
      }
    }
    float W = 0.f, O = 0.f;
    if (ok && M != -INFINITY)
#pragma unroll
      for (int p = 0; p < kXMaxRanks; ++p)
        if (p < a.world) {
          const float w = lse[p] == -INFINITY ? 0.f : expf(lse[p] - M);
          W += w;
          O += w * o[p];
        }
    const float v = !ok ? __int_as_float(0x7fc00000) : W > 0.f ? O / W : 0.f;
    if (a.out_dtype == FS_F16)
      static_cast<__half*>(a.out)[i] = __float2half_rn(v);
    else
      static_cast<float*>(a.out)[i] = v;
  }
  if (!ok && a.device_status != nullptr) atomicOr(a.device_status, FS_DEV_TIMEOUT);
  // 3. record the completed call (read by this CTA's next call on this GPU)
  __syncthreads();
  if (tid == 0) calls[c] = e;
}

size_t exchange_bytes(int64_t slot_floats) { return kXDataOffset + 2ull * kXMaxRanks * (size_t)slot_floats * 8; }

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
  if ((e = cudaMemcpy(static_cast<uint8_t*>(p) + kXSlotSizeOffset, &slot_floats, sizeof(slot_floats),
                      cudaMemcpyHostToDevice)) != cudaSuccess) {
    cudaFree(p);
    return fail_cuda("cudaMemcpy of the exchange buffer's slot size", e);
  }
  if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
    cudaFree(p);
    return fail_cuda("cudaIpcGetMemHandle of the exchange buffer", e);
  }
  remember_buffer(p, slot_floats);
  static_assert(sizeof(h) == FS_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return FS_OK;
}

int fs_exchange_open(const void* ipc_handle, void** peer_buf) {
  if (ipc_handle == nullptr || peer_buf == nullptr) return FS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fsb::fail_cuda("cudaIpcOpenMemHandle of a peer exchange buffer", e);
  int64_t slot_floats = 0;
  e = cudaMemcpy(&slot_floats, static_cast<const uint8_t*>(*peer_buf) + fsb::kXSlotSizeOffset, sizeof(slot_floats),
                 cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    cudaIpcCloseMemHandle(*peer_buf);
    *peer_buf = nullptr;
    return fsb::fail_cuda("cudaMemcpy of a peer exchange buffer's slot size", e);
  }
  fsb::remember_buffer(*peer_buf, slot_floats);
  return FS_OK;
}

int fs_exchange_close(void* peer_buf) {
  fsb::forget_buffer(peer_buf);
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
  return e == cudaSuccess ? FS_OK : fsb::fail_cuda("cudaIpcCloseMemHandle", e);
}

int fs_exchange_destroy(void* buf) {
  fsb::forget_buffer(buf);
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
  // every buffer must come from fs_exchange_create / fs_exchange_open with this slot size:
  // a larger one would make the kernel store past the end of a peer's buffer
  if (!exchange_buffers_match(a)) return FS_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(a->o_mine) & 15) return FS_ERR_ALIGNMENT;
  // slices of whole rows whose O part is a multiple of 4 floats
  int rows_per_cta = (int)((a->rows + kXMaxCtas - 1) / kXMaxCtas);
  const int ctas = (int)((a->rows + rows_per_cta - 1) / rows_per_cta);
  exchange_merge_kernel<<<ctas, kXThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a, rows_per_cta);
  return launch_status("exchange merge kernel launch");
}

}  // extern "C"

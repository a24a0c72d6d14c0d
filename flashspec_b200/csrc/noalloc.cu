// fs_paged_decode_noalloc: paged decode attention that never allocates device memory.
//
// Who needs this: some hosts cannot hand the library a workspace and must not see it
// call cudaMalloc either -- e.g. a plugin running inside an inference server whose
// memory manager owns every device allocation, or a serving loop that cannot afford
// the implicit device synchronisation cudaMalloc/cudaFree may cause.  This entry point
// takes the same FsDecodeArgs as fs_paged_decode, ignores args->workspace/tickets, and
// uses a fixed scratch array compiled into the library instead.
//
// The scratch is one file-scope __device__ array: every GPU that loads the library
// holds its kScratchBytes until the process exits.  Its first kTicketBytes hold the
// split-merge counters, the rest the split-K partial results.  Host code must not pass
// the array's name to a kernel (on the host it only names a stand-in object); the
// device address is obtained once per device with cudaGetSymbolAddress, with that
// device current, on the first call made on that device.  Make that first call before
// any stream capture begins.
//
// All calls share the one array and each call leaves its last contents there:
// calls that can overlap on the GPU (different streams, no ordering) race on it and
// must be serialised by the caller.  Whenever the plan merges partial results (the
// split kernel with more than one split, or the balanced kernel, which merges the
// pieces of a (request, kv head) pair that several warps share) the counters of the
// call's pairs are cleared (cudaMemsetAsync on the call's stream, not an allocation)
// before the launch, so a call that an earlier timeout left with non-zero counters
// still merges correctly.
#include <cuda_runtime.h>

#include <mutex>
#include <stdint.h>

#include "../../include/flashspec_b200.h"
#include "common.h"

namespace fsb {

constexpr size_t kTicketBytes = 256 * 1024;             // 65536 (request, kv head) counters
constexpr size_t kPartialBytes = 8 * 1024 * 1024;       // split partials (O + LSE)
constexpr size_t kScratchBytes = kTicketBytes + kPartialBytes;
constexpr int kHeadDim = 128;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

static size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

// Scratch the decode needs for these arguments with `splits` partitions (same layout
// the workspace of fs_paged_decode uses: partial O fp32 then partial LSE fp32).
static size_t partial_bytes(const FsDecodeArgs* a, int64_t splits) {
  if (splits <= 1) return 0;
  const size_t g = (size_t)(a->q_heads / a->kv_heads);
  const size_t units = (size_t)a->batch * (size_t)a->kv_heads * (size_t)splits * g;
  return round256(units * kHeadDim * 4) + round256(units * 4);
}

static int scratch_address(int device, unsigned char** out) {
  static unsigned char* addr[kMaxDevices] = {};
  static std::mutex mu;
  if (device < 0 || device >= kMaxDevices) return fail_cuda("device ordinal beyond the library's table");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    if (cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch); e != cudaSuccess || p == nullptr)
      return fail_cuda("cudaGetSymbolAddress of the no-alloc scratch", e);
    addr[device] = static_cast<unsigned char*>(p);
  }
  *out = addr[device];
  return FS_OK;
}

}  // namespace fsb

extern "C" int fs_paged_decode_noalloc(const FsDecodeArgs* args, void* stream) {
  using namespace fsb;
  if (args == nullptr || args->layout != FS_LAYOUT_PAGED || args->batch <= 0 || args->kv_heads <= 0 ||
      args->q_heads <= 0 || args->q_heads % args->kv_heads != 0)
    return FS_ERR_INVALID_ARGUMENT;
  if ((int64_t)args->batch * args->kv_heads * 4 > (int64_t)kTicketBytes) return FS_ERR_SCRATCH_LIMIT;
  // An explicit split count is checked against the fixed scratch before any CUDA call.
  if (args->num_splits > 0 && partial_bytes(args, args->num_splits) > kPartialBytes) return FS_ERR_SCRATCH_LIMIT;

  FsDecodeArgs a = *args;
  size_t need = 0;
  int32_t splits = 0;
  int st = fs_decode_workspace_size(&a, &need, &splits);
  if (st != FS_OK) return st;
  if (need > kPartialBytes) return FS_ERR_SCRATCH_LIMIT;
  a.num_splits = splits;  // the launch below must use the split count checked here

  int device = 0;
  if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
  unsigned char* scratch = nullptr;
  if ((st = scratch_address(device, &scratch)) != FS_OK) return st;
  a.tickets = reinterpret_cast<uint32_t*>(scratch);
  a.ticket_count = (int64_t)(kTicketBytes / 4);
  a.workspace = scratch + kTicketBytes;
  a.workspace_bytes = kPartialBytes;
  // fs_decode_workspace_size reports 0 splits for the balanced kernel and 1 for a
  // split kernel that writes the output directly; every other plan uses the counters.
  if (splits != 1) {
    const cudaError_t e =
        cudaMemsetAsync(a.tickets, 0, (size_t)a.batch * a.kv_heads * 4, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail_cuda("cudaMemsetAsync of the no-alloc tickets", e);
  }
  return fs_paged_decode(&a, stream);
}

// Tagged 8-byte words and the buffer layout of the peer-memory exchange, shared by the
// stand-alone exchange kernel (exchange.cu) and the decode kernel's fused exchange
// epilogue (decode.cu).
//
// Every value travels as one naturally aligned 8-byte word (value bits, call epoch):
// the store is single-copy atomic, so a receiver knows a word has arrived when its tag
// equals the epoch it expects, without fences or separate flags.
//
// Buffer layout (bytes):
//   [0, 256)        call counters of the stand-alone kernel, one per CTA (<= 64)
//   [256, 264)      slot size (floats) the buffer was created with
//   [512, 16896)    call counters of the fused decode epilogue, one per (request, kv head)
//                   pair (<= 4096)
//   [16896, ...)    two epoch parities x kXMaxRanks slots of slot_floats words
//                   (O [rows][D], then LSE [rows])
// A buffer serves one of the two modes: their counters are separate, but both use the
// same data slots, so a group must not alternate modes on one set of buffers.
#pragma once

#include <stdint.h>

#include "../../include/flashspec_b200.h"
#include "ptx.cuh"

namespace fsb {

constexpr int kXMaxRanks = FS_EXCHANGE_MAX_RANKS;
constexpr int kXMaxCtas = 64;
constexpr size_t kXCountersBytes = 256;
constexpr size_t kXSlotSizeOffset = kXCountersBytes;
constexpr size_t kXPairCountersOffset = 512;
constexpr int kXMaxPairs = 4096;
constexpr size_t kXDataOffset = kXPairCountersOffset + 4 * kXMaxPairs;
static_assert(kXMaxCtas * 4 <= kXCountersBytes, "call counters");
static_assert(kXDataOffset % 256 == 0, "data slots stay 256-byte aligned");

__host__ __device__ constexpr size_t exchange_parity_offset(uint32_t epoch, int64_t slot_floats) {
  return kXDataOffset + (size_t)(epoch & 1u) * kXMaxRanks * (size_t)slot_floats * 8;
}

__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Value of the word at p once it carries tag e; false when the deadline passes first.
__device__ __forceinline__ bool wait_word(const uint64_t* p, uint32_t e, uint64_t deadline, float& v) {
  for (unsigned n = 0;; ++n) {
    const uint64_t w = ld_word(p);
    if ((uint32_t)(w >> 32) == e) {
      v = __uint_as_float((uint32_t)w);
      return true;
    }
    if ((n & 255u) == 255u && globaltimer_ns() > deadline) return false;
  }
}

// Host: true when every buffer of the call was created or mapped by this process with
// exactly this slot size (exchange.cu keeps the table).
bool exchange_buffers_match(const FsExchangeArgs* a);

}  // namespace fsb

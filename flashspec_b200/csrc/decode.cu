// Decode attention over INT8 KV (contiguous or block_table-paged) for sm_100a.
//
// Replaces the reference Triton kernels _fused_dequant_attention_kernel,
// _fused_dequant_attention_split_kernel, _combine_splits_kernel
// (src/flashspec/triton_fused.py:203-503) and _paged_quant_attention_kernel
// (src/flashspec/triton_paged.py:120-299).  Same math: scores = q.dequant(k)*sm_scale,
// masked softmax over min(len, max_seq_len) tokens, out = softmax . dequant(v),
// fp32 accumulation, fp16 output, empty sequences -> 0 (triton_utils.py:181-186).
//
// Design.  A CTA is 4 consumer warps plus 1 producer warp; 3 CTAs per SM.
//  * A (page, kv head) block is 16 tokens x 128 B of K plus the same of V, contiguous
//    in HBM.  The producer keeps a ring of 16 stages full: 8 lanes issue 8 pages per
//    warp instruction, each two 2-D TMA tile loads (128B-swizzled into shared memory)
//    and 4-byte cp.async copies of the page's scale / zero-point words, completing on
//    the stage's full mbarrier.  Page i goes to consumer warp i % 4, stage i % 16.
//  * QK^T runs on the int8 tensor cores straight from the stored bytes (q held as
//    16-bit fixed point split into two signed bytes, mma.sync m16n8k32 s8); the zero
//    point is applied per page with the exact integer sum of q.  PV runs on fp16
//    tensor cores: a V byte becomes the exact fp16 1024+u (XOR + byte permute against
//    0x64 exponent bytes) and the zero point is subtracted once per piece from a
//    per-row sum of the fp16 probabilities.  The page's V scale is folded into them.
//  * Online softmax in the log2 domain with fp32 (m, l) per query; rescaling only when
//    a row max grows.
//  * Two ways to deal pages: decode_kernel (one CTA per (request, kv head, split); the
//    last CTA of a pair merges the splits' (O, LSE)) and decode_balanced_kernel (a
//    persistent grid, contiguous per-warp shares of all pages, the last contributor of
//    a pair merging its pieces).  The host plan picks one per call.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <algorithm>
#include <mutex>
#include <stdint.h>

#include "../../include/flashspec_b200.h"
#include "common.h"
#include "generic.h"
#include "ptx.cuh"
#include "xwords.cuh"

namespace fsb {

constexpr int kD = 128;
constexpr int kPage = 16;
constexpr int kPageBytes = kPage * kD;     // 2048
constexpr int kStageBytes = 2 * kPageBytes;  // K + V
constexpr int kMetaBytes = 160;  // 32 bytes of page qparams + 128 bytes of per-token scales
constexpr int kMaxG = 8;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint32_t kProducerSleepNs = 1000;  // default suspend hint of the producer's free-stage waits

// The producer's wait for a free stage: suspending (with a time hint) leaves issue slots
// to the consumer warps; hint 0 spins.
__device__ __forceinline__ bool producer_wait(uint32_t bar, uint32_t parity, int sleep_ns) {
  return sleep_ns > 0 ? mbar_wait_sleepy(bar, parity, (uint32_t)sleep_ns, kTimeoutNs)
                      : mbar_spin_bounded(bar, parity, kTimeoutNs);
}

struct DecodeParams {
  const __half* q;
  const float* k_scale;
  const int16_t* k_zero;
  const float* v_scale;
  const int16_t* v_zero;
  const int64_t* table;
  const int64_t* lengths;
  __half* out;
  float* shard_o;
  float* shard_lse;
  float* part_o;
  float* part_lse;
  unsigned* counters;
  uint32_t* status;
  unsigned long long* trace;  // profiling only: per-warp globaltimer stamps, usually null
  int B, Hq, Hkv, G, S, cols;
  int64_t num_blocks;
  int64_t max_seq_len;
  int64_t page_begin, page_end;
  int64_t zp_count;
  float qk_scale_log2;
  int tier_ctas, skew;  // balanced kernel: CTAs per tier (the SM count) and the tier weight step
  int piece_cost;       // balanced kernel: virtual pages charged per (request, kv head) pair
  int debug_mode;       // profiling only (FLASHSPEC_DEBUG_MODE)
  int sym;              // FS_KV_SYMMETRIC: per-token scales [blocks, 16], no zero points
  int producer_sleep_ns;  // suspend hint of the producer's free-stage waits; 0 = spin
  // fused exchange epilogue (fs_paged_decode_exchange); xworld == 0 otherwise
  void* xbufs[kXMaxRanks];
  void* xout;
  uint32_t* xstatus;
  int64_t xslot;
  int64_t xtimeout_ns;
  int xworld, xrank, xout_dtype;
};

// Shared-memory plan of one CTA: a ring of kNS page stages (K 2 KB + V 2 KB, 1024-byte
// aligned for the 128-byte TMA swizzle), 32 bytes of qparams per stage
// (k_scale, v_scale, k zero-point word, v zero-point word, flags), and a full / empty
// mbarrier pair per stage.  The warp merge at the end reuses the ring.
// Pages the producer warp issues per loop trip (one lane each): 8, or 4 when 8 does not
// divide the ring.
__host__ __device__ constexpr int issue_batch(int stages) { return stages % 8 == 0 ? 8 : 4; }

template <int kW, int kNS>
struct SmemLayout {
  static constexpr int kStageRegion = kNS * kStageBytes;
  static constexpr int kMetaRegion = kNS * kMetaBytes;
  static constexpr int kBarRegion = kNS * 16;
  static constexpr int kMergeBytes = kW * (2 * kMaxG + kMaxG * kD) * 4;
  static_assert(kMergeBytes <= kStageRegion, "merge scratch reuses the stage ring");
  // Every stage must always be consumed by the same warp (page i -> warp i % kW, stage
  // i % kNS).  Otherwise a warp can wait on a stage's full barrier a whole phase early
  // and the parity test aliases with the previous phase.
  static_assert(kNS % kW == 0, "stage count must be a multiple of the consumer warps");
  static constexpr int kTotal = 1024 /*alignment slack*/ + kStageRegion + kMetaRegion + kBarRegion;
};

constexpr uint32_t kMagic = 0x64646464u;  // fp16 exponent bytes: half 0x64xx == 1024 + xx

// qparams of one stage as the consumers read them; tok != 0 (symmetric format) is the
// shared address of the stage's 16 K then 16 V per-token scales
struct StageInfo {
  float ks, vs;
  uint32_t kz, vz;
  uint32_t tok;
};

constexpr uint32_t kStageSym = 4u;  // meta flag: the stage carries per-token scales

// Producer side, one lane: fill stage `st` with the (page, kv head) block whose index in
// the [blocks, 16, 128] view is `e` (< 0: nothing to load, the stage is marked invalid).
__device__ __forceinline__ void issue_page(const DecodeParams& p, const CUtensorMap* tmk, const CUtensorMap* tmv,
                                           uint32_t base_s, uint32_t* meta_p, uint32_t meta_s, uint32_t full,
                                           int st, int64_t e, uint64_t policy) {
  uint32_t* m = meta_p + st * (kMetaBytes / 4);
  if (e < 0) {
    m[4] = 0u;
    mbar_arrive(full);
    mbar_arrive(full);
    return;
  }
  if (p.sym) {  // symmetric format: 16 K and 16 V per-token scales, 64 bytes each
    m[4] = 1u | kStageSym;
    mbar_arrive_expect_tx(full, kStageBytes + 128);
    const uint32_t dst = base_s + st * kStageBytes;
    tma_load_2d(dst, tmk, 0, (int32_t)(e * kPage), full, policy);
    tma_load_2d(dst + kPageBytes, tmv, 0, (int32_t)(e * kPage), full, policy);
    const uint32_t ms = meta_s + st * kMetaBytes + 32;
    bulk_load(ms, p.k_scale + e * kPage, 64, full);
    bulk_load(ms + 64, p.v_scale + e * kPage, 64, full);
    mbar_arrive(full);
    return;
  }
  const bool word_ok = (e | 1) < p.zp_count;
  if (!word_ok) {  // last element of an odd-sized zero-point array: plain loads
    m[2] = (uint32_t)(uint16_t)p.k_zero[e];
    m[3] = (uint32_t)(uint16_t)p.v_zero[e];
  }
  m[4] = 1u | (word_ok ? ((uint32_t)(e & 1) << 1) : 0u);
  mbar_arrive_expect_tx(full, kStageBytes);
  const uint32_t dst = base_s + st * kStageBytes;
  tma_load_2d(dst, tmk, 0, (int32_t)(e * kPage), full, policy);
  tma_load_2d(dst + kPageBytes, tmv, 0, (int32_t)(e * kPage), full, policy);
  const uint32_t ms = meta_s + st * kMetaBytes;
  if (p.debug_mode >= 3) {  // profiling: no qparam copies
    mbar_arrive(full);
    return;
  }
  cp_async_4(ms + 0, p.k_scale + e);
  cp_async_4(ms + 4, p.v_scale + e);
  if (word_ok) {
    cp_async_4(ms + 8, p.k_zero + (e & ~1ll));
    cp_async_4(ms + 12, p.v_zero + (e & ~1ll));
  }
  cp_async_mbar_arrive_noinc(full);
}

// Index of the (page, kv head) block of table entry `phys` (paged) or logical page `phys`
// (contiguous); -1 when the entry is unallocated or outside the pool (the latter is
// reported in the status word).
template <bool kPaged>
__device__ __forceinline__ int64_t block_index(const DecodeParams& p, int b, int h, long long phys) {
  if (kPaged) {
    if (phys < 0) return -1;
    if (phys >= p.num_blocks) {
      if (p.status != nullptr) atomicOr(p.status, FS_DEV_BAD_PAGE);
      return -1;
    }
    return (int64_t)phys * p.Hkv + h;
  }
  return ((int64_t)b * p.Hkv + h) * p.num_blocks + phys;
}

__device__ __forceinline__ bool read_stage_info(const uint32_t* meta_p, int st, StageInfo& si, uint32_t meta_s) {
  const volatile uint32_t* m = meta_p + st * (kMetaBytes / 4);
  const uint32_t flags = m[4];
  if (!(flags & 1u)) return false;
  if (flags & kStageSym) {  // stored values are the signed integers: zero point 128 in the u domain
    si.ks = si.vs = 1.f;
    si.kz = si.vz = 128u;
    si.tok = meta_s + st * kMetaBytes + 32;
    return true;
  }
  si.tok = 0u;
  si.ks = __uint_as_float(m[0]);
  si.vs = __uint_as_float(m[1]);
  const uint32_t sh = (flags & 2u) ? 16u : 0u;
  si.kz = (m[2] >> sh) & 0xffffu;
  si.vz = (m[3] >> sh) & 0xffffu;
  return true;
}

// Per-thread shared-memory offsets inside a stage (128-byte swizzle: the 16-byte chunk
// index of row r is XOR-ed with r & 7).  K: rows g and g+8, chunks 2c and 2c+1.  V:
// ldmatrix.x4.trans #k reads 8x8 b16 matrices (chunk 2k | 2k+1) x (tokens 0-7 | 8-15);
// lane l supplies row (l & 7) of matrix (l >> 3).
struct StageOffsets {
  uint32_t k[2][2];
  uint32_t v[4];
  __device__ __forceinline__ explicit StageOffsets(int lane) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) k[nt][e2] = (g + 8 * nt) * 128 + (((2 * c + e2) ^ g) << 4);
    const int mat = lane >> 3, r = lane & 7;
    const int tok = 8 * (mat & 1) + r;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) v[kk] = kPageBytes + tok * 128 + (((2 * kk + (mat >> 1)) ^ r) << 4);
  }
};

// Query fragment of one (request, kv head) for S = Q K^T on the int8 tensor cores.
// Row g of q is held as 16-bit fixed point q ~= q16 * qscale (q16 = rint(q / qscale),
// |q16| <= 32639, qscale = max|q| / 32639), split as q16 = 256 * hi + lo with signed
// bytes hi, lo: two int8 MMAs give sum(q16 * s) exactly in int32.  Thread (g,c) holds
// head dims [32c, 32c+32): word w covers dims 32c+4w .. 32c+4w+3, and k-step j uses
// words 2j (logical k 4c..4c+3) and 2j+1 (logical k 16+4c..).  q16sum = sum of q16 over
// the row (exact), used to apply the zero point once per page.
struct QueryFrag {
  uint32_t hi[8], lo[8];
  int q16sum;
  float qscale;
  __device__ __forceinline__ void load(const DecodeParams& p, int b, int h, int lane) {
    const int g = lane >> 2, c = lane & 3;
    uint32_t raw[16];
    if (g < p.G) {
      const uint4* qp =
          reinterpret_cast<const uint4*>(p.q + ((size_t)b * p.Hq + (size_t)h * p.G + g) * kD + 32 * c);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = __ldg(qp + i);
        raw[4 * i] = v.x;
        raw[4 * i + 1] = v.y;
        raw[4 * i + 2] = v.z;
        raw[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) raw[i] = 0u;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&raw[i]));
      amax = fmaxf(amax, fmaxf(fabsf(f2.x), fabsf(f2.y)));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float inv = amax > 0.f ? 32639.0f / amax : 0.f;
    qscale = amax > 0.f ? amax / 32639.0f : 0.f;
    int sum = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      uint32_t hw = 0u, lw = 0u;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&raw[2 * w + k]));
        const float v2[2] = {f2.x, f2.y};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int q16 = __float2int_rn(v2[e] * inv);
          const int qh = (q16 + 128) >> 8;
          const int ql = q16 - (qh << 8);
          sum += q16;
          hw |= (uint32_t)(qh & 0xff) << (8 * (2 * k + e));
          lw |= (uint32_t)(ql & 0xff) << (8 * (2 * k + e));
        }
      }
      hi[w] = hw;
      lo[w] = lw;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    q16sum = sum;
  }
};

// Online-softmax state of one warp: running max (log2 domain, finite so exp2 never sees
// inf - inf), this thread's share of the denominator, and the PV accumulator
// acc[i][0..3] = O[d = 16i+2g (+1 for [2],[3])][query 2c | 2c+1].
// The PV MMAs multiply P by 1024 + u (the exact fp16 form of the stored byte) rather than
// by u - zp; z_run collects this thread's share of sum_t P16[g][t] * (1024 + zp_page) for
// query row g, and fold_zero_point() subtracts it once, when the warp's pages are done.
struct WarpState {
  float m_run, l_run, z_run;
  float acc[8][4];
  __device__ __forceinline__ void reset() {
    m_run = -1.0e30f;
    l_run = 0.f;
    z_run = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[i][k] = 0.f;
  }
  // acc[.][0|2] belong to query 2c and acc[.][1|3] to query 2c+1, whose corrections sit
  // (summed over the 4 lanes of a row) in lanes 8c and 8c+4.
  __device__ __forceinline__ void fold_zero_point(int lane) {
    float z = z_run;
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    z += __shfl_xor_sync(0xffffffffu, z, 2);
    const int c = lane & 3;
    const float z0 = __shfl_sync(0xffffffffu, z, 8 * c), z1 = __shfl_sync(0xffffffffu, z, 8 * c + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[i][0] -= z0;
      acc[i][1] -= z1;
      acc[i][2] -= z0;
      acc[i][3] -= z1;
    }
    z_run = 0.f;
  }
};

// Consumer side: load stage `sbase`, release it on `empty_bar`, then fold the page into
// the warp state.  pos0 = first token position of the page, len_eff = tokens that count.
// kMode 1 stops after the loads (profiling).
template <int kMode>
__device__ __forceinline__ void consume_page(uint32_t sbase, const StageOffsets& off, uint32_t empty_bar, int lane,
                                             const StageInfo& si, const QueryFrag& qf, float qk_scale_log2,
                                             int pos0, int len_eff, WarpState& ws) {
  const int c = lane & 3;
  // ---- S = Q K^T on the int8 tensor cores, straight from the stored bytes s = u - 128:
  // sum_d q16 * s = 256 * (hi . s) + (lo . s); u - zp = s + (128 - zp) is applied per page
  int shi[2][4], slo[2][4];
  {
    uint4 kr[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) kr[nt][e2] = lds128(sbase + off.k[nt][e2]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int k = 0; k < 4; ++k) shi[nt][k] = slo[nt][k] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint4 kv = kr[nt][j >> 1];
        const uint32_t b0 = (j & 1) ? kv.z : kv.x;
        const uint32_t b1 = (j & 1) ? kv.w : kv.y;
        mma_16832_s8(shi[nt], qf.hi[2 * j], 0u, qf.hi[2 * j + 1], 0u, b0, b1);
        mma_16832_s8(slo[nt], qf.lo[2 * j], 0u, qf.lo[2 * j + 1], 0u, b0, b1);
      }
    }
  }
  uint32_t vr[16];
#pragma unroll
  for (int k = 0; k < 4; ++k) ldsm_x4_trans(sbase + off.v[k], vr[4 * k], vr[4 * k + 1], vr[4 * k + 2], vr[4 * k + 3]);
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);  // the stage may be refilled now
  if (kMode == 1) {
    ws.acc[0][0] += __uint_as_float(((uint32_t)shi[0][0] ^ (uint32_t)slo[1][1] ^ vr[0] ^ vr[15]) & 0x007fffffu);
    return;
  }
  const float f = si.ks * qf.qscale * qk_scale_log2;
  const int zc = (128 - (int)si.kz) * qf.q16sum;
  // per-token scales of this thread's tokens 2c, 2c+1, 8+2c, 9+2c (symmetric format)
  float fk[4] = {f, f, f, f}, vk[4] = {si.vs, si.vs, si.vs, si.vs};
  if (si.tok != 0u) {
    const float2 k01 = lds64f(si.tok + 8 * c), k89 = lds64f(si.tok + 32 + 8 * c);
    const float2 v01 = lds64f(si.tok + 64 + 8 * c), v89 = lds64f(si.tok + 96 + 8 * c);
    fk[0] = f * k01.x;
    fk[1] = f * k01.y;
    fk[2] = f * k89.x;
    fk[3] = f * k89.y;
    vk[0] = v01.x;
    vk[1] = v01.y;
    vk[2] = v89.x;
    vk[3] = v89.y;
  }
  float t[4];
  t[0] = (float)((shi[0][0] << 8) + slo[0][0] + zc) * fk[0];  // token 2c
  t[1] = (float)((shi[0][1] << 8) + slo[0][1] + zc) * fk[1];  // token 2c+1
  t[2] = (float)((shi[1][0] << 8) + slo[1][0] + zc) * fk[2];  // token 8+2c
  t[3] = (float)((shi[1][1] << 8) + slo[1][1] + zc) * fk[3];  // token 9+2c
  if (pos0 + kPage > len_eff) {
    if (pos0 + 2 * c >= len_eff) t[0] = -INFINITY;
    if (pos0 + 2 * c + 1 >= len_eff) t[1] = -INFINITY;
    if (pos0 + 8 + 2 * c >= len_eff) t[2] = -INFINITY;
    if (pos0 + 9 + 2 * c >= len_eff) t[3] = -INFINITY;
  }
  float mx = fmaxf(fmaxf(t[0], t[1]), fmaxf(t[2], t[3]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  if (__any_sync(0xffffffffu, mx > ws.m_run)) {
    const float m_new = fmaxf(ws.m_run, mx);
    const float alpha = ex2_approx(ws.m_run - m_new);
    ws.m_run = m_new;
    ws.l_run *= alpha;
    ws.z_run *= alpha;
    const float a0 = __shfl_sync(0xffffffffu, alpha, 8 * c);
    const float a1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);
#pragma unroll
    for (int i2 = 0; i2 < 8; ++i2) {
      ws.acc[i2][0] *= a0;
      ws.acc[i2][1] *= a1;
      ws.acc[i2][2] *= a0;
      ws.acc[i2][3] *= a1;
    }
  }
  float pr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) pr[k] = ex2_approx(t[k] - ws.m_run);
  ws.l_run += (pr[0] + pr[1]) + (pr[2] + pr[3]);
  const uint32_t pb0 = pack_half2(pr[0] * vk[0], pr[1] * vk[1]);
  const uint32_t pb1 = pack_half2(pr[2] * vk[2], pr[3] * vk[3]);
  {  // the zero point, applied per page to the exact fp16 P values the MMAs see
    const float2 p01 = __half22float2(*reinterpret_cast<const __half2*>(&pb0));
    const float2 p23 = __half22float2(*reinterpret_cast<const __half2*>(&pb1));
    ws.z_run = fmaf(1024.f + (float)si.vz, (p01.x + p01.y) + (p23.x + p23.y), ws.z_run);
  }
  // ---- O += P V: vr(chunk i, tokens 0-7 | 8-15) hold bytes
  // [V[2c][d], V[2c][d+1], V[2c+1][d], V[2c+1][d+1]] with d = 16i + 2g; the stored byte
  // is u - 128, so XOR 0x80 gives u and PRMT with exponent bytes 0x64 the fp16 1024 + u.
#pragma unroll
  for (int i2 = 0; i2 < 8; ++i2) {
    const uint32_t x0 = vr[4 * (i2 >> 1) + 2 * (i2 & 1)] ^ 0x80808080u;
    const uint32_t x1 = vr[4 * (i2 >> 1) + 2 * (i2 & 1) + 1] ^ 0x80808080u;
    mma_16816(ws.acc[i2], prmt(x0, kMagic, 0x5240u), prmt(x0, kMagic, 0x5341u), prmt(x1, kMagic, 0x5240u),
              prmt(x1, kMagic, 0x5341u), pb0, pb1);
  }
}

// Writes one normalised output value: fp16 `out`, or (O, LSE) into the shard outputs.
__device__ __forceinline__ void write_final(const DecodeParams& p, size_t row, int d, float o, float lse) {
  if (p.shard_o != nullptr) {
    p.shard_o[row * kD + d] = o;
    if (d == 0) p.shard_lse[row] = lse;
  } else {
    p.out[row * kD + d] = __float2half_rn(o);
  }
}

// Profiling aid of the split kernel (FLASHSPEC_TRACE_PTR): thread 0 stamps %globaltimer
// into trace[k]; per CTA c: [4c] entry, [4c + 1] pages consumed, [4c + 2] partial
// written; per pair q, from 4 * gridDim.x: [16q] merge start, [16q + 1] rows ready,
// [16q + 2] exchange stores issued, [16q + 3] every rank's rows merged, [16q + 4] end,
// [16q + 5] partial LSEs loaded, [16q + 6] weights formed, [16q + 7] partial rows
// summed, [16q + 8 + 2r] staging round r arrived, [16q + 9 + 2r] round r summed.
__device__ __forceinline__ void split_mark(const DecodeParams& p, size_t k) {
  if (p.trace != nullptr && threadIdx.x == 0) p.trace[k] = globaltimer_ns();
}

// Fused exchange epilogue of a sequence-sharded step: this rank's normalised (O, LSE)
// rows of pair (b, h) -- staged in shared memory as xo [G][128], xl [G] -- go as tagged
// words (xwords.cuh) into slot `xrank` of every rank's exchange buffer; then the CTA
// merges every rank's rows of the pair with the log-sum-exp rule (the combine of
// triton_fused.py:446-503 on one partial per rank) as they arrive, and writes them to
// xout.  Waits end at xtimeout_ns: the CTA then sets FS_DEV_TIMEOUT and writes NaN.
// The pair's call counter in this rank's buffer gives the epoch (tag and parity).  The
// LSE words come first (one per rank and row, giving the weights), then the O words,
// each thread loading all of its elements of a peer at once.
template <int kThreads>
__device__ __forceinline__ void exchange_pair(const DecodeParams& p, int b, int h, int bh, const float* xo,
                                              float* xl, int tid) {
  uint8_t* own = static_cast<uint8_t*>(p.xbufs[p.xrank]);
  uint32_t* calls = reinterpret_cast<uint32_t*>(own + kXPairCountersOffset);
  const uint32_t e = calls[bh] + 1u;  // written by this pair's previous call on this GPU
  const size_t poff = exchange_parity_offset(e, p.xslot);
  const int64_t rows = (int64_t)p.B * p.Hq;
  const int64_t row0 = (int64_t)b * p.Hq + (int64_t)h * p.G;
  const int G = p.G, n = G * kD;
  for (int r = 0; r < p.xworld; ++r) {
    if (r == p.xrank) continue;  // this rank's rows are merged from shared memory
    uint64_t* dst = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(p.xbufs[r]) + poff) + (size_t)p.xrank * p.xslot;
    for (int i = tid; i < n; i += kThreads) st_word(dst + row0 * kD + i, xo[i], e);
    if (tid < G) st_word(dst + rows * kD + row0 + tid, xl[tid], e);
  }
  const size_t tr = 4 * (size_t)gridDim.x + 16 * (size_t)bh;
  split_mark(p, tr + 2);
  const uint64_t* data = reinterpret_cast<const uint64_t*>(own + poff);
  const uint64_t deadline = globaltimer_ns() + (uint64_t)p.xtimeout_ns;
  // 1. every rank's LSE of the pair's G rows -> normalised weights w[r][q] in shared
  //    memory (after xl); the output is O only, so the merged LSE is not formed
  float* w = xl + kMaxG;  // [kXMaxRanks][kMaxG]
  bool ok = true;
  if (tid < p.xworld * G) {
    const int r = tid / G, qg = tid - r * G;
    float l = xl[qg];
    if (r != p.xrank) ok = wait_word(data + (size_t)r * p.xslot + rows * kD + row0 + qg, e, deadline, l);
    w[r * kMaxG + qg] = l;
  }
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (tid < G) {
    float M = -INFINITY;
    for (int r = 0; r < p.xworld; ++r) M = fmaxf(M, w[r * kMaxG + tid]);
    float W = 0.f;
    for (int r = 0; r < p.xworld; ++r) {
      const float l = w[r * kMaxG + tid];
      const float x = (M == -INFINITY || l == -INFINITY) ? 0.f : expf(l - M);
      w[r * kMaxG + tid] = x;
      W += x;
    }
    const float inv = W > 0.f ? 1.f / W : 0.f;
    for (int r = 0; r < p.xworld; ++r) w[r * kMaxG + tid] *= inv;
  }
  __syncthreads();
  // 2. the rows: per peer rank, every element of this thread is loaded at once (one
  //    round trip), then any word still missing is waited for
  constexpr int kPer = (kMaxG * kD + kThreads - 1) / kThreads;
  float acc[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = tid + j * kThreads;
    acc[j] = i < n ? w[p.xrank * kMaxG + (i >> 7)] * xo[i] : 0.f;
  }
  for (int r = 0; r < p.xworld && ok; ++r) {
    if (r == p.xrank) continue;
    const uint64_t* src = data + (size_t)r * p.xslot + row0 * kD;
    uint64_t v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = tid + j * kThreads;
      v[j] = i < n ? ld_word(src + i) : 0ull;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = tid + j * kThreads;
      if (i >= n || !ok) continue;
      float o = __uint_as_float((uint32_t)v[j]);
      if ((uint32_t)(v[j] >> 32) != e) ok = wait_word(src + i, e, deadline, o);
      acc[j] = fmaf(w[r * kMaxG + (i >> 7)], o, acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = tid + j * kThreads;
    if (i >= n) continue;
    const float v = ok ? acc[j] : __int_as_float(0x7fc00000);
    const size_t at = (size_t)row0 * kD + i;
    if (p.xout_dtype == FS_F16)
      static_cast<__half*>(p.xout)[at] = __float2half_rn(v);
    else
      static_cast<float*>(p.xout)[at] = v;
  }
  if (!ok && p.xstatus != nullptr) atomicOr(p.xstatus, FS_DEV_TIMEOUT);
  __syncthreads();  // every thread has read this call's words before the epoch advances
  split_mark(p, tr + 3);
  if (tid == 0) calls[bh] = e;
}

// ==================================================================================
// Split kernel: one CTA = one (request, kv head, split).  Warps 0..kW-1 consume pages;
// warp kW is the producer that keeps the ring full with TMA tile loads and cp.async
// qparam copies.  kMode is a profiling aid: 0 = normal; 1 = consumers read the stage and
// release it but skip the math; 2 = consumers only wait and release (data movement).
// ==================================================================================
template <bool kPaged, int kW, int kNS, int kMinBlocks, int kMode>
__global__ void __launch_bounds__((kW + 1) * 32, kMinBlocks)
    decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const DecodeParams p) {
  using L = SmemLayout<kW, kNS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base_s = (raw_s + 1023u) & ~1023u;
  uint8_t* base_p = smem_raw + (base_s - raw_s);
  const uint32_t meta_s = base_s + L::kStageRegion;
  uint32_t* meta_p = reinterpret_cast<uint32_t*>(base_p + L::kStageRegion);
  const uint32_t full_s = base_s + L::kStageRegion + L::kMetaRegion;
  const uint32_t empty_s = full_s + kNS * 8;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int c = lane & 3;

  // ---- work item ------------------------------------------------------------
  const int S = p.S;
  const int split = blockIdx.x % S;
  const int bh = blockIdx.x / S;
  const int h = bh % p.Hkv;
  const int b = bh / p.Hkv;
  int64_t len64 = p.max_seq_len;
  if (p.lengths != nullptr) len64 = min(len64, p.lengths[b]);
  const int len = (int)max(len64, (int64_t)0);
  int npages = (len + kPage - 1) / kPage;
  npages = kPaged ? min(npages, p.cols) : (int)min((int64_t)npages, p.num_blocks);
  const int len_eff = min(len, npages * kPage);
  const int lo = (int)max(p.page_begin, (int64_t)0);
  const int hi = p.page_end > 0 ? (int)min(p.page_end, (int64_t)npages) : npages;
  const int span = hi > lo ? hi - lo : 0;
  __shared__ alignas(8) uint64_t s_merge_bar;  // the final merge's bulk copies
  const int chunk = (span + S - 1) / S;
  const int p0 = min(lo + split * chunk, max(hi, lo));
  const int n = max(min(hi, p0 + chunk) - p0, 0);  // pages of this CTA
  split_mark(p, 4 * (size_t)blockIdx.x);

  if (tid == 0) {
    for (int st = 0; st < kNS; ++st) {
      mbar_init(full_s + 8 * st, 2);
      mbar_init(empty_s + 8 * st, 1);
    }
    mbar_init(smem_u32(&s_merge_bar), 1);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  bool aborted = false;
  WarpState ws;
  ws.reset();

  if (warp == kW) {
    // ============================ producer warp ===============================
    // Pages are issued in batches of kIssue: lane j handles page i + j, so one warp
    // instruction issues kIssue TMA loads.
    constexpr int kIssue = issue_batch(kNS);
    static_assert(kNS % kIssue == 0 && 32 % kIssue == 0, "issue batch must divide the ring");
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
    const uint64_t policy = l2_policy_evict_first();
    const int64_t* trow = kPaged ? p.table + (size_t)b * p.cols + p0 : nullptr;
    long long tcur = (kPaged && lane < n) ? (long long)trow[lane] : -1;
    long long tnxt = (kPaged && 32 + lane < n) ? (long long)trow[32 + lane] : -1;
    for (int i0 = 0; i0 < n; i0 += kIssue) {
      long long phys;
      if (kPaged) {
        if ((i0 & 31) == 0 && i0 > 0) {
          tcur = tnxt;
          tnxt = (i0 + 32 + lane < n) ? (long long)trow[i0 + 32 + lane] : -1;
        }
        phys = __shfl_sync(0xffffffffu, tcur, (i0 + (lane & (kIssue - 1))) & 31);
      } else {
        phys = p0 + i0 + lane;
      }
      const int i = i0 + lane;
      if (lane < kIssue && i < n) {
        const int st = (int)((unsigned)i % kNS);
        if (i >= kNS && !producer_wait(empty_s + 8 * st, (((unsigned)i / kNS) - 1u) & 1u, p.producer_sleep_ns)) {
          if (p.status != nullptr) atomicOr(p.status, FS_DEV_TIMEOUT);
          aborted = true;
        }
        if (!aborted)
          issue_page(p, &tmk, &tmv, base_s, meta_p, meta_s, full_s + 8 * st, st, block_index<kPaged>(p, b, h, phys),
                     policy);
      }
      if (__any_sync(0xffffffffu, aborted)) {
        aborted = true;
        break;
      }
    }
  } else {
    // ============================ consumer warps ===============================
    QueryFrag qf;
    qf.load(p, b, h, lane);
    const StageOffsets off(lane);
    for (int i = warp; i < n; i += kW) {
      const int st = (int)((unsigned)i % kNS);
      if (!mbar_wait_bounded(full_s + 8 * st, ((unsigned)i / kNS) & 1u, kTimeoutNs)) {
        if (lane == 0 && p.status != nullptr) atomicOr(p.status, FS_DEV_TIMEOUT);
        aborted = true;
        break;
      }
      StageInfo si;
      if (kMode == 2 || !read_stage_info(meta_p, st, si, meta_s)) {  // masked page (or data-only profiling)
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_s + 8 * st);
        continue;
      }
      consume_page<kMode>(base_s + st * kStageBytes, off, empty_s + 8 * st, lane, si, qf, p.qk_scale_log2,
                          (p0 + i) * kPage, len_eff, ws);
    }
    ws.l_run += __shfl_xor_sync(0xffffffffu, ws.l_run, 1);
    ws.l_run += __shfl_xor_sync(0xffffffffu, ws.l_run, 2);
    ws.fold_zero_point(lane);
  }

  // ---- merge the consumer warps through shared memory ---------------------------
  __syncthreads();  // every page has been consumed, so no copy still targets the ring
  const bool any_abort = __syncthreads_or(aborted ? 1 : 0);
  if (any_abort) return;  // status word carries FS_DEV_TIMEOUT; outputs are not written
  split_mark(p, 4 * (size_t)blockIdx.x + 1);
  float* ms = reinterpret_cast<float*>(base_p);
  float* ls = ms + kW * kMaxG;
  float* accs = ls + kW * kMaxG;  // [kW][kMaxG][kD]
  if (warp < kW) {
    if (c == 0) {
      ms[warp * kMaxG + g] = ws.m_run;
      ls[warp * kMaxG + g] = ws.l_run;
    }
#pragma unroll
    for (int i2 = 0; i2 < 8; ++i2) {
      const int d = 16 * i2 + 2 * g;
      float* a0p = accs + (warp * kMaxG + 2 * c) * kD;
      float* a1p = accs + (warp * kMaxG + 2 * c + 1) * kD;
      a0p[d] = ws.acc[i2][0];
      a1p[d] = ws.acc[i2][1];
      a0p[d + 1] = ws.acc[i2][2];
      a1p[d + 1] = ws.acc[i2][3];
    }
  }
  __syncthreads();

  constexpr int kThreads = (kW + 1) * 32;
  const int nout = p.G * kD;
  const float kLn2 = 0.6931471805599453f;
  // fused exchange: the pair's merged rows are staged at the end of the ring region
  constexpr int kXStage = (L::kStageRegion - (kMaxG * kD + kMaxG + kXMaxRanks * kMaxG) * 4) & ~15;
  static_assert(kXStage >= ((3 + kD) * kW * kMaxG + kMaxG) * 4, "exchange staging overlaps the warp merge");
  const bool xmode = p.xworld > 0;
  float* xo = reinterpret_cast<float*>(base_p + kXStage);
  float* xl = xo + kMaxG * kD;
  // per query: the warps' scale factors exp2(m_w - M) / L folded into one weight each,
  // and the LSE, formed once (G threads) so the row loop below is loads and FMAs only
  float* fw = accs + kW * kMaxG * kD;  // [kW][kMaxG] weights, then [kMaxG] LSE
  float* flse = fw + kW * kMaxG;
  if (tid < p.G) {
    float M = -1.0e30f;
#pragma unroll
    for (int w = 0; w < kW; ++w) M = fmaxf(M, ms[w * kMaxG + tid]);
    float sc[kW], Lsum = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      sc[w] = exp2f(ms[w * kMaxG + tid] - M);
      Lsum += ls[w * kMaxG + tid] * sc[w];
    }
    const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) fw[w * kMaxG + tid] = sc[w] * inv;
    flse[tid] = Lsum > 0.f ? (M + log2f(Lsum)) * kLn2 : -INFINITY;
  }
  __syncthreads();
  for (int u4 = tid; u4 < nout / 4; u4 += kThreads) {
    const int idx = 4 * u4;
    const int qg = idx >> 7;
    const int d = idx & (kD - 1);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      const float f = fw[w * kMaxG + qg];
      const float4 a4 = *reinterpret_cast<const float4*>(accs + (w * kMaxG + qg) * kD + d);
      o.x = fmaf(a4.x, f, o.x);
      o.y = fmaf(a4.y, f, o.y);
      o.z = fmaf(a4.z, f, o.z);
      o.w = fmaf(a4.w, f, o.w);
    }
    const float lse = flse[qg];
    const size_t row = (size_t)b * p.Hq + (size_t)h * p.G + qg;
    if (S == 1 && xmode) {
      *reinterpret_cast<float4*>(xo + idx) = o;
      if (d == 0) xl[qg] = lse;
    } else if (S == 1) {
      write_final(p, row, d, o.x, lse);
      write_final(p, row, d + 1, o.y, lse);
      write_final(p, row, d + 2, o.z, lse);
      write_final(p, row, d + 3, o.w, lse);
    } else {
      const size_t prow = ((size_t)bh * S + split) * p.G + qg;
      *reinterpret_cast<float4*>(p.part_o + prow * kD + d) = o;
      if (d == 0) p.part_lse[prow] = lse;
    }
  }
  if (S == 1) {
    if (xmode) {
      __syncthreads();
      split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 1);
      exchange_pair<kThreads>(p, b, h, bh, xo, xl, tid);
    }
    split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 4);
    return;
  }

  // ---- split-K: the last CTA of this (request, kv head) merges -------------------
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned ticket = atomicAdd(p.counters + bh, 1u);
    s_last = (ticket == (unsigned)(S - 1)) ? 1 : 0;
  }
  __syncthreads();
  split_mark(p, 4 * (size_t)blockIdx.x + 2);
  if (!s_last) return;
  __threadfence();
  split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh);
  // the S partial LSEs of each query, staged in shared memory (the ring is free now)
  float* wsm = reinterpret_cast<float*>(base_p);  // [S][G]
  const int nw = S * p.G;
  const bool fits = (nw + 3 * kMaxG) * 4 + 1024 + p.G * kD * 4 <= kXStage;
  // staging of the partial rows (bulk copies, below): the first round is issued before
  // the weights are computed, so its latency overlaps theirs
  const int rows_bytes = p.G * kD * 4;
  const int stage_off = (((nw + 3 * kMaxG) * 4) + 1023) & ~1023;
  const int per_round = max(1, (kXStage - stage_off) / rows_bytes);
  const uint32_t mbar = smem_u32(&s_merge_bar);
  const float* src0 = p.part_o + (size_t)bh * S * p.G * kD;
  auto issue_round = [&](int s0) {
    const int cnt = min(per_round, S - s0);
    // the partials were written by other CTAs through the generic proxy, and the
    // stage was last read through it
    asm volatile("fence.proxy.async.global;" ::: "memory");
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(mbar, (uint32_t)(cnt * rows_bytes));
    for (int u = 0; u < cnt; ++u)
      bulk_load(base_s + stage_off + u * rows_bytes, src0 + (size_t)(s0 + u) * p.G * kD, (uint32_t)rows_bytes, mbar);
  };
  if (fits && tid == 0) issue_round(0);
  if (fits) {
    const size_t prow0 = (size_t)bh * S * p.G;
    for (int k = tid; k < nw; k += kThreads) wsm[k] = __ldcg(p.part_lse + prow0 + k);
    __syncthreads();
    split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 5);
  }
  if (fits) {
    // every split wrote its partial rows [G][128] (an empty one with weight 0), 4 KB
    // contiguous per split at most: bulk copies stage them in shared memory behind the
    // LSEs, as many splits per round as fit, so a round costs one copy latency
    const float* stage_p = reinterpret_cast<const float*>(base_p + stage_off);
    // weights w[s][q] = exp(lse_s - M_q) (empty partials 0) in place of the LSEs, each
    // phase spread over the threads so that no thread runs a long dependent chain;
    // 1 / sum_s w and the merged LSE per query go behind them
    float* wM = wsm + nw;  // [G] max, then [G] 1 / W, then [G] merged LSE
    float* wI = wM + kMaxG;
    float* wL = wI + kMaxG;
    if (tid < p.G) {
      float M = -INFINITY;
#pragma unroll 8
      for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, wsm[s2 * p.G + tid]);
      wM[tid] = M;
    }
    __syncthreads();
    for (int k = tid; k < nw; k += kThreads) {
      const float l = wsm[k], M = wM[k % p.G];
      wsm[k] = (l == -INFINITY || M == -INFINITY) ? 0.f : expf(l - M);
    }
    __syncthreads();
    if (tid < p.G) {
      float W = 0.f;
#pragma unroll 8
      for (int s2 = 0; s2 < S; ++s2) W += wsm[s2 * p.G + tid];
      wI[tid] = W > 0.f ? 1.f / W : 0.f;
      wL[tid] = W > 0.f ? wM[tid] + logf(W) : -INFINITY;
    }
    split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 6);
    // each thread accumulates 4 head dims of a query per column
    constexpr int kCols = (kMaxG * kD / 4 + kThreads - 1) / kThreads;
    float4 acc[kCols];
#pragma unroll
    for (int c4 = 0; c4 < kCols; ++c4) acc[c4] = make_float4(0.f, 0.f, 0.f, 0.f);
    int round = 0;
    for (int s0 = 0; s0 < S; s0 += per_round, ++round) {
      const int cnt = min(per_round, S - s0);
      if (tid == 0 && s0 > 0) issue_round(s0);
      if (!mbar_spin_bounded(mbar, (uint32_t)(round & 1), kTimeoutNs) && tid == 0 && p.status != nullptr)
        atomicOr(p.status, FS_DEV_TIMEOUT);
      if (round < 4) split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 8 + 2 * round);
#pragma unroll
      for (int c4 = 0; c4 < kCols; ++c4) {
        const int u4 = tid + c4 * kThreads;
        if (u4 >= nout / 4) continue;
        const int qg = (4 * u4) >> 7;
#pragma unroll 7
        for (int u = 0; u < cnt; ++u) {
          const float w = wsm[(s0 + u) * p.G + qg];
          const float4 v = *reinterpret_cast<const float4*>(stage_p + (size_t)u * p.G * kD + 4 * u4);
          acc[c4].x = fmaf(w, v.x, acc[c4].x);
          acc[c4].y = fmaf(w, v.y, acc[c4].y);
          acc[c4].z = fmaf(w, v.z, acc[c4].z);
          acc[c4].w = fmaf(w, v.w, acc[c4].w);
        }
      }
      __syncthreads();  // the stage is free for the next round
      if (round < 4) split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 9 + 2 * round);
    }
    split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 7);
#pragma unroll
    for (int c4 = 0; c4 < kCols; ++c4) {
      const int u4 = tid + c4 * kThreads;
      if (u4 >= nout / 4) continue;
      const int qg = (4 * u4) >> 7;
      const int d = (4 * u4) & (kD - 1);
      const float inv = wI[qg];
      const float4 o = make_float4(acc[c4].x * inv, acc[c4].y * inv, acc[c4].z * inv, acc[c4].w * inv);
      const float lse_out = wL[qg];
      const size_t row = (size_t)b * p.Hq + (size_t)h * p.G + qg;
      if (xmode) {
        *reinterpret_cast<float4*>(xo + 4 * u4) = o;
        if (d == 0) xl[qg] = lse_out;
      } else {
        write_final(p, row, d, o.x, lse_out);
        write_final(p, row, d + 1, o.y, lse_out);
        write_final(p, row, d + 2, o.z, lse_out);
        write_final(p, row, d + 3, o.w, lse_out);
      }
    }
  }
  for (int idx = fits ? nout : tid; idx < nout; idx += kThreads) {
    const int qg = idx >> 7;
    const int d = idx & (kD - 1);
    const size_t prow0 = (size_t)bh * S * p.G + qg;
    float o = 0.f, lse_out;
    {
      float M = -INFINITY;
      for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, __ldcg(p.part_lse + prow0 + (size_t)s2 * p.G));
      float W = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int s2 = 0; s2 < S; ++s2) {
          const size_t pr = prow0 + (size_t)s2 * p.G;
          const float lse = __ldcg(p.part_lse + pr);
          const float w = lse == -INFINITY ? 0.f : expf(lse - M);
          W += w;
          O += w * __ldcg(p.part_o + pr * kD + d);
        }
      }
      o = W > 0.f ? O / W : 0.f;
      lse_out = W > 0.f ? M + logf(W) : -INFINITY;
    }
    if (xmode) {
      xo[idx] = o;
      if (d == 0) xl[qg] = lse_out;
    } else {
      write_final(p, (size_t)b * p.Hq + (size_t)h * p.G + qg, d, o, lse_out);
    }
  }
  if (tid == 0) p.counters[bh] = 0u;  // leave the ticket clean for the next call
  if (xmode) {
    __syncthreads();
    split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 1);
    exchange_pair<kThreads>(p, b, h, bh, xo, xl, tid);
  }
  split_mark(p, 4 * (size_t)gridDim.x + 16 * (size_t)bh + 4);
}

// ==================================================================================
// Balanced kernel (stream-K over pages): a persistent grid of C CTAs with kW consumer
// warps each.  The flattened work space is every (request, kv head, page of the window)
// in request-major order, T pages in total; consumer warp k of the Wt = C*kW warps owns
// a contiguous share of it (Shares below), so the warps stream equal amounts of work
// whatever the lengths.  Per-request page counts come from `lengths` on the device
// (a block-wide prefix sum at start), so the host never synchronises.  The producer warp
// interleaves its CTA's kW shares through one ring (issue index i -> warp i % kW, step
// i / kW, stage i % kNS).  A consumer warp closes a "piece" whenever its share crosses a
// (request, kv head) boundary: a piece covering the whole pair writes the output
// directly; otherwise its normalised (O, LSE) goes to slot 0 (the warp's first piece)
// or slot 1 (a later piece) and an atomic ticket elects the last contributor of the
// pair to merge them.
// ==================================================================================
constexpr int kMaxSKBatch = 1536;  // requests whose prefix sums fit the shared-memory table

// Division of the T flat pages between the Wt consumer warps.  A full grid places
// `tiers` CTAs on every SM (CTA b in tier b / tier_ctas), and on B200 the CTAs of an SM
// do not stream at the same rate: the first one resident on the SM gets its warps
// issued first and finishes about 5% sooner than the second, which beats the third by
// as much again.  A warp of tier t therefore gets weight 1024 - skew * t, and warp k's
// share starts at floor(T * C(k) / Ctot), C(k) being the summed weight of warps 0..k-1.
// skew 0 (or one tier) gives every warp T / Wt pages.
// floor(a / b) for 0 <= a < 2^53, 0 < b < 2^31: a double-precision quotient, exact up to
// one unit, then corrected with integer products (cheaper than a 64-bit division).
__device__ __forceinline__ int64_t floordiv53(int64_t a, int64_t b) {
  int64_t q = (int64_t)((double)a / (double)b);
  if (q * b > a) --q;
  else if ((q + 1) * b <= a) ++q;
  return q;
}

// T < 2^31 pages and Ctot <= Wt * 1024 < 2^22, so every product below stays under 2^53.
struct Shares {
  int T, Wt;
  int tier_warps;  // warps per tier
  int tiers, skew;
  __device__ __forceinline__ int weight(int t) const { return 1024 - skew * t; }
  // summed weight of the warps before tier t (t <= tiers)
  __device__ __forceinline__ int64_t tier_base(int t) const {
    return (int64_t)tier_warps * (1024 * t - skew * (t * (t - 1) / 2));
  }
  __device__ __forceinline__ int64_t cum(int k) const {
    const int t = min(k / tier_warps, tiers - 1);
    return tier_base(t) + (int64_t)(k - t * tier_warps) * weight(t);
  }
  __device__ __forceinline__ int start(int k) const { return (int)floordiv53((int64_t)T * cum(k), tier_base(tiers)); }
  // the warp whose share holds flat page f: the largest k with start(k) <= f, i.e.
  // cum(k) <= X = ceil((f + 1) * Ctot / T) - 1
  __device__ __forceinline__ int owner(int f) const {
    const int64_t tot = tier_base(tiers);
    const int64_t X = floordiv53((int64_t)(f + 1) * tot + T - 1, T) - 1;
    int t = tiers - 1;
    while (t > 0 && tier_base(t) > X) --t;
    const int k = t * tier_warps + (int)((X - tier_base(t)) / weight(t));
    return min(k, Wt - 1);
  }
};

// The shares are divided in a cost space in which every (request, kv head) pair is
// charged `ovh` virtual pages ahead of its real ones, for the fixed cost of the piece a
// warp closes on it (partial write, ticket, merge); a share's bounds are then mapped
// back to real pages.  Request r starts at cost cpre(r) = pre[r] + ovh * Hkv * r.
struct CostMap {
  const int* pre;
  int B, Hkv, ovh;
  __device__ __forceinline__ int cpre(int r) const { return pre[r] + ovh * Hkv * r; }
  __device__ __forceinline__ int total() const { return cpre(B); }
  // real pages before cost position x, 0 <= x <= total()
  __device__ __forceinline__ int realpos(int x) const {
    int lo = 0, hi = B;  // the largest r with cpre(r) <= x; its block is never empty unless r == B
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cpre(mid) <= x) lo = mid; else hi = mid - 1;
    }
    if (lo == B) return pre[B];
    const int nbr = (pre[lo + 1] - pre[lo]) / Hkv, blk = nbr + ovh;
    const int off = x - cpre(lo), h = off / blk, o = off - h * blk;
    return pre[lo] + h * nbr + max(0, o - ovh);
  }
  // cost position of the first real page of pair (r, h), whose request has nbr pages per head
  __device__ __forceinline__ int pair_cost(int r, int h, int nbr) const { return cpre(r) + h * (nbr + ovh) + ovh; }
};

template <int kW>
__device__ __forceinline__ Shares make_shares(const DecodeParams& p, int T) {
  const int Wt = (int)gridDim.x * kW;
  const int tiers = (p.tier_ctas > 0 && (int)gridDim.x % p.tier_ctas == 0) ? (int)gridDim.x / p.tier_ctas : 1;
  // every tier keeps at least a quarter of the base weight
  return Shares{T, Wt, Wt / tiers, tiers, tiers > 1 ? min(p.skew, 768 / (tiers - 1)) : 0};
}

// The last contributor of a (request, kv head) pair merges the partial (O, LSE) slots of
// warps k0..k1 into the final rows row0 .. row0 + G - 1.  Warp k's slot is 2k, or 2k + 1
// for k0 when the pair starts inside k0's share (its second piece).  Every partial
// load is issued without waiting on another: lane j gathers contributor j's LSE together
// with the first four partial rows, then each lane accumulates head dims 4*lane .. +3
// four rows at a time.  (Inlined: as an out-of-line call it cost the streaming loop
// around it 3-5% on B200.)
__device__ __forceinline__ void merge_pair(const float* part_o, const float* part_lse, __half* out, float* shard_o,
                                        float* shard_lse, int G, int64_t k0, int64_t k1, bool k0_first,
                                        size_t row0, int lane) {
  const int n = (int)(k1 - k0 + 1);
  auto slot = [&](int j) -> size_t { return ((size_t)(k0 + j) * 2 + ((j == 0 && !k0_first) ? 1 : 0)) * G; };
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int qg = 0; qg < G; ++qg) {
    auto row = [&](int j) { return __ldcg(reinterpret_cast<const float4*>(part_o + (slot(j) + qg) * kD) + lane); };
    const float lse_l = lane < n ? __ldcg(part_lse + slot(lane) + qg) : -INFINITY;
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = u < n ? row(u) : zero4;
    float M = lse_l;
    for (int j = lane + 32; j < n; j += 32) M = fmaxf(M, __ldcg(part_lse + slot(j) + qg));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float W = 0.f;
    float4 acc = zero4;
    if (M != -INFINITY) {
      for (int j0 = 0; j0 < n; j0 += 32) {
        const int j = j0 + lane;
        const float lse = j0 == 0 ? lse_l : (j < n ? __ldcg(part_lse + slot(j) + qg) : -INFINITY);
        const float w = lse == -INFINITY ? 0.f : expf(lse - M);
        W += w;
        const int cnt = min(32, n - j0);
        for (int q = 0; q < cnt; q += 4) {
          if (q > 0 || j0 > 0) {
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = q + u < cnt ? row(j0 + q + u) : zero4;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float wu = __shfl_sync(0xffffffffu, w, (q + u) & 31);
            acc.x = fmaf(wu, v[u].x, acc.x);
            acc.y = fmaf(wu, v[u].y, acc.y);
            acc.z = fmaf(wu, v[u].z, acc.z);
            acc.w = fmaf(wu, v[u].w, acc.w);
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) W += __shfl_xor_sync(0xffffffffu, W, o);
    }
    const float inv = W > 0.f ? 1.f / W : 0.f;
    const float lse_out = W > 0.f ? M + logf(W) : -INFINITY;
    const size_t r = row0 + qg;
    const int d = 4 * lane;
    if (shard_o != nullptr) {
      *reinterpret_cast<float4*>(shard_o + r * kD + d) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      if (lane == 0) shard_lse[r] = lse_out;
    } else {
      const __half2 h01 = __floats2half2_rn(acc.x * inv, acc.y * inv), h23 = __floats2half2_rn(acc.z * inv, acc.w * inv);
      uint2 pk;
      pk.x = *reinterpret_cast<const uint32_t*>(&h01);
      pk.y = *reinterpret_cast<const uint32_t*>(&h23);
      *reinterpret_cast<uint2*>(out + r * kD + d) = pk;
    }
  }
}

// largest r with pre[r] <= f (pre ascending, pre[0] = 0, pre[B] = T > f)
__device__ __forceinline__ int find_request(const int* pre, int B, int f) {
  int lo = 0, hi = B;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pre[mid] <= f) lo = mid; else hi = mid;
  }
  return lo;
}

template <bool kPaged>
__device__ __forceinline__ int window_pages(const DecodeParams& p, int r, int lo, int hi_cap, int* len_eff) {
  int64_t len = p.max_seq_len;
  if (p.lengths != nullptr) len = min(len, p.lengths[r]);
  len = max(len, (int64_t)0);
  const int np = kPaged ? min((int)((len + kPage - 1) / kPage), p.cols) : (int)min((len + kPage - 1) / kPage, p.num_blocks);
  if (len_eff) *len_eff = (int)min(len, (int64_t)np * kPage);
  return max(0, min(np, hi_cap) - lo);
}

// Profiling aid: warp w of CTA b stamps %globaltimer into trace[(b * (kW + 1) + w) * 8 + k]:
// k = 0 kernel entry, 1 after the prologue, 2 first page ready (producer: first issue),
// 3 last page consumed (producer: last issue), 4 warp done, 5 pages handled, 6 SM id.
template <bool kTrace>
__device__ __forceinline__ void trace_mark(const DecodeParams& p, int nwarps, int lane, int k,
                                           unsigned long long v = 0ull) {
  if (kTrace && p.trace != nullptr && lane == 0)
    p.trace[((size_t)blockIdx.x * nwarps + (threadIdx.x >> 5)) * 8 + k] = k >= 5 ? v : globaltimer_ns();
}

template <bool kPaged, int kW, int kNS, int kMaxRegs, bool kTrace>
__global__ void __maxnreg__(kMaxRegs)
    decode_balanced_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                           const DecodeParams p) {
  using L = SmemLayout<kW, kNS>;
  constexpr int kThreads = (kW + 1) * 32;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base_s = (raw_s + 1023u) & ~1023u;
  uint8_t* base_p = smem_raw + (base_s - raw_s);
  const uint32_t meta_s = base_s + L::kStageRegion;
  uint32_t* meta_p = reinterpret_cast<uint32_t*>(base_p + L::kStageRegion);
  const uint32_t full_s = base_s + L::kStageRegion + L::kMetaRegion;
  const uint32_t empty_s = full_s + kNS * 8;
  int* pre = reinterpret_cast<int*>(base_p + L::kStageRegion + L::kMetaRegion + L::kBarRegion);  // [B + 1]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.B, Hkv = p.Hkv;
  int* starts = pre + B + 1;  // [kW + 1]
  const int lo = (int)max(p.page_begin, (int64_t)0);
  const int hi_cap = p.page_end > 0 ? (int)min(p.page_end, (int64_t)0x7fffffff) : 0x7fffffff;
  trace_mark<kTrace>(p, kW + 1, lane, 0);

  if (tid == 0) {
    for (int st = 0; st < kNS; ++st) {
      mbar_init(full_s + 8 * st, 2);
      mbar_init(empty_s + 8 * st, 1);
    }
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  for (int r = tid; r < B; r += kThreads) pre[r + 1] = window_pages<kPaged>(p, r, lo, hi_cap, nullptr) * Hkv;
  __syncthreads();
  if (warp == 0) {  // inclusive prefix sum of the per-request page counts (x Hkv)
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      int x = base + lane < B ? pre[base + lane + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (base + lane < B) pre[base + lane + 1] = carry + x;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) pre[0] = 0;
    __syncwarp();
    // the first flat page of this CTA's warps' shares, and the end of the last one
    if (lane <= kW) {
      const CostMap cm{pre, B, Hkv, p.piece_cost};
      starts[lane] = cm.realpos(make_shares<kW>(p, cm.total()).start((int)blockIdx.x * kW + lane));
    }
  }
  __syncthreads();
  const int64_t T = pre[B];
  const float kLn2 = 0.6931471805599453f;
  trace_mark<kTrace>(p, kW + 1, lane, 1);

  if (warp == kW) {
    // ============================ producer warp ===============================
    constexpr int kIssue = issue_batch(kNS);
    static_assert(kNS % kIssue == 0 && 32 % kIssue == 0, "issue batch must divide the ring");
    if (T == 0) return;
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
    const uint64_t policy = l2_policy_evict_first();
    int64_t sh_start[kW];
    int sh_len[kW];
    int max_len = 0;
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      sh_start[w] = starts[w];
      sh_len[w] = starts[w + 1] - starts[w];
      max_len = max(max_len, sh_len[w]);
    }
    const int n_issue = max_len * kW;
    // block index of issue slot i; -2 when the slot lies past its warp's share
    auto entry = [&](int i) -> long long {
      if (i >= n_issue) return -2;
      const int w = i % kW, j = i / kW;
      int64_t s0 = sh_start[0];
      int ln = sh_len[0];
#pragma unroll
      for (int ww = 1; ww < kW; ++ww)
        if (w == ww) {
          s0 = sh_start[ww];
          ln = sh_len[ww];
        }
      if (j >= ln) return -2;
      const int f = (int)(s0 + j);
      const int r = find_request(pre, B, f);
      const int nb = (pre[r + 1] - pre[r]) / Hkv;
      const int off = f - pre[r];
      const int h = off / nb;
      const int pg = lo + (off - h * nb);
      if (kPaged) return (long long)block_index<true>(p, r, h, (long long)p.table[(size_t)r * p.cols + pg]);
      return (long long)block_index<false>(p, r, h, pg);
    };
    long long tcur = entry(lane);
    long long tnxt = entry(32 + lane);
    bool aborted = false;
    for (int i0 = 0; i0 < n_issue; i0 += kIssue) {
      if ((i0 & 31) == 0 && i0 > 0) {
        tcur = tnxt;
        tnxt = entry(i0 + 32 + lane);
      }
      const long long e = __shfl_sync(0xffffffffu, tcur, (i0 + (lane & (kIssue - 1))) & 31);
      const int i = i0 + lane;
      if (lane < kIssue && e != -2) {
        const int st = (int)((unsigned)i % kNS);
        if (i >= kNS && !producer_wait(empty_s + 8 * st, (((unsigned)i / kNS) - 1u) & 1u, p.producer_sleep_ns)) {
          if (p.status != nullptr) atomicOr(p.status, FS_DEV_TIMEOUT);
          aborted = true;
        }
        if (!aborted) issue_page(p, &tmk, &tmv, base_s, meta_p, meta_s, full_s + 8 * st, st, e, policy);
      }
      if (i0 == 0) trace_mark<kTrace>(p, kW + 1, lane, 2);
      if (__any_sync(0xffffffffu, aborted)) break;
    }
    trace_mark<kTrace>(p, kW + 1, lane, 3);
    trace_mark<kTrace>(p, kW + 1, lane, 4);
    trace_mark<kTrace>(p, kW + 1, lane, 5, (unsigned long long)n_issue);
    return;  // the producer takes no part in the epilogue
  }

  // ============================ consumer warps ===============================
  const int g = lane >> 2, c = lane & 3;
  {  // pairs without pages in the window still need an output: zeros (LSE -inf)
    const int pairs = B * Hkv;
    const int p_lo = (int)((int64_t)blockIdx.x * pairs / gridDim.x);
    const int p_hi = (int)((int64_t)(blockIdx.x + 1) * pairs / gridDim.x);
    for (int pr = p_lo + warp; pr < p_hi; pr += kW) {
      const int r = pr / Hkv, h = pr % Hkv;
      if (pre[r + 1] != pre[r]) continue;
      for (int idx = lane; idx < p.G * kD; idx += 32)
        write_final(p, (size_t)r * p.Hq + (size_t)h * p.G + (idx >> 7), idx & (kD - 1), 0.f, -INFINITY);
    }
  }
  if (T == 0) return;
  const int64_t k = (int64_t)blockIdx.x * kW + warp;
  const int64_t f_begin = starts[warp];
  const int len_w = starts[warp + 1] - starts[warp];
  const StageOffsets off(lane);
  QueryFrag qf;
  WarpState ws;
  ws.reset();
  int r = 0, h = 0, nb = 1, len_eff = 0;
  int64_t pair_P = 0, pair_end = -1, piece_f0 = 0;
  bool first_piece = true;
  for (int j = 0; j < len_w; ++j) {
    const int64_t f = f_begin + j;
    if (f >= pair_end) {  // a new (request, kv head) piece starts
      r = find_request(pre, B, (int)f);
      nb = (pre[r + 1] - pre[r]) / Hkv;
      h = (int)((f - pre[r]) / nb);
      pair_P = pre[r] + (int64_t)h * nb;
      pair_end = pair_P + nb;
      piece_f0 = f;
      window_pages<kPaged>(p, r, lo, hi_cap, &len_eff);
      qf.load(p, r, h, lane);
    }
    const int i = j * kW + warp;
    const int st = (int)((unsigned)i % kNS);
    if (!mbar_wait_bounded(full_s + 8 * st, ((unsigned)i / kNS) & 1u, kTimeoutNs)) {
      if (lane == 0 && p.status != nullptr) atomicOr(p.status, FS_DEV_TIMEOUT);
      return;
    }
    if (j == 0) trace_mark<kTrace>(p, kW + 1, lane, 2);
    StageInfo si;
    if (read_stage_info(meta_p, st, si, meta_s) && p.debug_mode != 2 && p.debug_mode != 4) {
      consume_page<0>(base_s + st * kStageBytes, off, empty_s + 8 * st, lane, si, qf, p.qk_scale_log2,
                      (lo + (int)(f - pair_P)) * kPage, len_eff, ws);
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_s + 8 * st);
    }
    if (j + 1 == len_w) trace_mark<kTrace>(p, kW + 1, lane, 3);
    if (f + 1 != pair_end && j + 1 != len_w) continue;

    // ---- close the piece ------------------------------------------------------------
    ws.fold_zero_point(lane);
    float l = ws.l_run;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    // normaliser / max of the queries 2c, 2c+1 of this thread's accumulator columns
    const float l0 = __shfl_sync(0xffffffffu, l, 8 * c), l1 = __shfl_sync(0xffffffffu, l, 8 * c + 4);
    const float m0 = __shfl_sync(0xffffffffu, ws.m_run, 8 * c), m1 = __shfl_sync(0xffffffffu, ws.m_run, 8 * c + 4);
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    const float lse0 = l0 > 0.f ? (m0 + log2f(l0)) * kLn2 : -INFINITY;
    const float lse1 = l1 > 0.f ? (m1 + log2f(l1)) * kLn2 : -INFINITY;
    const size_t row0 = (size_t)r * p.Hq + (size_t)h * p.G;
    if (piece_f0 == pair_P && f + 1 == pair_end) {  // the whole pair: final output
#pragma unroll
      for (int i2 = 0; i2 < 8; ++i2) {
        const int d = 16 * i2 + 2 * g;
        if (2 * c < p.G) {
          write_final(p, row0 + 2 * c, d, ws.acc[i2][0] * inv0, lse0);
          write_final(p, row0 + 2 * c, d + 1, ws.acc[i2][2] * inv0, lse0);
        }
        if (2 * c + 1 < p.G) {
          write_final(p, row0 + 2 * c + 1, d, ws.acc[i2][1] * inv1, lse1);
          write_final(p, row0 + 2 * c + 1, d + 1, ws.acc[i2][3] * inv1, lse1);
        }
      }
    } else {
      // partial slot of this warp: O [Wt][2][G][kD], LSE [Wt][2][G]
      const size_t slot = ((size_t)k * 2 + (first_piece ? 0 : 1)) * p.G;
#pragma unroll
      for (int i2 = 0; i2 < 8; ++i2) {
        const int d = 16 * i2 + 2 * g;
        if (2 * c < p.G)
          *reinterpret_cast<float2*>(p.part_o + (slot + 2 * c) * kD + d) =
              make_float2(ws.acc[i2][0] * inv0, ws.acc[i2][2] * inv0);
        if (2 * c + 1 < p.G)
          *reinterpret_cast<float2*>(p.part_o + (slot + 2 * c + 1) * kD + d) =
              make_float2(ws.acc[i2][1] * inv1, ws.acc[i2][3] * inv1);
      }
      const float lq = __shfl_sync(0xffffffffu, l, (4 * lane) & 31);
      const float mq = __shfl_sync(0xffffffffu, ws.m_run, (4 * lane) & 31);
      if (lane < p.G) p.part_lse[slot + lane] = lq > 0.f ? (mq + log2f(lq)) * kLn2 : -INFINITY;
      // rebuilt here (T re-read from shared memory) so the loop above keeps no registers for it
      const CostMap cm{pre, B, Hkv, p.piece_cost};
      const Shares sh = make_shares<kW>(p, cm.total());
      const int c0 = cm.pair_cost(r, h, nb);  // cost position of the pair's first page
      const int64_t k0 = sh.owner(c0), k1 = sh.owner(c0 + nb - 1);
      const unsigned contributors = (unsigned)(k1 - k0 + 1);
      const int pair_id = r * Hkv + h;
      fence_acq_rel_gpu();  // releases this warp's partial before the ticket
      __syncwarp();
      unsigned ticket = 0;
      if (lane == 0) ticket = atomicAdd(p.counters + pair_id, 1u);
      ticket = __shfl_sync(0xffffffffu, ticket, 0);
      if (ticket == contributors - 1) {  // last contributor: merge the pair
        fence_acq_rel_gpu();
        merge_pair(p.part_o, p.part_lse, p.out, p.shard_o, p.shard_lse, p.G, k0, k1, sh.start(k0) >= c0 - cm.ovh,
                   row0, lane);
        if (lane == 0) p.counters[pair_id] = 0u;  // leave the ticket clean for the next call
      }
    }
    first_piece = false;
    ws.reset();
  }
  trace_mark<kTrace>(p, kW + 1, lane, 4);
  trace_mark<kTrace>(p, kW + 1, lane, 5, (unsigned long long)len_w);
  trace_mark<kTrace>(p, kW + 1, lane, 6, (unsigned long long)smid());
}

// ---------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------

// CTA shapes (consumer warps, ring stages, CTAs per SM the register budget must allow).
// FLASHSPEC_NUM_WARPS picks the shape by consumer-warp count (the reference's
// num_warps knob, triton_utils.py:101-116); FLASHSPEC_KERNEL_SHAPE picks by index.
struct Shape {
  int warps, stages, min_blocks, max_regs;  // max_regs: register cap of the balanced kernel
};
using DecodeKernelFn = void (*)(CUtensorMap, CUtensorMap, DecodeParams);
// Measured alternatives on B200 (cfg1): one CTA per SM with 11-12 consumer warps behind a
// single producer, 1.7-2x slower (one slow warp stalls the in-order producer and with it
// the whole SM); 2 CTAs of 6 consumer warps, 10% slower; 4 CTAs of 3, no faster.
constexpr Shape kShapes[] = {{4, 16, 3, 128}, {8, 16, 2, 112}};
constexpr int kNumShapes = 2;
constexpr int kDefaultShape = 0;          // split kernel
constexpr int kDefaultBalancedShape = 0;  // balanced kernel

template <bool kPaged, int kSi, int kMode>
__host__ DecodeKernelFn kernel_inst() {
  constexpr Shape sh = kShapes[kSi];
  return decode_kernel<kPaged, sh.warps, sh.stages, sh.min_blocks, kMode>;
}

template <bool kPaged, int kSi>
static DecodeKernelFn kernel_mode(int mode) {
  switch (mode) {
    case 1: return kernel_inst<kPaged, kSi, 1>();
    case 2: return kernel_inst<kPaged, kSi, 2>();
    default: return kernel_inst<kPaged, kSi, 0>();
  }
}

template <bool kPaged>
static DecodeKernelFn kernel_for(int shape, int mode) {
  return shape == 1 ? kernel_mode<kPaged, 1>(mode) : kernel_mode<kPaged, 0>(mode);
}

template <bool kPaged, int kSi, bool kTrace = false>
__host__ DecodeKernelFn balanced_inst() {
  constexpr Shape sh = kShapes[kSi];
  return decode_balanced_kernel<kPaged, sh.warps, sh.stages, sh.max_regs, kTrace>;
}

// FLASHSPEC_TRACE_PTR (profiling only): device address of a zeroed uint64 buffer of
// ctas * (warps + 1) * 8 words; the balanced kernel of shape 0 then records its
// per-warp timeline there (trace_mark), the split kernel its per-CTA and per-pair
// timeline (4 * ctas + 8 * pairs words, split_mark).
static unsigned long long* trace_ptr() {
  const char* v = getenv("FLASHSPEC_TRACE_PTR");
  return v ? reinterpret_cast<unsigned long long*>(strtoull(v, nullptr, 0)) : nullptr;
}

template <bool kPaged>
static DecodeKernelFn balanced_for_untraced(int shape) {
  return shape == 1 ? balanced_inst<kPaged, 1>() : balanced_inst<kPaged, 0>();
}

template <bool kPaged>
static DecodeKernelFn balanced_for(int shape) {
  if (shape == 1) return balanced_inst<kPaged, 1>();
  return trace_ptr() != nullptr ? balanced_inst<kPaged, 0, true>() : balanced_inst<kPaged, 0>();
}

static int smem_bytes(int shape) {
  const Shape sh = kShapes[shape];
  return 1024 + sh.stages * (kStageBytes + kMetaBytes + 16);
}

// the balanced kernel adds its per-request prefix table
static int smem_balanced(int shape, int batch) {
  return smem_bytes(shape) + ((4 * (batch + 1) + 4 * (kShapes[shape].warps + 1) + 15) & ~15);
}

// FLASHSPEC_DEBUG_MODE (profiling only, results are wrong when set): 1 = skip the math,
// 2 = data movement only (split kernel; the balanced kernel honours 2), 3 = no copies of
// the pages' scale / zero-point words, 4 = 2 and 3 (balanced kernel).
static int debug_mode() {
  const char* v = getenv("FLASHSPEC_DEBUG_MODE");
  const int m = v ? atoi(v) : 0;
  return (m >= 1 && m <= 4) ? m : 0;
}

static int shape_choice() {
  if (const char* v = getenv("FLASHSPEC_KERNEL_SHAPE")) {
    const int s = atoi(v);
    if (s >= 0 && s < kNumShapes) return s;
  }
  if (const char* v = getenv("FLASHSPEC_NUM_WARPS")) {
    const int w = atoi(v);
    for (int s = 0; s < kNumShapes; ++s)
      if (kShapes[s].warps == w) return s;
  }
  return -1;
}

template <bool kPaged>
static int configure_kernel(int device, int shape) {
  static bool done[2][kNumShapes][kMaxDevices] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= kMaxDevices) return fail_cuda("device ordinal beyond the library's table");
  if (done[kPaged][shape][device]) return FS_OK;
  cudaError_t e;
  for (int mode = 0; mode < 3; ++mode)
    if ((e = cudaFuncSetAttribute(kernel_for<kPaged>(shape, mode), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smem_bytes(shape))) != cudaSuccess)
      return fail_cuda("shared-memory limit of the split decode kernel", e);
  const DecodeKernelFn balanced[2] = {balanced_for_untraced<kPaged>(shape),
                                      shape == 0 ? balanced_inst<kPaged, 0, true>() : balanced_for_untraced<kPaged>(shape)};
  for (DecodeKernelFn fn : balanced)
    if ((e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_balanced(shape, kMaxSKBatch))) !=
        cudaSuccess)
      return fail_cuda("shared-memory limit of the balanced decode kernel", e);
  done[kPaged][shape][device] = true;
  return FS_OK;
}

// Raises the shared-memory limits of every kernel a plan may pick (the occupancy queries
// of the planner need them); the paged instantiations are the ones those queries use.
template <bool kPaged>
static int configure_shapes(int device, int forced) {
  const int shapes[2] = {forced >= 0 ? forced : kDefaultShape, forced >= 0 ? forced : kDefaultBalancedShape};
  for (int sh : shapes) {
    int st = configure_kernel<kPaged>(device, sh);
    if (st == FS_OK) st = configure_kernel<true>(device, sh);
    if (st != FS_OK) return st;
  }
  return FS_OK;
}

static int resident_ctas(int device, int shape) {
  static int cached[kNumShapes][kMaxDevices] = {};
  static std::mutex mu;
  // the occupancy query needs the kernel's dynamic shared-memory limit raised first
  if (configure_kernel<true>(device, shape) != FS_OK) return device_sm_count(device);
  std::lock_guard<std::mutex> lock(mu);
  if (cached[shape][device] > 0) return cached[shape][device];
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel_for<true>(shape, 0),
                                                    (kShapes[shape].warps + 1) * 32, smem_bytes(shape)) != cudaSuccess ||
      per_sm <= 0)
    per_sm = 1;
  cached[shape][device] = per_sm * device_sm_count(device);
  return cached[shape][device];
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// View of an int8 KV array as rows of 128 bytes; one box = one 16-row page block,
// landing in shared memory with the 128-byte swizzle.
static int make_kv_map(CUtensorMap* map, const void* base, uint64_t rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail_cuda("cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kD};
  cuuint32_t box[2] = {(cuuint32_t)kD, (cuuint32_t)kPage};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FS_OK : fail_cuda("cuTensorMapEncodeTiled", r);
}

// Tensor maps depend only on the base address and the row count (box, swizzle and
// strides are fixed), so the last few are kept: a serving loop calls with the same
// pools every step and saves the driver's encode.
static int cached_kv_map(CUtensorMap* map, const void* base, uint64_t rows) {
  struct Entry {
    const void* base;
    uint64_t rows;
    CUtensorMap map;
  };
  static Entry cache[16] = {};
  static int next = 0;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& e : cache)
      if (e.base == base && e.rows == rows && base != nullptr) {
        *map = e.map;
        return FS_OK;
      }
  }
  const int st = make_kv_map(map, base, rows);
  if (st != FS_OK) return st;
  std::lock_guard<std::mutex> lock(mu);
  cache[next] = Entry{base, rows, *map};
  next = (next + 1) % 16;
  return FS_OK;
}

static int64_t max_pages_of(const FsDecodeArgs* a) {
  int64_t np = ((int64_t)a->max_seq_len + kPage - 1) / kPage;
  if (a->layout == FS_LAYOUT_PAGED)
    np = np < a->table_cols ? np : a->table_cols;
  else
    np = np < a->num_blocks ? np : a->num_blocks;
  int64_t lo = a->page_begin > 0 ? a->page_begin : 0;
  int64_t hi = a->page_end > 0 && a->page_end < np ? a->page_end : np;
  return hi > lo ? hi - lo : 0;
}

// Split policy.  Every CTA carries a fixed cost (set-up latency before its first page
// lands, the warp merge, the ticket) worth roughly kCtaOverheadPages pages of streaming,
// and CTAs run in waves of `slots` (resident CTAs).  With fewer (request, kv head) pairs
// than slots, split to fill exactly one wave; otherwise pick the S minimising
// waves(S) * (pages per CTA + overhead).  Fitted on B200 sweeps of the benchmark
// configurations.
static int resolve_splits(const FsDecodeArgs* a, int device, int shape) {
  if (a->num_splits > 0) return a->num_splits;
  constexpr int64_t kCtaOverheadPages = 24;
  const int64_t pairs = (int64_t)a->batch * a->kv_heads;
  const int64_t maxp = max_pages_of(a);
  const int64_t slots = resident_ctas(device, shape);
  const int64_t cap = maxp / (kShapes[shape].warps * 4) > 1 ? maxp / (kShapes[shape].warps * 4) : 1;
  if (pairs <= 0 || maxp <= 0) return 1;
  int64_t best = 1;
  if (pairs <= slots) {  // one wave: split each pair as far as the wave allows
    best = slots / pairs;
  } else {
    double best_cost = 1e300;
    for (int64_t s = 1; s <= 64; ++s) {
      const int64_t waves = (pairs * s + slots - 1) / slots;
      const double cost = (double)waves * (double)((maxp + s - 1) / s + kCtaOverheadPages);
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        best = s;
      }
    }
  }
  if (best > cap) best = cap;
  if (best < 1) best = 1;
  if (best > 256) best = 256;
  return (int)best;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Plan of one call: the balanced kernel on `ctas` CTAs, or the split kernel with `splits`.
struct Plan {
  bool balanced;
  int splits;
  int ctas;
  int shape;
};

static int balanced_per_sm(int device, int shape, int batch) {
  static int cached[kNumShapes][kMaxDevices][16] = {};  // by 512-byte bucket of the prefix table
  static std::mutex mu;
  const int smem = smem_balanced(shape, batch);
  int bucket = (smem - smem_bytes(shape)) / 512;
  if (bucket > 15) bucket = 15;
  std::lock_guard<std::mutex> lock(mu);
  int& c = cached[shape][device][bucket];
  if (c == 0) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, balanced_for<true>(shape), (kShapes[shape].warps + 1) * 32,
                                                      smem_bytes(shape) + (bucket + 1) * 512) != cudaSuccess ||
        per_sm <= 0)
      per_sm = 1;
    c = per_sm;
  }
  return c;
}

// Weight step between CTA tiers of the balanced kernel, in 1/1024 (Shares).
// FLASHSPEC_TIER_SKEW overrides it (profiling).
static int tier_skew() {
  constexpr int kDefaultSkew = 26;  // B200 sweep of the benchmark configurations
  if (const char* v = getenv("FLASHSPEC_TIER_SKEW")) {
    const int s = atoi(v);
    if (s >= 0 && s <= 256) return s;
  }
  return kDefaultSkew;
}

// Virtual pages the balanced kernel charges per (request, kv head) pair (CostMap).
// FLASHSPEC_PIECE_COST overrides it (profiling).
constexpr int kDefaultPieceCost = 6;  // B200 sweep of the benchmark configurations
static int piece_cost() {
  if (const char* v = getenv("FLASHSPEC_PIECE_COST")) {
    const int c = atoi(v);
    if (c >= 0 && c <= 64) return c;
  }
  return kDefaultPieceCost;
}

// FLASHSPEC_PRODUCER_SLEEP_NS overrides the producer's suspend hint (profiling; 0 spins).
static int producer_sleep_ns() {
  if (const char* v = getenv("FLASHSPEC_PRODUCER_SLEEP_NS")) {
    const int n = atoi(v);
    if (n >= 0 && n <= 100000) return n;
  }
  return (int)kProducerSleepNs;
}

// FLASHSPEC_DECODE_KERNEL=split|balanced forces a kernel (profiling, tests).
static int kernel_override() {
  const char* v = getenv("FLASHSPEC_DECODE_KERNEL");
  if (v == nullptr) return 0;
  if (strcmp(v, "split") == 0) return 1;
  if (strcmp(v, "balanced") == 0) return 2;
  return 0;
}

// An explicit num_splits selects the split kernel.  Otherwise the balanced kernel runs
// when there are more (request, kv head) pairs than resident CTAs (then split CTAs come
// in several unequal waves); with fewer pairs the split kernel fills exactly one wave.
// `forced` is a shape from FLASHSPEC_KERNEL_SHAPE / FLASHSPEC_NUM_WARPS or -1; each kernel
// otherwise runs its own default shape.
static Plan make_plan(const FsDecodeArgs* a, int device, int forced) {
  Plan pl{false, 1, 0, 0};
  const int ov = kernel_override();
  const int64_t pairs = (int64_t)a->batch * a->kv_heads;
  const int64_t maxp = max_pages_of(a);
  const int shape = forced >= 0 ? forced : kDefaultBalancedShape;
  const int split_shape = forced >= 0 ? forced : kDefaultShape;
  const int warps = kShapes[shape].warps;
  bool balanced = a->num_splits <= 0 && a->batch <= kMaxSKBatch && maxp > 0 && pairs * (maxp + 64) < (1ll << 31);
  if (balanced) {
    const int64_t slots = (int64_t)balanced_per_sm(device, shape, a->batch) * device_sm_count(device);
    const int64_t t_est = pairs * maxp;
    pl.ctas = (int)std::max<int64_t>(1, std::min<int64_t>(slots, t_est / (warps * 4)));
    // the share arithmetic (Shares) needs fewer than 4096 warps
    pl.ctas = (int)std::min<int64_t>(pl.ctas, 4095 / warps);
    // With no more pairs than resident CTAs the split kernel already fills one wave with
    // equal CTAs (measured faster); with few long pairs the merges would serialise.
    const int64_t split_slots = resident_ctas(device, split_shape);
    const int64_t contributors = (int64_t)pl.ctas * warps / pairs + 1;
    if ((contributors > 16 || pairs <= split_slots) && ov != 2) balanced = false;
    if (ov == 1) balanced = false;
  }
  if (balanced) {
    pl.balanced = true;
    pl.splits = 0;
    pl.shape = shape;
  } else {
    pl.splits = resolve_splits(a, device, split_shape);
    pl.shape = split_shape;
  }
  return pl;
}

static size_t workspace_balanced(const FsDecodeArgs* a, int ctas, int shape) {
  const size_t G = (size_t)(a->q_heads / a->kv_heads);
  const size_t slots = (size_t)ctas * kShapes[shape].warps * 2 * G;
  return align256(slots * kD * 4) + align256(slots * 4);
}

static size_t workspace_for(const FsDecodeArgs* a, int splits) {
  if (splits <= 1) return 0;
  const size_t G = (size_t)(a->q_heads / a->kv_heads);
  const size_t units = (size_t)a->batch * a->kv_heads * splits * G;
  return align256(units * kD * 4) + align256(units * 4);
}

// The shapes of the tuned TMA kernels: D = 128, pages = quant blocks = 16 tokens, fp16 q.
static bool tuned_shape(const FsDecodeArgs* a) {
  return a->head_dim == kD && a->block_size == kPage && (a->page_size == 0 || a->page_size == kPage) &&
         a->q_dtype == FS_F16;
}

static int validate(const FsDecodeArgs* a, int layout) {
  if (a == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if (a->layout != layout) return FS_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->q_heads <= 0 || a->kv_heads <= 0) return FS_ERR_INVALID_ARGUMENT;
  if (a->q_heads % a->kv_heads) return FS_ERR_INVALID_ARGUMENT;
  const int G = a->q_heads / a->kv_heads;
  if (G > kMaxG) return FS_ERR_UNSUPPORTED;
  if (a->q_dtype != FS_F16 && a->q_dtype != FS_BF16) return FS_ERR_UNSUPPORTED;
  if (a->block_size <= 0 || a->page_size < 0) return FS_ERR_INVALID_ARGUMENT;
  if (layout == FS_LAYOUT_PAGED && a->page_size > 0 && a->page_size % a->block_size) return FS_ERR_INVALID_ARGUMENT;
  if (!tuned_shape(a) && !generic_supports(a)) return FS_ERR_UNSUPPORTED;
  if (a->kv_format != FS_KV_AFFINE_BLOCK && a->kv_format != FS_KV_SYMMETRIC) return FS_ERR_INVALID_ARGUMENT;
  if (a->q == nullptr || a->k_values == nullptr || a->v_values == nullptr || a->k_scale == nullptr ||
      a->v_scale == nullptr)
    return FS_ERR_INVALID_ARGUMENT;
  if (a->kv_format == FS_KV_AFFINE_BLOCK && (a->k_zero == nullptr || a->v_zero == nullptr))
    return FS_ERR_INVALID_ARGUMENT;
  if (a->shard_o == nullptr && a->out == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if ((a->shard_o == nullptr) != (a->shard_lse == nullptr)) return FS_ERR_INVALID_ARGUMENT;
  if (a->num_blocks <= 0 || a->max_seq_len < 0) return FS_ERR_INVALID_ARGUMENT;
  if (layout == FS_LAYOUT_PAGED) {
    if (a->block_table == nullptr || a->lengths == nullptr || a->table_cols <= 0) return FS_ERR_INVALID_ARGUMENT;
    const int64_t page = a->page_size > 0 ? a->page_size : a->block_size;
    if ((uint64_t)a->num_blocks * a->kv_heads * page >= (1ull << 31)) return FS_ERR_UNSUPPORTED;
  } else {
    if ((uint64_t)a->batch * a->kv_heads * a->num_blocks * a->block_size >= (1ull << 31)) return FS_ERR_UNSUPPORTED;
    if ((int64_t)a->max_seq_len > a->num_blocks * a->block_size) return FS_ERR_INVALID_ARGUMENT;
  }
  if ((reinterpret_cast<uintptr_t>(a->k_values) | reinterpret_cast<uintptr_t>(a->v_values) |
       reinterpret_cast<uintptr_t>(a->q)) & 15)
    return FS_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(a->k_zero) | reinterpret_cast<uintptr_t>(a->v_zero) |
       reinterpret_cast<uintptr_t>(a->k_scale) | reinterpret_cast<uintptr_t>(a->v_scale)) & 3)
    return FS_ERR_ALIGNMENT;
  // the symmetric format's per-token scales travel as 64-byte bulk copies
  if (a->kv_format == FS_KV_SYMMETRIC &&
      ((reinterpret_cast<uintptr_t>(a->k_scale) | reinterpret_cast<uintptr_t>(a->v_scale)) & 15))
    return FS_ERR_ALIGNMENT;
  return FS_OK;
}

// Plan of a decode with the fused exchange epilogue: the split kernel, one wave at most
// (every CTA resident at once, so a CTA waiting for its peers never holds a slot that
// another CTA of the same call needs); FS_ERR_UNSUPPORTED when the pairs alone exceed
// one wave or the exchange's per-pair counters.
static int exchange_plan(const FsDecodeArgs* a, int device, int forced, Plan* pl) {
  const int shape = forced >= 0 ? forced : kDefaultShape;
  const int64_t pairs = (int64_t)a->batch * a->kv_heads;
  const int64_t slots = resident_ctas(device, shape);
  if (pairs > slots || pairs > kXMaxPairs) return FS_ERR_UNSUPPORTED;
  int64_t s = resolve_splits(a, device, shape);
  if (s * pairs > slots) s = slots / pairs;
  *pl = Plan{false, (int)std::max<int64_t>(s, 1), 0, shape};
  return FS_OK;
}

static int validate_exchange(const FsDecodeArgs* a, const FsExchangeArgs* x) {
  if (x == nullptr || x->world < 1 || x->world > kXMaxRanks || x->rank < 0 || x->rank >= x->world ||
      x->out == nullptr || x->timeout_ns <= 0)
    return FS_ERR_INVALID_ARGUMENT;
  if (x->out_dtype != FS_F16 && x->out_dtype != FS_F32) return FS_ERR_UNSUPPORTED;
  if (a->shard_o != nullptr || a->shard_lse != nullptr) return FS_ERR_INVALID_ARGUMENT;
  const int64_t rows = (int64_t)a->batch * a->q_heads;
  if (x->slot_floats < rows * (a->head_dim + 1) || x->slot_floats % 64) return FS_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < x->world; ++r)
    if (x->bufs[r] == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if (!exchange_buffers_match(x)) return FS_ERR_INVALID_ARGUMENT;
  if (!tuned_shape(a)) return FS_ERR_UNSUPPORTED;
  return FS_OK;
}

template <bool kPaged>
static int launch_decode(const FsDecodeArgs* a_in, void* stream, const FsExchangeArgs* x = nullptr) {
  FsDecodeArgs ax;
  const FsDecodeArgs* a = a_in;
  if (x != nullptr && a_in != nullptr) {  // the exchange writes x->out; the decode's own output is unused
    ax = *a_in;
    ax.out = x->out;
    a = &ax;
  }
  int st = validate(a, kPaged ? FS_LAYOUT_PAGED : FS_LAYOUT_CONTIGUOUS);
  if (st != FS_OK) return st;
  if (x != nullptr && (st = validate_exchange(a_in, x)) != FS_OK) return st;
  int device = 0;
  if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
  if (!tuned_shape(a)) return launch_generic_decode(a, device, stream);
  const int forced = shape_choice();
  if ((st = configure_shapes<kPaged>(device, forced)) != FS_OK) return st;
  Plan pl;
  if (x != nullptr) {
    if ((st = exchange_plan(a, device, forced, &pl)) != FS_OK) return st;
  } else {
    pl = make_plan(a, device, forced);
  }
  const int shape = pl.shape;
  const size_t need = pl.balanced ? workspace_balanced(a, pl.ctas, shape) : workspace_for(a, pl.splits);
  if (need > 0 && (a->workspace == nullptr || a->workspace_bytes < need)) return FS_ERR_WORKSPACE;
  if ((pl.balanced || pl.splits > 1) && (a->tickets == nullptr || a->ticket_count < (int64_t)a->batch * a->kv_heads))
    return FS_ERR_WORKSPACE;

  const uint64_t rows = kPaged ? (uint64_t)a->num_blocks * a->kv_heads * kPage
                               : (uint64_t)a->batch * a->kv_heads * a->num_blocks * kPage;
  CUtensorMap tmk, tmv;
  if ((st = cached_kv_map(&tmk, a->k_values, rows)) != FS_OK) return st;
  if ((st = cached_kv_map(&tmv, a->v_values, rows)) != FS_OK) return st;

  DecodeParams p{};
  p.q = reinterpret_cast<const __half*>(a->q);
  p.k_scale = a->k_scale;
  p.k_zero = a->k_zero;
  p.v_scale = a->v_scale;
  p.v_zero = a->v_zero;
  p.table = a->block_table;
  p.lengths = a->lengths;
  p.out = reinterpret_cast<__half*>(a->out);
  p.shard_o = a->shard_o;
  p.shard_lse = a->shard_lse;
  p.status = a->device_status;
  p.trace = trace_ptr();
  p.B = a->batch;
  p.Hq = a->q_heads;
  p.Hkv = a->kv_heads;
  p.G = a->q_heads / a->kv_heads;
  p.S = pl.balanced ? 1 : pl.splits;
  p.cols = a->table_cols;
  p.num_blocks = a->num_blocks;
  p.max_seq_len = a->max_seq_len;
  p.page_begin = a->page_begin;
  p.page_end = a->page_end;
  p.zp_count = kPaged ? a->num_blocks * a->kv_heads : (int64_t)a->batch * a->kv_heads * a->num_blocks;
  p.qk_scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.tier_ctas = device_sm_count(device);
  p.skew = tier_skew();
  p.piece_cost = piece_cost();
  p.debug_mode = debug_mode();
  p.sym = a->kv_format == FS_KV_SYMMETRIC;
  p.producer_sleep_ns = producer_sleep_ns();
  if (x != nullptr) {
    for (int r = 0; r < x->world; ++r) p.xbufs[r] = x->bufs[r];
    p.xout = x->out;
    p.xstatus = x->device_status;
    p.xslot = x->slot_floats;
    p.xtimeout_ns = x->timeout_ns;
    p.xworld = x->world;
    p.xrank = x->rank;
    p.xout_dtype = x->out_dtype;
  }
  if (need > 0) {
    const size_t G = (size_t)p.G;
    const size_t units = pl.balanced ? (size_t)pl.ctas * kShapes[shape].warps * 2 * G
                                     : (size_t)a->batch * a->kv_heads * pl.splits * G;
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
    p.part_o = reinterpret_cast<float*>(ws);
    p.part_lse = reinterpret_cast<float*>(ws + align256(units * kD * 4));
  }
  p.counters = reinterpret_cast<unsigned*>(a->tickets);
  const int threads = (kShapes[shape].warps + 1) * 32;
  if (pl.balanced) {
    balanced_for<kPaged>(shape)<<<(unsigned)pl.ctas, threads, smem_balanced(shape, a->batch),
                                  reinterpret_cast<cudaStream_t>(stream)>>>(tmk, tmv, p);
  } else {
    const int64_t grid = (int64_t)a->batch * a->kv_heads * pl.splits;
    if (grid >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
    kernel_for<kPaged>(shape, debug_mode())<<<(unsigned)grid, threads, smem_bytes(shape),
                                              reinterpret_cast<cudaStream_t>(stream)>>>(tmk, tmv, p);
  }
  return launch_status(pl.balanced ? "balanced decode kernel launch" : "split decode kernel launch");
}

}  // namespace fsb

extern "C" {

int fs_decode_workspace_size(const FsDecodeArgs* a, size_t* bytes, int32_t* splits_out) {
  if (a == nullptr || bytes == nullptr) return FS_ERR_INVALID_ARGUMENT;
  int st = fsb::validate(a, a->layout);
  if (st != FS_OK) return st;
  int device = 0;
  if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return fsb::fail_cuda("cudaGetDevice", e);
  if (!fsb::tuned_shape(a)) {
    int splits = 1;
    *bytes = fsb::generic_workspace(a, device, &splits);
    if (splits_out) *splits_out = splits;
    return FS_OK;
  }
  const int forced = fsb::shape_choice();
  if ((st = fsb::configure_shapes<true>(device, forced)) != FS_OK) return st;
  const fsb::Plan pl = fsb::make_plan(a, device, forced);
  *bytes = pl.balanced ? fsb::workspace_balanced(a, pl.ctas, pl.shape) : fsb::workspace_for(a, pl.splits);
  if (splits_out) *splits_out = pl.balanced ? 0 : pl.splits;
  return FS_OK;
}

int fs_paged_decode_exchange_workspace_size(const FsDecodeArgs* a, size_t* bytes, int32_t* splits_out) {
  if (a == nullptr || bytes == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if (a->layout != FS_LAYOUT_PAGED || !fsb::tuned_shape(a)) return FS_ERR_UNSUPPORTED;
  int device = 0;
  if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return fsb::fail_cuda("cudaGetDevice", e);
  const int forced = fsb::shape_choice();
  int st = fsb::configure_shapes<true>(device, forced);
  if (st != FS_OK) return st;
  fsb::Plan pl;
  if ((st = fsb::exchange_plan(a, device, forced, &pl)) != FS_OK) return st;
  *bytes = fsb::workspace_for(a, pl.splits);
  if (splits_out) *splits_out = pl.splits;
  return FS_OK;
}

int fs_paged_decode_exchange(const FsDecodeArgs* args, const FsExchangeArgs* x, void* stream) {
  if (x == nullptr) return FS_ERR_INVALID_ARGUMENT;
  return fsb::launch_decode<true>(args, stream, x);
}

int fs_fused_decode(const FsDecodeArgs* args, void* stream) { return fsb::launch_decode<false>(args, stream); }

int fs_paged_decode(const FsDecodeArgs* args, void* stream) { return fsb::launch_decode<true>(args, stream); }

}  // extern "C"

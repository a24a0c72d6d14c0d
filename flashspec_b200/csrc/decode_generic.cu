// Decode attention for the INT8 cache shapes outside the tuned kernels of decode.cu:
// head_dim 32/64/128/256, any quantization block up to 64 tokens, pages of several
// quantization blocks, and fp16 or bf16 q / out.  The reference accepts all of these
// (src/flashspec/triton_paged.py:242-246 page = multiple of the quant block;
// triton_utils.py:40-45 head_dim <= 256; its own GPU parity tests run head_dim 64,
// tests/test_flashspec.py:92-125,177-198).
//
// Design.  One CTA of kGW warps per (request, kv head, split).  The warps take the
// split's quantization blocks ("units", qb tokens each) round robin; a warp stages a
// unit's K and V bytes in its own shared-memory buffers with 16-byte cp.async copies
// (two buffers: the next unit loads while this one is used; rows padded by 16 bytes so
// the row-per-lane reads below are free of bank conflicts), then
//   * scores: lane t takes token t of a 32-token slice, s_q = sum_d q_q[d] (u_d - zp)
//     * scale, q read from shared memory as a broadcast (fp32);
//   * online softmax per query with warp reductions (log2 domain, exp2);
//   * O: lane l owns head dims [l*D/32, (l+1)*D/32) and accumulates
//     sum_t p_q[t] * scale_v * (u_td - zp_v) for every query of the kv head.
// The warps' (m, l, O) are merged in shared memory at the end; one split writes the
// output (or the (O, LSE) partial of a sequence shard), several write partials that
// fs_merge_partials combines.  fp32 arithmetic throughout; empty sequences give 0.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <stdint.h>

#include "../../include/flashspec_b200.h"
#include "common.h"
#include "generic.h"

namespace fsb {

constexpr int kGW = 4;             // warps per CTA
constexpr int kGMaxG = 8;          // query heads per kv head
constexpr int kGMaxUnitBytes = 12 * 1024;  // qb * (D + 16), one staged K or V unit

struct GenericParams {
  const void* q;
  const int8_t* kval;
  const int8_t* vval;
  const float* kscale;
  const float* vscale;
  const int16_t* kzero;
  const int16_t* vzero;
  const int64_t* table;
  const int64_t* lengths;
  void* out;
  float* shard_o;
  float* shard_lse;
  float* part_o;    // [S][B * Hq][D] when S > 1
  float* part_lse;  // [S][B * Hq]
  uint32_t* status;
  int B, Hq, Hkv, G, S, cols, qb, bpp, paged, bf16;
  int sym;             // FS_KV_SYMMETRIC: per-token scales, no zero points
  int64_t num_blocks;  // paged: pages; contiguous: quant blocks per (request, kv head)
  int64_t max_seq_len, page_begin, page_end;
  float qk_scale_log2;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Tokens of request r that count, and the quantization blocks that hold them.
__device__ __forceinline__ void generic_extent(const GenericParams& p, int r, int& len, int& units) {
  int64_t n = p.max_seq_len;
  if (p.lengths != nullptr) n = min(n, p.lengths[r]);
  n = max(n, (int64_t)0);
  const int64_t cap = p.paged ? (int64_t)p.cols * p.bpp * p.qb : p.num_blocks * p.qb;
  n = min(n, cap);
  len = (int)n;
  units = (int)((n + p.qb - 1) / p.qb);
}

// Block index (in quant blocks of the values array) of unit u of (r, h); -1 when the
// page is unallocated or outside the pool (reported in the status word).
__device__ __forceinline__ int64_t generic_block(const GenericParams& p, int r, int h, int u) {
  if (!p.paged) return ((int64_t)r * p.Hkv + h) * p.num_blocks + u;
  const int lp = u / p.bpp, sub = u - lp * p.bpp;
  const int64_t phys = p.table[(size_t)r * p.cols + lp];
  if (phys < 0) return -1;
  if (phys >= p.num_blocks) {
    if (p.status != nullptr) atomicOr(p.status, FS_DEV_BAD_PAGE);
    return -1;
  }
  return (phys * p.Hkv + h) * p.bpp + sub;
}

template <int kDim>
__global__ void __launch_bounds__(kGW * 32) decode_generic_kernel(const GenericParams p) {
  constexpr int kRow = kDim + 16;  // padded shared-memory row of one token
  constexpr int kDpl = kDim / 32;  // head dims per lane in the O accumulation
  extern __shared__ __align__(16) uint8_t gsm[];
  const int qb = p.qb;
  const int unit_bytes = qb * kRow;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t* wbuf = gsm + (size_t)warp * 4 * unit_bytes;  // [2 buffers][K | V]
  float* qs = reinterpret_cast<float*>(gsm + (size_t)kGW * 4 * unit_bytes);  // [G][D]
  float* ps = qs + kGMaxG * kDim + warp * kGMaxG * 64;  // [G][64] probabilities of this warp

  const int S = p.S, split = blockIdx.x % S, bh = blockIdx.x / S;
  const int h = bh % p.Hkv, r = bh / p.Hkv, G = p.G;
  int len, units;
  generic_extent(p, r, len, units);
  const int lo = (int)min((int64_t)units, max(p.page_begin, (int64_t)0) * p.bpp);
  const int hi = p.page_end > 0 ? (int)min((int64_t)units, p.page_end * p.bpp) : units;
  const int span = max(hi - lo, 0), chunk = (span + S - 1) / S;
  const int u0 = min(lo + split * chunk, max(hi, lo)), u1 = min(u0 + chunk, max(hi, lo));

  // q of the kv head's G query heads, fp32
  for (int i = threadIdx.x; i < G * kDim; i += kGW * 32) {
    const size_t src = ((size_t)r * p.Hq + (size_t)h * G + i / kDim) * kDim + (i % kDim);
    qs[i] = p.bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[src])
                   : __half2float(reinterpret_cast<const __half*>(p.q)[src]);
  }
  __syncthreads();

  float m[kGMaxG], l[kGMaxG], acc[kGMaxG][kDpl];
#pragma unroll
  for (int g = 0; g < kGMaxG; ++g) {
    m[g] = -1.0e30f;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < kDpl; ++j) acc[g][j] = 0.f;
  }

  // stage unit u (if any) of this warp into buffer b; returns its block index
  auto stage = [&](int u, int b) -> int64_t {
    int64_t e = -1;
    if (u < u1) e = generic_block(p, r, h, u);
    if (e >= 0) {
      const int8_t* ks = p.kval + e * (int64_t)qb * kDim;
      const int8_t* vs = p.vval + e * (int64_t)qb * kDim;
      uint8_t* kd = wbuf + (size_t)b * 2 * unit_bytes;
      uint8_t* vd = kd + unit_bytes;
      const int chunks = qb * kDim / 16;
      for (int c = lane; c < chunks; c += 32) {
        const int row = c / (kDim / 16), col = (c % (kDim / 16)) * 16;
        cp_async16(kd + row * kRow + col, ks + (size_t)c * 16);
        cp_async16(vd + row * kRow + col, vs + (size_t)c * 16);
      }
    }
    cp_async_commit();
    return e;
  };

  int u = u0 + warp;
  int64_t e_cur = stage(u, 0);
  for (int it = 0; u < u1; ++it, u += kGW) {
    const int b = it & 1;
    const int64_t e_next = stage(u + kGW, b ^ 1);
    cp_async_wait_prev();
    __syncwarp();
    if (e_cur >= 0) {
      // affine: one (scale, zero point) per unit, values stored as u - 128; symmetric:
      // one scale per token (read per lane / per token below), values as stored
      const float ksc_u = p.sym ? 1.f : p.kscale[e_cur], vsc_u = p.sym ? 1.f : p.vscale[e_cur];
      const float kz = p.sym ? 128.f : (float)p.kzero[e_cur], vz = p.sym ? 128.f : (float)p.vzero[e_cur];
      const uint8_t* kd = wbuf + (size_t)b * 2 * unit_bytes;
      const uint8_t* vd = kd + unit_bytes;
      for (int t0 = 0; t0 < qb; t0 += 32) {
        const int nt = min(32, qb - t0);
        const int tok = u * qb + t0 + lane;
        // ---- scores of token t0 + lane for every query
        float s[kGMaxG];
#pragma unroll
        for (int g = 0; g < kGMaxG; ++g) s[g] = 0.f;
        if (lane < nt) {
          const uint8_t* row = kd + (t0 + lane) * kRow;
#pragma unroll 2
          for (int d0 = 0; d0 < kDim; d0 += 16) {
            const uint4 w = *reinterpret_cast<const uint4*>(row + d0);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            float kf[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
              kf[j] = (float)((int)(int8_t)(ww[j >> 2] >> (8 * (j & 3))) + 128) - kz;
#pragma unroll
            for (int g = 0; g < kGMaxG; ++g) {
              if (g < G) {
                const float4* qv = reinterpret_cast<const float4*>(qs + g * kDim + d0);
                float a = s[g];
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                  const float4 q4 = qv[j4];
                  a = fmaf(q4.x, kf[4 * j4], a);
                  a = fmaf(q4.y, kf[4 * j4 + 1], a);
                  a = fmaf(q4.z, kf[4 * j4 + 2], a);
                  a = fmaf(q4.w, kf[4 * j4 + 3], a);
                }
                s[g] = a;
              }
            }
          }
        }
        const bool valid = lane < nt && tok < len;
        const size_t tok_at = (size_t)e_cur * qb + t0 + lane;  // this lane's token in the scale arrays
        const float ksc = p.sym ? (lane < nt ? p.kscale[tok_at] : 0.f) : ksc_u;
        const float vsc = p.sym ? (lane < nt ? p.vscale[tok_at] : 0.f) : vsc_u;
        // ---- online softmax per query (log2 domain)
#pragma unroll
        for (int g = 0; g < kGMaxG; ++g) {
          if (g < G) {
            const float t = valid ? s[g] * ksc * p.qk_scale_log2 : -INFINITY;
            float mx = t;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_new = fmaxf(m[g], mx);
            const float alpha = exp2f(m[g] - m_new);
            m[g] = m_new;
            const float pr = valid ? exp2f(t - m_new) : 0.f;
            l[g] = l[g] * alpha + pr;
#pragma unroll
            for (int j = 0; j < kDpl; ++j) acc[g][j] *= alpha;
            ps[g * 64 + lane] = pr * vsc;
          }
        }
        __syncwarp();
        // ---- O += P (V - zp): lane owns head dims lane*kDpl ..
        for (int t = 0; t < nt; ++t) {
          const uint8_t* vrow = vd + (t0 + t) * kRow + lane * kDpl;
          float vf[kDpl];
#pragma unroll
          for (int j = 0; j < kDpl; ++j) vf[j] = (float)((int)(int8_t)vrow[j] + 128) - vz;
#pragma unroll
          for (int g = 0; g < kGMaxG; ++g) {
            if (g < G) {
              const float pg = ps[g * 64 + t];
#pragma unroll
              for (int j = 0; j < kDpl; ++j) acc[g][j] = fmaf(pg, vf[j], acc[g][j]);
            }
          }
        }
        __syncwarp();
      }
    }
    e_cur = e_next;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");

  // ---- merge the warps' states through shared memory (the unit buffers are free now)
  __syncthreads();
  float* ms = reinterpret_cast<float*>(gsm);         // [kGW][G]
  float* ls = ms + kGW * kGMaxG;                      // [kGW][G]
  float* os = ls + kGW * kGMaxG;                      // [kGW][G][D]
#pragma unroll
  for (int g = 0; g < kGMaxG; ++g) {
    if (g < G) {
      float lsum = l[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
      if (lane == 0) {
        ms[warp * kGMaxG + g] = m[g];
        ls[warp * kGMaxG + g] = lsum;
      }
#pragma unroll
      for (int j = 0; j < kDpl; ++j) os[(warp * kGMaxG + g) * kDim + lane * kDpl + j] = acc[g][j];
    }
  }
  __syncthreads();
  const float kLn2 = 0.6931471805599453f;
  for (int idx = threadIdx.x; idx < G * kDim; idx += kGW * 32) {
    const int g = idx / kDim, d = idx % kDim;
    float M = -1.0e30f;
    for (int w = 0; w < kGW; ++w) M = fmaxf(M, ms[w * kGMaxG + g]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kGW; ++w) {
      const float sc = exp2f(ms[w * kGMaxG + g] - M);
      L += ls[w * kGMaxG + g] * sc;
      O += os[(w * kGMaxG + g) * kDim + d] * sc;
    }
    const float o = L > 0.f ? O / L : 0.f;
    const float lse = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    const size_t row = (size_t)r * p.Hq + (size_t)h * G + g;
    if (S > 1) {
      const size_t prow = (size_t)split * p.B * p.Hq + row;
      p.part_o[prow * kDim + d] = o;
      if (d == 0) p.part_lse[prow] = lse;
    } else if (p.shard_o != nullptr) {
      p.shard_o[row * kDim + d] = o;
      if (d == 0) p.shard_lse[row] = lse;
    } else if (p.bf16) {
      reinterpret_cast<__nv_bfloat16*>(p.out)[row * kDim + d] = __float2bfloat16_rn(o);
    } else {
      reinterpret_cast<__half*>(p.out)[row * kDim + d] = __float2half_rn(o);
    }
  }
}

template <int kDim>
static size_t generic_smem(int qb) {
  const size_t units = (size_t)kGW * 4 * qb * (kDim + 16);
  const size_t merge = (size_t)(2 * kGW * kGMaxG + kGW * kGMaxG * kDim) * 4;
  const size_t extra = (size_t)(kGMaxG * kDim + kGW * kGMaxG * 64) * 4;
  return (units > merge ? units : merge) + extra;
}

static size_t generic_smem_for(int dim, int qb) {
  switch (dim) {
    case 32: return generic_smem<32>(qb);
    case 64: return generic_smem<64>(qb);
    case 128: return generic_smem<128>(qb);
    default: return generic_smem<256>(qb);
  }
}

bool generic_supports(const FsDecodeArgs* a) {
  const int d = a->head_dim, qb = a->block_size;
  if (d != 32 && d != 64 && d != 128 && d != 256) return false;
  if (qb <= 0 || qb > 64 || qb * (d + 16) > kGMaxUnitBytes) return false;
  const int page = a->page_size > 0 ? a->page_size : qb;
  if (a->layout == FS_LAYOUT_PAGED && page % qb) return false;
  if (a->q_heads / a->kv_heads > kGMaxG) return false;
  if (a->kv_format == FS_KV_SYMMETRIC && a->layout == FS_LAYOUT_PAGED && page != qb) return false;
  return a->q_dtype == FS_F16 || a->q_dtype == FS_BF16;
}

// Split count: enough CTAs for about two waves of resident CTAs, at least 8 quant blocks
// per split; sequence-shard calls (partial outputs) use one split.
static int generic_splits(const FsDecodeArgs* a, int device, size_t smem) {
  if (a->shard_o != nullptr) return 1;
  if (a->num_splits > 0) return a->num_splits;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_generic_kernel<128>, kGW * 32, smem);
  if (per_sm <= 0) per_sm = 1;
  const int64_t slots = (int64_t)per_sm * device_sm_count(device) * 2;
  const int64_t pairs = (int64_t)a->batch * a->kv_heads;
  const int page = a->page_size > 0 ? a->page_size : a->block_size;
  const int64_t max_units = (((int64_t)a->max_seq_len + a->block_size - 1) / a->block_size);
  (void)page;
  int64_t s = (slots + pairs - 1) / pairs;
  const int64_t cap = max_units / 8 > 1 ? max_units / 8 : 1;
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return (int)s;
}

static size_t align256g(size_t x) { return (x + 255) & ~(size_t)255; }

size_t generic_workspace(const FsDecodeArgs* a, int device, int* splits_out) {
  const size_t smem = generic_smem_for(a->head_dim, a->block_size);
  const int s = generic_splits(a, device, smem);
  if (splits_out) *splits_out = s;
  if (s <= 1) return 0;
  const size_t rows = (size_t)a->batch * a->q_heads;
  return align256g((size_t)s * rows * a->head_dim * 4) + align256g((size_t)s * rows * 4);
}

int launch_generic_decode(const FsDecodeArgs* a, int device, void* stream) {
  const size_t smem = generic_smem_for(a->head_dim, a->block_size);
  int S = 1;
  const size_t need = generic_workspace(a, device, &S);
  if (need > 0 && (a->workspace == nullptr || a->workspace_bytes < need)) return FS_ERR_WORKSPACE;
  GenericParams p{};
  p.q = a->q;
  p.kval = a->k_values;
  p.vval = a->v_values;
  p.kscale = a->k_scale;
  p.vscale = a->v_scale;
  p.kzero = a->k_zero;
  p.vzero = a->v_zero;
  p.table = a->block_table;
  p.lengths = a->lengths;
  p.out = a->out;
  p.shard_o = a->shard_o;
  p.shard_lse = a->shard_lse;
  p.status = a->device_status;
  p.B = a->batch;
  p.Hq = a->q_heads;
  p.Hkv = a->kv_heads;
  p.G = a->q_heads / a->kv_heads;
  p.S = S;
  p.cols = a->table_cols;
  p.qb = a->block_size;
  p.bpp = a->layout == FS_LAYOUT_PAGED ? (a->page_size > 0 ? a->page_size : a->block_size) / a->block_size : 1;
  p.paged = a->layout == FS_LAYOUT_PAGED;
  p.bf16 = a->q_dtype == FS_BF16;
  p.sym = a->kv_format == FS_KV_SYMMETRIC;
  p.num_blocks = a->num_blocks;
  p.max_seq_len = a->max_seq_len;
  p.page_begin = a->page_begin;
  p.page_end = a->page_end;
  p.qk_scale_log2 = a->sm_scale * 1.4426950408889634f;
  if (S > 1) {
    const size_t rows = (size_t)a->batch * a->q_heads;
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
    p.part_o = reinterpret_cast<float*>(ws);
    p.part_lse = reinterpret_cast<float*>(ws + align256g((size_t)S * rows * a->head_dim * 4));
  }
  const int64_t grid = (int64_t)a->batch * a->kv_heads * S;
  if (grid >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto go = [&](auto kernel) -> int {
    if (cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        e != cudaSuccess)
      return fail_cuda("shared-memory limit of the generic decode kernel", e);
    kernel<<<(unsigned)grid, kGW * 32, smem, st>>>(p);
    return launch_status("generic decode kernel launch");
  };
  int rc;
  switch (a->head_dim) {
    case 32: rc = go(decode_generic_kernel<32>); break;
    case 64: rc = go(decode_generic_kernel<64>); break;
    case 128: rc = go(decode_generic_kernel<128>); break;
    default: rc = go(decode_generic_kernel<256>); break;
  }
  if (rc != FS_OK || S <= 1) return rc;
  const int64_t rows = (int64_t)a->batch * a->q_heads;
  return fs_merge_partials(p.part_o, p.part_lse, S, rows, a->head_dim, 0, a->out, a->q_dtype, stream);
}

}  // namespace fsb

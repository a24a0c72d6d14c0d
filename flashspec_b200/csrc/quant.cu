// Quantize / page-update / dequantize / merge kernels.
//
// The quantizer must be bit-exact with the reference (src/flashspec/quant.py:141-158),
// which torch evaluates as separate fp32 operations with round-to-nearest-even:
//   scale = max((max - min) / 255, 1e-8)
//   zp    = clamp(rint(-min / scale), 0, 255)
//   u     = clamp(rint(x / scale + zp), 0, 255);  value = u - 128
// Every operation below is an explicitly rounded intrinsic (__fsub_rn, __fdiv_rn,
// __fadd_rn, __fmul_rn) so the compiler cannot contract or approximate them, and
// this file must not be built with --use_fast_math.  min/max are exact.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <cstdlib>
#include <stdint.h>

#include "common.h"

#include "../../include/flashspec_b200.h"

namespace fsb {

__device__ __forceinline__ float load_as_f32(const void* base, int64_t idx, int dtype) {
  if (dtype == FS_F16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  if (dtype == FS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  return reinterpret_cast<const float*>(base)[idx];
}

// 16 consecutive source elements from index idx as fp32: 16-byte loads when aligned.
__device__ __forceinline__ void load16_as_f32(const void* base, int64_t idx, int dtype, float* out) {
  const int esz = dtype == FS_F32 ? 4 : 2;
  const char* p = reinterpret_cast<const char*>(base) + idx * esz;
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    if (dtype == FS_F32) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float4 f = reinterpret_cast<const float4*>(p)[c];
        out[4 * c] = f.x, out[4 * c + 1] = f.y, out[4 * c + 2] = f.z, out[4 * c + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 u = reinterpret_cast<const uint4*>(p)[c];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const unsigned short lo = (unsigned short)(w[k] & 0xffffu), hi = (unsigned short)(w[k] >> 16);
          if (dtype == FS_F16) {
            out[8 * c + 2 * k] = __half2float(__ushort_as_half(lo));
            out[8 * c + 2 * k + 1] = __half2float(__ushort_as_half(hi));
          } else {
            out[8 * c + 2 * k] = __bfloat162float(__ushort_as_bfloat16(lo));
            out[8 * c + 2 * k + 1] = __bfloat162float(__ushort_as_bfloat16(hi));
          }
        }
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = load_as_f32(base, idx + j, dtype);
}

struct QParams {
  float scale, zp;
};

__device__ __forceinline__ QParams qparams_from_range(float mn, float mx) {
  QParams q;
  q.scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), 255.0f), 1.0e-8f);
  q.zp = fminf(fmaxf(rintf(__fdiv_rn(-mn, q.scale)), 0.0f), 255.0f);
  return q;
}

__device__ __forceinline__ int8_t quantize_one(float x, QParams q) {
  const float u = fminf(fmaxf(rintf(__fadd_rn(__fdiv_rn(x, q.scale), q.zp)), 0.0f), 255.0f);
  return (int8_t)((int)u - 128);
}

__device__ __forceinline__ float dequant_one(int8_t v, float scale, int16_t zp) {
  return __fmul_rn(__fsub_rn((float)((int)v + 128), (float)zp), scale);
}

// Block-wide min/max; every thread gets the result.
template <int kThreads>
__device__ __forceinline__ void block_minmax(float& mn, float& mx) {
  __shared__ float smn[32], smx[32];
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    smn[w] = mn;
    smx[w] = mx;
  }
  __syncthreads();
  mn = smn[0];
  mx = smx[0];
  for (int i = 1; i < kThreads / 32; ++i) {
    mn = fminf(mn, smn[i]);
    mx = fmaxf(mx, smx[i]);
  }
}

constexpr int kQThreads = 256;

// One CTA per (leading index, block): x [n_lead, seq, D] -> values [n_lead, nblk, bs, D].
__global__ void __launch_bounds__(kQThreads)
    quantize_blocks_kernel(const void* __restrict__ x, int dtype, int seq, int D, int bs, int nblk,
                           int8_t* __restrict__ values, float* __restrict__ scale, int16_t* __restrict__ zp) {
  const int64_t blkid = blockIdx.x;
  const int64_t lead = blkid / nblk;
  const int blk = (int)(blkid % nblk);
  const int E = bs * D;
  float mn = INFINITY, mx = -INFINITY;
  for (int e = threadIdx.x; e < E; e += kQThreads) {
    const int t = blk * bs + e / D;
    const float v = t < seq ? load_as_f32(x, (lead * seq + t) * D + e % D, dtype) : 0.0f;
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  block_minmax<kQThreads>(mn, mx);
  const QParams q = qparams_from_range(mn, mx);
  int8_t* out = values + blkid * E;
  for (int e = threadIdx.x; e < E; e += kQThreads) {
    const int t = blk * bs + e / D;
    const float v = t < seq ? load_as_f32(x, (lead * seq + t) * D + e % D, dtype) : 0.0f;
    out[e] = quantize_one(v, q);
  }
  if (threadIdx.x == 0) {
    scale[blkid] = q.scale;
    zp[blkid] = (int16_t)q.zp;
  }
}

constexpr int kUThreads = 256;

// One CTA per (item, head); K then V.  Dynamic smem: bs*D floats.
__global__ void __launch_bounds__(kUThreads) page_update_kernel(const FsPageUpdate* __restrict__ items,
                                                                const FsPageUpdateArgs a) {
  extern __shared__ float buf[];
  const FsPageUpdate it = items[blockIdx.x];
  const int h = blockIdx.y;
  const int D = a.head_dim, bs = a.block_size, E = bs * D;
  if (it.page < 0 || it.page >= a.num_pages) return;  // host validates; never touch memory out of range
  const int64_t blk = it.page * a.heads + h;
#pragma unroll 1
  for (int kv = 0; kv < 2; ++kv) {
    // pages written from zeros may lie beyond the input pool: never read it for them
    const int8_t* vin = it.from_zero ? nullptr : (kv ? a.v_values_in : a.k_values_in) + blk * E;
    const float sin = it.from_zero ? 0.0f : (kv ? a.v_scale_in : a.k_scale_in)[blk];
    const int16_t zin = it.from_zero ? (int16_t)0 : (kv ? a.v_zero_in : a.k_zero_in)[blk];
    const void* src = kv ? a.v_src : a.k_src;
    float mn = INFINITY, mx = -INFINITY;
    for (int e = threadIdx.x; e < E; e += kUThreads) {
      const int r = e / D;
      float v;
      if (r >= it.dst_row && r < it.dst_row + it.n_rows) {
        const int64_t si = (int64_t)it.src_b * a.src_stride_b + (int64_t)h * a.src_stride_h +
                           (int64_t)(it.src_t + r - it.dst_row) * a.src_stride_t + (e % D);
        v = load_as_f32(src, si, a.src_dtype);
      } else if (it.from_zero) {
        v = 0.0f;
      } else {
        v = dequant_one(vin[e], sin, zin);
      }
      buf[e] = v;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    block_minmax<kUThreads>(mn, mx);  // contains __syncthreads: all old values are read
    const QParams q = qparams_from_range(mn, mx);
    int8_t* vout = (kv ? a.v_values_out : a.k_values_out) + blk * E;
    for (int e = threadIdx.x; e < E; e += kUThreads) vout[e] = quantize_one(buf[e], q);
    if (threadIdx.x == 0) {
      (kv ? a.v_scale_out : a.k_scale_out)[blk] = q.scale;
      (kv ? a.v_zero_out : a.k_zero_out)[blk] = (int16_t)q.zp;
    }
    __syncthreads();  // buf is reused by the V pass
  }
}

// Out of line so that the unrolled fast path carries one copy of the division.
__device__ __noinline__ int8_t quantize_one_exact(float x, QParams q) { return quantize_one(x, q); }

// 16 x quantize_one, bit-identical, packed as 16 int8 bytes, with almost no divisions.
//   qa = RN(x * RN(1/s)) is within |x/s| (2^-23 + 2^-24 + 2^-47) of q = RN(x/s) (1/s is a
//   normal float: 1e-8 <= s < 2^128 / 255), so wherever ta = RN(qa + zp) lies in [0, 255]
//   (|q| < 511) it is within 1.0e-4 + ulp(ta) < 1.4e-4 of t = RN(q + zp).  The reference
//   code is clamp(rint(t), 0, 255) = rint(clamp(t, 0, 255)) (integer bounds); rint is
//   constant between half-integers, so when tc = clamp(ta, 0, 255) lies more than 2^-11
//   (4.9e-4) from the nearest half-integer the code is rint(tc), and a ta that clamps is
//   off by less than the margin from a t that clamps the same way.  rint(tc) is the low
//   byte of RN(tc + 1.5 * 2^23) (round-to-nearest-even, tc < 2^22), d = tc - rint(tc) is
//   exact, and the elements with |d| >= 0.5 - 2^-11 (about 0.1%) take the division.
//   NaN: fmaxf(NaN, 0) = 0, the same code as the division path gives.
__device__ __forceinline__ uint4 quantize16_fast(const float* v, QParams q) {
  const float rcp = __frcp_rn(q.scale);
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  uint32_t bits[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float ta = __fadd_rn(__fmul_rn(v[j], rcp), q.zp);
    const float tc = fminf(fmaxf(ta, 0.0f), 255.0f);
    const float r = __fadd_rn(tc, kMagic);
    const float d = __fsub_rn(tc, __fsub_rn(r, kMagic));
    bits[j] = __float_as_uint(r);  // low byte = rint(tc)
    if (fabsf(d) >= 0.5f - 4.8828125e-4f) bits[j] = (uint32_t)(uint8_t)quantize_one_exact(v[j], q) ^ 0x80u;
  }
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = __byte_perm(bits[4 * k], bits[4 * k + 1], 0x0040);
    const uint32_t hi = __byte_perm(bits[4 * k + 2], bits[4 * k + 3], 0x0040);
    w[k] = __byte_perm(lo, hi, 0x5410) ^ 0x80808080u;  // code - 128 as int8
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// dequant_one of the 16 int8 codes in raw, bit-identical: the byte u = code + 128 is put
// in the mantissa of 2^23 (the float 2^23 + u, exact), and (2^23 + u) - (2^23 + zp) = u - zp
// exactly (|zp| < 2^23), which is dequant_one's first step; then the same RN product.
__device__ __forceinline__ void dequant16(int4 raw, float scale, int16_t zp, float* out) {
  const float base = __fadd_rn(8388608.0f, (float)zp);
  const uint32_t w4[4] = {(uint32_t)raw.x ^ 0x80808080u, (uint32_t)raw.y ^ 0x80808080u,
                          (uint32_t)raw.z ^ 0x80808080u, (uint32_t)raw.w ^ 0x80808080u};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float f = __uint_as_float(__byte_perm(w4[j >> 2], 0x4B000000u, 0x7540 | (j & 3)));
    out[j] = __fmul_rn(__fsub_rn(f, base), scale);
  }
}

// Register-resident page update for blocks of E = bs * D bytes (D % 16 == 0) with E % (512 G) == 0 and
// E <= 16384: one CTA per (item, head, K|V) of E / (16 G) threads; thread t owns the G
// 16-byte chunks t, t + blockDim, ... (each inside one row) -- one 16-byte load of old
// values and one 16-byte store per chunk, all loads issued before any arithmetic.  Same
// per-element arithmetic as page_update_kernel (kFast: quantize16_fast / dequant16 above,
// bit-identical to it), so the result is bit-identical (min and max are exact whatever
// the order).  In place is safe: a thread loads its chunks before the block barrier and
// stores after it.
template <int G, bool kFast>
__global__ void __launch_bounds__(512) page_update_vec_kernel(const FsPageUpdate* __restrict__ items,
                                                              const FsPageUpdateArgs a) {
  __shared__ float smn[16], smx[16];
  const FsPageUpdate it = items[blockIdx.x];
  const int h = blockIdx.y, kv = blockIdx.z;
  if (it.page < 0 || it.page >= a.num_pages) return;
  const int D = a.head_dim, E = a.block_size * D;
  const int64_t blk = it.page * a.heads + h;
  float v[G][16];
  if (it.from_zero) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 16; ++j) v[g][j] = 0.0f;
  } else {
    const float sin = (kv ? a.v_scale_in : a.k_scale_in)[blk];
    const int16_t zin = (kv ? a.v_zero_in : a.k_zero_in)[blk];
    const int4* vin = reinterpret_cast<const int4*>((kv ? a.v_values_in : a.k_values_in) + blk * E);
    int4 raw[G];
#pragma unroll
    for (int g = 0; g < G; ++g) raw[g] = vin[threadIdx.x + g * blockDim.x];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (kFast) {
        dequant16(raw[g], sin, zin, v[g]);
      } else {
        const int w4[4] = {raw[g].x, raw[g].y, raw[g].z, raw[g].w};
#pragma unroll
        for (int j = 0; j < 16; ++j) v[g][j] = dequant_one((int8_t)(w4[j >> 2] >> (8 * (j & 3))), sin, zin);
      }
    }
  }
  const void* src = kv ? a.v_src : a.k_src;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int e0 = (threadIdx.x + g * blockDim.x) * 16, r = e0 / D;
    if (r >= it.dst_row && r < it.dst_row + it.n_rows) {
      const int64_t si = (int64_t)it.src_b * a.src_stride_b + (int64_t)h * a.src_stride_h +
                         (int64_t)(it.src_t + r - it.dst_row) * a.src_stride_t + e0 % D;
      load16_as_f32(src, si, a.src_dtype, v[g]);
    }
  }
  float mn = v[0][0], mx = v[0][0];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      mn = fminf(mn, v[g][j]);
      mx = fmaxf(mx, v[g][j]);
    }
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    smn[w] = mn;
    smx[w] = mx;
  }
  __syncthreads();
  mn = smn[0];
  mx = smx[0];
  for (int i = 1; i < nw; ++i) {
    mn = fminf(mn, smn[i]);
    mx = fmaxf(mx, smx[i]);
  }
  const QParams q = qparams_from_range(mn, mx);
  uint4* vout = reinterpret_cast<uint4*>((kv ? a.v_values_out : a.k_values_out) + blk * E);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (kFast) {
      vout[threadIdx.x + g * blockDim.x] = quantize16_fast(v[g], q);
    } else {
      uint32_t wd[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int j = 0; j < 16; ++j) wd[j >> 2] |= (uint32_t)(uint8_t)quantize_one(v[g][j], q) << (8 * (j & 3));
      vout[threadIdx.x + g * blockDim.x] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
  }
  if (threadIdx.x == 0) {
    (kv ? a.v_scale_out : a.k_scale_out)[blk] = q.scale;
    (kv ? a.v_zero_out : a.k_zero_out)[blk] = (int16_t)q.zp;
  }
}

// quantize_blocks_kernel for blocks of E = bs * D elements (D % 16 == 0) with E % (512 G) == 0: one CTA
// of E / (16 G) threads per block, thread t owning the G 16-element chunks t, t + blockDim,
// ... (each inside one row): 16-element source loads, one 16-byte store per chunk, codes
// from quantize16_fast (bit-identical to quantize_one).  Rows past seq are zeros.
template <int G>
__global__ void __launch_bounds__(512) quantize_blocks_vec_kernel(const void* __restrict__ x, int dtype, int seq,
                                                                  int D, int bs, int nblk,
                                                                  int8_t* __restrict__ values,
                                                                  float* __restrict__ scale,
                                                                  int16_t* __restrict__ zp) {
  __shared__ float smn[16], smx[16];
  const int64_t blkid = blockIdx.x;
  const int64_t lead = blkid / nblk;
  const int blk = (int)(blkid % nblk);
  float v[G][16];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int e0 = (threadIdx.x + g * blockDim.x) * 16, t = blk * bs + e0 / D;
    if (t < seq) {
      load16_as_f32(x, (lead * seq + t) * D + e0 % D, dtype, v[g]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[g][j] = 0.0f;
    }
  }
  float mn = v[0][0], mx = v[0][0];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      mn = fminf(mn, v[g][j]);
      mx = fmaxf(mx, v[g][j]);
    }
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    smn[w] = mn;
    smx[w] = mx;
  }
  __syncthreads();
  mn = smn[0];
  mx = smx[0];
  for (int i = 1; i < nw; ++i) {
    mn = fminf(mn, smn[i]);
    mx = fmaxf(mx, smx[i]);
  }
  const QParams q = qparams_from_range(mn, mx);
  uint4* out = reinterpret_cast<uint4*>(values + blkid * (int64_t)bs * D);
#pragma unroll
  for (int g = 0; g < G; ++g) out[threadIdx.x + g * blockDim.x] = quantize16_fast(v[g], q);
  if (threadIdx.x == 0) {
    scale[blkid] = q.scale;
    zp[blkid] = (int16_t)q.zp;
  }
}

// 16-byte chunks per thread of page_update_vec_kernel for blocks of E bytes (E % 512 == 0):
// 2 by default (FLASHSPEC_PAGE_UPDATE_CHUNKS = 1 | 2 | 4 overrides), fewer where E is
// not a multiple of 512 * chunks, more where the CTA would exceed 512 threads.
static int page_update_chunks(int64_t E) {
  const char* gs = std::getenv("FLASHSPEC_PAGE_UPDATE_CHUNKS");
  int g = gs ? std::atoi(gs) : 2;
  if (g != 1 && g != 4) g = 2;
  while (g > 1 && E % (512 * g) != 0) g /= 2;
  while (g < 4 && E / (16 * g) > 512 && E % (1024 * g) == 0) g *= 2;
  return g;
}

__global__ void dequantize_pages_kernel(const int8_t* __restrict__ values, const float* __restrict__ scale,
                                        const int16_t* __restrict__ zp, const int64_t* __restrict__ pages,
                                        int64_t num_pages, int H, int bs, int D, float* __restrict__ out) {
  const int64_t i = blockIdx.x;
  const int h = blockIdx.y;
  const int E = bs * D;
  const int64_t page = pages[i];
  float* o = out + (i * H + h) * E;
  if (page < 0 || page >= num_pages) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) o[e] = 0.0f;
    return;
  }
  const int64_t blk = page * H + h;
  const float s = scale[blk];
  const int16_t z = zp[blk];
  for (int e = threadIdx.x; e < E; e += blockDim.x) o[e] = dequant_one(values[blk * E + e], s, z);
}

__global__ void merge_partials_kernel(const float* __restrict__ o, const float* __restrict__ lse, int n,
                                      int64_t rows, int D, int64_t stride, void* __restrict__ out, int out_dtype) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * D) return;
  const int64_t row = idx / D;
  const int64_t so = stride ? stride : rows * D, sl = stride ? stride : rows;
  float M = -INFINITY;
  for (int i = 0; i < n; ++i) M = fmaxf(M, lse[i * sl + row]);
  float W = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int i = 0; i < n; ++i) {
      const float l = lse[i * sl + row];
      const float w = l == -INFINITY ? 0.f : expf(l - M);
      W += w;
      O += w * o[i * so + idx];
    }
  }
  const float r = W > 0.f ? O / W : 0.f;
  if (out_dtype == FS_F16)
    reinterpret_cast<__half*>(out)[idx] = __float2half_rn(r);
  else if (out_dtype == FS_BF16)
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(r);
  else
    reinterpret_cast<float*>(out)[idx] = r;
}

// Symmetric per-token quantization (the format of the benchmark configurations'
// wording, doc/TODO.MD:241-255 "symmetric INT8"): one fp32 scale per (token, head),
// scale = max(absmax / 127, 1e-8), q = clamp(rint(x / scale), -127, 127), each step an
// explicitly rounded fp32 operation.  One warp per token row of D values.
__global__ void quantize_sym_kernel(const void* __restrict__ x, int dtype, int64_t rows, int D,
                                    int8_t* __restrict__ values, float* __restrict__ scale) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float amax = 0.f;
  for (int d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(load_as_f32(x, row * D + d, dtype)));
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-8f);
  for (int d = lane; d < D; d += 32) {
    const float q = fminf(fmaxf(rintf(__fdiv_rn(load_as_f32(x, row * D + d, dtype), s)), -127.0f), 127.0f);
    values[row * D + d] = (int8_t)(int)q;
  }
  if (lane == 0) scale[row] = s;
}

}  // namespace fsb

extern "C" {

/* args->x is [n_lead, seq_len, head_dim]; writes values [n_lead, seq_len, head_dim] and
 * one scale per (lead, token) into args->scale; block_size and zero_point are unused. */
int fs_quantize_symmetric(const FsQuantizeArgs* a, void* stream) {
  if (a == nullptr || a->x == nullptr || a->values == nullptr || a->scale == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if (a->n_lead <= 0 || a->seq_len <= 0 || a->head_dim <= 0) return FS_ERR_INVALID_ARGUMENT;
  if (a->x_dtype != FS_F16 && a->x_dtype != FS_BF16 && a->x_dtype != FS_F32) return FS_ERR_UNSUPPORTED;
  const int64_t rows = a->n_lead * a->seq_len;
  const int64_t blocks = (rows + 7) / 8;
  if (blocks >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
  fsb::quantize_sym_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      a->x, a->x_dtype, rows, a->head_dim, a->values, a->scale);
  return fsb::launch_status("symmetric quantize kernel launch");
}

int fs_abi_version(void) { return FS_ABI_VERSION; }

const char* fs_status_string(int s) {
  switch (s) {
    case FS_OK: return "ok";
    case FS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FS_ERR_UNSUPPORTED: return "unsupported shape or dtype for this kernel";
    case FS_ERR_CUDA: return "CUDA error";
    case FS_ERR_WORKSPACE: return "workspace missing or too small";
    case FS_ERR_ALIGNMENT: return "pointer misaligned";
    case FS_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of fs_paged_decode_noalloc";
    default: return "unknown status";
  }
}

const char* fs_last_error_detail(void) { return fsb::g_error_detail; }

int fs_quantize_blocks(const FsQuantizeArgs* a, void* stream) {
  if (a == nullptr || a->x == nullptr || a->values == nullptr || a->scale == nullptr || a->zero_point == nullptr)
    return FS_ERR_INVALID_ARGUMENT;
  if (a->n_lead <= 0 || a->seq_len <= 0 || a->head_dim <= 0 || a->block_size <= 0) return FS_ERR_INVALID_ARGUMENT;
  if (a->x_dtype != FS_F16 && a->x_dtype != FS_BF16 && a->x_dtype != FS_F32) return FS_ERR_UNSUPPORTED;
  const int nblk = (a->seq_len + a->block_size - 1) / a->block_size;
  const int64_t grid = a->n_lead * nblk;
  if (grid >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
  const int64_t E = (int64_t)a->block_size * a->head_dim;
  if (E % 512 == 0 && E <= 16384 && a->head_dim % 16 == 0 && (reinterpret_cast<uintptr_t>(a->values) & 15) == 0 &&
      std::getenv("FLASHSPEC_PAGE_UPDATE_SCALAR") == nullptr) {
    const int g = E % 1024 == 0 ? 2 : 1;
    auto st = reinterpret_cast<cudaStream_t>(stream);
    if (g == 1)
      fsb::quantize_blocks_vec_kernel<1><<<(unsigned)grid, (unsigned)(E / 16), 0, st>>>(
          a->x, a->x_dtype, a->seq_len, a->head_dim, a->block_size, nblk, a->values, a->scale, a->zero_point);
    else
      fsb::quantize_blocks_vec_kernel<2><<<(unsigned)grid, (unsigned)(E / 32), 0, st>>>(
          a->x, a->x_dtype, a->seq_len, a->head_dim, a->block_size, nblk, a->values, a->scale, a->zero_point);
    return fsb::launch_status("quantize kernel launch");
  }
  fsb::quantize_blocks_kernel<<<(unsigned)grid, fsb::kQThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      a->x, a->x_dtype, a->seq_len, a->head_dim, a->block_size, nblk, a->values, a->scale, a->zero_point);
  return fsb::launch_status("quantize kernel launch");
}

int fs_page_update(const FsPageUpdateArgs* a, void* stream) {
  if (a == nullptr) return FS_ERR_INVALID_ARGUMENT;
  if (a->n_items == 0) return FS_OK;
  if (a->n_items < 0 || a->items == nullptr || a->heads <= 0 || a->head_dim <= 0 || a->block_size <= 0 ||
      a->num_pages <= 0)
    return FS_ERR_INVALID_ARGUMENT;
  if (a->src_dtype != FS_F16 && a->src_dtype != FS_BF16 && a->src_dtype != FS_F32) return FS_ERR_UNSUPPORTED;
  if (a->heads > 65535) return FS_ERR_UNSUPPORTED;
  const int64_t E = (int64_t)a->block_size * a->head_dim;
  const bool aligned16 = ((reinterpret_cast<uintptr_t>(a->k_values_out) | reinterpret_cast<uintptr_t>(a->v_values_out) |
                           reinterpret_cast<uintptr_t>(a->k_values_in) | reinterpret_cast<uintptr_t>(a->v_values_in)) &
                          15) == 0;
  if (E % 512 == 0 && E <= 16384 && a->head_dim % 16 == 0 && aligned16 &&
      std::getenv("FLASHSPEC_PAGE_UPDATE_SCALAR") == nullptr &&
      E / (16 * fsb::page_update_chunks(E)) <= 512) {
    const int g = fsb::page_update_chunks(E);
    dim3 grid((unsigned)a->n_items, (unsigned)a->heads, 2);
    const unsigned threads = (unsigned)(E / (16 * g));
    auto st = reinterpret_cast<cudaStream_t>(stream);
    const bool fast = std::getenv("FLASHSPEC_PAGE_UPDATE_EXACT_DIV") == nullptr;
    if (g == 1)
      fast ? fsb::page_update_vec_kernel<1, true><<<grid, threads, 0, st>>>(a->items, *a)
           : fsb::page_update_vec_kernel<1, false><<<grid, threads, 0, st>>>(a->items, *a);
    else if (g == 2)
      fast ? fsb::page_update_vec_kernel<2, true><<<grid, threads, 0, st>>>(a->items, *a)
           : fsb::page_update_vec_kernel<2, false><<<grid, threads, 0, st>>>(a->items, *a);
    else
      fast ? fsb::page_update_vec_kernel<4, true><<<grid, threads, 0, st>>>(a->items, *a)
           : fsb::page_update_vec_kernel<4, false><<<grid, threads, 0, st>>>(a->items, *a);
    return fsb::launch_status("page update kernel launch");
  }
  const size_t smem = (size_t)E * sizeof(float);
  if (smem > 48 * 1024) return FS_ERR_UNSUPPORTED;
  dim3 grid((unsigned)a->n_items, (unsigned)a->heads);
  fsb::page_update_kernel<<<grid, fsb::kUThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a->items, *a);
  return fsb::launch_status("page update kernel launch");
}

int fs_dequantize_pages(const int8_t* values, const float* scale, const int16_t* zero_point, const int64_t* pages,
                        int64_t n_listed, int64_t num_pages, int32_t heads, int32_t block_size, int32_t head_dim,
                        float* out, void* stream) {
  if (n_listed == 0) return FS_OK;
  if (values == nullptr || scale == nullptr || zero_point == nullptr || pages == nullptr || out == nullptr ||
      n_listed < 0 || heads <= 0 || heads > 65535 || block_size <= 0 || head_dim <= 0)
    return FS_ERR_INVALID_ARGUMENT;
  if (n_listed >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
  dim3 grid((unsigned)n_listed, (unsigned)heads);
  fsb::dequantize_pages_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      values, scale, zero_point, pages, num_pages, heads, block_size, head_dim, out);
  return fsb::launch_status("dequantize kernel launch");
}

int fs_merge_partials(const float* o_parts, const float* lse_parts, int32_t n_parts, int64_t rows, int32_t head_dim,
                      int64_t part_stride, void* out, int32_t out_dtype, void* stream) {
  if (o_parts == nullptr || lse_parts == nullptr || out == nullptr || n_parts <= 0 || rows < 0 || head_dim <= 0)
    return FS_ERR_INVALID_ARGUMENT;
  if (out_dtype != FS_F16 && out_dtype != FS_BF16 && out_dtype != FS_F32) return FS_ERR_UNSUPPORTED;
  const int64_t n = rows * head_dim;
  if (n == 0) return FS_OK;
  const int64_t blocks = (n + 255) / 256;
  if (blocks >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
  fsb::merge_partials_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      o_parts, lse_parts, n_parts, rows, head_dim, part_stride < 0 ? 0 : part_stride, out, out_dtype);
  return fsb::launch_status("merge kernel launch");
}

}  // extern "C"

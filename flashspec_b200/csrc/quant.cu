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
#include <stdint.h>

#include "common.h"

#include "../../include/flashspec_b200.h"

namespace fsb {

__device__ __forceinline__ float load_as_f32(const void* base, int64_t idx, int dtype) {
  if (dtype == FS_F16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  if (dtype == FS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  return reinterpret_cast<const float*>(base)[idx];
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
  const size_t smem = (size_t)a->block_size * a->head_dim * sizeof(float);
  if (smem > 48 * 1024) return FS_ERR_UNSUPPORTED;
  if (a->heads > 65535) return FS_ERR_UNSUPPORTED;
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

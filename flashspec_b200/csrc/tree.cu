// Tree-attention verify for speculative decoding: the draft-tree half of the step and
// the merge with the committed prefix.
//
// A verify step scores every node of a draft tree at once.  Node i of request b attends
// to the request's committed prefix (the paged INT8 cache) and to the draft tokens on
// its own root path (its ancestors and itself), never to siblings or other branches.
// The prefix half is a paged decode in which the tree's nodes share the kv head's reads
// (the caller folds the nodes into the query-head axis and asks for partial (O, LSE)
// outputs); this kernel adds the path half and merges the two with the log-sum-exp rule.
// The reference lists this kernel in doc/TODO.MD:186-237 (a tree mask instead of the
// causal one, parent pointers, per-node outputs) without implementing it.
//
// One warp per (request, node, q head): lane l owns head dims [l*D/32, (l+1)*D/32); the
// warp walks parent pointers from the node to the root (the path is at most `nodes`
// long), scoring each path token against q with a warp reduction and folding it into an
// online softmax; then it merges with the prefix partial and writes the output row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <stdint.h>

#include "../../include/flashspec_b200.h"
#include "common.h"

namespace fsb {

constexpr int kTreeWarps = 4;

__device__ __forceinline__ float ld_act(const void* base, size_t i, bool bf16) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i])
              : __half2float(reinterpret_cast<const __half*>(base)[i]);
}

template <int kDim>
__global__ void __launch_bounds__(kTreeWarps * 32) tree_attend_kernel(const FsTreeArgs a) {
  constexpr int kDpl = kDim / 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kTreeWarps + (threadIdx.x >> 5);  // (b, i, hq)
  const int64_t rows = (int64_t)a.batch * a.nodes * a.q_heads;
  if (row >= rows) return;
  const int hq = (int)(row % a.q_heads);
  const int64_t bi = row / a.q_heads;
  const int i = (int)(bi % a.nodes), b = (int)(bi / a.nodes);
  const int hkv = hq / (a.q_heads / a.kv_heads);
  const bool bf16 = a.q_dtype == FS_BF16;
  const float scale_log2 = a.sm_scale * 1.4426950408889634f;

  float q[kDpl], o[kDpl];
#pragma unroll
  for (int j = 0; j < kDpl; ++j) {
    q[j] = ld_act(a.q, (size_t)row * kDim + lane * kDpl + j, bf16);
    o[j] = 0.f;
  }
  // path tokens: the node, its parent, ... up to the root (parents[] < own index)
  float m = -INFINITY, l = 0.f;
  int node = i, steps = 0;
  while (node >= 0 && steps <= a.nodes) {
    const size_t kv = (((size_t)b * a.nodes + node) * a.kv_heads + hkv) * kDim + lane * kDpl;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kDpl; ++j) s = fmaf(q[j], ld_act(a.tree_k, kv + j, bf16), s);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float t = s * scale_log2;
    const float m_new = fmaxf(m, t);
    const float alpha = exp2f(m - m_new), pr = exp2f(t - m_new);
    l = l * alpha + pr;
#pragma unroll
    for (int j = 0; j < kDpl; ++j) o[j] = fmaf(pr, ld_act(a.tree_v, kv + j, bf16), o[j] * alpha);
    m = m_new;
    node = a.parents[(size_t)b * a.nodes + node];
    ++steps;
  }
  // merge with the prefix partial: (O_p, LSE_p) normalised, natural log
  const float kLn2 = 0.6931471805599453f;
  const float lse_tree = (m + log2f(l)) * kLn2;  // the path holds at least the node itself
  const float lse_pre = a.prefix_lse != nullptr ? a.prefix_lse[row] : -INFINITY;
  const float M = fmaxf(lse_tree, lse_pre);
  const float w_tree = expf(lse_tree - M), w_pre = lse_pre == -INFINITY ? 0.f : expf(lse_pre - M);
  const float inv = 1.f / (w_tree + w_pre);
#pragma unroll
  for (int j = 0; j < kDpl; ++j) {
    const size_t idx = (size_t)row * kDim + lane * kDpl + j;
    const float pre = w_pre > 0.f ? a.prefix_o[idx] : 0.f;
    const float v = (w_tree * (o[j] / l) + w_pre * pre) * inv;
    if (bf16)
      reinterpret_cast<__nv_bfloat16*>(a.out)[idx] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<__half*>(a.out)[idx] = __float2half_rn(v);
  }
}

}  // namespace fsb

extern "C" int fs_tree_attend(const FsTreeArgs* a, void* stream) {
  using namespace fsb;
  if (a == nullptr || a->q == nullptr || a->tree_k == nullptr || a->tree_v == nullptr || a->parents == nullptr ||
      a->out == nullptr || a->batch <= 0 || a->nodes <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 ||
      a->q_heads % a->kv_heads)
    return FS_ERR_INVALID_ARGUMENT;
  if ((a->prefix_o == nullptr) != (a->prefix_lse == nullptr)) return FS_ERR_INVALID_ARGUMENT;
  if (a->q_dtype != FS_F16 && a->q_dtype != FS_BF16) return FS_ERR_UNSUPPORTED;
  const int64_t rows = (int64_t)a->batch * a->nodes * a->q_heads;
  const int64_t blocks = (rows + kTreeWarps - 1) / kTreeWarps;
  if (blocks >= (1ll << 31)) return FS_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->head_dim) {
    case 32: tree_attend_kernel<32><<<(unsigned)blocks, kTreeWarps * 32, 0, st>>>(*a); break;
    case 64: tree_attend_kernel<64><<<(unsigned)blocks, kTreeWarps * 32, 0, st>>>(*a); break;
    case 128: tree_attend_kernel<128><<<(unsigned)blocks, kTreeWarps * 32, 0, st>>>(*a); break;
    case 256: tree_attend_kernel<256><<<(unsigned)blocks, kTreeWarps * 32, 0, st>>>(*a); break;
    default: return FS_ERR_UNSUPPORTED;
  }
  return launch_status("tree attend kernel launch");
}

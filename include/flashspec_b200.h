/*
 * flashspec_b200 -- C ABI of the B200 (sm_100a) INT8 decode-attention library.
 *
 * Plain C: raw device pointers, sizes and a CUDA stream passed as void*.  No torch
 * types cross this boundary.  Every entry point is asynchronous on the given
 * stream, never synchronises, and returns an FsStatus (0 = ok).
 *
 * Data formats are those of the FlashSpec reference (src/flashspec/quant.py:9-43,
 * paged.py:258-300): affine INT8 per (page|block, head): values int8 = uint8-128,
 * fp32 scale, int16 zero_point in the uint8 domain, one (scale, zp) per
 * [block_size x head_dim] block.
 *   contiguous KV : values [B, Hkv, nblk, 16, D], scale/zp [B, Hkv, nblk]
 *   paged KV pool : values [P, Hkv, 16, D],        scale/zp [P, Hkv]
 *   block_table   : int64 [B, cols], -1 = unallocated; lengths int64 [B]
 *   q / out       : fp16 or bf16 [B, Hq, D]; q head h reads kv head h / (Hq/Hkv)
 * Shapes: head_dim 32/64/128/256, quant block 1..64 tokens (block * (D + 16) <= 12 KB),
 * pages of one or more quant blocks, Hq/Hkv in 1..8.  D = 128 with pages and blocks of
 * 16 tokens and fp16 q runs the tuned TMA kernels; every other shape the generic kernel.
 */
#ifndef FLASHSPEC_B200_H_
#define FLASHSPEC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FS_ABI_VERSION 3

typedef enum FsStatus {
  FS_OK = 0,
  FS_ERR_INVALID_ARGUMENT = 1, /* shape / size / pointer inconsistency      */
  FS_ERR_UNSUPPORTED = 2,      /* valid input outside the kernel's limits    */
  FS_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed          */
  FS_ERR_WORKSPACE = 4,        /* workspace missing or too small             */
  FS_ERR_ALIGNMENT = 5,        /* pointer not aligned as the kernel needs    */
  FS_ERR_SCRATCH_LIMIT = 6     /* request needs more than the fixed scratch of
                                  fs_paged_decode_noalloc                     */
} FsStatus;

/* bits OR-ed into the optional device status word by kernels */
#define FS_DEV_BAD_PAGE 1u /* block_table entry outside [0, num_pages): page skipped */
#define FS_DEV_TIMEOUT 2u  /* a bounded wait gave up; outputs of that CTA invalid   */

typedef enum FsDtype { FS_F16 = 0, FS_BF16 = 1, FS_F32 = 2 } FsDtype;

typedef enum FsKvLayout { FS_LAYOUT_CONTIGUOUS = 0, FS_LAYOUT_PAGED = 1 } FsKvLayout;

/* KV formats.  FS_KV_AFFINE_BLOCK is the reference's (quant.py:94-165): values int8 =
 * u - 128, fp32 scale and int16 zero point per [block_size x D] block.
 * FS_KV_SYMMETRIC (no counterpart in the reference, which lists symmetric INT8 as future
 * work, doc/TODO.MD:241-255): values int8 = rint(x / s), fp32 scale s = absmax / 127 per
 * (token, head), no zero points (k_zero / v_zero unused); scales laid out like the values
 * without the head_dim axis ([P, Hkv, page] paged, [B, Hkv, S] contiguous), 16-byte
 * aligned; one page = one block (block_size = page_size <= 64).  D = 128 with 16-token
 * pages and fp16 q runs the tuned kernels (the stage carries the page's 2 x 64 bytes of
 * token scales), every other shape the generic kernel. */
typedef enum FsKvFormat { FS_KV_AFFINE_BLOCK = 0, FS_KV_SYMMETRIC = 1 } FsKvFormat;

/* Arguments of one decode-attention call (one query token per request). */
typedef struct FsDecodeArgs {
  int32_t layout;             /* FsKvLayout                                          */
  const void* q;              /* [B, Hq, D], dtype q_dtype                            */
  const int8_t* k_values;     /* see layouts above; 16-byte aligned                  */
  const float* k_scale;
  const int16_t* k_zero;      /* 4-byte aligned                                      */
  const int8_t* v_values;
  const float* v_scale;
  const int16_t* v_zero;
  const int64_t* block_table; /* paged: [B, table_cols]; contiguous: NULL            */
  const int64_t* lengths;     /* [B]; NULL (contiguous only) = every request is seq_len */
  void* out;                  /* q_dtype [B, Hq, D]; unused when shard_o is set       */
  int32_t batch, q_heads, kv_heads, head_dim, block_size;
  int64_t num_blocks;         /* paged: physical pages P; contiguous: nblk per (b,h)  */
  int32_t table_cols;         /* paged only                                          */
  int32_t max_seq_len;        /* paged: cache.max_seq_len; contiguous: seq_len        */
  int32_t num_splits;         /* split-K factor; 0 = library policy                   */
  float sm_scale;             /* softmax scale, normally 1/sqrt(D)                    */
  /* optional logical page window [page_begin, page_end) per request (sequence
   * sharding across GPUs); page_end <= 0 means "to the end" */
  int64_t page_begin, page_end;
  /* optional partial outputs: when shard_o != NULL the call writes the normalised
   * partial O fp32 [B, Hq, D] and LSE fp32 [B, Hq] (natural log, -inf if empty)
   * instead of `out`, for a later fs_merge_partials */
  float* shard_o;
  float* shard_lse;
  void* workspace;            /* device scratch for split partials,
                                 fs_decode_workspace_size() bytes (any contents)   */
  size_t workspace_bytes;
  uint32_t* tickets;          /* device merge counters, >= batch*kv_heads entries when
                                 num_splits > 1; must be zero at call time; every call
                                 that completes leaves them zero                    */
  int64_t ticket_count;
  uint32_t* device_status;    /* optional device word receiving FS_DEV_* bits         */
  int32_t q_dtype;            /* FsDtype of q and out: FS_F16 or FS_BF16              */
  int32_t page_size;          /* paged: tokens per page, a multiple of block_size
                                 (0 = block_size); contiguous: ignored                 */
  int32_t kv_format;          /* FsKvFormat of K and V                                */
} FsDecodeArgs;

/* Library version / ABI check. */
int fs_abi_version(void);
const char* fs_status_string(int status);
/* After a call returned FS_ERR_CUDA: which CUDA call failed and its error, for this
 * thread (empty before the first such failure).  No reference counterpart: the
 * reference surfaces CUDA errors as Python exceptions from its launcher. */
const char* fs_last_error_detail(void);

/* Bytes of workspace a call with these arguments needs (0 when num_splits
 * resolves to 1; the call then needs batch*kv_heads zeroed tickets as well).  Resolves num_splits==0 with the library policy and reports
 * the value used in *splits_out (may be NULL). */
int fs_decode_workspace_size(const FsDecodeArgs* args, size_t* bytes, int32_t* splits_out);

/* Contiguous INT8 KV decode attention.
 * Replaces _run_fused_dequant_attention_triton (src/flashspec/triton_fused.py:604-761)
 * i.e. the kernels _fused_dequant_attention_kernel / _split_kernel /
 * _combine_splits_kernel (triton_fused.py:203-503).  args->layout must be
 * FS_LAYOUT_CONTIGUOUS. */
int fs_fused_decode(const FsDecodeArgs* args, void* stream);

/* Paged INT8 KV decode attention through block_table.
 * Replaces _run_paged_quant_attention_triton (src/flashspec/triton_paged.py:338-450)
 * and _paged_quant_attention_kernel (triton_paged.py:120-299), adding split-K,
 * GQA and page windows.  args->layout must be FS_LAYOUT_PAGED. */
int fs_paged_decode(const FsDecodeArgs* args, void* stream);

/* Paged decode attention that allocates nothing, for callers that cannot provide
 * device memory and must not see the library allocate it (e.g. a plugin whose host
 * owns every device allocation, or a loop that cannot tolerate cudaMalloc's implicit
 * synchronisation).  No counterpart in the reference: it is fs_paged_decode with the
 * workspace/tickets fields ignored and replaced by one fixed scratch array compiled
 * into the library (8 MiB of split partials + 256 KiB of counters, held on every GPU
 * that loads the library until exit).  Limits: batch*kv_heads <= 65536 and
 * batch*kv_heads*splits*(q_heads/kv_heads)*516 bytes (rounded) <= 8 MiB, else
 * FS_ERR_SCRATCH_LIMIT (checked before any launch).  The first call on a device looks
 * up the array's device address (make it before any stream capture).  All calls share
 * the array: calls that may overlap on the GPU race and must be serialised. */
int fs_paged_decode_noalloc(const FsDecodeArgs* args, void* stream);

/* Log-sum-exp merge of n_parts partial results (split-K partials, or per-GPU
 * shards gathered over NVLink).  Part i's O is o_parts + i*S ([rows, head_dim] fp32)
 * and its LSE lse_parts + i*S' ([rows] fp32), where S = part_stride and S' =
 * part_stride (both in floats) when part_stride > 0 -- e.g. parts packed as
 * [O | LSE] slots of one all-gather buffer -- and S = rows*head_dim, S' = rows when
 * part_stride == 0 (dense stacks).  Writes out [rows, head_dim] as out_dtype (FS_F16
 * or FS_F32); rows whose partials are all empty produce 0.
 * Same math as _combine_splits_kernel (src/flashspec/triton_fused.py:446-503). */
int fs_merge_partials(const float* o_parts, const float* lse_parts, int32_t n_parts, int64_t rows,
                      int32_t head_dim, int64_t part_stride, void* out, int32_t out_dtype, void* stream);

/* Peer-memory exchange for decode steps whose pages are split across the GPUs of one
 * node (one process per GPU).  It stands where the gather of per-rank partials plus
 * fs_merge_partials would: the reference has no multi-GPU path, and its combine of
 * partials (_combine_splits_kernel, src/flashspec/triton_fused.py:446-503) is the
 * merge applied here to one partial per rank.
 *
 * Set-up, once per group: every rank calls fs_exchange_create (a cudaMalloc'd, zeroed
 * buffer for slots of slot_floats elements -- a multiple of 64, at least
 * rows*(head_dim+1); each element travels as an 8-byte (value, call tag) word -- and its FS_EXCHANGE_HANDLE_BYTES-byte IPC handle), sends the
 * handle to the other ranks (e.g. through torch.distributed), and maps each peer's
 * buffer with fs_exchange_open.  Tear-down: fs_exchange_close on the peers' mappings,
 * then fs_exchange_destroy on its own buffer.
 *
 * fs_exchange_merge, per step, on every rank (the same number of calls on each): one
 * kernel stores this rank's partial rows into every rank's buffer (plain peer stores
 * over NVLink) and waits for every rank's rows -- up to timeout_ns, after which it sets
 * FS_DEV_TIMEOUT in device_status and writes NaN to the rows it could not merge -- and
 * writes the merged rows [rows, head_dim] to `out` (FS_F16 or FS_F32).  No host sync
 * and no collective library call, so a step that uses it can be recorded in a CUDA
 * graph.  Every buffer in bufs[] must come from fs_exchange_create / fs_exchange_open of
 * this process with the same slot_floats, else FS_ERR_INVALID_ARGUMENT (a larger slot
 * would store past the end of a peer's buffer).  After a timeout the ranks' call
 * counters may disagree: every rank must close and destroy its buffers and create new
 * ones. */
#define FS_EXCHANGE_MAX_RANKS 8
#define FS_EXCHANGE_HANDLE_BYTES 64
typedef struct FsExchangeArgs {
  int32_t world, rank;
  void* bufs[FS_EXCHANGE_MAX_RANKS]; /* exchange buffer of every rank, as mapped here */
  int64_t slot_floats;
  const float* o_mine;        /* this rank's partial O fp32 [rows, head_dim], 16-byte aligned */
  const float* lse_mine;      /* this rank's partial LSE fp32 [rows] (natural log)          */
  int64_t rows;
  int32_t head_dim;
  void* out;
  int32_t out_dtype;
  int64_t timeout_ns;
  uint32_t* device_status;    /* optional device word receiving FS_DEV_TIMEOUT           */
} FsExchangeArgs;

int fs_exchange_create(int64_t slot_floats, void** buf, void* ipc_handle);
int fs_exchange_open(const void* ipc_handle, void** peer_buf);
int fs_exchange_close(void* peer_buf);
int fs_exchange_destroy(void* buf);
int fs_exchange_merge(const FsExchangeArgs* args, void* stream);

/* Sequence-sharded decode step in ONE kernel: the paged decode of this rank's page
 * window (args->page_begin / page_end) whose epilogue is the exchange -- the CTA that
 * finishes a (request, kv head) pair stores the pair's normalised (O, LSE) rows straight
 * into every rank's exchange buffer and merges every rank's rows of the pair into
 * x->out [batch, q_heads, head_dim] (FS_F16 or FS_F32), with no partial round trip
 * through this GPU's memory and no second launch.  Same buffers, waits, timeout and
 * status word as fs_exchange_merge (x->o_mine, lse_mine, rows, head_dim are ignored);
 * args->out and shard_o / shard_lse must be NULL.  Tuned shapes only (head_dim 128,
 * pages = quant blocks = 16 tokens, fp16 q) and at most one wave of CTAs per call
 * (batch * kv_heads <= resident CTAs, <= 4096 pairs), else FS_ERR_UNSUPPORTED.  The
 * split-K workspace and tickets are those fs_paged_decode_exchange_workspace_size names.
 * A set of exchange buffers serves either this entry point or fs_exchange_merge, not
 * both.  Replaces the same step as fs_exchange_merge: the reference has no multi-GPU
 * path; per GPU it is paged_quant_attention_triton (src/flashspec/triton_paged.py:453)
 * over a page range, and the merge is _combine_splits_kernel
 * (src/flashspec/triton_fused.py:446-503) across ranks. */
int fs_paged_decode_exchange_workspace_size(const FsDecodeArgs* args, size_t* workspace_bytes, int32_t* splits);
int fs_paged_decode_exchange(const FsDecodeArgs* args, const FsExchangeArgs* x, void* stream);

/* Affine INT8 quantization of x [n_lead, seq_len, head_dim] (dtype x_dtype,
 * contiguous) in blocks of block_size tokens, zero-padding the last block:
 * values [n_lead, nblk, block_size, head_dim], scale/zero_point [n_lead, nblk].
 * Bit-exact with quantize_int8_per_block (src/flashspec/quant.py:94-165). */
typedef struct FsQuantizeArgs {
  const void* x;
  int32_t x_dtype;
  int64_t n_lead;
  int32_t seq_len, head_dim, block_size;
  int8_t* values;
  float* scale;
  int16_t* zero_point;
} FsQuantizeArgs;
int fs_quantize_blocks(const FsQuantizeArgs* args, void* stream);

/* Symmetric per-token quantization into the FS_KV_SYMMETRIC format: x [n_lead, seq_len,
 * head_dim] -> values [n_lead, seq_len, head_dim] (rint(x / s) clamped to [-127, 127])
 * and scale [n_lead, seq_len] (s = max(absmax / 127, 1e-8)); block_size and zero_point
 * are unused.  No counterpart in the reference (doc/TODO.MD:241-255 lists it). */
int fs_quantize_symmetric(const FsQuantizeArgs* args, void* stream);

/* One page rewrite: rows [dst_row, dst_row+n_rows) of physical page `page`
 * take tokens [src_t, src_t+n_rows) of source request src_b; the other rows
 * are the page's dequantized current contents (from_zero=0, i.e. stale rows of
 * a reused page are kept) or zeros (from_zero=1); then the page is requantized. */
typedef struct FsPageUpdate {
  int64_t page;
  int32_t src_b, src_t, dst_row, n_rows, from_zero, reserved;
} FsPageUpdate;

typedef struct FsPageUpdateArgs {
  const FsPageUpdate* items;  /* DEVICE array [n_items]; pages distinct            */
  int32_t n_items;
  const void* k_src;          /* [Bsrc, H, T, D] with the strides below (elements) */
  const void* v_src;
  int32_t src_dtype;
  int64_t src_stride_b, src_stride_h, src_stride_t; /* D stride must be 1 */
  int32_t heads, head_dim, block_size;
  int64_t num_pages;          /* pool pages (bounds of items[].page)               */
  /* pool read before the update (may equal the *_out pointers: in place)          */
  const int8_t* k_values_in; const float* k_scale_in; const int16_t* k_zero_in;
  const int8_t* v_values_in; const float* v_scale_in; const int16_t* v_zero_in;
  int8_t* k_values_out; float* k_scale_out; int16_t* k_zero_out;
  int8_t* v_values_out; float* v_scale_out; int16_t* v_zero_out;
} FsPageUpdateArgs;

/* Page append / prefill with re-quantization, bit-exact with the reference
 * allocator (PagedKVAllocator.add_request / append_request / _write_quantized_block,
 * src/flashspec/paged.py:66-136,226-255) and with the whole-store requantization of
 * PagedKVCache.append (paged.py:463-557) when every page is listed. */
int fs_page_update(const FsPageUpdateArgs* args, void* stream);

/* Dequantize pages into fp32 [n_pages_listed, H, block_size, D]; pages is a device
 * int64 list (entries < 0 give zeros).  Same arithmetic as
 * dequantize_int8_per_block (src/flashspec/quant.py:168-204). */
int fs_dequantize_pages(const int8_t* values, const float* scale, const int16_t* zero_point,
                        const int64_t* pages, int64_t n_pages_listed, int64_t num_pages, int32_t heads,
                        int32_t block_size, int32_t head_dim, float* out, void* stream);

/* Tree-attention verify (speculative decoding), the draft-tree half: for node i of
 * request b, attention of q [B, nodes, Hq, D] over the draft tokens on i's root path
 * (tree_k / tree_v [B, nodes, Hkv, D], parents int32 [B, nodes], parents[b][i] < i,
 * -1 = the node hangs off the committed prefix), merged with the normalised partial
 * (prefix_o fp32 [B, nodes, Hq, D], prefix_lse fp32 [B, nodes, Hq], natural log) of the
 * same rows over the committed prefix, or with nothing when prefix_o is NULL.  out has
 * q's dtype (FS_F16 / FS_BF16); head_dim 32/64/128/256.  The reference plans this kernel
 * (doc/TODO.MD:186-237, "Kernel 3") without implementing it; parents are validated by
 * the caller (the Python wrapper raises on cycles and orphans). */
typedef struct FsTreeArgs {
  const void* q;
  const void* tree_k;
  const void* tree_v;
  const int32_t* parents;
  const float* prefix_o;
  const float* prefix_lse;
  void* out;
  int32_t batch, nodes, q_heads, kv_heads, head_dim, q_dtype;
  float sm_scale;
} FsTreeArgs;
int fs_tree_attend(const FsTreeArgs* args, void* stream);

/* Measurement aid, no counterpart in the reference: streams `bytes` (a multiple of 16,
 * 16-byte aligned buffer) through a read-only kernel and stores one 32-bit XOR per CTA
 * into sink[0 .. *ctas_used) (sink_count entries at least as many as the CTAs used, at
 * most resident CTAs).  Time it with events to get the GPU's read-only HBM bandwidth,
 * the denominator for kernels that mostly read (the decode kernels). */
int fs_read_bandwidth_probe(const void* buf, size_t bytes, uint32_t* sink, int32_t sink_count, int32_t* ctas_used,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHSPEC_B200_H_ */

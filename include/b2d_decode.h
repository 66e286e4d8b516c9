/*
 * b2d_decode.h — C ABI of the B200 (sm_100a) decode-attention library
 * (libb2d.so).  Plain pointers, sizes and enums only: no C++ or torch types.
 *
 * What this boundary replaces.  The reference (meinie0826/Roofline-Analysis,
 * decodebench/) times one library call per backend inside a
 * `<X>Kernel(DecodeShape).run()` adapter.  These entry points are the single
 * call such an adapter makes:
 *
 *   b2d_decode_gqa  replaces
 *     decodebench/flashattn_kvcache_kernel.py:150-169
 *         flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens,
 *                                 block_table, causal=True) -> (out, lse)
 *     decodebench/flashinfer_kernel.py:115-116
 *         BatchDecodeWithPagedKVCacheWrapper.run(q, (k_cache, v_cache))
 *     decodebench/trtllm_decode_kernel.py:102-113
 *         trtllm_batch_decode_with_kv_cache(...)  (HND cache: pass strides)
 *     decodebench/vllm_paged_kernel.py:203-222
 *         ops.paged_attention_v2(...)  (split-KV partials + reduce)
 *   b2d_decode_mla  replaces
 *     decodebench/trtllm_mla_kernel.py:115-132
 *         trtllm_batch_decode_with_kv_cache_mla(query, kv_cache, ...)
 *   the split merge inside both follows
 *     cute_attention/cluster_decode/cluster_decode_reduce.py:67-91
 *         merge_split_kv_decode_partials (M = max m; L = sum l e^(m-M); ...)
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise.  Strides are
 *     in ELEMENTS; the innermost (head_dim) dimension must be contiguous.
 *   - All calls are enqueue-only on `stream` (a cudaStream_t, NULL = legacy
 *     default stream); none synchronises or allocates.  The caller owns all
 *     memory including the workspace (size from the *_workspace_bytes call).
 *   - Return value 0 = success, negative = b2d_status code; a human-readable
 *     message comes from b2d_error_string().  Nothing aborts the process.
 *   - lse is the natural-log log-sum-exp of the scaled scores, fp32.
 */
#ifndef B2D_DECODE_H_
#define B2D_DECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (0 = ok). */
enum b2d_status {
  B2D_OK = 0,
  B2D_ERR_INVALID_ARG = -1,      /* null pointer, bad size, bad stride      */
  B2D_ERR_UNSUPPORTED = -2,      /* head_dim / dtype / group not built      */
  B2D_ERR_ALIGNMENT = -3,        /* base or stride not 16-byte aligned      */
  B2D_ERR_WORKSPACE = -4,        /* workspace missing or too small          */
  B2D_ERR_CUDA = -5,             /* a CUDA runtime/driver call failed       */
  B2D_ERR_DEVICE_TIMEOUT = -6,   /* a kernel gave up waiting (status word)  */
  B2D_ERR_DEVICE_BOUNDS = -7,    /* a kernel saw a page id out of range     */
  B2D_ERR_TOO_LARGE = -8         /* a size beyond the documented maximum    */
};

/* Launch flags, for measuring the two kernels of a decode separately.
 * SKIP_COMBINE enqueues only the split-KV kernel (rows split across CTAs are
 * then left as partials in the workspace); COMBINE_ONLY enqueues only the
 * merge, over the partials the previous identical call left.  When the GQA
 * plan merges inside the split-KV kernel (many rows per CTA wave), there is
 * no combine kernel: SKIP_COMBINE changes nothing and COMBINE_ONLY enqueues
 * nothing.  TEST_NO_LOADS is for testing the bounded waits: the producer
 * issues no loads, so every consumer wait runs out after wait_limit_us,
 * records B2D_ERR_DEVICE_TIMEOUT in the status word and returns (no copy is
 * in flight when the kernel ends); out and lse are then undefined. */
enum b2d_flags {
  B2D_FLAG_SKIP_COMBINE = 1,
  B2D_FLAG_COMBINE_ONLY = 2,
  B2D_FLAG_TEST_NO_LOADS = 4
};

/* Paged-cache layouts (b2d_gqa_args.kv_layout). */
enum b2d_kv_layout {
  /* [page, token, head, head_dim] in any order given by the strides: NHD
   * [pages, P, Hkv, D], TRT-LLM HND [pages, 2, Hkv, P, D], ... */
  B2D_KV_STRIDED = 0,
  /* vLLM paged_attention: K [blocks, Hkv, D/8, P, 8] (8 elements = 16 bytes
   * innermost), V [blocks, Hkv, D, P] (tokens innermost); each head's block
   * contiguous, blocks of all heads contiguous (stride_page = Hkv *
   * stride_head = Hkv * D * P elements).  16-bit caches, page_size % 16 == 0.
   * The *_stride_tok fields are ignored. */
  B2D_KV_VLLM = 1
};

/* Element types. */
enum b2d_dtype {
  B2D_BF16 = 0,
  B2D_FP16 = 1,
  B2D_FP8_E4M3 = 2,
  B2D_FP32 = 3
};

/*
 * Paged GQA/MHA/MQA decode: one query token per sequence.
 *   q        [batch, num_q_heads, head_dim]               (bf16 | fp16)
 *   k_cache  [num_pages, page_size, num_kv_heads, head_dim] (NHD, default) or
 *            any other order of (page, token, head) given by the strides, e.g.
 *            TRT-LLM HND [num_pages, 2, num_kv_heads, page_size, head_dim].
 *            Element type = q's type, or FP8_E4M3 with k_scale/v_scale.
 *   cache_seqlens [batch] int32, block_table [batch, max_pages_per_seq] int32
 *   k_scale, v_scale: fp32 [num_kv_heads] dequantisation scales (FP8 only;
 *            value = e4m3 * scale).  NULL means 1.0.
 *   out      [batch, num_q_heads, head_dim] in q's type;  lse [batch,
 *            num_q_heads] fp32 (may be NULL).
 * Query head h reads KV head h / (num_q_heads / num_kv_heads).
 * A sequence of length 0 yields out = 0 and lse = -inf.
 * Built: head_dim 64, 128 and 256 (any page size, all cache types) and 192
 * (bf16/fp16 caches with page_size % 16 == 0); group (num_q_heads /
 * num_kv_heads) <= 32.  Other combinations return B2D_ERR_UNSUPPORTED.
 */
typedef struct b2d_gqa_args {
  const void* q;
  int64_t q_stride_b, q_stride_h;
  const void* k_cache;
  const void* v_cache;
  int64_t k_stride_page, k_stride_tok, k_stride_head;
  int64_t v_stride_page, v_stride_tok, v_stride_head;
  int64_t num_pages;
  const int32_t* cache_seqlens;
  const int32_t* block_table;
  int64_t block_table_stride;
  const float* k_scale;
  const float* v_scale;
  void* out;
  int64_t out_stride_b, out_stride_h;
  float* lse;
  int64_t lse_stride_b;
  int32_t batch, num_q_heads, num_kv_heads, head_dim, page_size;
  int32_t max_pages_per_seq;
  int32_t q_dtype, kv_dtype;
  float softmax_scale;
  void* workspace;
  size_t workspace_bytes;
  int32_t num_ctas;        /* 0 = one resident wave on this device          */
  int32_t flags;           /* B2D_FLAG_* (0 = normal decode)                */
  int32_t kv_layout;       /* B2D_KV_* (0 = strided NHD/HND)                */
  int32_t wait_limit_us;   /* in-kernel wait limit, microseconds (0 = 2 s)  */
} b2d_gqa_args;

/* Workspace bytes that b2d_decode_gqa needs for these arguments (pointers
 * may be NULL here; only sizes, dtypes and num_ctas are read).  Every
 * workspace starts with a 256-byte status word and 64 KiB of split-merge
 * arrival counters (B2D_WORKSPACE_HEADER_BYTES in all); both must be zero
 * before the first call (cudaMemset once after allocating).  The kernels
 * leave them zero; b2d_check_device_status(clear = 1) re-zeroes them after a
 * device error. */
#define B2D_WORKSPACE_HEADER_BYTES 65792
int b2d_gqa_workspace_bytes(const b2d_gqa_args* args, size_t* bytes);

/* Enqueue the decode (split-KV kernel, then the LSE combine when a
 * sequence was split across CTAs). */
int b2d_decode_gqa(const b2d_gqa_args* args, void* stream);

/*
 * Same decode as b2d_decode_gqa, for callers that cannot allocate device
 * memory — e.g. a plugin whose enqueue step may not allocate, or a serving
 * loop that reserved all free HBM for its KV cache at start-up — and so
 * cannot pass a workspace.  No counterpart in the reference.  args->workspace
 * and args->workspace_bytes are ignored: the scratch is a 16 MiB array of
 * device memory inside this library, held on every GPU that loads it until
 * the process exits.  Problems needing more than 16 MiB of workspace
 * (b2d_gqa_workspace_bytes) return B2D_ERR_TOO_LARGE.  The first call on a
 * device looks up the array's address and clears its status word (make it before any
 * stream capture).  All calls share the array, so calls that overlap on the
 * GPU race; serialise them.  Allocates nothing.
 */
int b2d_decode_gqa_static_scratch(const b2d_gqa_args* args, void* stream);

/*
 * Absorbed-MLA decode (DeepSeek-V3 shape): every query head attends to one
 * shared latent KV head.  Scores use all head_dim_qk (= 576: 512 latent + 64
 * rope) columns; V is the first head_dim_v (= 512) columns of the same row.
 *   q        [batch, num_heads, head_dim_qk] bf16
 *   kv_cache [num_pages, page_size, head_dim_qk] bf16 (row stride given)
 *   out      [batch, num_heads, head_dim_v] bf16; lse [batch, num_heads] fp32
 */
typedef struct b2d_mla_args {
  const void* q;
  int64_t q_stride_b, q_stride_h;
  const void* kv_cache;
  int64_t kv_stride_page, kv_stride_tok;
  int64_t num_pages;
  const int32_t* cache_seqlens;
  const int32_t* block_table;
  int64_t block_table_stride;
  void* out;
  int64_t out_stride_b, out_stride_h;
  float* lse;
  int64_t lse_stride_b;
  int32_t batch, num_heads, head_dim_qk, head_dim_v, page_size;
  int32_t max_pages_per_seq;
  int32_t dtype;
  float softmax_scale;
  void* workspace;
  size_t workspace_bytes;
  int32_t num_ctas;        /* 0 = auto                                      */
  int32_t flags;           /* B2D_FLAG_* (0 = normal decode)                */
  int32_t wait_limit_us;   /* in-kernel wait limit, microseconds (0 = 2 s)  */
  int32_t reserved;
} b2d_mla_args;

int b2d_mla_workspace_bytes(const b2d_mla_args* args, size_t* bytes);
int b2d_decode_mla(const b2d_mla_args* args, void* stream);

/*
 * KV-cache append (the write side of the paged cache that the decode reads):
 * token t's key/value rows go to slot slot_mapping[t] = page * page_size +
 * offset, optionally quantised to FP8-e4m3 as round-to-nearest-even of
 * x / scale[kv_head], saturated to +-448.  Replaces
 * decodebench/vllm_paged_kernel.py:160-172 ops.reshape_and_cache(key, value,
 * key_cache, value_cache, slot_mapping, kv_cache_dtype, k_scale, v_scale)
 * for the NHD / HND page layouts (strides as in b2d_gqa_args).
 *   key, value   [num_tokens, num_kv_heads, head_dim] (bf16 | fp16)
 *   slot_mapping int64 [num_tokens]; a negative slot skips the token
 *   caches       in the source type, or FP8_E4M3 with k_scale / v_scale
 *   bad_slots    optional int counter (device), incremented for every
 *                slot >= num_pages * page_size (such tokens are skipped)
 */
typedef struct b2d_append_args {
  const void* key;
  const void* value;
  int64_t src_stride_t, src_stride_h;
  void* k_cache;
  void* v_cache;
  int64_t k_stride_page, k_stride_tok, k_stride_head;
  int64_t v_stride_page, v_stride_tok, v_stride_head;
  int64_t num_pages;
  const int64_t* slot_mapping;
  const float* k_scale;
  const float* v_scale;
  int* bad_slots;
  int32_t num_tokens, num_kv_heads, head_dim, page_size;
  int32_t src_dtype, cache_dtype;
  int32_t kv_layout;       /* B2D_KV_* ; for B2D_KV_VLLM only the page and
                              head strides are read (16-bit caches)         */
  int32_t reserved;
} b2d_append_args;

int b2d_append_kv(const b2d_append_args* args, void* stream);

/*
 * Reads (and clears, when clear != 0) the device status word that kernels
 * set when an in-kernel wait ran out of time or a page id was out of range.
 * Synchronises `stream`.  Returns 0 or the matching negative b2d_status.
 */
int b2d_check_device_status(void* workspace, int clear, void* stream);
/*
 * The same read-back for b2d_decode_gqa_static_scratch, whose status word
 * lives in the library's own scratch array on the current device (a caller
 * never sees that array's address).  No counterpart in the reference.
 * Returns B2D_OK when no call on this device has used the array yet.
 */
int b2d_static_scratch_check_status(int clear, void* stream);

/* Split plan the GQA kernel would use: number of CTAs (0 when num_ctas is 0:
 * one resident wave, resolved at launch from the kernel's occupancy), KV
 * tokens per pipeline chunk and KV heads per CTA (host-only). */
int b2d_gqa_plan(const b2d_gqa_args* args, int32_t* num_ctas,
                 int32_t* chunk_tokens, int32_t* kv_heads_per_cta);

/* Number of kernel launches one b2d_decode_gqa call with these arguments
 * enqueues (the split-KV kernel per batch slice, plus a combine kernel per
 * slice when the merge is not done in-kernel).  Launches nothing; needs a
 * current device (the plan depends on its SM count and occupancy).  No
 * counterpart in the reference. */
int b2d_gqa_launch_count(const b2d_gqa_args* args, int32_t* launches);
const char* b2d_error_string(int status);
const char* b2d_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B2D_DECODE_H_ */

/*
 * slokv.h - C ABI of the B200 (sm_100a) KV-cache hot path.
 *
 * Every entry point takes plain device pointers, element strides and a
 * cudaStream_t passed as `void*`; nothing here knows about torch.  All calls are
 * asynchronous on `stream`, allocate nothing, never synchronise, and are safe to
 * capture in a CUDA graph (fixed-address workspace supplied by the caller).
 *
 * Return value: SLOKV_OK (0) or a negative SLOKV_ERR_* status for arguments the
 * host side rejects before any launch.  Invalid *device-resident* metadata
 * (a slot or block id outside the pool, a context length longer than the block
 * table) never traps: the kernel skips the offending row, and ORs a
 * SLOKV_DEVERR_* bit into the caller's `dev_error` word (may be NULL).
 *
 * KV pool layout (same as the reference engine): one tensor per layer and per
 * K/V, shape [num_blocks, block_size, num_kv_heads, head_dim], with the inner
 * [block_size, num_kv_heads, head_dim] contiguous.  A "slot" is
 * block_id * block_size + offset.
 */
#ifndef SLOKV_H
#define SLOKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host-side argument checks) ---------------------------- */
#define SLOKV_OK                 0
#define SLOKV_ERR_INVALID_ARG   -1  /* null pointer, negative size, bad geometry  */
#define SLOKV_ERR_ALIGNMENT     -2  /* pointer/stride not aligned as required     */
#define SLOKV_ERR_UNSUPPORTED   -3  /* dtype / head_dim / group size not built    */
#define SLOKV_ERR_CUDA          -4  /* a CUDA runtime call failed                 */
#define SLOKV_ERR_WORKSPACE     -5  /* workspace missing or too small             */
#define SLOKV_ERR_SCRATCH_LIMIT -6  /* geometry needs more than the fixed scratch of
                                       slokv_paged_decode_noalloc                 */

/* ---- device error word bits ---------------------------------------------- */
#define SLOKV_DEVERR_SLOT_RANGE   0x1u  /* slot_mapping entry < -1 or >= num_slots  */
#define SLOKV_DEVERR_BLOCK_RANGE  0x2u  /* block_tables entry outside [0, num_blocks) */
#define SLOKV_DEVERR_CONTEXT_LEN  0x4u  /* context length > table width * block_size */
#define SLOKV_DEVERR_TIMEOUT      0x8u  /* a bounded wait (mbarrier, peer flag) gave up */
#define SLOKV_DEVERR_NONFINITE    0x10u /* FP8 encode met NaN/Inf (stored as code 0x7F) */

/* ---- element types --------------------------------------------------------- */
#define SLOKV_DTYPE_BF16      0
#define SLOKV_DTYPE_F16       1
#define SLOKV_DTYPE_F32       2
#define SLOKV_DTYPE_FP8_E4M3  3

/* Human-readable text for a status code. */
const char *slokv_status_string(int status);

/* ABI version: bumped whenever a signature below changes. */
int slokv_abi_version(void);

/*
 * Paged KV append.
 * Replaces the Triton `store_kvcache_kernel` / `store_kvcache`
 * (nanovllm/layers/attention.py:10-40).
 *
 * For every token i < num_tokens with slot = slot_mapping[i] != -1, copies the
 * `row_elems` contiguous elements (num_kv_heads * head_dim) of key row i to
 * k_cache[slot * row_elems ...] and of value row i to v_cache[...].  Rows of
 * key/value may have any stride (value is a strided view of the fused QKV
 * output in the reference); the cache rows are contiguous.  Bit copy for any
 * element type (elem_bytes 1, 2 or 4).  Uses 16-byte vector loads/stores when
 * every pointer and stride allows it, narrower vectors otherwise.
 */
int slokv_kv_append(const void *key, int64_t key_row_stride,
                    const void *value, int64_t value_row_stride,
                    void *k_cache, void *v_cache,
                    const int32_t *slot_mapping, int32_t num_tokens,
                    int32_t row_elems, int32_t elem_bytes, int64_t num_slots,
                    uint32_t *dev_error, void *stream);

/*
 * Workspace needed by slokv_paged_decode for a given geometry, in bytes.
 * The decode kernel is persistent (one CTA per SM); the workspace holds the
 * split-K partial states of the context segments that straddle two warps'
 * ranges, so its size does not depend on the batch or on the context lengths.
 * device: CUDA ordinal whose SM count sizes the grid (-1 = current device).
 */
size_t slokv_paged_decode_workspace_bytes(int32_t device, int32_t num_q_heads,
                                          int32_t num_kv_heads, int32_t head_dim);

/*
 * Paged decode attention (one query token per sequence, GQA).
 * Replaces `flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
 * cache_seqlens=context_lens, block_table=block_tables, softmax_scale, causal=True)`
 * (nanovllm/layers/attention.py:75-78, nanovllm/layers/mixed_attention.py:117-121).
 *
 *   out[b, hq, :] = softmax(scale * q[b, hq] . K[b, 0:L_b, hq / G]^T) . V[...]
 *
 * with K/V gathered through block_tables[b, pos / block_size], L_b =
 * context_lens[b] (already including the token appended this step) and
 * G = num_q_heads / num_kv_heads.  Rows with L_b <= 0 produce zeros.
 * Table entries past ceil(L_b / block_size) are never read.
 *
 * q/out: element (b, h, d) at base + b*stride_b + h*stride_h + d.
 * k_cache/v_cache: [num_blocks, block_size, num_kv_heads, head_dim] with the
 * given block stride (elements).
 * dtype: SLOKV_DTYPE_BF16 or SLOKV_DTYPE_F16 for q/out/cache (tensor-core
 * path), or SLOKV_DTYPE_F32 for an fp32 pool (the reference's fp32
 * configuration: CUDA-core fp32 arithmetic, groups of 1, 2, 4, 8 or 16 query
 * heads per KV head, cache bases 16-byte aligned; the workspace is not used).
 * workspace: >= slokv_paged_decode_workspace_bytes(...) bytes, 256-byte aligned.
 */
int slokv_paged_decode(void *out, int64_t out_stride_b, int64_t out_stride_h,
                       const void *q, int64_t q_stride_b, int64_t q_stride_h,
                       const void *k_cache, const void *v_cache,
                       int64_t k_block_stride, int64_t v_block_stride,
                       int32_t num_blocks, int32_t block_size,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                       const int32_t *block_tables, int64_t block_table_stride,
                       int32_t max_blocks_per_seq,
                       const int32_t *context_lens, int32_t batch,
                       float softmax_scale, int32_t dtype,
                       void *workspace, size_t workspace_bytes,
                       uint32_t *dev_error, void *stream);

/*
 * Causal varlen attention for prefill chunks, prefix-cached prefill and the
 * prefill rows of a mixed batch.
 * Replaces flash_attn_varlen_func(q, k|k_cache, v|v_cache, cu_seqlens_q,
 * cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale, causal=True,
 * block_table) (nanovllm/layers/attention.py:69-74,
 * nanovllm/layers/mixed_attention.py:123-133).
 *
 * Row r has q_len = cu_q[r+1]-cu_q[r] queries and k_len = cu_k[r+1]-cu_k[r]
 * keys; query i sees keys 0 .. k_len-q_len+i (bottom-right aligned).  Keys come
 * from the paged pool through block_tables[r, key / block_size] when
 * block_tables is non-null (k/v are the [num_blocks, block_size, Hkv, 128]
 * caches, block strides in elements), else from rows cu_k[r] .. of contiguous
 * k/v ([kv_rows, Hkv, 128] with row strides kv_stride_t / v_stride_t).
 * q/out: [q_rows, Hq, 128] with the given token / head strides.  bf16 or f16.
 * tcgen05.mma with TMEM accumulators; block_size must be a multiple of 128.
 * k_page_scale (NULL: none): fp32 [num_blocks, Hkv]; when given, the paged K
 * holds unscaled FP8 code values and the logits of keys in page b are
 * S * k_page_scale[b * Hkv + kv head] (FP8 pools; even GQA groups only, else
 * SLOKV_ERR_UNSUPPORTED).
 */
int slokv_paged_prefill(void *out, int64_t out_stride_t, int64_t out_stride_h,
                        const void *q, int64_t q_stride_t, int64_t q_stride_h, int64_t q_rows,
                        const void *k, const void *v, int64_t kv_stride_t, int64_t v_stride_t,
                        int64_t kv_rows, int64_t k_block_stride, int64_t v_block_stride,
                        const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                        int32_t num_rows, int32_t max_seqlen_q,
                        const int32_t *block_tables, int64_t block_table_stride,
                        int32_t max_blocks_per_seq, int32_t num_blocks, int32_t block_size,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                        float softmax_scale, int32_t dtype, const float *k_page_scale,
                        void *workspace, size_t workspace_bytes, uint32_t *dev_error,
                        void *stream);

/* Bytes of the optional prefill workspace: num_rows * ceil(max_seqlen_q / 128)
 * int32 (rounded up to 256), holding the longest-first order of the query
 * tiles that a small pre-kernel writes on the same stream.  With a null or
 * smaller workspace slokv_paged_prefill runs the tiles in row-major order
 * (same results, longer tail).  No counterpart in the reference (its
 * flash-attn call schedules internally). */
size_t slokv_paged_prefill_workspace_bytes(int32_t num_rows, int32_t max_seqlen_q);

/*
 * Fused q/k RMSNorm + rotary embedding + append (the layer chain between the
 * qkv projection and attention: nanovllm/models/qwen3.py:76-86 with
 * nanovllm/layers/layernorm.py, nanovllm/layers/rotary_embedding.py and
 * store_kvcache, nanovllm/layers/attention.py:10-40).  qkv: [T, (Hq + 2 Hkv) x
 * 128] rows (element stride qkv_row_stride); q_weight / k_weight: [128];
 * positions: [T] int64; cos_sin: fp32 [max_position, 128] = cos[64] | sin[64]
 * per position (the reference's cos_sin_cache); q_out: [T, Hq, 128] (token
 * stride q_out_row_stride); k_out: [T, Hkv, 128] or NULL.  Cache row
 * slot_mapping[t] (slot -1 skips) receives the normed, rotated k and the raw v.
 * RMS statistics in fp32, the normed row rounded, times the weight (rounded),
 * rotation in fp32 of the rounded values, rounded.  head_dim 128, bf16/f16.  A
 * position outside [0, max_position) sets SLOKV_DEVERR_CONTEXT_LEN. */
int slokv_qk_norm_rope_append(const void *qkv, int64_t qkv_row_stride, int32_t num_tokens,
                              int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                              const void *q_weight, const void *k_weight, float eps,
                              const int64_t *positions, const float *cos_sin,
                              int32_t max_position, const int32_t *slot_mapping, void *k_cache,
                              void *v_cache, int64_t num_slots, void *q_out,
                              int64_t q_out_row_stride, void *k_out, int64_t k_out_row_stride,
                              int32_t dtype, uint32_t *dev_error, void *stream);

/*
 * FP8-E4M3 KV cache.
 *
 * Pool: codes uint8 [num_blocks, block_size, num_kv_heads, head_dim] (one tensor
 * for K, one for V, as in the bf16 layout) and fp32 scales [num_blocks,
 * num_kv_heads] for K and for V.  A scale of 0 means "nothing nonzero stored
 * yet".  The scales need no reset when a block is (re)assigned: a write that
 * starts at offset 0 of a block ignores the stored scale (a block's first
 * token always lands at offset 0, and shared prefix blocks are full and never
 * written), so a reused page never inherits its previous owner's amax and the
 * block manager (nanovllm/engine/block_manager.py:43-92) stays unchanged.
 * The reference has the E4M3FN codec (benchmarks/v0/probe_quant_support.py:24-56)
 * but no quantised KV path; this is the per-(block, kv-head) contract of the
 * north star, written out in oracle/kv_oracle.py (fp8_append):
 *   s_old = 0 if the block's new tokens start at offset 0, else the stored scale;
 *   s_new = max(s_old, amax(new tokens of the block, this head) / 448);
 *   if s_new > s_old > 0 the block/head's earlier positions are re-encoded as
 *   encode(fp32(decode(c) * s_old) / s_new); new tokens get encode(x / s_new)
 *   (divisor 1 while s_new == 0); RNE everywhere, saturation at 448.
 * The new tokens of one block must be adjacent in slot_mapping with
 * consecutive offsets (decode: one token per block; prefill: a run).
 */

/* Quantising append; counterpart of slokv_kv_append for the FP8 pool
 * (replaces store_kvcache, nanovllm/layers/attention.py:33-40, when the pool is
 * FP8).  in_dtype: SLOKV_DTYPE_BF16, _F16 or _F32 for key/value.  head_dim 128. */
int slokv_kv_append_fp8(const void *key, int64_t key_row_stride,
                        const void *value, int64_t value_row_stride,
                        void *k_codes, void *v_codes, float *k_scale, float *v_scale,
                        const int32_t *slot_mapping, int32_t num_tokens,
                        int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                        int32_t num_blocks, int32_t in_dtype,
                        uint32_t *dev_error, void *stream);

/* Prefix-cache prefill over an FP8 pool (the prefill half of
 * flash_attn_varlen_func / forward_mixed, nanovllm/layers/attention.py:69-74,
 * nanovllm/layers/mixed_attention.py:123-133, when the pool is FP8): page p of
 * row r (p < pages_per_row, p * block_size < cu_seqlens_k[r+1] - cu_seqlens_k[r])
 * is written to page r * pages_per_row + p of f16 buffers dst_k / dst_v
 * ([num_rows * pages_per_row, block_size, Hkv, 128]): K as its unscaled code
 * values (exact in f16) with the page's K scale in dst_k_scale[page * Hkv + h],
 * V as decode(code) * scale in fp32 rounded to f16.  slokv_paged_prefill (f16,
 * k_page_scale = dst_k_scale) then attends through table row r = r *
 * pages_per_row + 0 .. pages_per_row - 1, applying the K scale to the logits as
 * the FP8 decode does.  Pages past a row's keys are not written; an id outside
 * the pool writes zeros (scale 0) and sets SLOKV_DEVERR_BLOCK_RANGE.  Codes,
 * strides and destinations 16-byte aligned. */
int slokv_fp8_pages_dequant(const void *k_codes, const void *v_codes, int64_t k_block_stride,
                            int64_t v_block_stride, const float *k_scale, const float *v_scale,
                            int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                            int32_t head_dim, const int32_t *block_tables,
                            int64_t block_table_stride, int32_t max_blocks_per_seq,
                            const int32_t *cu_seqlens_k, int32_t num_rows, int32_t pages_per_row,
                            void *dst_k, void *dst_v, float *dst_k_scale, uint32_t *dev_error,
                            void *stream);

/* Prefix-cache prefill over an FP8 pool, reading the code pages directly (the
 * prefill half of flash_attn_varlen_func / forward_mixed,
 * nanovllm/layers/attention.py:69-74, nanovllm/layers/mixed_attention.py:123-133,
 * when the pool is FP8).  Arguments as slokv_paged_prefill with paged K/V, the
 * pool being k_codes / v_codes (uint8 [num_blocks, block_size, Hkv, 128],
 * block strides in bytes, 16-byte multiples) and its fp32 scales k_scale /
 * v_scale [num_blocks, Hkv].  Each 128-key tile of codes is TMA-loaded from its
 * page.  S = Q K^T runs on the K codes (E4M3 x E4M3 MMAs, fp32 accumulate)
 * against each query row split into two E4M3 rows (a power-of-two row scale,
 * hi = e4m3(q), lo = e4m3(q - hi): exact for every element at least 2^-10 of
 * its row's largest), times the page's K scale; V codes are widened in shared
 * memory to their f16 values and the page's V scale applied to P.  Out is
 * written in q_dtype (bf16 or f16).  Within the FP8 attention bar of the fp32
 * result on the dequantised pool.  Even GQA groups only, block_size % 128 == 0,
 * max_blocks_per_seq <= 4330 (a K and a V scale per page in shared memory;
 * pass the pages the longest row reaches), else SLOKV_ERR_UNSUPPORTED.  An id
 * outside the pool loads zero codes (scale 0) and sets
 * SLOKV_DEVERR_BLOCK_RANGE. */
int slokv_paged_prefill_fp8(void *out, int64_t out_stride_t, int64_t out_stride_h,
                            const void *q, int64_t q_stride_t, int64_t q_stride_h, int64_t q_rows,
                            const void *k_codes, const void *v_codes, int64_t k_block_stride,
                            int64_t v_block_stride, const float *k_scale, const float *v_scale,
                            const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                            int32_t num_rows, int32_t max_seqlen_q, const int32_t *block_tables,
                            int64_t block_table_stride, int32_t max_blocks_per_seq,
                            int32_t num_blocks, int32_t block_size, int32_t num_q_heads,
                            int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                            int32_t q_dtype, void *workspace, size_t workspace_bytes,
                            uint32_t *dev_error, void *stream);

/* slokv_kv_append_fp8 for calls with long runs (prefill chunks: up to a block
 * of new tokens per (block, kv head)), token-parallel in three launches: each
 * (token, head, K|V) takes its row's amax into a per-(block, head, K|V) word
 * (atomicMax on the float bits), then every token is encoded with s_new =
 * max(s_old, amax / 448) (the run's first token re-encodes the block's earlier
 * positions when the scale grows), then the run's first token stores s_new and
 * clears the word.  Same arguments, codes and scales as slokv_kv_append_fp8,
 * plus `workspace`: slokv_kv_append_fp8_runs_workspace_bytes(num_blocks,
 * num_kv_heads) bytes, 4-byte aligned, zero before the first call (each call
 * leaves it zero); else SLOKV_ERR_WORKSPACE. */
size_t slokv_kv_append_fp8_runs_workspace_bytes(int32_t num_blocks, int32_t num_kv_heads);
int slokv_kv_append_fp8_runs(const void *key, int64_t key_row_stride, const void *value,
                             int64_t value_row_stride, void *k_codes, void *v_codes,
                             float *k_scale, float *v_scale, const int32_t *slot_mapping,
                             int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                             int32_t block_size, int32_t num_blocks, int32_t in_dtype,
                             void *workspace, size_t workspace_bytes, uint32_t *dev_error,
                             void *stream);

/* Workspace of slokv_paged_decode_fp8 (8 warp slots per SM), in bytes. */
size_t slokv_paged_decode_fp8_workspace_bytes(int32_t device, int32_t num_q_heads,
                                              int32_t num_kv_heads, int32_t head_dim);

/* Paged decode over the FP8 pool, dequantisation fused into the tile load
 * (replaces flash_attn_with_kvcache, nanovllm/layers/attention.py:76-78, when
 * the pool is FP8).  Same arguments as slokv_paged_decode plus the two scale
 * arrays; q/out are bf16 or f16 (q_dtype).  QK^T runs in f16 on the raw codes
 * with the K scale applied to the scores; PV runs in f16 with the output kept
 * in units of the current page's V scale.  q must lie within the f16 range. */
int slokv_paged_decode_fp8(void *out, int64_t out_stride_b, int64_t out_stride_h,
                           const void *q, int64_t q_stride_b, int64_t q_stride_h,
                           const void *k_codes, const void *v_codes,
                           int64_t k_block_stride, int64_t v_block_stride,
                           const float *k_scale, const float *v_scale,
                           int32_t num_blocks, int32_t block_size,
                           int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                           const int32_t *block_tables, int64_t block_table_stride,
                           int32_t max_blocks_per_seq,
                           const int32_t *context_lens, int32_t batch,
                           float softmax_scale, int32_t q_dtype,
                           void *workspace, size_t workspace_bytes,
                           uint32_t *dev_error, void *stream);

/* E4M3FN codec on device arrays (the encoder of
 * benchmarks/v0/probe_quant_support.py:39-56 and decoder of :24-33):
 * RNE to the nearest code, ties to even, saturate at 448; NaN/Inf encode as
 * 0x7F and flag SLOKV_DEVERR_NONFINITE. */
int slokv_fp8_e4m3_encode(const float *x, uint8_t *codes, int64_t n,
                          uint32_t *dev_error, void *stream);
int slokv_fp8_e4m3_decode(const uint8_t *codes, float *x, int64_t n, void *stream);

/*
 * Allocation-free paged decode.  No counterpart in the reference engine.
 *
 * Same arguments and result as slokv_paged_decode, minus the workspace.  It is
 * for callers that cannot call cudaMalloc: a host runtime that binds only this
 * C ABI and owns no device allocator, or an engine whose caching allocator has
 * already given ~90% of HBM to the KV pool, where a new cudaMalloc would fail
 * or would synchronise the device in the middle of a step.  The split-K
 * scratch lives in a file-scope __device__ array of
 * slokv_paged_decode_noalloc_scratch_bytes() bytes (6 MiB) that every GPU
 * loading the library keeps until the process exits.  Nothing is allocated,
 * freed or zeroed per call.
 *
 * Limits and rules:
 *  - the partials take SMs x 3 x (2 x G x 132 x 4 + 16) bytes for G query
 *    heads per KV head; a call that slokv_paged_decode would run but whose
 *    partials exceed the scratch (on a 148-SM B200: G > 13) returns
 *    SLOKV_ERR_SCRATCH_LIMIT and launches nothing; every other argument error
 *    returns the same status as slokv_paged_decode;
 *  - the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current, so make the first call
 *    on each device before any stream capture;
 *  - every call on a device shares the one scratch array, which keeps the last
 *    call's contents; no part of it needs to start at zero (each partial is
 *    written before it is read within a call), but calls that overlap on the
 *    GPU -- on different streams, or graphs replayed concurrently -- race on it.
 */
int slokv_paged_decode_noalloc(void *out, int64_t out_stride_b, int64_t out_stride_h,
                               const void *q, int64_t q_stride_b, int64_t q_stride_h,
                               const void *k_cache, const void *v_cache,
                               int64_t k_block_stride, int64_t v_block_stride,
                               int32_t num_blocks, int32_t block_size,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               const int32_t *block_tables, int64_t block_table_stride,
                               int32_t max_blocks_per_seq,
                               const int32_t *context_lens, int32_t batch,
                               float softmax_scale, int32_t dtype,
                               uint32_t *dev_error, void *stream);

/* Size in bytes of the fixed device scratch used by slokv_paged_decode_noalloc. */
size_t slokv_paged_decode_noalloc_scratch_bytes(void);

/*
 * Block-pool page copy.
 * Device counterpart of the page copy `pool[:, :, page].copy_(saved[:, :, j])`
 * (diagnostics/online_token_replay/tensors.py:34-43) and of copy-on-write /
 * swap of whole blocks for prefix sharing and preemption.
 *
 * Copies `num_pages` pages.  A page is `page_bytes` contiguous bytes (one block
 * of one layer of K or V: block_size * num_kv_heads * head_dim * elem_bytes).
 * The pool is addressed as [num_planes][num_pages_total] pages, where a
 * "plane" is one (K|V, layer) pair: page p of plane j lives at
 * base + j * plane_stride_bytes + p * page_stride_bytes.
 * Page i copies src page src_ids[i] to dst page dst_ids[i], in every plane.
 * src_ids / dst_ids may be NULL, meaning the identity i (used to gather pages
 * into, or scatter them out of, a compact buffer).  A pair with a negative id
 * is skipped; a pair with an id >= the side's capacity (pages per plane) is
 * skipped and sets SLOKV_DEVERR_BLOCK_RANGE.  Pointers, strides and page_bytes
 * must be 16-byte aligned.
 */
int slokv_kv_block_copy(const void *src, int64_t src_plane_stride_bytes,
                        int64_t src_page_stride_bytes, const int32_t *src_ids,
                        int32_t src_capacity,
                        void *dst, int64_t dst_plane_stride_bytes,
                        int64_t dst_page_stride_bytes, const int32_t *dst_ids,
                        int32_t dst_capacity,
                        int32_t num_pages, int32_t num_planes, int64_t page_bytes,
                        uint32_t *dev_error, void *stream);

/* ---- row-parallel linear + tensor-parallel all-reduce (one kernel) --------
 *
 * Replaces RowParallelLinear.forward (nanovllm/layers/linear.py:152-156):
 *   y = F.linear(x, W_rank, bias if rank == 0 else None); dist.all_reduce(y)
 * for the o_proj and down_proj of every decoder layer.  Every rank computes
 * its partial x_r W_r^T on the tensor cores and the ranks exchange 128 x 128
 * output tiles through each other's symmetric buffer over NVLink peer memory
 * (owner-reduce, then broadcast of the reduced tile), all inside one launch.
 * GEMMs of at least 2^34 multiply-adds (tokens x n_features x k_features) run
 * on CTA pairs (tcgen05.mma.cta_group::2, 256 x 256 tiles); smaller ones on one
 * CTA per 128 x 128 tile (slokv_row_parallel_plan reports the choice).
 * Result: y = round(bias + sum_r round(x_r W_r^T)) on every rank (the per-rank
 * rounding is the reference's F.linear output; the sum is fp32 in rank order,
 * rounded once), identical on every rank.
 *
 * x[i]: [tokens, k_features] (row stride x_row_stride elements), w[i]: [n_features,
 * k_features] (nn.Linear weight of rank rank_base + i), bias[i]: [n_features] or
 * NULL (bias may be NULL), y[i]: [tokens, n_features] output, for the
 * `local_ranks` ranks rank_base .. rank_base + local_ranks - 1 this launch runs
 * (1 in a one-process-per-GPU deployment; all ranks when one GPU emulates the
 * group).  rank_buffers[r] (r < world): the symmetric buffer of rank r as mapped
 * in this process (its own allocation, or a peer's opened with
 * slokv_ipc_import), slokv_row_parallel_buffer_bytes(max_tokens, n_features,
 * world) bytes each, zeroed once before first use; ignored when world == 1.
 * state: 2 device uint32 of this process, zeroed once (the call counter the
 * flags are compared against).  Every rank must make the same sequence of calls
 * with the same tokens / geometry.  world in {1, 2, 4, 8}, n_features % 128 == 0, k_features % 64 ==
 * 0, tokens <= max_tokens, 16-bit dtype, row strides multiples of 8 elements,
 * pointers 16-byte aligned (rank buffers 256-byte).  A peer that does not
 * arrive within the wait limit sets SLOKV_DEVERR_TIMEOUT (the output is then
 * undefined and the buffers must be zeroed again on every rank). */
size_t slokv_row_parallel_buffer_bytes(int32_t max_tokens, int32_t n_features, int32_t world);
int slokv_row_parallel_linear(const void *const *x, int64_t x_row_stride, const void *const *w,
                              int64_t w_row_stride, const void *const *bias, void *const *y,
                              int64_t y_row_stride, int32_t tokens, int32_t n_features,
                              int32_t k_features, void *const *rank_buffers, int32_t world,
                              int32_t rank_base, int32_t local_ranks, int32_t max_tokens,
                              uint32_t *state, int32_t dtype, uint32_t *dev_error, void *stream);

/* The grid slokv_row_parallel_linear would launch for this geometry on the
 * current device (no launch): plan[0] = kernel (1: one CTA per 128 x 128 tile,
 * 2: CTA pairs on 256 x 256 tiles with tcgen05.mma.cta_group::2), plan[1] =
 * CTAs per rank, plan[2] = CTAs of a rank with GEMM work, plan[3] = CTAs per
 * rank launched, plan[4] = co-resident two-CTA clusters on the device (0 when
 * the single-CTA kernel is chosen without querying it). */
int slokv_row_parallel_plan(int32_t tokens, int32_t n_features, int32_t k_features,
                            int32_t world, int32_t local_ranks, int32_t *plan);

/* Symmetric-buffer plumbing: a zeroed device allocation owned by the library,
 * and CUDA IPC export / import / close of it between the ranks' processes
 * (handles are slokv_ipc_handle_size() bytes, exchanged by the host). */
int slokv_device_alloc(size_t bytes, void **ptr);
int slokv_device_free(void *ptr);
int slokv_ipc_handle_size(void);
int slokv_ipc_export(const void *ptr, void *handle_out);
int slokv_ipc_import(const void *handle, void **ptr);
int slokv_ipc_close(void *ptr);

#ifdef __cplusplus
}
#endif

#endif /* SLOKV_H */

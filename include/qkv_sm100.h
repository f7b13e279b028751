/*
 * qkv_sm100.h — C ABI of libqkv_sm100.so, the B200 (sm_100a) kernels behind the
 * quantized-KV attention path of vllm-ascend-quantized-kv-cache
 * (dtype literals "int8" and "kivi_int4").
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are DEVICE pointers to contiguous memory in the
 *     layouts written next to each function; sizes are element counts.
 *   - `stream` is a cudaStream_t (0 = legacy default stream). Launches are
 *     asynchronous on that stream; no entry point synchronises the device.
 *   - Return value: QKV_OK (0) or a negative qkv_status. On error nothing was
 *     launched and qkv_last_error() returns the message (thread-local).
 *   - Kernels bounds-check every index they read from device memory (slots,
 *     block ids, residual rows). An out-of-range index is skipped, never
 *     dereferenced, and recorded in a device error word that
 *     qkv_device_error() reads back.
 *   - Floating-point element types are selected with qkv_dtype; index arrays
 *     (slot_mapping) with qkv_index.
 *
 * Every entry point names the reference interface it replaces (paths are
 * relative to src/vllm_ascend_quantized_kv_cache/ of the reference project).
 */
#ifndef QKV_SM100_H
#define QKV_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define QKV_API __attribute__((visibility("default")))
#else
#define QKV_API
#endif

typedef struct CUstream_st* qkv_stream_t; /* identical to cudaStream_t */

enum qkv_status {
  QKV_OK = 0,
  QKV_ERR_INVALID = -1,     /* bad argument: shape, alignment, geometry */
  QKV_ERR_UNSUPPORTED = -2, /* valid for the reference, not built here */
  QKV_ERR_CUDA = -3,        /* a CUDA runtime call failed */
  QKV_ERR_WORKSPACE = -4,   /* caller workspace too small */
  QKV_ERR_DEVICE = -5       /* a kernel recorded a bad index */
};

enum qkv_dtype { QKV_F32 = 0, QKV_BF16 = 1, QKV_F16 = 2 };
enum qkv_index { QKV_I32 = 0, QKV_I64 = 1 };

/* Library version string, e.g. "qkv_sm100 0.1.0 (sm_100a)". */
QKV_API const char* qkv_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len). Returns the status of the failed call (0 if none). */
QKV_API int qkv_last_error(char* buf, int len);

/* Synchronises `stream`, then reads and clears the device error word of the
 * current device. *code receives 0 or the first recorded kernel error
 * (1 = slot out of range, 2 = block id out of range, 3 = residual row out of
 * range, 4 = block-table entry negative for a live token, 5 = a bounded wait
 * on an in-kernel copy gave up, 6 = window plan source or lane out of
 * range, 7 = a bounded wait for the other ranks of a peer all-gather gave
 * up). Returns QKV_OK or QKV_ERR_CUDA. */
QKV_API int qkv_device_error(int* code, qkv_stream_t stream);

/* ------------------------------------------------------------------------
 * INT8 dynamic per-channel
 * ---------------------------------------------------------------------- */

/* Per-(kv_head, channel) scales from the first K/V batch of a layer.
 * Replaces AscendInt8AttentionBackendMixin._prepare_int8_scales
 * (methods/int8_dynamic/attention_backend.py:130-150; the same math as
 * Int8DynamicSemantics.calc_scales, methods/int8_dynamic/semantics.py:49-70).
 *   key, value        bf16 [num_tokens, num_kv_heads, head_size]
 *   k_inv_scale, ...  bf16 [num_kv_heads, head_size]
 * inv = bf16(bf16(1 / max(amax_t |x|, bf16(1e-12))) * 127), aq = bf16(1 / inv),
 * i.e. torch's bf16 `127.0 / amax` and `1.0 / inv` rounding sequence. */
QKV_API int qkv_int8_scales(const void* key, const void* value, int64_t num_tokens,
                    int num_kv_heads, int head_size, void* k_inv_scale,
                    void* v_inv_scale, void* k_aq_scale, void* v_aq_scale,
                    qkv_stream_t stream);

/* Quantise K/V and scatter them into the paged int8 caches.
 * Replaces AscendInt8AttentionBackendMixin._quantize_kv_to_runtime_int8
 * (methods/int8_dynamic/attention_backend.py:152-171) followed by the host's
 * reshape_and_cache (attention_backend.py:86-88).
 *   key, value            bf16 [num_tokens, num_kv_heads, head_size]
 *   slot_mapping          int32/int64 [num_tokens]; slot < 0 = padding, skipped
 *   k_inv_scale, v_inv..  bf16 [num_kv_heads, head_size]
 *   key_cache, value_c.   int8 [num_blocks, block_size, num_kv_heads, head_size]
 * code = clamp(rint(bf16(x * inv)), -128, 127). */
QKV_API int qkv_int8_quant_store(const void* key, const void* value,
                         const void* slot_mapping, int slot_dtype,
                         int64_t num_tokens, int num_kv_heads, int head_size,
                         int block_size, int64_t num_blocks,
                         const void* k_inv_scale, const void* v_inv_scale,
                         int8_t* key_cache, int8_t* value_cache,
                         qkv_stream_t stream);

/* Bytes of workspace qkv_int8_paged_decode needs for this batch shape. */
QKV_API size_t qkv_int8_paged_decode_workspace(int batch, int num_heads,
                                       int num_kv_heads, int head_size,
                                       int block_size, int max_seq_len);

/* GQA decode attention, one query token per request, over the paged int8
 * caches with per-channel antiquant folded into the kernel. Replaces the FIA
 * call of AscendInt8AttentionBackendMixin._forward_int8_decode
 * (methods/int8_dynamic/attention_backend.py:173-205); numerically it follows
 * the dequantise-then-attend path of _dequant_int8_paged_kv_to_dense
 * (attention_backend.py:370-404) + fp32 softmax attention.
 *   query        bf16, row b at query + b*q_stride, heads contiguous [Hq, D]
 *   key_cache..  int8 [num_blocks, block_size, num_kv_heads, head_size]
 *   k_aq_scale.. bf16 [num_kv_heads, head_size]
 *   block_table  int32, row b at block_table + b*bt_stride (>= max_blocks)
 *   seq_lens     int32 [batch]
 *   out          bf16, row b at out + b*out_stride, [Hq, D]
 * max_seq_len bounds seq_lens (used to plan the split-KV grid only). */
QKV_API int qkv_int8_paged_decode(const void* query, int64_t q_stride,
                          const int8_t* key_cache, const int8_t* value_cache,
                          const void* k_aq_scale, const void* v_aq_scale,
                          const int32_t* block_table, int64_t bt_stride,
                          const int32_t* seq_lens, int batch, int num_heads,
                          int num_kv_heads, int head_size, int block_size,
                          int64_t num_blocks, int max_seq_len, float scale,
                          void* workspace, size_t workspace_bytes, void* out,
                          int64_t out_stride, qkv_stream_t stream);

/* ------------------------------------------------------------------------
 * KIVI INT4 (int4 history + full-precision residual window)
 * ---------------------------------------------------------------------- */

/* Pack whole token groups of keys into the paged int4 key cache.
 * Replaces kivi_pack_key_cache / _kivi_pack_key_cache_kernel
 * (ops/triton/kivi_pack.py:287-348, :134-226).
 *   key       key_dtype [num_tokens, num_kv_heads, head_size], num_tokens % g == 0
 *   slot_map  [num_tokens]; each group of g slots contiguous, g-aligned and
 *             inside one block (validated by the host before the call)
 *   k_quant   int32 [num_blocks, num_kv_heads, head_size, block_size/8]
 *   k_scale   f32   [num_blocks, num_kv_heads, head_size, block_size/g]
 *   k_mn      f32   same shape as k_scale
 * scale = max((mx - mn) / 15, 1e-6); code = clamp(floor((x - mn)/scale + 0.5), 0, 15),
 * token offset o of the block goes to nibble o % 8 of word o / 8. */
QKV_API int qkv_kivi_pack_key(const void* key, int key_dtype, const void* slot_mapping,
                      int slot_dtype, int64_t num_tokens, int num_kv_heads,
                      int head_size, int group_size, int block_size,
                      int64_t num_blocks, int32_t* k_quant, float* k_scale,
                      float* k_mn, qkv_stream_t stream);

/* Pack values, one token at a time, grouped along head_size.
 * Replaces kivi_pack_value_cache / _kivi_pack_value_cache_kernel
 * (ops/triton/kivi_pack.py:229-284, :61-131).
 *   value     value_dtype [num_tokens, num_kv_heads, head_size]
 *   slot_map  [num_tokens]; slot < 0 skipped
 *   v_quant   int32 [num_blocks, block_size, num_kv_heads, head_size/8]
 *   v_scale   f32   [num_blocks, block_size, num_kv_heads, head_size/g]
 *   v_mn      f32   same shape as v_scale */
QKV_API int qkv_kivi_pack_value(const void* value, int value_dtype,
                        const void* slot_mapping, int slot_dtype,
                        int64_t num_tokens, int num_kv_heads, int head_size,
                        int group_size, int block_size, int64_t num_blocks,
                        int32_t* v_quant, float* v_scale, float* v_mn,
                        qkv_stream_t stream);

/* Pack keys and values of the SAME tokens in one launch: the results of
 * qkv_kivi_pack_key followed by qkv_kivi_pack_value on (key, slot_mapping)
 * and (value, slot_mapping). Replaces the pair of launches the reference
 * makes when a bulk prompt write flushes floor(n / r) * r tokens of both sides
 * to the int4 history (methods/kivi_int4/attention_backend.py:608-674 ->
 * kivi_pack_key_cache + kivi_pack_value_cache, ops/triton/kivi_pack.py:229-348).
 * Keys need whole groups (num_tokens % group_size == 0, every slot valid and
 * each group contiguous and aligned inside one block, as for
 * qkv_kivi_pack_key). bf16 at head_size 128, group 64 / 128 runs one fused
 * kernel; other geometries run the two packs back to back. */
QKV_API int qkv_kivi_pack_kv(const void* key, const void* value, int dtype,
                             const void* slot_mapping, int slot_dtype,
                             int64_t num_tokens, int num_kv_heads, int head_size,
                             int group_size, int block_size, int64_t num_blocks,
                             int32_t* k_quant, float* k_scale, float* k_mn,
                             int32_t* v_quant, float* v_scale, float* v_mn,
                             qkv_stream_t stream);

/* Bytes of workspace qkv_kivi_paged_decode needs for this batch shape. */
QKV_API size_t qkv_kivi_paged_decode_workspace(int batch, int num_heads,
                                       int num_kv_heads, int head_size,
                                       int group_size, int block_size,
                                       int max_seq_len);

/* Fused KIVI decode attention: streams the int4 pages of each request,
 * dequantises in registers and merges the bf16 residual window into the same
 * online softmax; no dense K/V copy is materialised. Replaces
 * _forward_kivi_paged_decode_attention (methods/kivi_int4/attention_backend.py:1193-1230),
 * i.e. _gather_dequant_kivi_paged_cache (:849-935) = kivi_dequant_gather_cache
 * (ops/kivi_gather.py:36-156) + residual tail overwrite, then FIA TND.
 *   query, out           as for qkv_int8_paged_decode
 *   k_quant..v_mn        the six KIVI views (see qkv_kivi_pack_key/value)
 *   res_key, res_value   bf16 [res_rows, res_capacity, num_kv_heads, head_size]
 *   seq_lens             int32 [batch]: row b attends to positions [0, seq_lens[b])
 *                        (the new token included; a prefill query row passes its
 *                        causal length, with the request's table row repeated)
 *   res_state            int32 [batch, 6] = row, k_start, k_len, v_start, v_len, end
 *                        (row < 0 or NULL: no residual). The key window holds
 *                        positions [end - k_len, end): position p in it reads
 *                        residual lane (k_start + p - (end - k_len)) % res_capacity,
 *                        every other position reads its int4 page
 *                        block_table[b][p / block_size]; values likewise. */
QKV_API int qkv_kivi_paged_decode(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* workspace, size_t workspace_bytes,
    void* out, int64_t out_stride, qkv_stream_t stream);
/* qkv_kivi_paged_decode for a consumer that merges the split partials itself
 * (qkv_peer_combine_allgather): when the page-pipelined kernel runs with
 * several splits, the [B, Hq, splits, D] fp32 sums and the [B, Hq, splits, 2]
 * (max, sum) pairs that follow them stay at the start of `workspace`, no
 * combine runs, and *splits_used receives the split count; otherwise `out`
 * is written as by qkv_kivi_paged_decode and *splits_used = 1. */
QKV_API int qkv_kivi_paged_decode_partials(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* workspace, size_t workspace_bytes,
    void* out, int64_t out_stride, int* splits_used, qkv_stream_t stream);

/* qkv_kivi_paged_decode for callers that cannot allocate device memory. This
 * entry point has no counterpart in the reference; it exists for callers of
 * this library that cannot hand it a workspace: an engine that has given all
 * free device memory to its own KV-cache pool, a host in another language with
 * no device allocator of its own behind the C ABI, or a serving loop that must
 * not call cudaMalloc because that call can synchronise the device.
 * Same arguments and result as qkv_kivi_paged_decode minus the workspace: the
 * split-KV partials live in a static device array of 8 MiB inside the library
 * (held on every GPU that loads it until the process exits). A batch whose
 * partials need more (see qkv_kivi_paged_decode_workspace) is rejected with
 * QKV_ERR_WORKSPACE. The call allocates nothing. Its first call on a device,
 * with that device current, looks the array's address up once, so make it
 * before any stream capture. All calls on a device share the array: calls
 * that overlap on the GPU race on it and must be serialised by the caller. */
QKV_API int qkv_kivi_paged_decode_noalloc(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* out, int64_t out_stride,
    qkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Dense prefill attention (TND)
 * ---------------------------------------------------------------------- */

/* Bytes of workspace qkv_dense_prefill needs. */
QKV_API size_t qkv_dense_prefill_workspace(int total_q, int num_heads,
                                   int num_kv_heads, int head_size,
                                   int max_kv_len);

/* Prompt attention over full-precision K/V in the TND layout, one request per
 * [cu_seqlens_q[b], cu_seqlens_q[b+1]) query range. Replaces the FIA calls of
 * the all-new prefill branches: _forward_kivi_prefill_fia and the prompt rows
 * of _forward_kivi_chunked_prefill (methods/kivi_int4/attention_backend.py:
 * 1232-1266, :1315-1338), and the PrefillNoCache / all-new rows of
 * _forward_int8_prefill / _forward_int8_chunked_prefill
 * (methods/int8_dynamic/attention_backend.py:246-368). With causal != 0 query
 * i of a request with q_len queries over kv_len keys sees keys
 * j <= kv_len - q_len + i (FIA sparse_mode 3, the mask of build_causal_mask,
 * methods/kivi_int4/semantics.py:285-299).
 *   query, out     bf16 [total_q, num_heads, head_size]
 *   key, value     bf16 [cu_seqlens_k[num_reqs], num_kv_heads, head_size]
 *   cu_seqlens_*   int32 [num_reqs + 1], cu[0] = 0
 *   total_k        cu_seqlens_k[num_reqs] (the rows of key / value)
 * Head size 128 with num_heads / num_kv_heads in {1, 2, 4, 8} runs on the
 * tcgen05 tensor cores (no workspace); other geometries on CUDA cores. */
QKV_API int qkv_dense_prefill(const void* query, const void* key, const void* value,
                      const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                      int num_reqs, int total_q, int total_k, int num_heads,
                      int num_kv_heads, int head_size, int causal,
                      int max_kv_len, float scale, void* workspace,
                      size_t workspace_bytes, void* out, qkv_stream_t stream);

/* Dense bf16 K/V of whole requests from the KIVI int4 pages and the bf16
 * residual windows: kivi_dequant_gather_cache (ops/kivi_gather.py:36-156) +
 * the residual overwrite of _gather_dequant_kivi_paged_cache
 * (methods/kivi_int4/attention_backend.py:849-935). Position t of request b
 * (t < seq_lens[b]) lands in row cu_seqlens_k[b] + t of out_key / out_value
 * bf16 [total_k, num_kv_heads, head_size]; a history element is
 * bf16(code * scale + mn) with the product and sum rounded in fp32, a window
 * element is copied. Views, windows, block table and res_state as for
 * qkv_kivi_paged_decode (res_state may be NULL: no windows). */
QKV_API int qkv_kivi_dequant_gather(
    const int32_t* k_quant, const float* k_scale, const float* k_mn,
    const int32_t* v_quant, const float* v_scale, const float* v_mn,
    const void* res_key, const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* cu_seqlens_k, const int32_t* res_state, int batch,
    int num_kv_heads, int head_size, int group_size, int block_size,
    int64_t num_blocks, int total_k, void* out_key, void* out_value,
    qkv_stream_t stream);

/* Dense bf16 K/V of whole requests from the int8 pages:
 * _dequant_int8_paged_kv_to_dense (methods/int8_dynamic/attention_backend.py:
 * 370-404). Position t of request b (t < seq_lens[b]) lands in row
 * cu_seqlens_k[b] + t of out_key / out_value bf16 [total_k, num_kv_heads,
 * head_size]; an element is bf16(code * aq) (the product is exact in fp32, so
 * this is the reference's bf16 multiply). Caches, scales and block table as
 * for qkv_int8_paged_decode; head_size a multiple of 16. */
QKV_API int qkv_int8_dequant_gather(
    const int8_t* key_cache, const int8_t* value_cache, const void* k_aq_scale,
    const void* v_aq_scale, const int32_t* block_table, int64_t bt_stride,
    const int32_t* seq_lens, const int32_t* cu_seqlens_k, int batch,
    int num_kv_heads, int head_size, int block_size, int64_t num_blocks,
    int total_k, void* out_key, void* out_value, qkv_stream_t stream);

/* ------------------------------------------------------------------------
 * FP8 per-token-head (E4M3 codes + one fp32 scale per (token, head))
 * ---------------------------------------------------------------------- */

/* Quantise K/V per (token, head) and scatter into the paged views: the
 * store of the fp8_per_token_head method (reference
 * ops/triton/per_token_head_store.py:262-294 with the numerics of
 * methods/fp8_per_token_head/semantics.py:52-66): scale = max(amax / 448,
 * 1e-6), code = E4M3(clamp(x / scale, -448, 448)), round to nearest even.
 *   key, value   kv_dtype [num_tokens, num_kv_heads, head_size] (head % 4 == 0)
 *   slot_mapping slot_dtype [num_tokens]; slot < 0 skipped
 *   k_data/v_data uint8 [num_blocks, block_size, num_kv_heads, head_size]
 *   k_scale/v_scale f32 [num_blocks, block_size, num_kv_heads, 1] */
QKV_API int qkv_fp8_store(const void* key, const void* value, int kv_dtype,
                          const void* slot_mapping, int slot_dtype,
                          int64_t num_tokens, int num_kv_heads, int head_size,
                          int block_size, int64_t num_blocks, uint8_t* k_data,
                          float* k_scale, uint8_t* v_data, float* v_scale,
                          qkv_stream_t stream);

/* Bytes of workspace qkv_fp8_paged_decode needs for this batch shape. */
QKV_API size_t qkv_fp8_paged_decode_workspace(int batch, int num_heads,
                                              int num_kv_heads, int head_size,
                                              int block_size, int max_seq_len);

/* GQA decode attention over the FP8 pages, per-token-head scales applied in
 * the kernel (the read path the reference's method lacks): numerically the
 * dequantise-then-attend of semantics.dequantize + fp32 softmax attention.
 * Query / out / block table / seq_lens as for qkv_int8_paged_decode. */
QKV_API int qkv_fp8_paged_decode(const void* query, int64_t q_stride,
                                 const uint8_t* k_data, const float* k_scale,
                                 const uint8_t* v_data, const float* v_scale,
                                 const int32_t* block_table, int64_t bt_stride,
                                 const int32_t* seq_lens, int batch,
                                 int num_heads, int num_kv_heads, int head_size,
                                 int block_size, int64_t num_blocks,
                                 int max_seq_len, float scale, void* workspace,
                                 size_t workspace_bytes, void* out,
                                 int64_t out_stride, qkv_stream_t stream);

/* Dense bf16 K/V of whole requests from the FP8 pages: bf16(code * scale)
 * (the product rounded to fp32 first, as semantics.dequantize computes it),
 * rows laid out as for qkv_int8_dequant_gather; head_size % 16 == 0. */
QKV_API int qkv_fp8_dequant_gather(const uint8_t* k_data, const float* k_scale,
                                   const uint8_t* v_data, const float* v_scale,
                                   const int32_t* block_table, int64_t bt_stride,
                                   const int32_t* seq_lens,
                                   const int32_t* cu_seqlens_k, int batch,
                                   int num_kv_heads, int head_size,
                                   int block_size, int64_t num_blocks,
                                   int total_k, void* out_key, void* out_value,
                                   qkv_stream_t stream);

/* ------------------------------------------------------------------------
 * KIVI residual windows: host planner and device apply
 * ---------------------------------------------------------------------- */

/* Host-side planner of the residual windows (no GPU): the reference's state
 * machine _store_kivi_residual_entries / _flush_kivi_residual_prefix /
 * _set_kivi_residual_window (methods/kivi_int4/attention_backend.py:377-462,
 * :813-836) over caller-owned int64 state arrays: per side, slots
 * [rows, capacity] (-1 = empty lane), FIFO start [rows] and length [rows].
 * Returns an opaque handle (NULL on bad arguments); the arrays must outlive
 * it. A plan collects flushes and ring writes between qkv_window_begin and
 * qkv_window_plan_export; source codes s >= 0 name ring lane s (row *
 * capacity + lane), s < 0 new token -1 - s. */
QKV_API void* qkv_window_create(int rows, int capacity, int group_size,
                                int64_t* key_slots, int64_t* key_start,
                                int64_t* key_length, int64_t* value_slots,
                                int64_t* value_start, int64_t* value_length);
QKV_API void qkv_window_destroy(void* window);
QKV_API void qkv_window_begin(void* window);
/* Appends n tokens (slots[i] holds new token tokens[i]) to one row's window:
 * a held slot is overwritten in place; at capacity a key window flushes whole
 * (gated by is_aligned_key_window, semantics.py:254-283, when
 * gate_block_size > 0; a misaligned window returns QKV_ERR_INVALID), a value
 * window evicts its oldest lane. */
QKV_API int qkv_window_store(void* window, int row, int n, const int64_t* slots,
                             const int64_t* tokens, int is_key,
                             int gate_block_size);
/* One token for each of n distinct rows (a decode step). */
QKV_API int qkv_window_store_one_each(void* window, int n, const int64_t* rows,
                                      const int64_t* slots,
                                      const int64_t* tokens, int is_key,
                                      int gate_block_size);
/* Tokens that go straight to the int4 history (bulk prompt write,
 * attention_backend.py:608-674). */
QKV_API int qkv_window_flush_direct(void* window, int n, const int64_t* slots,
                                    const int64_t* tokens, int is_key);
/* Drops lanes whose slot is not among live_slots; survivors move to lanes
 * 0.. in FIFO order. */
QKV_API int qkv_window_prune(void* window, int row, int n_live,
                             const int64_t* live_slots, int is_key);
QKV_API int qkv_window_reset_row(void* window, int row);
/* Sizes of the open plan of one side after deduplication (the last flush of
 * a slot, for keys of a whole group, is kept). */
QKV_API int qkv_window_plan_counts(void* window, int is_key, int64_t* n_flush,
                                   int64_t* n_writes);
/* flush_src / flush_slots [n_flush], write_lanes / write_src [n_writes]
 * (lanes ascending). */
QKV_API int qkv_window_plan_export(void* window, int is_key, int64_t* flush_src,
                                   int64_t* flush_slots, int64_t* write_lanes,
                                   int64_t* write_src);
/* ok[i] = 1 when both windows of rows[i] hold exactly the last positions of a
 * request of seq_lens[i] tokens (block-table row i of table [n, table_cols]);
 * the fast check of _sync_kivi_residual_windows. */
QKV_API int qkv_window_expected_live(void* window, int n, const int64_t* rows,
                                     const int64_t* seq_lens,
                                     const int64_t* table, int table_cols,
                                     int block_size, uint8_t* ok);

/* Device side of a plan, both sides in one launch: out_k[i] = the token row
 * named by k_src[i] (ring_key lane or new_key row), likewise for values.
 * Rings [ring_lanes, row_bytes], new tokens [n_new, row_bytes] (new_key may
 * be NULL when no source names a new token), row_bytes a multiple of 16. A
 * source out of range writes zeros and sets the device error word. Replaces
 * the index_select calls of the reference's window writes
 * (methods/kivi_int4/attention_backend.py:411-462). */
QKV_API int qkv_kivi_window_gather(const void* ring_key, const void* ring_value,
                                   int64_t ring_lanes, const void* new_key,
                                   const void* new_value, int64_t n_new,
                                   const int64_t* k_src, int64_t nk,
                                   const int64_t* v_src, int64_t nv,
                                   int64_t row_bytes, void* out_k, void* out_v,
                                   qkv_stream_t stream);
/* ring_key[k_lanes[i]] = k_data[i], ring_value[v_lanes[i]] = v_data[i]; a
 * lane out of range is skipped and sets the device error word. */
QKV_API int qkv_kivi_window_scatter(void* ring_key, void* ring_value,
                                    int64_t ring_lanes, const int64_t* k_lanes,
                                    int64_t nk, const void* k_data,
                                    const int64_t* v_lanes, int64_t nv,
                                    const void* v_data, int64_t row_bytes,
                                    qkv_stream_t stream);

/* A whole KIVI decode step (one new token per request) in one call: the
 * DecodeOnly branch of AscendKiviInt4AttentionBackendMixin.forward
 * (methods/kivi_int4/attention_backend.py:1006-1040): _write_kivi_cache
 * (:562-606) through the window planner, _sync_kivi_residual_windows
 * (:813-836), then _forward_kivi_paged_decode_attention (:1193-1230). Every
 * index the device needs is staged in one pinned buffer and copied once; the
 * value pack, ring scatter and decode launch on `stream` with no host sync
 * (a steady step reads the flushed lanes and new tokens in place; a step
 * with a key-window flush, or a ring write from a ring lane, first gathers
 * the plan's rows and also packs keys). qkv_kivi_step_create returns the runtime (staging buffers) of one
 * caller; destroy releases it.
 *   window            a qkv_window_create handle (its state is updated)
 *   rows, slots       int64 [batch] host: residual row and new-token slot
 *   seq_lens          int32 [batch] host, including the new token
 *   block_table_host  int32 [batch, table_cols] host (liveness check)
 *   block_table       int32 device [batch, >= max blocks], row stride bt_stride;
 *                     NULL: the host table is staged with the indices (one
 *                     copy for the whole step) and bt_stride is ignored
 *   query, out        bf16 [batch, num_heads, head_size], row strides in elements
 *   new_key/new_value bf16 [batch, num_kv_heads, head_size] device, contiguous
 *   k_quant..v_mn     the six KIVI views; res_key/res_value the bf16 rings
 *                     [rows, capacity, num_kv_heads, head_size]
 *   workspace         qkv_kivi_paged_decode_workspace bytes for this batch
 * A key window that must flush but is not whole aligned groups returns
 * QKV_ERR_INVALID with the reference's message. */
QKV_API void* qkv_kivi_step_create(void);
QKV_API void qkv_kivi_step_destroy(void* step);
QKV_API int qkv_kivi_decode_step(
    void* step, void* window, int batch, const int64_t* rows,
    const int64_t* slots, const int32_t* seq_lens,
    const int32_t* block_table_host, int table_cols,
    const int32_t* block_table, int64_t bt_stride, const void* query,
    int64_t q_stride, const void* new_key, const void* new_value,
    int32_t* k_quant, float* k_scale, float* k_mn, int32_t* v_quant,
    float* v_scale, float* v_mn, void* res_key, void* res_value,
    int num_heads, int num_kv_heads, int head_size, int group_size,
    int block_size, int64_t num_blocks, float scale, void* workspace,
    size_t workspace_bytes, void* out, int64_t out_stride,
    qkv_stream_t stream);

/* ------------------------------------------------------------------------
 * NVLink peer all-gather of the KV-head-sharded outputs
 *
 * With the KV heads sharded over N GPUs (rank i owns KV heads
 * [KVH i/N, KVH (i+1)/N) and the query heads reading them; the per-head cache
 * layout is the reference's with num_kv_heads = KVH/N, as its host-TP test
 * builds it, tests/test_kivi_int4.py:1484-1494), the outputs [B, Hq/N, D]
 * are reassembled into [B, Hq, D] on every rank by one kernel per call: each
 * 4-byte word of this rank's slice goes to every peer's receive buffer
 * (peer memory opened through CUDA IPC) as one 64-bit scalar store that
 * carries the call's epoch in its high half, and the receivers poll those
 * words. No barrier; the epoch is kept on the device, so the call can be
 * captured in a CUDA graph. Waits give up after about a second (device
 * error 7). Every rank makes the same calls in the same order, and the
 * call's CTAs (at most 128) must be able to run at once (no other kernel
 * filling the GPU). Calls on one rank that use the same buffer set must be
 * ordered on one stream (or by events): each call reads its epoch from the
 * buffer's control word, which the previous call's last CTA advances, so two
 * calls that overlap on the GPU (two streams, two graphs replaying at once)
 * would take the same epoch and corrupt each other's receive words.
 *
 * qkv_peer_alloc     one rank's receive buffer for slices of up to
 *                    slice_bytes_max bytes (a multiple of 16) from `world`
 *                    ranks, zeroed; qkv_peer_buffer_bytes gives its size
 * qkv_ipc_handle     the 64-byte CUDA IPC handle of such a buffer, to send to
 *                    the other ranks; qkv_ipc_open maps a peer's, _close
 *                    unmaps it
 * qkv_peer_allgather local [batch, row_bytes] (this rank's heads of each
 *                    request), buffers[r] = rank r's buffer as mapped here
 *                    (this rank's own at [rank]), out [batch, world *
 *                    row_bytes] on this rank: rank r's row b lands at byte
 *                    (b * world + r) * row_bytes.
 * ---------------------------------------------------------------------- */
#define QKV_IPC_HANDLE_BYTES 64
QKV_API size_t qkv_peer_buffer_bytes(int64_t slice_bytes_max, int world);
QKV_API int qkv_peer_alloc(int64_t slice_bytes_max, int world, void** ptr);
QKV_API int qkv_peer_free(void* ptr);
QKV_API int qkv_ipc_handle(const void* ptr, void* handle_out);
QKV_API int qkv_ipc_open(const void* handle, void** ptr);
QKV_API int qkv_ipc_close(void* ptr);
QKV_API int qkv_peer_allgather(const void* local, int64_t batch,
                               int64_t row_bytes, void* const* buffers,
                               int64_t slice_bytes_max, void* out, int rank,
                               int world, qkv_stream_t stream);
/* qkv_peer_allgather fused with the split combine of a decode: with
 * splits > 1, one warp per (request, local head) row merges the splits left
 * by qkv_kivi_paged_decode_partials (partial_acc [batch, local_heads, splits,
 * head_size] fp32, partial_ml [batch, local_heads, splits, 2]) exactly as the
 * decode's own combine does, and the bf16 results go out as in
 * qkv_peer_allgather; with splits <= 1 `local` (the decode's output) is
 * gathered as is. */
QKV_API int qkv_peer_combine_allgather(const float* partial_acc,
                                       const float* partial_ml, int splits,
                                       int64_t batch, int local_heads,
                                       int head_size, const void* local,
                                       void* const* buffers,
                                       int64_t slice_bytes_max, void* out,
                                       int rank, int world,
                                       qkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QKV_SM100_H */

/*
 * vasr_pa.h — C ABI of the B200 (sm_100a) paged KV-cache kernels.
 *
 * These entry points are what the Rust crate `vasr-paged-attn` binds through
 * `extern "C"` in place of the third-party crate `mistralrs-paged-attn` 0.8.3
 * (pinned at vasr-paged-attn/Cargo.toml:46, Cargo.lock:2601-2609), so that the
 * decoder call sites in vasr-models/src/model/thinker_text.rs stay unchanged.
 *
 * Conventions shared by every entry point
 * ---------------------------------------
 *  - Plain pointers and sizes only. Every tensor pointer is a device address
 *    (or, for swap, a device-accessible pinned host address) that the caller
 *    owns. No entry point allocates, frees or synchronises; all work is
 *    enqueued on `stream` (NULL = legacy default stream). Every call except
 *    vasr_pa_paged_attention_noalloc (see its own notes) is safe inside CUDA
 *    stream capture.
 *  - Cache layout is the vLLM layout the reference allocates in
 *    vasr-paged-attn/src/paged_kv_cache.rs:285-294:
 *        key_cache   [num_blocks, num_kv_heads, head_dim / x, block_size, x]
 *        value_cache [num_blocks, num_kv_heads, head_dim, block_size]
 *    with x = 16 / sizeof(element). Both are contiguous.
 *  - Return value: VASR_PA_OK (0) or a negative vasr_pa_status. Shape,
 *    dtype and pointer checks run on the host before anything is launched;
 *    a rejected call leaves device memory untouched. Kernels never trap.
 *    Out-of-range slot or block ids met on the device are skipped and
 *    recorded in the device error word (vasr_pa_get_device_error).
 */
#ifndef VASR_PA_H
#define VASR_PA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t, declared without the CUDA headers. */
typedef struct CUstream_st *vasr_pa_stream_t;

#define VASR_PA_ABI_VERSION 1

/* Element types of q, k, v and the caches (candle DType names).
 * VASR_PA_FP8_E4M3 is a cache storage type only (the _fp8 entry points). */
typedef enum vasr_pa_dtype {
  VASR_PA_F32 = 0,
  VASR_PA_BF16 = 1,
  VASR_PA_F16 = 2,
  VASR_PA_FP8_E4M3 = 3
} vasr_pa_dtype;

typedef enum vasr_pa_status {
  VASR_PA_OK = 0,
  VASR_PA_EINVAL_SHAPE = -1,     /* a size is zero/negative/inconsistent   */
  VASR_PA_EINVAL_DTYPE = -2,     /* dtype not in vasr_pa_dtype             */
  VASR_PA_EINVAL_BLOCKSIZE = -3, /* block_size not in {8, 16, 32}          */
  VASR_PA_EINVAL_ALIGN = -4,     /* pointer/stride not 16-byte aligned     */
  VASR_PA_EINVAL_WORKSPACE = -5, /* workspace missing or too small         */
  VASR_PA_ENOT_SUPPORTED = -6,   /* head_dim / GQA group not instantiated  */
  VASR_PA_ELAUNCH = -7,          /* cudaLaunchKernel reported an error     */
  VASR_PA_EDEVICE = -8,          /* no usable sm_100 device current        */
  VASR_PA_EINVAL_POINTER = -9,   /* NULL or host-only pointer              */
  VASR_PA_ESCRATCH_LIMIT = -10   /* sizes exceed the fixed no-alloc scratch */
} vasr_pa_status;

/* Device error word bits (set by kernels, read with vasr_pa_get_device_error). */
#define VASR_PA_DERR_SLOT_RANGE 0x1    /* slot >= num_blocks * block_size     */
#define VASR_PA_DERR_BLOCK_RANGE 0x2   /* block id >= num_blocks              */
#define VASR_PA_DERR_CTX_RANGE 0x4     /* context_len > max_context_len bound */
#define VASR_PA_DERR_WAIT_TIMEOUT 0x8  /* a bounded mbarrier wait gave up     */
#define VASR_PA_DERR_MAPPING_RANGE 0x10 /* copy/swap pair out of range        */
#define VASR_PA_DERR_QLEN_RANGE 0x20   /* prefill q_len > max_query_len       */

int32_t vasr_pa_abi_version(void);
const char *vasr_pa_status_string(int32_t status);

/*
 * KV append. Replaces mistralrs_paged_attn::reshape_and_cache, called at
 * vasr-models/src/model/thinker_text.rs:1101-1109 (decode and padded prefill)
 * and :1324-1332 (packed prefill).
 *
 * For every t in [0, num_tokens) with slot = slot_mapping[t] >= 0:
 *   key_cache[slot / bs, h, d / x, slot % bs, d % x] = key[t, h, d]
 *   value_cache[slot / bs, h, d, slot % bs]          = value[t, h, d]
 * Negative slots (PAD_SLOT_ID = -1, paged_kv_cache.rs:7) are skipped.
 * key/value are [num_tokens, num_kv_heads, head_dim] with unit dim stride,
 * head stride head_dim and the given token strides (in elements).
 * k_scale / v_scale are the fp8 scales of the reference signature; with a
 * cache dtype equal to the input dtype they are unused and may be NULL.
 */
int32_t vasr_pa_reshape_and_cache(const void *key, const void *value,
                                  void *key_cache, void *value_cache,
                                  const int64_t *slot_mapping,
                                  int64_t num_tokens, int32_t num_kv_heads,
                                  int32_t head_dim, int32_t block_size,
                                  int64_t num_blocks, int64_t key_token_stride,
                                  int64_t value_token_stride, int32_t dtype,
                                  const float *k_scale, const float *v_scale,
                                  vasr_pa_stream_t stream);

/*
 * Bytes of scratch that vasr_pa_paged_attention needs for these sizes
 * (split-K partials + per-(sequence, kv head) arrival counters + error word).
 * The workspace must be zero-filled once after allocation; every call leaves
 * the counters at zero again, so it can be reused by later calls of any shape
 * and by CUDA graph replays without re-clearing. One workspace serves one
 * stream at a time (concurrent calls sharing it race). Supports
 * num_seqs * num_kv_heads <= 65536.
 */
size_t vasr_pa_paged_attention_workspace_size(int32_t num_seqs,
                                              int32_t num_heads,
                                              int32_t num_kv_heads,
                                              int32_t head_dim,
                                              int32_t block_size,
                                              int32_t max_context_len,
                                              int32_t dtype);

/*
 * Single-query paged decode attention. Replaces
 * mistralrs_paged_attn::paged_attention, called at thinker_text.rs:1126-1139
 * with softmax_scale = head_dim^-0.5 (thinker_text.rs:598), softcapping = 1.0,
 * alibi = None, sinks = None.
 *
 * out[b, h, :] = softmax(scale * q[b, h, :] . K_b^T) . V_b, where K_b / V_b
 * are the first context_lens[b] tokens of sequence b, token j read from
 * block block_tables[b * max_num_blocks_per_seq + j / bs] at offset j % bs,
 * and kv head h / (num_heads / num_kv_heads). softcapping != 1.0 applies
 * s = softcapping * tanh(s / softcapping) after scaling.
 * max_context_len is only an upper bound on context_lens[] (CUDA-graph
 * bucket, vasr-paged-attn/src/cuda_graph.rs:141); the grid is sized from it
 * and the true lengths are read on the device. Rows with context_len 0 get
 * zeros. q/out are [num_seqs, num_heads, head_dim], sequence stride
 * q_seq_stride (elements; out is contiguous).
 */
int32_t vasr_pa_paged_attention(void *out, const void *query,
                                const void *key_cache, const void *value_cache,
                                const uint32_t *block_tables,
                                const uint32_t *context_lens, int32_t num_seqs,
                                int32_t num_heads, int32_t num_kv_heads,
                                int32_t head_dim, int32_t block_size,
                                int64_t num_blocks,
                                int32_t max_num_blocks_per_seq,
                                int32_t max_context_len, float scale,
                                float softcapping, int64_t q_seq_stride,
                                int32_t dtype, void *workspace,
                                size_t workspace_bytes,
                                vasr_pa_stream_t stream);

/*
 * vasr_pa_paged_attention issued right behind this step's KV append on the
 * same stream (vasr_pa_fused_qk_norm_rope_append or vasr_pa_reshape_and_cache,
 * the pair at thinker_text.rs:1101-1139), as a programmatic dependent launch:
 * its CTAs start while the append still runs and stream every page before
 * each sequence's last one, then wait for the append to complete before
 * reading q, the last page or writing anything. Same arguments, results
 * and errors as vasr_pa_paged_attention. Contract: the kernel immediately
 * before it on the stream writes nothing this call reads except q and
 * tokens in each sequence's last page (as a decode append does), and was
 * itself launched in ordinary stream order. Other dtypes and GQA groups than
 * the 16-bit GQA-2 kernel launch as vasr_pa_paged_attention does.
 */
int32_t vasr_pa_paged_attention_after_append(void *out, const void *query,
                                             const void *key_cache, const void *value_cache,
                                             const uint32_t *block_tables,
                                             const uint32_t *context_lens, int32_t num_seqs,
                                             int32_t num_heads, int32_t num_kv_heads,
                                             int32_t head_dim, int32_t block_size,
                                             int64_t num_blocks,
                                             int32_t max_num_blocks_per_seq,
                                             int32_t max_context_len, float scale,
                                             float softcapping, int64_t q_seq_stride,
                                             int32_t dtype, void *workspace,
                                             size_t workspace_bytes,
                                             vasr_pa_stream_t stream);

/*
 * Decode attention for callers that cannot allocate device memory.
 * No counterpart in the reference: it is an addition of this library.
 *
 * Same arguments and results as vasr_pa_paged_attention minus the workspace.
 * The split-K scratch is a fixed buffer inside the library (a file-scope
 * device array of vasr_pa_noalloc_scratch_bytes() = 16 MiB that every GPU
 * loading the library keeps until exit), so a caller whose device memory is
 * owned by someone else — a plugin enqueue path that must not allocate, a
 * fixed-budget host framework, a real-time thread that must not block in the
 * allocator — passes only inputs and outputs. Sizes whose workspace
 * (vasr_pa_paged_attention_workspace_size) exceeds the buffer return
 * VASR_PA_ESCRATCH_LIMIT. The first call on a device looks up the buffer's
 * device address; make that first call before any stream capture. All calls
 * on a device share the buffer: calls that overlap on the GPU race.
 */
int32_t vasr_pa_paged_attention_noalloc(void *out, const void *query,
                                        const void *key_cache,
                                        const void *value_cache,
                                        const uint32_t *block_tables,
                                        const uint32_t *context_lens,
                                        int32_t num_seqs, int32_t num_heads,
                                        int32_t num_kv_heads, int32_t head_dim,
                                        int32_t block_size, int64_t num_blocks,
                                        int32_t max_num_blocks_per_seq,
                                        int32_t max_context_len, float scale,
                                        float softcapping, int64_t q_seq_stride,
                                        int32_t dtype, vasr_pa_stream_t stream);

/* Size in bytes of the fixed scratch used by vasr_pa_paged_attention_noalloc. */
size_t vasr_pa_noalloc_scratch_bytes(void);

/*
 * Gather the first kv_len tokens of each sequence out of the pages into
 * packed [total_tokens, num_kv_heads, head_dim] K and V. Replaces
 * mistralrs_paged_attn::gather_kv_cache, called at thinker_text.rs:190-198
 * and :1344-1352. Sequence b owns packed rows
 * [cu_seqlens_kv[b], cu_seqlens_kv[b + 1]); total_tokens must equal
 * cu_seqlens_kv[num_seqs] (the caller reads it when sizing the outputs).
 */
int32_t vasr_pa_gather_kv_cache(void *key_out, void *value_out,
                                const void *key_cache, const void *value_cache,
                                const uint32_t *block_tables,
                                const uint32_t *cu_seqlens_kv, int32_t num_seqs,
                                int32_t max_num_blocks_per_seq,
                                int64_t total_tokens, int32_t num_kv_heads,
                                int32_t head_dim, int32_t block_size,
                                int64_t num_blocks, int32_t dtype,
                                vasr_pa_stream_t stream);

/*
 * Causal varlen (chunked) prefill attention that reads K/V straight from the
 * pages. Same argument meaning as the reference's
 * paged_attention_varlen_prefill (vasr-paged-attn/src/metal/varlen_prefill.rs:291-427):
 * query/out are packed [total_q_tokens, num_heads, head_dim]; sequence b owns
 * query rows [cu_seqlens_q[b], cu_seqlens_q[b + 1]) and has context_lens[b]
 * tokens in the cache (its new tokens already appended). Query row i of
 * sequence b sits at absolute position context_lens[b] - q_len_b + i and sees
 * key j iff j <= that position: the cached causal mask of
 * vasr-models/src/model/attention.rs:86-149 with cache_len = context - q_len.
 * This replaces gather_kv_cache + flash_attn_varlen
 * (thinker_text.rs:1344-1365, attention.rs:580-657) in one kernel.
 * max_query_len bounds every q_len (flash_attn_varlen's max_seqlen_q); the
 * kernel schedules num_seqs x ceil(max_query_len / rows per CTA) work items
 * per kv head, so a sequence longer than it is cut short and sets
 * VASR_PA_DERR_QLEN_RANGE. 0 means "unknown" and schedules for the worst case
 * (total_q_tokens). When the items are few next to the SM count (a long
 * context with few new tokens), each item's key range is shared by a
 * thread-block cluster of up to 8 CTAs (bf16 / f16 pages of 16 tokens,
 * head_dim 128); the results are the same computation up to float rounding.
 */
int32_t vasr_pa_paged_attention_varlen_prefill(
    void *out, const void *query, const void *key_cache,
    const void *value_cache, const uint32_t *block_tables,
    const uint32_t *context_lens, const uint32_t *cu_seqlens_q,
    int32_t num_seqs, int64_t total_q_tokens, int32_t max_query_len,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t block_size, int64_t num_blocks, int32_t max_num_blocks_per_seq,
    float scale, float softcapping, int64_t q_token_stride, int32_t dtype,
    vasr_pa_stream_t stream);

/*
 * Copy whole blocks inside each layer's K and V caches (scheduler fork and
 * compaction). vLLM-style copy_blocks; the reference has no counterpart call
 * site but frees/trims blocks at vasr-paged-attn/src/paged_cache_runtime.rs:320-357.
 * key_caches / value_caches are HOST arrays of num_layers device pointers
 * (num_layers <= 128); block_mapping is a device array of num_pairs
 * (src, dst) int64 pairs; block_bytes is the size of one block of one
 * layer's K cache (= of its V cache). Pairs are applied concurrently: a
 * block that is both a source and a destination gives an unspecified result.
 */
int32_t vasr_pa_copy_blocks(void *const *key_caches, void *const *value_caches,
                            int32_t num_layers, const int64_t *block_mapping,
                            int64_t num_pairs, int64_t num_blocks,
                            int64_t block_bytes, vasr_pa_stream_t stream);

/*
 * Swap blocks between two caches of the same geometry, typically device and
 * pinned host memory (eviction / restore). dst[pair.dst] = src[pair.src] for
 * every (src, dst) int64 pair of block_mapping. src, dst and block_mapping
 * must be device-accessible: device memory or page-locked host memory
 * (cudaHostAlloc / cudaHostRegister / torch pin_memory); the copy is done by
 * a kernel that reads and writes through the unified address space, so it
 * needs no per-block cudaMemcpyAsync. src_num_blocks / dst_num_blocks bound
 * the ids.
 */
int32_t vasr_pa_swap_blocks(void *dst, const void *src,
                            const int64_t *block_mapping, int64_t num_pairs,
                            int64_t src_num_blocks, int64_t dst_num_blocks,
                            int64_t block_bytes, vasr_pa_stream_t stream);

/*
 * Fused pre-attention step of one decoder layer: per-head q/k RMSNorm, rotary
 * embedding of q and k, and the KV append. Replaces the chain at
 * vasr-models/src/model/thinker_text.rs:1041-1109 (q_norm, k_norm,
 * apply_multimodal_rotary_pos_emb — 1-D RoPE when the three mRoPE position
 * streams are equal, as for text and audio tokens — then reshape_and_cache).
 * qkv is the fused projection output [num_tokens, (Hq + 2 Hkv) * D] with
 * token stride qkv_token_stride (elements): q heads, then k heads, then v
 * heads. Writes q_out [num_tokens, Hq, D] (normed + rotated) and appends the
 * normed + rotated k and the raw v at slot_mapping[t] (negative = skip).
 * cos_table / sin_table are f32 [max_position, D / 2]; positions i64 [T].
 * RMSNorm: x * rsqrt(mean(x^2) + eps) * w in f32, rounded to the element
 * type; RoPE in f32 on the rounded values, rounded again. bf16/f16, D = 128.
 */
int32_t vasr_pa_fused_qk_norm_rope_append(
    void *q_out, const void *qkv, int64_t qkv_token_stride,
    const void *q_norm_weight, const void *k_norm_weight, float eps,
    const float *cos_table, const float *sin_table, int64_t max_position,
    const int64_t *positions, void *key_cache, void *value_cache,
    const int64_t *slot_mapping, int64_t num_tokens, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t num_blocks, int32_t dtype, vasr_pa_stream_t stream);

/*
 * fp8 (E4M3) KV cache with per-tensor scales — the k_scale / v_scale
 * arguments that reshape_and_cache and paged_attention carry in the
 * reference API (thinker_text.rs:23-28, 586-590; the Metal fp8 path,
 * metal/varlen_prefill.rs:276-288). Pages keep the same layout with one
 * byte per element: K [nb, Hkv, D/16, bs, 16], V [nb, Hkv, D, bs].
 *
 * reshape_and_cache_fp8: key/value of element type src_dtype (f32, bf16,
 * f16) are stored as fp8(value / scale), rounded to nearest even and
 * saturated to +-448 (NaN stays NaN); k_scale / v_scale are device f32
 * scalars (required). Otherwise as vasr_pa_reshape_and_cache.
 */
int32_t vasr_pa_reshape_and_cache_fp8(
    const void *key, const void *value, void *key_cache, void *value_cache,
    const int64_t *slot_mapping, int64_t num_tokens, int32_t num_kv_heads,
    int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int64_t key_token_stride, int64_t value_token_stride, int32_t src_dtype,
    const float *k_scale, const float *v_scale, vasr_pa_stream_t stream);

/*
 * gather_kv_cache_fp8: vasr_pa_gather_kv_cache over fp8 pages, the form the
 * call site at thinker_text.rs:190-198 / :1344-1352 takes with k_scale /
 * v_scale and the model dtype as out_dtype: packed rows of out_dtype (f32,
 * bf16, f16) holding float(stored byte) * scale, rounded to nearest even.
 */
int32_t vasr_pa_gather_kv_cache_fp8(void *key_out, void *value_out,
                                    const void *key_cache, const void *value_cache,
                                    const uint32_t *block_tables,
                                    const uint32_t *cu_seqlens_kv, int32_t num_seqs,
                                    int32_t max_num_blocks_per_seq,
                                    int64_t total_tokens, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t block_size,
                                    int64_t num_blocks, int32_t out_dtype,
                                    const float *k_scale, const float *v_scale,
                                    vasr_pa_stream_t stream);

/*
 * paged_attention_varlen_prefill_fp8: the varlen prefill over fp8 pages for
 * bf16 / f16 queries (dtype). 16-token pages with num_heads / num_kv_heads
 * in {1, 2, 4}: the tcgen05 kernel reads the fp8 pages itself, converting
 * each byte exactly to f16 on its way into shared memory (the products run
 * in f16 with f32 accumulation; k_scale scales the scores, v_scale the
 * output), and the workspace is not touched. Other page sizes: the pages of
 * each sequence's context are first written to a 16-bit scratch pool in the
 * workspace (byte * scale in dtype, the 16-bit page layouts), then the
 * prefill runs on that pool — the same numbers as gather_kv_cache_fp8
 * followed by attention, without the packed copy. workspace_size: bytes for
 * num_seqs x max_num_blocks_per_seq pages of every kv head (K and V) plus a
 * block table; required in every case. The workspace is scratch (its
 * contents are overwritten): not the paged_attention workspace, whose
 * counters must stay zero. head_dim 128.
 */
int32_t vasr_pa_paged_attention_varlen_prefill_fp8(
    void *out, const void *query, const void *key_cache,
    const void *value_cache, const uint32_t *block_tables,
    const uint32_t *context_lens, const uint32_t *cu_seqlens_q,
    int32_t num_seqs, int64_t total_q_tokens, int32_t max_query_len,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t block_size, int64_t num_blocks, int32_t max_num_blocks_per_seq,
    float scale, float softcapping, int64_t q_token_stride, int32_t dtype,
    const float *k_scale, const float *v_scale, void *workspace,
    size_t workspace_bytes, vasr_pa_stream_t stream);
size_t vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size(
    int32_t num_seqs, int32_t num_kv_heads, int32_t head_dim,
    int32_t block_size, int32_t max_num_blocks_per_seq);

/*
 * paged_attention_fp8: decode attention of bf16 / f16 queries (dtype) over
 * fp8 pages; scores use K = stored * k_scale and the output V = stored *
 * v_scale. GQA group 2, head_dim 128 (the Qwen3-ASR shape); other shapes
 * return VASR_PA_ENOT_SUPPORTED. Workspace as vasr_pa_paged_attention.
 */
int32_t vasr_pa_paged_attention_fp8(
    void *out, const void *query, const void *key_cache,
    const void *value_cache, const uint32_t *block_tables,
    const uint32_t *context_lens, int32_t num_seqs, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t num_blocks, int32_t max_num_blocks_per_seq,
    int32_t max_context_len, float scale, float softcapping,
    int64_t q_seq_stride, int32_t dtype, const float *k_scale,
    const float *v_scale, void *workspace, size_t workspace_bytes,
    vasr_pa_stream_t stream);

/*
 * Device-side decode step bookkeeping (no counterpart call in the reference,
 * which does this on the host every step; it replaces the host work of
 * paged_batch_decode_step, vasr-models/src/model/paged_batch_engine.rs:634-712,
 * with decode_metadata_for_batch_step, vasr-paged-attn/src/paged_kv_cache.rs:
 * 924-1059, so a captured decode step replays without a host round trip).
 * For each row b, with step = *step (a device u32):
 *   - a row not yet finished takes tok = next_ids[b]; tok in eos_ids marks it
 *     finished (finished[b] = 1); otherwise tok is recorded
 *     (history[b * history_cols + generated[b]] when there is room, then
 *     generated[b] += 1; generated/history may be NULL) and the row gets
 *     input_ids = tok, positions = prompt_lens[b] + step, slot_mapping =
 *     block_tables[b][pos / block_size] * block_size + pos % block_size and
 *     context_lens = pos + 1 (slot_for_block_table_position,
 *     paged_kv_cache.rs:74-103);
 *   - a finished row becomes a padding row of pad_decode_batch_to_max
 *     (cuda_graph.rs:373-486): input 0, position 0, slot 0, context 1.
 * block_table_lens[b] (may be NULL = all columns valid) is the number of
 * valid table entries; a position past it gets slot -1 and sets
 * VASR_PA_DERR_SLOT_RANGE (the host must allocate blocks ahead of the steps
 * it replays without syncing). Capture-safe.
 */
int32_t vasr_pa_decode_step_prepare(
    const uint32_t *next_ids, const uint32_t *eos_ids, int32_t num_eos,
    const uint32_t *prompt_lens, const uint32_t *step,
    const uint32_t *block_tables, const uint32_t *block_table_lens,
    int32_t max_num_blocks_per_seq, int32_t block_size, int64_t num_blocks,
    int32_t num_seqs, uint8_t *finished, uint32_t *generated,
    uint32_t *history, int32_t history_cols, int64_t *input_ids,
    int64_t *positions, int64_t *slot_mapping, uint32_t *context_lens,
    vasr_pa_stream_t stream);

/*
 * Greedy next tokens on the device: next_ids[b] = argmax over v < vocab of
 * logits[b * row_stride + v] (argmax_token_ids_from_logits,
 * vasr-models/src/model/generation.rs:443-460; the lowest index among equal
 * maxima, NaN never wins, a row without a value above -inf gives 0). Rows
 * with finished[b] != 0 are skipped (finished may be NULL). If step is not
 * NULL, *step is incremented once (the decode step counter read by
 * vasr_pa_decode_step_prepare). workspace: at least
 * vasr_pa_greedy_argmax_workspace_size(num_seqs, vocab) bytes, zeroed once
 * before first use and left zeroed by every call; one call at a time per
 * workspace. dtype f32/bf16/f16. Capture-safe.
 */
size_t vasr_pa_greedy_argmax_workspace_size(int32_t num_seqs, int64_t vocab);
int32_t vasr_pa_greedy_argmax(uint32_t *next_ids, const void *logits,
                              int32_t num_seqs, int64_t vocab,
                              int64_t row_stride, int32_t dtype,
                              const uint8_t *finished, uint32_t *step,
                              void *workspace, size_t workspace_bytes,
                              vasr_pa_stream_t stream);

/*
 * Read (and optionally clear) the device error word of the current device.
 * Synchronises `stream` because it copies the word to the host; call it
 * outside stream capture.
 */
int32_t vasr_pa_get_device_error(int32_t *out_bits, int32_t clear,
                                 vasr_pa_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VASR_PA_H */

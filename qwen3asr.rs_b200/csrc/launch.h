// launch.h — internal interface between the C ABI (capi.cu) and the kernel
// translation units. Argument structs carry already-validated values.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/vasr_pa.h"

namespace vasr {

struct AppendArgs {
  const void *key;
  const void *value;
  void *key_cache;
  void *value_cache;
  const int64_t *slot_mapping;
  int64_t num_tokens;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int64_t num_blocks;
  int64_t key_token_stride;
  int64_t value_token_stride;
  int dtype;                       // element type of key / value
  int cache_dtype = -1;            // -1: same as dtype; VASR_PA_FP8_E4M3: scaled fp8 pages
  const float *k_scale = nullptr;  // fp8: device scalars, cache = value / scale
  const float *v_scale = nullptr;
};

struct DecodeArgs {
  void *out;
  const void *query;
  const void *key_cache;
  const void *value_cache;
  const uint32_t *block_tables;
  const uint32_t *context_lens;
  int num_seqs;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int64_t num_blocks;
  int max_num_blocks_per_seq;
  int max_context_len;
  float scale;
  float softcapping;
  int64_t q_seq_stride;
  int dtype;                       // element type of query / out
  void *workspace;
  size_t workspace_bytes;
  int cache_dtype = -1;            // -1: same as dtype; VASR_PA_FP8_E4M3: scaled fp8 pages
  const float *k_scale = nullptr;  // fp8: device scalars, real K = stored K * k_scale
  const float *v_scale = nullptr;
  // Launch as a programmatic dependent of the preceding kernel on the stream
  // (the KV append of this step); honoured by the GQA-2 tensor-core kernel.
  int overlap_append = 0;
};

struct GatherArgs {
  void *key_out;
  void *value_out;
  const void *key_cache;
  const void *value_cache;
  const uint32_t *block_tables;
  const uint32_t *cu_seqlens_kv;
  int num_seqs;
  int max_num_blocks_per_seq;
  int64_t total_tokens;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int64_t num_blocks;
  int dtype;  // element type of the outputs (and of the cache unless cache_dtype is set)
  int cache_dtype = -1;  // VASR_PA_FP8_E4M3: one-byte pages, outputs = byte * scale
  const float *k_scale = nullptr;
  const float *v_scale = nullptr;
};

struct PrefillArgs {
  void *out;
  const void *query;
  const void *key_cache;
  const void *value_cache;
  const uint32_t *block_tables;
  const uint32_t *context_lens;
  const uint32_t *cu_seqlens_q;
  int num_seqs;
  int64_t total_q_tokens;
  int max_query_len;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int64_t num_blocks;
  int max_num_blocks_per_seq;
  float scale;
  float softcapping;
  int64_t q_token_stride;
  int dtype;                       // element type of query / out (and of the pages by default)
  int cache_dtype = -1;            // VASR_PA_FP8_E4M3: one-byte pages, real K = byte * k_scale
  const float *k_scale = nullptr;  // device scalars (fp8 pages)
  const float *v_scale = nullptr;
};

struct FusedRopeArgs {
  void *q_out;
  const void *qkv;
  int64_t qkv_token_stride;
  const void *q_norm_weight;
  const void *k_norm_weight;
  float eps;
  const float *cos_table;
  const float *sin_table;
  int64_t max_position;
  const int64_t *positions;
  void *key_cache;
  void *value_cache;
  const int64_t *slot_mapping;
  int64_t num_tokens;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int64_t num_blocks;
  int dtype;
};
int launch_fused_rope(const FusedRopeArgs &a, cudaStream_t s);

struct DecodeStepArgs {
  const uint32_t *next_ids;
  const uint32_t *eos_ids;
  int num_eos;
  const uint32_t *prompt_lens;
  const uint32_t *step;
  const uint32_t *block_tables;
  const uint32_t *block_table_lens;  // may be null: every column valid
  int max_num_blocks_per_seq;
  int block_size;
  int64_t num_blocks;
  int num_seqs;
  uint8_t *finished;
  uint32_t *generated;  // may be null
  uint32_t *history;    // may be null
  int history_cols;
  int64_t *input_ids;
  int64_t *positions;
  int64_t *slot_mapping;
  uint32_t *context_lens;
};
int launch_decode_step_prepare(const DecodeStepArgs &a, cudaStream_t s);

struct ArgmaxArgs {
  uint32_t *next_ids;
  const void *logits;
  int num_seqs;
  int64_t vocab;
  int64_t row_stride;
  int dtype;
  const uint8_t *finished;  // may be null
  uint32_t *step;           // may be null: incremented once per call
  // filled by launch_greedy_argmax
  int num_chunks;
  int64_t chunk_elems;
  uint32_t *counters;
  void *partials;
};
void argmax_chunking(int64_t vocab, int *num_chunks, int64_t *chunk_elems);
size_t argmax_workspace_bytes(int num_seqs, int64_t vocab);
int launch_greedy_argmax(ArgmaxArgs a, void *workspace, cudaStream_t s);
int read_error_decode_loop(uint32_t *bits, bool clear, cudaStream_t s);
int read_error_fused(uint32_t *bits, bool clear, cudaStream_t s);

// Workspace layout of the decode kernel (all offsets 256-byte aligned):
// [counters: kDecodeMaxCounters x u32][partial o][partial (m, l)].
constexpr size_t kDecodeMaxCounters = 65536;  // num_seqs * num_kv_heads limit
struct DecodeWorkspace {
  int pages_per_split;
  int max_splits;
  size_t off_o, off_ml, off_counters, total;
};
DecodeWorkspace decode_workspace_layout(int num_seqs, int num_heads, int num_kv_heads,
                                        int head_dim, int block_size, int max_context_len);

int launch_append(const AppendArgs &a, cudaStream_t s);
int launch_decode(const DecodeArgs &a, cudaStream_t s);
int launch_gather(const GatherArgs &a, cudaStream_t s);

// fp8 pages of the block tables' live entries -> a 16-bit scratch pool
// (block b * cols + i) and the remapped table; dtype = the pool's type.
struct DequantArgs {
  const void *key_cache;
  const void *value_cache;
  const uint32_t *block_tables;
  const uint32_t *context_lens;
  int num_seqs;
  int cols;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int64_t num_blocks;
  int dtype;
  const float *k_scale;
  const float *v_scale;
  void *key_out;
  void *value_out;
  uint32_t *table_out;
};
int launch_dequant_pages(const DequantArgs &a, cudaStream_t s);
int launch_prefill(const PrefillArgs &a, cudaStream_t s);
// Position tiles per sequence for CTAs of `positions` query positions:
// ceil(max_query_len / positions); max_query_len 0 (unknown) counts as
// total_q_tokens, the largest length a single sequence can have.
inline int64_t prefill_tiles_per_seq(const PrefillArgs &a, int positions) {
  const int64_t mq = a.max_query_len > 0 ? a.max_query_len : a.total_q_tokens;
  return (mq + positions - 1) / positions;
}
// tcgen05 kernel (bf16/f16 queries, 16-token bf16/f16 or fp8 pages, head_dim
// 128, G in {1,2,4}); VASR_PA_ENOT_SUPPORTED for any other shape.
int launch_prefill_umma(const PrefillArgs &a, cudaStream_t s);
int launch_copy_blocks(void *const *k, void *const *v, int layers, const int64_t *mapping,
                       int64_t pairs, int64_t num_blocks, int64_t block_bytes, cudaStream_t s);
int launch_swap_blocks(void *dst, const void *src, const int64_t *mapping, int64_t pairs,
                       int64_t src_blocks, int64_t dst_blocks, int64_t block_bytes,
                       cudaStream_t s);

int read_error_kv_ops(uint32_t *bits, bool clear, cudaStream_t s);
int read_error_decode(uint32_t *bits, bool clear, cudaStream_t s);
int read_error_prefill(uint32_t *bits, bool clear, cudaStream_t s);
int read_error_prefill_umma(uint32_t *bits, bool clear, cudaStream_t s);

// Raise a kernel's dynamic shared-memory limit once per device. The
// attribute is not a stream operation, so this is legal during capture.
template <typename F>
inline bool ensure_smem_attr(F *func, int bytes, std::atomic<uint64_t> &done_mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return true;
  if (cudaFuncSetAttribute(reinterpret_cast<const void *>(func),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

// CTAs of `func` (block `threads`, dynamic shared memory `smem`) resident on
// the whole current device at once: SM count x blocks per SM, queried once
// per device (cache[dev] = 0 until then). 0 on error.
template <typename F>
inline int64_t resident_ctas(F *func, int threads, size_t smem, std::atomic<int64_t> (&cache)[64]) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int64_t v = cache[dev].load(std::memory_order_acquire);
  if (v > 0) return v;
  int sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void *>(func), threads,
                                                    smem) != cudaSuccess)
    return 0;
  v = (int64_t)sms * per_sm;
  cache[dev].store(v, std::memory_order_release);
  return v;
}

}  // namespace vasr

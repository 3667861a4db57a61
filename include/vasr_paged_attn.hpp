// vasr_paged_attn.hpp — C++ host mirror of the Rust crate `vasr-paged-attn`.
//
// Same type names, fields, methods and error behaviour as the crate's public
// API (re-exports at vasr-paged-attn/src/lib.rs:12-27), written in C++
// because this build has no Rust toolchain. Sizes are size_t where Rust has
// usize; tensors that Rust keeps as candle `Tensor`s on a Device are host
// vectors here (the metadata builders) or non-owning DeviceTensor views
// (the cache pages). Every `candle_core::bail!` of the reference becomes a
// thrown vasr_paged_attn::Error with the same message.
//
// Kernel entry points (namespace mistralrs_paged_attn) call the C ABI of
// vasr_pa.h; they are what thinker_text.rs calls through
// `vasr_paged_attn::mistralrs_paged_attn`.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <optional>
#include <set>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>
#include <deque>

#include "vasr_pa.h"

namespace vasr_paged_attn {

struct Error : std::runtime_error {
  explicit Error(const std::string &m) : std::runtime_error(m) {}
};

enum class DType { F32 = VASR_PA_F32, BF16 = VASR_PA_BF16, F16 = VASR_PA_F16 };
size_t dtype_size_in_bytes(DType d);

// Device placement of the cache pages. Cpu allocates host memory (the
// reference's CPU-device tests); Cuda allocates device memory on `ordinal`.
struct Device {
  enum class Kind { Cpu, Cuda } kind = Kind::Cpu;
  int ordinal = 0;
  static Device cpu() { return Device{}; }
  static Device cuda(int ordinal) { return Device{Kind::Cuda, ordinal}; }
  bool is_cuda() const { return kind == Kind::Cuda; }
};

// Non-owning view of a contiguous tensor (device or host memory).
struct DeviceTensor {
  void *ptr = nullptr;
  std::vector<size_t> dims;
  DType dtype = DType::F32;
  Device device;
  size_t elem_count() const;
};

constexpr int64_t PAD_SLOT_ID = -1;  // paged_kv_cache.rs:7

// ------------------------------------------------------------------ flash.rs
struct FlashKMeta {
  uint32_t max = 0;
  std::optional<std::vector<uint32_t>> cumulative_seqlens;
};

struct FlashParams {
  uint32_t max_q = 0;
  std::optional<std::vector<uint32_t>> cumulative_seqlens_q;
  FlashKMeta logical_k;
  bool causal = false;
  // flash.rs:28-42
  static std::optional<FlashParams> new_prefill(std::optional<size_t> max_q,
                                                std::optional<std::vector<uint32_t>> cu_q,
                                                std::optional<size_t> max_k,
                                                std::optional<std::vector<uint32_t>> cu_k,
                                                bool causal);
};

// --------------------------------------------------------- paged_kv_cache.rs
// paged_kv_cache.rs:22-38. Tensors are host vectors: slot_mapping i64 [T],
// block_tables u32 [rows, cols] row-major, context_lens u32 [B].
struct PagedInputMetadata {
  std::vector<int64_t> slot_mapping;
  std::vector<uint32_t> block_tables;
  size_t block_table_rows = 0;
  size_t block_table_cols = 0;
  std::vector<uint32_t> context_lens;
  size_t max_context_len = 0;
  std::optional<std::vector<uint32_t>> token_attention_mask;  // [rows, seq_len]
  size_t token_attention_mask_cols = 0;
  bool prefill_causal_only = false;
  std::optional<std::vector<size_t>> query_lens;
  std::optional<std::vector<size_t>> kv_lens;
  std::optional<FlashParams> prefill_flash_params_;
  std::optional<std::vector<uint32_t>> cu_seqlens_q;
  std::optional<std::vector<uint32_t>> cu_seqlens_kv;
  std::optional<size_t> max_query_len;
  std::optional<size_t> max_kv_len;

  const std::optional<FlashParams> &prefill_flash_params() const { return prefill_flash_params_; }
  std::optional<FlashParams> flash_params(bool causal) const;  // paged_kv_cache.rs:45-55
};

std::vector<uint32_t> cumulative_seqlens_from_lengths(const std::vector<size_t> &lengths);
int64_t slot_for_block_table_position(const std::vector<std::vector<size_t>> &block_tables,
                                      size_t block_size, size_t num_blocks, size_t seq,
                                      size_t position);

class PagedKvCache {
 public:
  // paged_kv_cache.rs:149-226
  static PagedKvCache create(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                             size_t block_size, size_t max_tokens, DType dtype, Device device);
  static PagedKvCache new_batched(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                  size_t block_size, size_t batch_size,
                                  size_t max_tokens_per_sequence, DType dtype, Device device);
  static PagedKvCache new_pool(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                               size_t block_size, size_t num_blocks, DType dtype, Device device);
  // Wrap caller-owned per-layer pages (e.g. torch tensors) without copying.
  static PagedKvCache from_external(std::vector<DeviceTensor> key_cache,
                                    std::vector<DeviceTensor> value_cache, size_t block_size);

  PagedKvCache(PagedKvCache &&) noexcept;
  PagedKvCache &operator=(PagedKvCache &&) noexcept;
  PagedKvCache(const PagedKvCache &) = delete;
  PagedKvCache &operator=(const PagedKvCache &) = delete;
  ~PagedKvCache();

  size_t estimated_bytes() const;
  size_t block_size() const { return block_size_; }
  size_t num_blocks() const { return num_blocks_; }
  size_t num_blocks_per_sequence() const { return num_blocks_per_sequence_; }
  size_t batch_size() const { return batch_size_; }
  size_t max_tokens_per_sequence() const { return max_tokens_per_sequence_; }
  size_t max_tokens() const { return max_tokens_; }
  size_t num_layers() const { return key_cache_.size(); }
  size_t num_kv_heads() const { return num_kv_heads_; }
  size_t head_dim() const { return head_dim_; }
  DType dtype() const { return dtype_; }
  const std::vector<uint32_t> &block_table_host() const { return block_table_host_; }
  std::vector<size_t> key_dims() const;
  std::vector<size_t> value_dims() const;

  int64_t slot_for_position(size_t position) const;
  int64_t slot_for_sequence_position(size_t sequence, size_t position) const;
  std::vector<int64_t> slot_mapping_for_range(size_t start, size_t len) const;
  std::vector<std::vector<uint32_t>> block_tables_tensor() const;
  std::vector<std::vector<uint32_t>> block_tables_tensor_for_batch(size_t batch) const;
  std::vector<uint32_t> context_lens_tensor(size_t context_len) const;

  PagedInputMetadata input_metadata_for_range(size_t start, size_t len, size_t context_len) const;
  PagedInputMetadata input_metadata_for_batch_ranges(const std::vector<size_t> &starts, size_t len,
                                                     const std::vector<size_t> &context_lens) const;
  PagedInputMetadata input_metadata_from_block_tables(
      const std::vector<std::vector<size_t>> &block_tables, const std::vector<size_t> &starts,
      size_t len, const std::vector<size_t> &context_lens) const;
  PagedInputMetadata input_metadata_from_attention_masks(
      const std::vector<std::vector<size_t>> &block_tables,
      const std::vector<std::vector<uint32_t>> &attention_masks) const;
  PagedInputMetadata input_metadata_from_query_lens(
      const std::vector<std::vector<size_t>> &block_tables,
      const std::vector<size_t> &query_lens) const;
  std::vector<PagedInputMetadata> decode_metadata_for_steps(size_t prompt_len, size_t steps) const;
  // `cuda_graph` = the crate's cuda-graph feature: block tables padded to
  // bucket_block_table_cols (paged_kv_cache.rs:948-952).
  std::vector<PagedInputMetadata> decode_metadata_for_batch_steps(
      const std::vector<std::vector<size_t>> &block_tables, const std::vector<size_t> &prompt_lens,
      size_t steps, bool cuda_graph = false) const;
  // Same result as the reference's decode_metadata_for_batch_step
  // (paged_kv_cache.rs:1046-1059), computed for the requested step only
  // instead of rebuilding steps 0..=step.
  PagedInputMetadata decode_metadata_for_batch_step(
      const std::vector<std::vector<size_t>> &block_tables, const std::vector<size_t> &prompt_lens,
      size_t step, bool cuda_graph = false) const;

  std::pair<const DeviceTensor &, const DeviceTensor &> key_value_cache(size_t layer_idx) const;

 private:
  PagedKvCache() = default;
  static PagedKvCache new_inner(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                size_t block_size, size_t num_blocks,
                                size_t num_blocks_per_sequence, size_t batch_size,
                                size_t max_tokens_per_sequence, DType dtype, Device device);
  void release();

  std::vector<DeviceTensor> key_cache_;
  std::vector<DeviceTensor> value_cache_;
  bool owns_ = false;
  std::vector<uint32_t> block_table_host_;
  size_t block_size_ = 0, num_blocks_ = 0, num_blocks_per_sequence_ = 0, batch_size_ = 0;
  size_t max_tokens_per_sequence_ = 0, max_tokens_ = 0, num_kv_heads_ = 0, head_dim_ = 0;
  DType dtype_ = DType::F32;
};

// ---------------------------------------------------- paged_cache_runtime.rs
struct PagedCacheMemory {  // paged_cache_runtime.rs:22-28
  enum class Kind { ContextSize, Blocks, GpuMemoryFraction } kind = Kind::GpuMemoryFraction;
  size_t value = 0;
  float fraction = 0.8f;
  static PagedCacheMemory context_size(size_t tokens) { return {Kind::ContextSize, tokens, 0.f}; }
  static PagedCacheMemory blocks(size_t n) { return {Kind::Blocks, n, 0.f}; }
  static PagedCacheMemory gpu_memory_fraction(float f) { return {Kind::GpuMemoryFraction, 0, f}; }
};

struct PagedCacheConfig {  // paged_cache_runtime.rs:30-43 (default bs 32, 0.8 of VRAM)
  size_t block_size = 32;
  PagedCacheMemory memory = PagedCacheMemory::gpu_memory_fraction(0.8f);
};

size_t bytes_per_paged_block(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                             size_t block_size, DType dtype);
size_t blocks_for_byte_budget(size_t byte_budget, size_t bytes_per_block);
// KV budget = fraction * total - used, from cudaMemGetInfo (the reference
// shells out to nvidia-smi, paged_cache_runtime.rs:89-149).
size_t cuda_kv_byte_budget(int ordinal, float fraction);
size_t resolve_num_blocks(PagedCacheMemory memory, size_t num_layers, size_t num_kv_heads,
                          size_t head_dim, size_t block_size, DType dtype, Device device);

struct PagedCacheStats {  // paged_cache_runtime.rs:203-210
  size_t block_size = 0, num_blocks = 0, free_blocks = 0, max_context_tokens = 0, bytes = 0;
};

class PagedBlockManager {  // paged_cache_runtime.rs:217-371
 public:
  PagedBlockManager(size_t num_blocks, size_t block_size);
  size_t block_size() const { return block_size_; }
  size_t free_blocks() const { return free_.size(); }
  bool slots_available_for(size_t request_id, size_t num_tokens) const;
  size_t blocks_for_request(size_t request_id) const;
  size_t total_allocated_blocks() const;
  static size_t allocatable_block_capacity(size_t num_blocks) {
    return num_blocks > 0 ? num_blocks - 1 : 0;
  }
  void allocate_slots(size_t request_id, size_t num_tokens);
  bool try_allocate_slots(size_t request_id, size_t num_tokens);
  void trim_request_to_num_tokens(size_t request_id, size_t num_tokens);
  const std::vector<size_t> &block_ids(size_t request_id) const;
  void free_request(size_t request_id);
  void free_many(const std::vector<size_t> &request_ids);
  std::vector<std::vector<size_t>> block_tables_for(const std::vector<size_t> &request_ids) const;

 private:
  size_t block_size_;
  std::deque<size_t> free_;
  std::unordered_map<size_t, std::vector<size_t>> request_blocks_;
};

// batch_scheduler.rs:100-113
bool can_admit_with_projected_kv(const PagedBlockManager &manager, size_t kv_block_capacity,
                                 size_t prompt_len, size_t projected_used_blocks,
                                 size_t projected_running);

// --------------------------------------------------------------- cuda_graph.rs
constexpr size_t CUDA_GRAPH_CONTEXT_BUCKET_TOKENS = 256;
constexpr size_t CUDA_DECODE_GRAPH_MAX_BATCH = 256;
constexpr size_t CUDA_DECODE_GRAPH_MAX_GRAPHS = 256;
std::optional<size_t> cuda_graph_batch_bucket(size_t actual_batch, size_t max_batch);
std::vector<size_t> cuda_graph_batch_buckets(size_t max_batch);
size_t cuda_graph_block_bucket(size_t block_size);
size_t bucket_block_table_cols(size_t blocks, size_t block_size);
size_t cuda_graph_prewarm_batch_limit(size_t max_batch);

// pad_decode_batch_to_max / pad_metadata_block_tables on host metadata
// (cuda_graph.rs:373-486): dummy rows get id 0, slot 0, context 1 and an
// all-zero block-table row; real rows are widened by repeating their last
// block id.
struct PaddedDecodeBatch {
  std::vector<int64_t> input_ids;
  PagedInputMetadata metadata;
};
PaddedDecodeBatch pad_decode_batch_to_max(size_t max_batch, const std::vector<int64_t> &input_ids,
                                          const PagedInputMetadata &metadata,
                                          size_t block_table_cols);
PagedInputMetadata pad_metadata_block_tables(const PagedInputMetadata &metadata, size_t cols);

struct CudaDecodeGraphKey {
  size_t batch = 0;
  size_t block_table_cols = 0;
  bool operator<(const CudaDecodeGraphKey &o) const {
    return batch != o.batch ? batch < o.batch : block_table_cols < o.block_table_cols;
  }
  bool operator==(const CudaDecodeGraphKey &o) const {
    return batch == o.batch && block_table_cols == o.block_table_cols;
  }
};

// Graph-key bookkeeping of PagedCacheRuntime (paged_cache_runtime.rs:478-553):
// the key of a decode step, and the per-key disable list used when a capture
// or replay fails (fallback to eager, paged_batch_engine.rs:750-761).
class DecodeGraphRegistry {
 public:
  DecodeGraphRegistry(size_t block_size, size_t max_batch)
      : block_size_(block_size), max_batch_(cuda_graph_prewarm_batch_limit(max_batch)) {}
  CudaDecodeGraphKey key(size_t actual_batch, size_t meta_cols) const;
  bool enabled() const { return !disabled_ && max_batch_ > 0; }
  bool enabled_for(size_t actual_batch, size_t meta_cols) const;
  void disable_for(size_t actual_batch, size_t meta_cols);
  void disable_all() { disabled_ = true; }
  size_t max_batch() const { return max_batch_; }

 private:
  size_t block_size_;
  size_t max_batch_;
  bool disabled_ = false;
  std::set<CudaDecodeGraphKey> disabled_keys_;
};

class PagedCacheRuntime {  // paged_cache_runtime.rs:381-705 (host parts)
 public:
  PagedCacheRuntime(size_t num_layers, size_t num_kv_heads, size_t head_dim, DType dtype,
                    Device device, PagedCacheConfig config);
  const PagedKvCache &cache() const { return cache_; }
  const PagedBlockManager &manager() const { return manager_; }
  PagedBlockManager &manager_mut() { return manager_; }
  std::vector<std::vector<size_t>> block_tables_for(const std::vector<size_t> &request_ids) const {
    return manager_.block_tables_for(request_ids);
  }
  PagedCacheStats stats() const;
  DecodeGraphRegistry &graphs() { return graphs_; }
  void set_cuda_graph_max_batch(size_t max_batch) {
    graphs_ = DecodeGraphRegistry(cache_.block_size(), max_batch);
  }

 private:
  PagedKvCache cache_;
  PagedBlockManager manager_;
  PagedCacheStats stats_;
  DecodeGraphRegistry graphs_;
};

// ---------------------------------------------------- mistralrs_paged_attn
// The kernel calls of thinker_text.rs with the reference argument order.
// Outputs and workspace are allocated by the caller (the C ABI never
// allocates); `stream` is a cudaStream_t.
namespace mistralrs_paged_attn {
void reshape_and_cache(const DeviceTensor &key, const DeviceTensor &value,
                       const DeviceTensor *k_scale, const DeviceTensor *v_scale,
                       const DeviceTensor &key_cache, const DeviceTensor &value_cache,
                       const DeviceTensor &slot_mapping, vasr_pa_stream_t stream);
size_t paged_attention_workspace_bytes(const DeviceTensor &q, const DeviceTensor &key_cache,
                                       size_t max_context_len);
void paged_attention(const DeviceTensor &out, const DeviceTensor &q, const DeviceTensor *k_scale,
                     const DeviceTensor *v_scale, const DeviceTensor &key_cache,
                     const DeviceTensor &value_cache, const DeviceTensor &block_tables,
                     const DeviceTensor &context_lens, const DeviceTensor *alibi,
                     size_t max_context_len, float softmax_scale, float softcapping,
                     const DeviceTensor *sinks, void *workspace, size_t workspace_bytes,
                     vasr_pa_stream_t stream);
void gather_kv_cache(const DeviceTensor &key_out, const DeviceTensor &value_out,
                     const DeviceTensor &key_cache, const DeviceTensor &value_cache,
                     const DeviceTensor *k_scale, const DeviceTensor *v_scale,
                     const DeviceTensor &block_tables, const DeviceTensor &cu_seqlens_kv,
                     vasr_pa_stream_t stream);
void copy_blocks(const std::vector<DeviceTensor> &key_caches,
                 const std::vector<DeviceTensor> &value_caches, const DeviceTensor &block_mapping,
                 vasr_pa_stream_t stream);
void swap_blocks(const DeviceTensor &src, const DeviceTensor &dst,
                 const DeviceTensor &block_mapping, vasr_pa_stream_t stream);
}  // namespace mistralrs_paged_attn

}  // namespace vasr_paged_attn

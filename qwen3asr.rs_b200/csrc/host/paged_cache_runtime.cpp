// paged_cache_runtime.cpp — pool sizing, block allocator, runtime, graph keys.
// Restates vasr-paged-attn/src/paged_cache_runtime.rs and the bucketing /
// padding helpers of vasr-paged-attn/src/cuda_graph.rs (host parts).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <limits>
#include <sstream>

#include "vasr_paged_attn.hpp"

namespace vasr_paged_attn {

namespace {
template <typename... A>
[[noreturn]] void bail(A &&...parts) {
  std::ostringstream os;
  (os << ... << parts);
  throw Error(os.str());
}
size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }
size_t next_power_of_two(size_t v) {
  size_t p = 1;
  while (p < v) p <<= 1;
  return p;
}
}  // namespace

// paged_cache_runtime.rs:46-71
size_t bytes_per_paged_block(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                             size_t block_size, DType dtype) {
  if (num_layers == 0 || num_kv_heads == 0 || head_dim == 0 || block_size == 0)
    bail("paged block sizing requires non-zero layer/head/block parameters");
  const size_t per_layer = num_kv_heads * head_dim * block_size * 2;
  if (per_layer / 2 / block_size / head_dim != num_kv_heads) bail("paged block element count overflow");
  const size_t elems = num_layers * per_layer;
  if (elems / num_layers != per_layer) bail("paged block element count overflow");
  const size_t es = dtype_size_in_bytes(dtype);
  if (elems > std::numeric_limits<size_t>::max() / es) bail("paged block byte count overflow");
  return elems * es;
}

// paged_cache_runtime.rs:74-86: +1 for the reserved null block 0.
size_t blocks_for_byte_budget(size_t byte_budget, size_t bytes_per_block) {
  if (bytes_per_block == 0) bail("paged block byte size must be non-zero");
  const size_t n = byte_budget / bytes_per_block + 1;
  if (n <= 1)
    bail("paged KV byte budget ", byte_budget, " is too small for one block (", bytes_per_block,
         " bytes)");
  return n;
}

// paged_cache_runtime.rs:135-149, with cudaMemGetInfo in place of the
// nvidia-smi subprocess of :89-133 (same quantities: total and used bytes).
size_t cuda_kv_byte_budget(int ordinal, float fraction) {
  if (!(fraction > 0.f && fraction <= 1.f))
    bail("GPU memory fraction must be in (0.0, 1.0]; got ", fraction);
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(ordinal) != cudaSuccess) bail("GpuMemoryFraction sizing: no CUDA device ", ordinal);
  size_t free_b = 0, total_b = 0;
  const cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
  cudaSetDevice(prev);
  if (e != cudaSuccess) bail("cudaMemGetInfo failed: ", cudaGetErrorString(e));
  const size_t mib = 1024 * 1024;
  const size_t total_mib = total_b / mib;
  const size_t used_mib = (total_b - free_b) / mib;
  const size_t target_mib = static_cast<size_t>(std::floor(static_cast<double>(total_mib) * fraction));
  const size_t budget_mib = target_mib > used_mib ? target_mib - used_mib : 0;
  if (budget_mib == 0)
    bail("GPU KV budget exhausted: total_mib=", total_mib, " used_mib=", used_mib,
         " fraction=", fraction);
  return budget_mib * mib;
}

// paged_cache_runtime.rs:151-201
size_t resolve_num_blocks(PagedCacheMemory memory, size_t num_layers, size_t num_kv_heads,
                          size_t head_dim, size_t block_size, DType dtype, Device device) {
  switch (memory.kind) {
    case PagedCacheMemory::Kind::ContextSize: return div_ceil(memory.value, block_size) + 1;
    case PagedCacheMemory::Kind::Blocks: return memory.value;
    case PagedCacheMemory::Kind::GpuMemoryFraction: {
      if (!device.is_cuda())
        bail("GpuMemoryFraction paged cache sizing requires a CUDA device");
      const size_t budget = cuda_kv_byte_budget(device.ordinal, memory.fraction);
      return blocks_for_byte_budget(
          budget, bytes_per_paged_block(num_layers, num_kv_heads, head_dim, block_size, dtype));
    }
  }
  bail("unknown paged cache memory policy");
}

// ------------------------------------------------------- PagedBlockManager
PagedBlockManager::PagedBlockManager(size_t num_blocks, size_t block_size)
    : block_size_(block_size) {
  for (size_t b = 1; b < num_blocks; ++b) free_.push_back(b);  // block 0 is the null block
}

bool PagedBlockManager::slots_available_for(size_t request_id, size_t num_tokens) const {
  const size_t required = div_ceil(num_tokens, block_size_);
  const size_t existing = blocks_for_request(request_id);
  const size_t needed = required > existing ? required - existing : 0;
  return needed <= free_.size();
}

size_t PagedBlockManager::blocks_for_request(size_t request_id) const {
  auto it = request_blocks_.find(request_id);
  return it == request_blocks_.end() ? 0 : it->second.size();
}

size_t PagedBlockManager::total_allocated_blocks() const {
  size_t n = 0;
  for (const auto &kv : request_blocks_) n += kv.second.size();
  return n;
}

void PagedBlockManager::allocate_slots(size_t request_id, size_t num_tokens) {
  if (!try_allocate_slots(request_id, num_tokens))
    bail("paged KV cache exhausted: request_id=", request_id, " num_tokens=", num_tokens,
         " free_blocks=", free_.size());
}

// paged_cache_runtime.rs:286-314: pops from the front of the FIFO free list.
bool PagedBlockManager::try_allocate_slots(size_t request_id, size_t num_tokens) {
  const size_t required = div_ceil(num_tokens, block_size_);
  const size_t existing = blocks_for_request(request_id);
  const size_t needed = required > existing ? required - existing : 0;
  if (needed == 0) return true;
  if (needed > free_.size()) return false;
  auto &ids = request_blocks_[request_id];
  for (size_t i = 0; i < needed; ++i) {
    ids.push_back(free_.front());
    free_.pop_front();
  }
  return true;
}

// paged_cache_runtime.rs:320-335: tail blocks return to the back in reverse.
void PagedBlockManager::trim_request_to_num_tokens(size_t request_id, size_t num_tokens) {
  const size_t keep = div_ceil(num_tokens, block_size_);
  auto it = request_blocks_.find(request_id);
  if (it == request_blocks_.end() || keep >= it->second.size()) return;
  auto &ids = it->second;
  for (size_t i = ids.size(); i > keep; --i)
    if (ids[i - 1] != 0) free_.push_back(ids[i - 1]);
  ids.resize(keep);
}

const std::vector<size_t> &PagedBlockManager::block_ids(size_t request_id) const {
  auto it = request_blocks_.find(request_id);
  if (it == request_blocks_.end())
    bail("paged KV request has no allocated blocks: request_id=", request_id);
  return it->second;
}

// paged_cache_runtime.rs:348-357
void PagedBlockManager::free_request(size_t request_id) {
  auto it = request_blocks_.find(request_id);
  if (it == request_blocks_.end()) return;
  const auto &ids = it->second;
  for (size_t i = ids.size(); i > 0; --i)
    if (ids[i - 1] != 0) free_.push_back(ids[i - 1]);
  request_blocks_.erase(it);
}

void PagedBlockManager::free_many(const std::vector<size_t> &request_ids) {
  for (size_t r : request_ids) free_request(r);
}

std::vector<std::vector<size_t>> PagedBlockManager::block_tables_for(
    const std::vector<size_t> &request_ids) const {
  std::vector<std::vector<size_t>> out;
  out.reserve(request_ids.size());
  for (size_t r : request_ids) out.push_back(block_ids(r));
  return out;
}

bool can_admit_with_projected_kv(const PagedBlockManager &manager, size_t kv_block_capacity,
                                 size_t prompt_len, size_t projected_used_blocks,
                                 size_t projected_running) {
  const size_t prompt_blocks = div_ceil(prompt_len, manager.block_size());
  const size_t headroom = std::max<size_t>(projected_running, 1);
  return projected_used_blocks + prompt_blocks + headroom <= kv_block_capacity;
}

// ------------------------------------------------------------- cuda_graph.rs
std::optional<size_t> cuda_graph_batch_bucket(size_t actual, size_t max_batch) {
  if (actual == 0 || max_batch == 0 || actual > max_batch) return std::nullopt;
  size_t b;
  if (actual <= 2) b = actual;
  else if (actual <= 4) b = 4;
  else if (actual <= 8) b = 8;
  else b = div_ceil(actual, 16) * 16;
  return std::min(b, max_batch);
}

size_t cuda_graph_prewarm_batch_limit(size_t max_batch) {
  return std::min(max_batch, CUDA_DECODE_GRAPH_MAX_BATCH);
}

std::vector<size_t> cuda_graph_batch_buckets(size_t max_batch) {
  const size_t m = cuda_graph_prewarm_batch_limit(max_batch);
  std::vector<size_t> out;
  if (m == 0) return out;
  for (size_t b : {1, 2, 4, 8})
    if (b <= m) out.push_back(b);
  for (size_t b = 16; b <= m; b += 16) out.push_back(b);
  if (out.back() != m) out.push_back(m);
  return out;
}

size_t cuda_graph_block_bucket(size_t block_size) {
  return std::max<size_t>(1, div_ceil(CUDA_GRAPH_CONTEXT_BUCKET_TOKENS, block_size));
}

size_t bucket_block_table_cols(size_t blocks, size_t block_size) {
  const size_t bb = cuda_graph_block_bucket(block_size);
  if (blocks == 0) return bb;
  return std::max(next_power_of_two(blocks), bb);
}

// cuda_graph.rs:432-449, 471-486
PagedInputMetadata pad_metadata_block_tables(const PagedInputMetadata &metadata, size_t cols) {
  const size_t meta_cols = metadata.block_table_cols;
  if (meta_cols > cols) bail("cannot pad block tables from ", meta_cols, " columns down to ", cols);
  if (meta_cols == cols) return metadata;
  PagedInputMetadata out = metadata;
  out.block_tables.assign(metadata.block_table_rows * cols, 0);
  for (size_t r = 0; r < metadata.block_table_rows; ++r) {
    for (size_t c = 0; c < cols; ++c) {
      uint32_t v = 0;
      if (meta_cols > 0) v = metadata.block_tables[r * meta_cols + std::min(c, meta_cols - 1)];
      out.block_tables[r * cols + c] = v;
    }
  }
  out.block_table_cols = cols;
  return out;
}

// cuda_graph.rs:373-430
PaddedDecodeBatch pad_decode_batch_to_max(size_t max_batch, const std::vector<int64_t> &input_ids,
                                          const PagedInputMetadata &metadata,
                                          size_t block_table_cols) {
  const size_t actual = input_ids.size();
  if (actual == 0 || actual > max_batch)
    bail("actual batch ", actual, " exceeds cuda graph max batch ", max_batch);
  PaddedDecodeBatch out;
  out.metadata = pad_metadata_block_tables(metadata, block_table_cols);
  out.input_ids = input_ids;
  if (actual == max_batch) return out;
  const size_t pad = max_batch - actual;
  out.input_ids.resize(max_batch, 0);
  auto &m = out.metadata;
  m.slot_mapping.resize(m.slot_mapping.size() + pad, 0);
  m.context_lens.resize(m.context_lens.size() + pad, 1);
  m.block_tables.resize((m.block_table_rows + pad) * m.block_table_cols, 0);
  m.block_table_rows += pad;
  m.token_attention_mask.reset();
  m.prefill_flash_params_.reset();
  m.prefill_causal_only = false;
  m.query_lens.reset();
  m.kv_lens.reset();
  m.cu_seqlens_q.reset();
  m.cu_seqlens_kv.reset();
  m.max_query_len.reset();
  m.max_kv_len.reset();
  return out;
}

// paged_cache_runtime.rs:498-529
CudaDecodeGraphKey DecodeGraphRegistry::key(size_t actual_batch, size_t meta_cols) const {
  if (max_batch_ == 0) bail("CUDA decode graphs are not prewarmed");
  if (actual_batch == 0 || actual_batch > max_batch_)
    bail("CUDA decode actual batch must be in 1..=", max_batch_, "; got ", actual_batch);
  const auto b = cuda_graph_batch_bucket(actual_batch, max_batch_);
  if (!b) bail("CUDA decode graph has no batch bucket for actual_batch=", actual_batch);
  return CudaDecodeGraphKey{*b, bucket_block_table_cols(meta_cols, block_size_)};
}

bool DecodeGraphRegistry::enabled_for(size_t actual_batch, size_t meta_cols) const {
  if (!enabled()) return false;
  return disabled_keys_.count(key(actual_batch, meta_cols)) == 0;
}

void DecodeGraphRegistry::disable_for(size_t actual_batch, size_t meta_cols) {
  disabled_keys_.insert(key(actual_batch, meta_cols));
}

// ------------------------------------------------------------ runtime
// paged_cache_runtime.rs:398-454
static PagedKvCache make_runtime_cache(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                       DType dtype, Device device, const PagedCacheConfig &config,
                                       size_t *num_blocks_out) {
  if (!(config.block_size == 8 || config.block_size == 16 || config.block_size == 32))
    bail("paged cache block size must be 8, 16, or 32; got ", config.block_size);
  const size_t nb = resolve_num_blocks(config.memory, num_layers, num_kv_heads, head_dim,
                                       config.block_size, dtype, device);
  if (nb <= 1) bail("paged cache requires at least 2 blocks including null block");
  *num_blocks_out = nb;
  return PagedKvCache::new_pool(num_layers, num_kv_heads, head_dim, config.block_size, nb, dtype,
                                device);
}

PagedCacheRuntime::PagedCacheRuntime(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                     DType dtype, Device device, PagedCacheConfig config)
    : cache_([&] {
        size_t nb = 0;
        return make_runtime_cache(num_layers, num_kv_heads, head_dim, dtype, device, config, &nb);
      }()),
      manager_(cache_.num_blocks(), config.block_size),
      graphs_(config.block_size, 0) {
  stats_.block_size = config.block_size;
  stats_.num_blocks = cache_.num_blocks();
  stats_.free_blocks = cache_.num_blocks() - 1;
  stats_.max_context_tokens = (cache_.num_blocks() - 1) * config.block_size;
  stats_.bytes = cache_.estimated_bytes();
}

PagedCacheStats PagedCacheRuntime::stats() const {
  PagedCacheStats s = stats_;
  s.free_blocks = manager_.free_blocks();
  return s;
}

}  // namespace vasr_paged_attn

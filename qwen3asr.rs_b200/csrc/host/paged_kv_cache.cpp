// paged_kv_cache.cpp — PagedKvCache and PagedInputMetadata builders.
// Restates vasr-paged-attn/src/paged_kv_cache.rs (and flash.rs) in C++; each
// method cites the Rust function it mirrors. Messages match the reference's
// candle_core::bail! texts.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
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

uint32_t to_u32(size_t v, const char *what) {
  if (v > std::numeric_limits<uint32_t>::max()) bail(what, " overflows u32: ", v);
  return static_cast<uint32_t>(v);
}

size_t checked_mul(size_t a, size_t b, const char *what) {
  if (a != 0 && b > std::numeric_limits<size_t>::max() / a) bail(what);
  return a * b;
}

size_t max_len(const std::vector<std::vector<size_t>> &t) {
  size_t m = 0;
  for (const auto &r : t) m = std::max(m, r.size());
  return m;
}

// Right-pad block tables with 0 to `width` columns (paged_kv_cache.rs:607-617).
std::vector<uint32_t> pad_tables(const std::vector<std::vector<size_t>> &tables, size_t width) {
  std::vector<uint32_t> out;
  out.reserve(tables.size() * width);
  for (const auto &t : tables) {
    for (size_t id : t) out.push_back(to_u32(id, "block id"));
    for (size_t i = t.size(); i < width; ++i) out.push_back(0);
  }
  return out;
}

struct Varlen {
  std::optional<FlashParams> flash;
  std::optional<std::vector<uint32_t>> cu_q, cu_kv;
  std::optional<size_t> max_q, max_kv;
};

// paged_kv_cache.rs:105-146
Varlen build_varlen_metadata(const std::optional<std::vector<size_t>> &query_lens,
                             const std::optional<std::vector<size_t>> &kv_lens) {
  Varlen v;
  if (query_lens) v.cu_q = cumulative_seqlens_from_lengths(*query_lens);
  if (kv_lens) v.cu_kv = cumulative_seqlens_from_lengths(*kv_lens);
  if (query_lens) {
    size_t m = 0;
    for (size_t n : *query_lens) m = std::max(m, n);
    v.max_q = m;
  }
  if (kv_lens) {
    size_t m = 0;
    for (size_t n : *kv_lens) m = std::max(m, n);
    v.max_kv = m;
  }
  bool causal = false;
  if (query_lens)
    for (size_t n : *query_lens) causal = causal || n > 1;
  v.flash = FlashParams::new_prefill(v.max_q, v.cu_q, v.max_kv, v.cu_kv, causal);
  return v;
}

void apply_varlen(PagedInputMetadata &m, std::optional<std::vector<size_t>> q,
                  std::optional<std::vector<size_t>> kv) {
  Varlen v = build_varlen_metadata(q, kv);
  m.query_lens = std::move(q);
  m.kv_lens = std::move(kv);
  m.prefill_flash_params_ = v.flash;
  m.cu_seqlens_q = v.cu_q;
  m.cu_seqlens_kv = v.cu_kv;
  m.max_query_len = v.max_q;
  m.max_kv_len = v.max_kv;
}

std::vector<uint32_t> context_u32(const std::vector<size_t> &lens, size_t *max_out) {
  std::vector<uint32_t> out;
  out.reserve(lens.size());
  size_t m = 0;
  for (size_t c : lens) {
    m = std::max(m, c);
    out.push_back(to_u32(c, "context length"));
  }
  *max_out = m;
  return out;
}

}  // namespace

size_t dtype_size_in_bytes(DType d) { return d == DType::F32 ? 4 : 2; }

size_t DeviceTensor::elem_count() const {
  size_t n = 1;
  for (size_t d : dims) n *= d;
  return n;
}

std::optional<FlashParams> FlashParams::new_prefill(std::optional<size_t> max_q,
                                                    std::optional<std::vector<uint32_t>> cu_q,
                                                    std::optional<size_t> max_k,
                                                    std::optional<std::vector<uint32_t>> cu_k,
                                                    bool causal) {
  if (!max_q || !max_k) return std::nullopt;
  if (*max_q > std::numeric_limits<uint32_t>::max() || *max_k > std::numeric_limits<uint32_t>::max())
    return std::nullopt;
  FlashParams p;
  p.max_q = static_cast<uint32_t>(*max_q);
  p.cumulative_seqlens_q = std::move(cu_q);
  p.logical_k.max = static_cast<uint32_t>(*max_k);
  p.logical_k.cumulative_seqlens = std::move(cu_k);
  p.causal = causal;
  return p;
}

std::optional<FlashParams> PagedInputMetadata::flash_params(bool causal) const {
  if (prefill_flash_params_) return prefill_flash_params_;
  return FlashParams::new_prefill(max_query_len, cu_seqlens_q, max_kv_len, cu_seqlens_kv, causal);
}

// paged_kv_cache.rs:58-72
std::vector<uint32_t> cumulative_seqlens_from_lengths(const std::vector<size_t> &lengths) {
  std::vector<uint32_t> out;
  out.reserve(lengths.size() + 1);
  out.push_back(0);
  uint64_t total = 0;
  for (size_t len : lengths) {
    const uint32_t l = to_u32(len, "sequence length");
    total += l;
    if (total > std::numeric_limits<uint32_t>::max()) bail("cumulative sequence length overflow");
    out.push_back(static_cast<uint32_t>(total));
  }
  return out;
}

// paged_kv_cache.rs:74-103
int64_t slot_for_block_table_position(const std::vector<std::vector<size_t>> &block_tables,
                                      size_t block_size, size_t num_blocks, size_t seq,
                                      size_t position) {
  if (seq >= block_tables.size()) bail("missing block table for sequence ", seq);
  const auto &table = block_tables[seq];
  const size_t block_idx = position / block_size;
  const size_t offset = position % block_size;
  if (block_idx >= table.size())
    bail("missing block table entry: seq=", seq, " block_idx=", block_idx, " position=", position,
         " block_size=", block_size, " table_len=", table.size());
  const size_t block_id = table[block_idx];
  if (block_id >= num_blocks)
    bail("block id exceeds paged cache capacity: block_id=", block_id, " num_blocks=", num_blocks);
  const size_t slot = checked_mul(block_id, block_size, "paged slot mapping overflow") + offset;
  if (slot > static_cast<size_t>(std::numeric_limits<int64_t>::max()))
    bail("paged slot overflows i64: ", slot);
  return static_cast<int64_t>(slot);
}

// ----------------------------------------------------------- construction
PagedKvCache PagedKvCache::create(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                  size_t block_size, size_t max_tokens, DType dtype,
                                  Device device) {
  return new_batched(num_layers, num_kv_heads, head_dim, block_size, 1, max_tokens, dtype, device);
}

PagedKvCache PagedKvCache::new_batched(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                       size_t block_size, size_t batch_size,
                                       size_t max_tokens_per_sequence, DType dtype,
                                       Device device) {
  if (block_size == 0) bail("paged kv cache requires non-zero block_size");
  const size_t nbps = (max_tokens_per_sequence + block_size - 1) / block_size;
  const size_t nb = checked_mul(batch_size, nbps, "paged kv cache block count overflow");
  return new_inner(num_layers, num_kv_heads, head_dim, block_size, nb, nbps, batch_size,
                   max_tokens_per_sequence, dtype, device);
}

PagedKvCache PagedKvCache::new_pool(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                    size_t block_size, size_t num_blocks, DType dtype,
                                    Device device) {
  const size_t max_tokens =
      checked_mul(num_blocks, block_size, "paged kv cache token capacity overflow");
  return new_inner(num_layers, num_kv_heads, head_dim, block_size, num_blocks, num_blocks, 1,
                   max_tokens, dtype, device);
}

// paged_kv_cache.rs:229-314
PagedKvCache PagedKvCache::new_inner(size_t num_layers, size_t num_kv_heads, size_t head_dim,
                                     size_t block_size, size_t num_blocks,
                                     size_t num_blocks_per_sequence, size_t batch_size,
                                     size_t max_tokens_per_sequence, DType dtype,
                                     Device device) {
  if (num_layers == 0) bail("paged kv cache requires at least one layer");
  if (num_kv_heads == 0) bail("paged kv cache requires at least one kv head");
  if (head_dim == 0) bail("paged kv cache requires non-zero head_dim");
  if (block_size == 0) bail("paged kv cache requires non-zero block_size");
  if (batch_size == 0) bail("paged kv cache requires non-zero batch_size");
  if (max_tokens_per_sequence == 0) bail("paged kv cache requires non-zero max_tokens");
  if (num_blocks == 0) bail("paged kv cache requires non-zero num_blocks");
  const size_t es = dtype_size_in_bytes(dtype);
  const size_t key_pack = 16 / es;
  if (head_dim % key_pack != 0)
    bail("head_dim must be divisible by key cache pack size: head_dim=", head_dim,
         " pack=", key_pack);
  const size_t max_tokens =
      checked_mul(num_blocks, block_size, "paged kv cache token capacity overflow");
  if (num_blocks - 1 > std::numeric_limits<uint32_t>::max())
    bail("block index overflows u32: ", num_blocks - 1);

  PagedKvCache c;
  c.block_table_host_.resize(num_blocks);
  for (size_t i = 0; i < num_blocks; ++i) c.block_table_host_[i] = static_cast<uint32_t>(i);
  c.block_size_ = block_size;
  c.num_blocks_ = num_blocks;
  c.num_blocks_per_sequence_ = num_blocks_per_sequence;
  c.batch_size_ = batch_size;
  c.max_tokens_per_sequence_ = max_tokens_per_sequence;
  c.max_tokens_ = max_tokens;
  c.num_kv_heads_ = num_kv_heads;
  c.head_dim_ = head_dim;
  c.dtype_ = dtype;
  c.owns_ = true;
  const std::vector<size_t> kdims{num_blocks, num_kv_heads, head_dim / key_pack, block_size,
                                  key_pack};
  const std::vector<size_t> vdims{num_blocks, num_kv_heads, head_dim, block_size};
  const size_t bytes = checked_mul(checked_mul(num_blocks, num_kv_heads * head_dim * block_size,
                                               "paged kv cache size overflow"),
                                   es, "paged kv cache size overflow");
  for (size_t l = 0; l < num_layers; ++l) {
    for (int kv = 0; kv < 2; ++kv) {
      DeviceTensor t;
      t.dims = kv == 0 ? kdims : vdims;
      t.dtype = dtype;
      t.device = device;
      if (device.is_cuda()) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device.ordinal);
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
        cudaSetDevice(prev);
        if (e != cudaSuccess) {
          c.release();
          bail("paged kv cache allocation failed: ", cudaGetErrorString(e));
        }
        t.ptr = p;
      } else {
        t.ptr = std::calloc(bytes, 1);
        if (!t.ptr) {
          c.release();
          bail("paged kv cache host allocation failed");
        }
      }
      (kv == 0 ? c.key_cache_ : c.value_cache_).push_back(t);
    }
  }
  return c;
}

PagedKvCache PagedKvCache::from_external(std::vector<DeviceTensor> key_cache,
                                         std::vector<DeviceTensor> value_cache,
                                         size_t block_size) {
  if (key_cache.empty() || key_cache.size() != value_cache.size())
    bail("paged kv cache requires at least one layer");
  const auto &k = key_cache[0];
  const auto &v = value_cache[0];
  if (k.dims.size() != 5 || v.dims.size() != 4) bail("paged cache shape mismatch");
  for (size_t l = 0; l < key_cache.size(); ++l)
    if (key_cache[l].dims != k.dims || value_cache[l].dims != v.dims)
      bail("paged cache shape mismatch across layers");
  if (k.dims[0] != v.dims[0] || k.dims[1] != v.dims[1] || k.dims[3] != block_size ||
      v.dims[3] != block_size || k.dims[2] * k.dims[4] != v.dims[2] ||
      k.dims[4] * dtype_size_in_bytes(k.dtype) != 16)
    bail("paged cache shape mismatch");
  PagedKvCache c;
  c.key_cache_ = std::move(key_cache);
  c.value_cache_ = std::move(value_cache);
  c.owns_ = false;
  c.block_size_ = block_size;
  c.num_blocks_ = v.dims[0];
  c.num_blocks_per_sequence_ = v.dims[0];
  c.batch_size_ = 1;
  c.max_tokens_ = c.num_blocks_ * block_size;
  c.max_tokens_per_sequence_ = c.max_tokens_;
  c.num_kv_heads_ = v.dims[1];
  c.head_dim_ = v.dims[2];
  c.dtype_ = k.dtype;
  c.block_table_host_.resize(c.num_blocks_);
  for (size_t i = 0; i < c.num_blocks_; ++i) c.block_table_host_[i] = static_cast<uint32_t>(i);
  return c;
}

void PagedKvCache::release() {
  if (owns_) {
    for (auto *vec : {&key_cache_, &value_cache_})
      for (auto &t : *vec) {
        if (!t.ptr) continue;
        if (t.device.is_cuda()) cudaFree(t.ptr);
        else std::free(t.ptr);
        t.ptr = nullptr;
      }
  }
  key_cache_.clear();
  value_cache_.clear();
}

PagedKvCache::PagedKvCache(PagedKvCache &&o) noexcept { *this = std::move(o); }
PagedKvCache &PagedKvCache::operator=(PagedKvCache &&o) noexcept {
  if (this != &o) {
    release();
    key_cache_ = std::move(o.key_cache_);
    value_cache_ = std::move(o.value_cache_);
    owns_ = o.owns_;
    o.owns_ = false;
    o.key_cache_.clear();
    o.value_cache_.clear();
    block_table_host_ = std::move(o.block_table_host_);
    block_size_ = o.block_size_;
    num_blocks_ = o.num_blocks_;
    num_blocks_per_sequence_ = o.num_blocks_per_sequence_;
    batch_size_ = o.batch_size_;
    max_tokens_per_sequence_ = o.max_tokens_per_sequence_;
    max_tokens_ = o.max_tokens_;
    num_kv_heads_ = o.num_kv_heads_;
    head_dim_ = o.head_dim_;
    dtype_ = o.dtype_;
  }
  return *this;
}
PagedKvCache::~PagedKvCache() { release(); }

size_t PagedKvCache::estimated_bytes() const {
  size_t n = 0;
  for (const auto *vec : {&key_cache_, &value_cache_})
    for (const auto &t : *vec) n += t.elem_count() * dtype_size_in_bytes(t.dtype);
  return n;
}

std::vector<size_t> PagedKvCache::key_dims() const {
  const size_t x = 16 / dtype_size_in_bytes(dtype_);
  return {num_blocks_, num_kv_heads_, head_dim_ / x, block_size_, x};
}
std::vector<size_t> PagedKvCache::value_dims() const {
  return {num_blocks_, num_kv_heads_, head_dim_, block_size_};
}

// --------------------------------------------------------------- slot math
int64_t PagedKvCache::slot_for_position(size_t position) const {
  return slot_for_sequence_position(0, position);
}

// paged_kv_cache.rs:356-378
int64_t PagedKvCache::slot_for_sequence_position(size_t sequence, size_t position) const {
  if (sequence >= batch_size_)
    bail("sequence exceeds paged kv cache batch: sequence=", sequence, " batch=", batch_size_);
  if (position >= max_tokens_per_sequence_)
    bail("position exceeds paged kv cache capacity: position=", position,
         " max_tokens_per_sequence=", max_tokens_per_sequence_);
  const size_t base = checked_mul(checked_mul(sequence, num_blocks_per_sequence_,
                                              "slot sequence base overflow"),
                                  block_size_, "slot sequence base overflow");
  return static_cast<int64_t>(base + position);
}

// paged_kv_cache.rs:380-399
std::vector<int64_t> PagedKvCache::slot_mapping_for_range(size_t start, size_t len) const {
  const size_t end = start + len;
  if (end < start) bail("slot range overflow");
  if (end > max_tokens_)
    bail("slot range exceeds paged kv cache capacity: start=", start, " len=", len,
         " max_tokens=", max_tokens_);
  std::vector<int64_t> out;
  out.reserve(len);
  for (size_t p = start; p < end; ++p) out.push_back(slot_for_position(p));
  return out;
}

// paged_kv_cache.rs:401-407
std::vector<std::vector<uint32_t>> PagedKvCache::block_tables_tensor() const {
  return {block_table_host_};
}

// paged_kv_cache.rs:409-424
std::vector<std::vector<uint32_t>> PagedKvCache::block_tables_tensor_for_batch(size_t batch) const {
  if (batch > batch_size_)
    bail("requested block table batch exceeds cache batch: requested=", batch,
         " cache_batch=", batch_size_);
  std::vector<std::vector<uint32_t>> out(batch);
  for (size_t b = 0; b < batch; ++b)
    out[b].assign(block_table_host_.begin() + b * num_blocks_per_sequence_,
                  block_table_host_.begin() + (b + 1) * num_blocks_per_sequence_);
  return out;
}

// paged_kv_cache.rs:426-437
std::vector<uint32_t> PagedKvCache::context_lens_tensor(size_t context_len) const {
  if (context_len > max_tokens_)
    bail("context length exceeds paged kv cache capacity: context_len=", context_len,
         " max_tokens=", max_tokens_);
  return {to_u32(context_len, "context length")};
}

// --------------------------------------------------------------- builders
// paged_kv_cache.rs:439-466
PagedInputMetadata PagedKvCache::input_metadata_for_range(size_t start, size_t len,
                                                          size_t context_len) const {
  PagedInputMetadata m;
  m.slot_mapping = slot_mapping_for_range(start, len);
  m.block_tables = block_table_host_;
  m.block_table_rows = 1;
  m.block_table_cols = num_blocks_;
  m.context_lens = context_lens_tensor(context_len);
  m.max_context_len = context_len;
  apply_varlen(m, std::vector<size_t>{len}, std::vector<size_t>{context_len});
  return m;
}

// paged_kv_cache.rs:468-545
PagedInputMetadata PagedKvCache::input_metadata_for_batch_ranges(
    const std::vector<size_t> &starts, size_t len, const std::vector<size_t> &context_lens) const {
  const size_t batch = starts.size();
  if (batch == 0) bail("paged metadata batch must be non-empty");
  if (context_lens.size() != batch)
    bail("context_lens batch mismatch: starts=", starts.size(),
         " context_lens=", context_lens.size());
  if (batch > batch_size_)
    bail("metadata batch exceeds cache batch: batch=", batch, " cache_batch=", batch_size_);
  PagedInputMetadata m;
  m.slot_mapping.reserve(batch * len);
  for (size_t seq = 0; seq < batch; ++seq) {
    const size_t end = starts[seq] + len;
    if (end > max_tokens_per_sequence_)
      bail("slot range exceeds paged kv cache sequence capacity: sequence=", seq,
           " start=", starts[seq], " len=", len,
           " max_tokens_per_sequence=", max_tokens_per_sequence_);
    for (size_t p = starts[seq]; p < end; ++p)
      m.slot_mapping.push_back(slot_for_sequence_position(seq, p));
  }
  for (size_t c : context_lens)
    if (c > max_tokens_per_sequence_)
      bail("context length exceeds paged kv cache sequence capacity: context_len=", c,
           " max_tokens_per_sequence=", max_tokens_per_sequence_);
  m.context_lens = context_u32(context_lens, &m.max_context_len);
  const auto tables = block_tables_tensor_for_batch(batch);
  m.block_table_rows = batch;
  m.block_table_cols = num_blocks_per_sequence_;
  for (const auto &r : tables) m.block_tables.insert(m.block_tables.end(), r.begin(), r.end());
  apply_varlen(m, std::vector<size_t>(batch, len), context_lens);
  return m;
}

// paged_kv_cache.rs:547-649
PagedInputMetadata PagedKvCache::input_metadata_from_block_tables(
    const std::vector<std::vector<size_t>> &block_tables, const std::vector<size_t> &starts,
    size_t len, const std::vector<size_t> &context_lens) const {
  const size_t batch = block_tables.size();
  if (batch == 0) bail("paged metadata batch must be non-empty");
  if (starts.size() != batch || context_lens.size() != batch)
    bail("paged metadata batch mismatch: block_tables=", batch, " starts=", starts.size(),
         " context_lens=", context_lens.size());
  const size_t max_blocks = max_len(block_tables);
  if (max_blocks == 0) bail("paged metadata requires at least one block per sequence");
  PagedInputMetadata m;
  m.slot_mapping.reserve(batch * len);
  for (size_t seq = 0; seq < batch; ++seq)
    for (size_t p = starts[seq]; p < starts[seq] + len; ++p)
      m.slot_mapping.push_back(
          slot_for_block_table_position(block_tables, block_size_, num_blocks_, seq, p));
  m.block_tables = pad_tables(block_tables, max_blocks);
  m.block_table_rows = batch;
  m.block_table_cols = max_blocks;
  m.context_lens = context_u32(context_lens, &m.max_context_len);
  apply_varlen(m, std::vector<size_t>(batch, len), context_lens);
  return m;
}

// paged_kv_cache.rs:651-773
PagedInputMetadata PagedKvCache::input_metadata_from_attention_masks(
    const std::vector<std::vector<size_t>> &block_tables,
    const std::vector<std::vector<uint32_t>> &attention_masks) const {
  const size_t batch = attention_masks.size();
  if (batch == 0) bail("paged metadata batch must be non-empty");
  if (block_tables.size() != batch)
    bail("paged metadata batch mismatch: block_tables=", block_tables.size(),
         " attention_masks=", batch);
  const size_t seq_len = attention_masks[0].size();
  if (seq_len == 0) bail("attention mask rows must be non-empty");
  const size_t max_blocks = max_len(block_tables);
  if (max_blocks == 0) bail("paged metadata requires at least one block per sequence");
  PagedInputMetadata m;
  std::vector<uint32_t> attn;
  std::vector<size_t> qlens;
  for (size_t seq = 0; seq < batch; ++seq) {
    const auto &row = attention_masks[seq];
    if (row.size() != seq_len)
      bail("attention_mask row len mismatch: expected=", seq_len, ", got=", row.size());
    size_t n = 0;
    for (size_t p = 0; p < seq_len; ++p) {
      attn.push_back(row[p]);
      if (row[p] == 0) {
        m.slot_mapping.push_back(PAD_SLOT_ID);
        continue;
      }
      m.slot_mapping.push_back(
          slot_for_block_table_position(block_tables, block_size_, num_blocks_, seq, p));
      ++n;
    }
    qlens.push_back(n);
  }
  m.block_tables = pad_tables(block_tables, max_blocks);
  m.block_table_rows = batch;
  m.block_table_cols = max_blocks;
  m.context_lens = context_u32(qlens, &m.max_context_len);
  m.token_attention_mask = std::move(attn);
  m.token_attention_mask_cols = seq_len;
  bool all_full = true;
  for (size_t n : qlens) all_full = all_full && n == seq_len;
  m.prefill_causal_only = all_full;
  apply_varlen(m, qlens, qlens);
  return m;
}

// paged_kv_cache.rs:775-869
PagedInputMetadata PagedKvCache::input_metadata_from_query_lens(
    const std::vector<std::vector<size_t>> &block_tables,
    const std::vector<size_t> &query_lens) const {
  const size_t batch = query_lens.size();
  if (batch == 0) bail("paged metadata batch must be non-empty");
  if (block_tables.size() != batch)
    bail("paged metadata batch mismatch: block_tables=", block_tables.size(),
         " query_lens=", batch);
  const size_t max_blocks = max_len(block_tables);
  if (max_blocks == 0) bail("paged metadata requires at least one block per sequence");
  size_t total = 0;
  for (size_t n : query_lens) {
    if (n == 0) bail("packed prefill query length must be non-zero");
    total += n;
  }
  PagedInputMetadata m;
  m.slot_mapping.reserve(total);
  for (size_t seq = 0; seq < batch; ++seq) {
    const size_t len = query_lens[seq];
    for (size_t p = 0; p < len; ++p)
      m.slot_mapping.push_back(
          slot_for_block_table_position(block_tables, block_size_, num_blocks_, seq, p));
    const size_t need = (len + block_size_ - 1) / block_size_;
    if (block_tables[seq].size() < need)
      bail("paged block table too short for packed prefill: seq=", seq, " len=", len,
           " have=", block_tables[seq].size(), " need=", need);
  }
  m.block_tables = pad_tables(block_tables, max_blocks);
  m.block_table_rows = batch;
  m.block_table_cols = max_blocks;
  m.context_lens = context_u32(query_lens, &m.max_context_len);
  m.prefill_causal_only = true;
  apply_varlen(m, query_lens, query_lens);
  return m;
}

// paged_kv_cache.rs:871-922
std::vector<PagedInputMetadata> PagedKvCache::decode_metadata_for_steps(size_t prompt_len,
                                                                        size_t steps) const {
  const size_t end = prompt_len + steps;
  if (end > max_tokens_)
    bail("decode metadata range exceeds paged kv cache capacity: prompt_len=", prompt_len,
         " steps=", steps, " max_tokens=", max_tokens_);
  std::vector<PagedInputMetadata> out;
  out.reserve(steps);
  for (size_t step = 0; step < steps; ++step) {
    PagedInputMetadata m;
    m.slot_mapping = {slot_for_position(prompt_len + step)};
    m.block_tables = block_table_host_;
    m.block_table_rows = 1;
    m.block_table_cols = num_blocks_;
    m.context_lens = {to_u32(prompt_len + step + 1, "context length")};
    m.max_context_len = prompt_len + step + 1;
    out.push_back(std::move(m));
  }
  return out;
}

// paged_kv_cache.rs:924-1044 (one step; shared by both batch builders)
PagedInputMetadata PagedKvCache::decode_metadata_for_batch_step(
    const std::vector<std::vector<size_t>> &block_tables, const std::vector<size_t> &prompt_lens,
    size_t step, bool cuda_graph) const {
  const size_t batch = block_tables.size();
  if (batch == 0) bail("paged batch decode metadata requires at least one sequence");
  if (prompt_lens.size() != batch)
    bail("paged batch decode metadata mismatch: block_tables=", batch,
         " prompt_lens=", prompt_lens.size());
  const size_t raw = max_len(block_tables);
  if (raw == 0) bail("paged batch decode metadata requires at least one block per sequence");
  const size_t width = cuda_graph ? bucket_block_table_cols(raw, block_size_) : raw;
  PagedInputMetadata m;
  m.block_tables = pad_tables(block_tables, width);
  m.block_table_rows = batch;
  m.block_table_cols = width;
  m.slot_mapping.reserve(batch);
  m.context_lens.reserve(batch);
  for (size_t seq = 0; seq < batch; ++seq) {
    const size_t position = prompt_lens[seq] + step;
    const size_t context_len = position + 1;
    if (context_len > max_tokens_per_sequence_)
      bail("batch decode context length exceeds paged kv cache sequence capacity: context_len=",
           context_len, " max_tokens_per_sequence=", max_tokens_per_sequence_);
    m.slot_mapping.push_back(
        slot_for_block_table_position(block_tables, block_size_, num_blocks_, seq, position));
    m.context_lens.push_back(to_u32(context_len, "context length"));
    m.max_context_len = std::max(m.max_context_len, context_len);
  }
  return m;
}

std::vector<PagedInputMetadata> PagedKvCache::decode_metadata_for_batch_steps(
    const std::vector<std::vector<size_t>> &block_tables, const std::vector<size_t> &prompt_lens,
    size_t steps, bool cuda_graph) const {
  if (block_tables.empty()) bail("paged batch decode metadata requires at least one sequence");
  if (prompt_lens.size() != block_tables.size())
    bail("paged batch decode metadata mismatch: block_tables=", block_tables.size(),
         " prompt_lens=", prompt_lens.size());
  if (max_len(block_tables) == 0)
    bail("paged batch decode metadata requires at least one block per sequence");
  std::vector<PagedInputMetadata> out;
  out.reserve(steps);
  for (size_t s = 0; s < steps; ++s)
    out.push_back(decode_metadata_for_batch_step(block_tables, prompt_lens, s, cuda_graph));
  return out;
}

// paged_kv_cache.rs:1061-1069
std::pair<const DeviceTensor &, const DeviceTensor &> PagedKvCache::key_value_cache(
    size_t layer_idx) const {
  if (layer_idx >= key_cache_.size()) bail("paged kv cache layer out of range: ", layer_idx);
  return {key_cache_[layer_idx], value_cache_[layer_idx]};
}

}  // namespace vasr_paged_attn

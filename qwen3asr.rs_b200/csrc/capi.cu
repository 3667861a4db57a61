// capi.cu — the extern "C" boundary declared in include/vasr_pa.h.
//
// Every entry point validates sizes, dtype, block size and pointer alignment
// on the host (mirroring the candle_core::bail! checks of
// vasr-paged-attn/src/paged_kv_cache.rs:241-272 and the block-size rule of
// paged_cache_runtime.rs:406-411) before anything is enqueued, then launches
// on the caller's stream. Nothing here allocates or synchronises.
#include <cuda_runtime.h>

#include <cstdint>

#include "launch.h"

namespace {

using vasr::AppendArgs;
using vasr::DecodeArgs;
using vasr::GatherArgs;
using vasr::PrefillArgs;

int elem_size(int32_t dtype) {
  switch (dtype) {
    case VASR_PA_F32: return 4;
    case VASR_PA_BF16: return 2;
    case VASR_PA_F16: return 2;
    default: return 0;
  }
}
bool block_size_ok(int32_t bs) { return bs == 8 || bs == 16 || bs == 32; }
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
cudaStream_t to_stream(vasr_pa_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Common cache-geometry checks shared by all page readers / writers.
int check_geometry(int32_t dtype, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                   int64_t num_blocks) {
  const int es = elem_size(dtype);
  if (es == 0) return VASR_PA_EINVAL_DTYPE;
  if (!block_size_ok(block_size)) return VASR_PA_EINVAL_BLOCKSIZE;
  if (num_kv_heads <= 0 || head_dim <= 0 || num_blocks <= 0) return VASR_PA_EINVAL_SHAPE;
  if (head_dim % (16 / es) != 0) return VASR_PA_EINVAL_SHAPE;  // key pack x must divide D
  return VASR_PA_OK;
}

}  // namespace

extern "C" {

int32_t vasr_pa_abi_version(void) { return VASR_PA_ABI_VERSION; }

const char *vasr_pa_status_string(int32_t status) {
  switch (status) {
    case VASR_PA_OK: return "ok";
    case VASR_PA_EINVAL_SHAPE: return "invalid shape";
    case VASR_PA_EINVAL_DTYPE: return "invalid dtype";
    case VASR_PA_EINVAL_BLOCKSIZE: return "paged cache block size must be 8, 16, or 32";
    case VASR_PA_EINVAL_ALIGN: return "pointer or stride not 16-byte aligned";
    case VASR_PA_EINVAL_WORKSPACE: return "workspace missing or too small";
    case VASR_PA_ENOT_SUPPORTED: return "configuration not supported by the sm_100a kernels";
    case VASR_PA_ELAUNCH: return "CUDA launch failed";
    case VASR_PA_EDEVICE: return "no usable CUDA device";
    case VASR_PA_EINVAL_POINTER: return "null or inaccessible pointer";
    case VASR_PA_ESCRATCH_LIMIT:
      return "sizes need more split-K scratch than the fixed 16 MiB no-alloc buffer holds";
    default: return "unknown status";
  }
}

int32_t vasr_pa_reshape_and_cache(const void *key, const void *value, void *key_cache,
                                  void *value_cache, const int64_t *slot_mapping,
                                  int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t block_size, int64_t num_blocks, int64_t key_token_stride,
                                  int64_t value_token_stride, int32_t dtype, const float *k_scale,
                                  const float *v_scale, vasr_pa_stream_t stream) {
  (void)k_scale;
  (void)v_scale;
  const int g = check_geometry(dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (num_tokens < 0) return VASR_PA_EINVAL_SHAPE;
  if (num_tokens == 0) return VASR_PA_OK;
  if (num_tokens > 0x7fffffffLL * 16) return VASR_PA_EINVAL_SHAPE;
  const int es = elem_size(dtype);
  if (key_token_stride < (int64_t)num_kv_heads * head_dim ||
      value_token_stride < (int64_t)num_kv_heads * head_dim)
    return VASR_PA_EINVAL_SHAPE;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping) return VASR_PA_EINVAL_POINTER;
  if (!aligned16(key) || !aligned16(value) || !aligned16(key_cache) || !aligned16(value_cache) ||
      (key_token_stride * es) % 16 != 0 || (value_token_stride * es) % 16 != 0 ||
      !aligned(slot_mapping, 8))
    return VASR_PA_EINVAL_ALIGN;
  AppendArgs a{key, value, key_cache, value_cache, slot_mapping, num_tokens, num_kv_heads,
               head_dim, block_size, num_blocks, key_token_stride, value_token_stride, dtype};
  return vasr::launch_append(a, to_stream(stream));
}

int32_t vasr_pa_reshape_and_cache_fp8(const void *key, const void *value, void *key_cache,
                                      void *value_cache, const int64_t *slot_mapping,
                                      int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                                      int32_t block_size, int64_t num_blocks,
                                      int64_t key_token_stride, int64_t value_token_stride,
                                      int32_t src_dtype, const float *k_scale, const float *v_scale,
                                      vasr_pa_stream_t stream) {
  const int es = elem_size(src_dtype);
  if (es == 0) return VASR_PA_EINVAL_DTYPE;
  if (!block_size_ok(block_size)) return VASR_PA_EINVAL_BLOCKSIZE;
  if (num_kv_heads <= 0 || head_dim <= 0 || num_blocks <= 0 || num_tokens < 0 ||
      head_dim % 16 != 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_tokens == 0) return VASR_PA_OK;
  if (key_token_stride < (int64_t)num_kv_heads * head_dim ||
      value_token_stride < (int64_t)num_kv_heads * head_dim)
    return VASR_PA_EINVAL_SHAPE;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping || !k_scale || !v_scale)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(key) || !aligned16(value) || !aligned16(key_cache) || !aligned16(value_cache) ||
      (key_token_stride * es) % 16 != 0 || (value_token_stride * es) % 16 != 0 ||
      !aligned(slot_mapping, 8) || !aligned(k_scale, 4) || !aligned(v_scale, 4))
    return VASR_PA_EINVAL_ALIGN;
  AppendArgs a{key, value, key_cache, value_cache, slot_mapping, num_tokens, num_kv_heads,
               head_dim, block_size, num_blocks, key_token_stride, value_token_stride, src_dtype,
               VASR_PA_FP8_E4M3, k_scale, v_scale};
  return vasr::launch_append(a, to_stream(stream));
}

int32_t vasr_pa_paged_attention_fp8(void *out, const void *query, const void *key_cache,
                                    const void *value_cache, const uint32_t *block_tables,
                                    const uint32_t *context_lens, int32_t num_seqs,
                                    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t block_size, int64_t num_blocks,
                                    int32_t max_num_blocks_per_seq, int32_t max_context_len,
                                    float scale, float softcapping, int64_t q_seq_stride,
                                    int32_t dtype, const float *k_scale, const float *v_scale,
                                    void *workspace, size_t workspace_bytes,
                                    vasr_pa_stream_t stream) {
  if (dtype != VASR_PA_BF16 && dtype != VASR_PA_F16) return VASR_PA_EINVAL_DTYPE;
  if (!block_size_ok(block_size)) return VASR_PA_EINVAL_BLOCKSIZE;
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_blocks <= 0 ||
      num_heads % num_kv_heads != 0 || head_dim % 16 != 0 || max_num_blocks_per_seq <= 0 ||
      max_context_len < 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0) return VASR_PA_OK;
  if (num_seqs > 65535 || num_kv_heads > 65535) return VASR_PA_EINVAL_SHAPE;
  if (q_seq_stride < (int64_t)num_heads * head_dim) return VASR_PA_EINVAL_SHAPE;
  if (!(softcapping > 0.f)) return VASR_PA_EINVAL_SHAPE;
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens || !k_scale ||
      !v_scale)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(query) || !aligned16(key_cache) || !aligned16(value_cache) ||
      (q_seq_stride * 2) % 16 != 0 || !aligned(out, 2) || !aligned(block_tables, 4) ||
      !aligned(context_lens, 4) || (workspace && !aligned(workspace, 256)) ||
      !aligned(k_scale, 4) || !aligned(v_scale, 4))
    return VASR_PA_EINVAL_ALIGN;
  DecodeArgs a{out, query, key_cache, value_cache, block_tables, context_lens, num_seqs,
               num_heads, num_kv_heads, head_dim, block_size, num_blocks, max_num_blocks_per_seq,
               max_context_len > 0 ? max_context_len : 1, scale, softcapping, q_seq_stride, dtype,
               workspace, workspace_bytes, VASR_PA_FP8_E4M3, k_scale, v_scale};
  return vasr::launch_decode(a, to_stream(stream));
}

size_t vasr_pa_paged_attention_workspace_size(int32_t num_seqs, int32_t num_heads,
                                              int32_t num_kv_heads, int32_t head_dim,
                                              int32_t block_size, int32_t max_context_len,
                                              int32_t dtype) {
  (void)dtype;
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      !block_size_ok(block_size) || num_heads % num_kv_heads != 0)
    return 0;
  const int ctx = max_context_len > 0 ? max_context_len : 1;
  return vasr::decode_workspace_layout(num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                       ctx)
      .total;
}

namespace {
int32_t paged_attention_impl(void *out, const void *query, const void *key_cache,
                             const void *value_cache, const uint32_t *block_tables,
                             const uint32_t *context_lens, int32_t num_seqs, int32_t num_heads,
                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                             int64_t num_blocks, int32_t max_num_blocks_per_seq,
                             int32_t max_context_len, float scale, float softcapping,
                             int64_t q_seq_stride, int32_t dtype, void *workspace,
                             size_t workspace_bytes, vasr_pa_stream_t stream, int overlap_append) {
  const int g = check_geometry(dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (num_seqs < 0 || num_heads <= 0 || num_heads % num_kv_heads != 0 ||
      max_num_blocks_per_seq <= 0 || max_context_len < 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0) return VASR_PA_OK;
  if (num_seqs > 65535 || num_kv_heads > 65535) return VASR_PA_EINVAL_SHAPE;
  if (q_seq_stride < (int64_t)num_heads * head_dim) return VASR_PA_EINVAL_SHAPE;
  if (!(softcapping > 0.f)) return VASR_PA_EINVAL_SHAPE;
  const int es = elem_size(dtype);
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(query) || !aligned16(key_cache) || !aligned16(value_cache) ||
      (q_seq_stride * es) % 16 != 0 || !aligned(out, es) || !aligned(block_tables, 4) ||
      !aligned(context_lens, 4) || (workspace && !aligned(workspace, 256)))
    return VASR_PA_EINVAL_ALIGN;
  DecodeArgs a{out, query, key_cache, value_cache, block_tables, context_lens, num_seqs,
               num_heads, num_kv_heads, head_dim, block_size, num_blocks, max_num_blocks_per_seq,
               max_context_len > 0 ? max_context_len : 1, scale, softcapping, q_seq_stride, dtype,
               workspace, workspace_bytes};
  a.overlap_append = overlap_append;
  return vasr::launch_decode(a, to_stream(stream));
}
}  // namespace

int32_t vasr_pa_paged_attention(void *out, const void *query, const void *key_cache,
                                const void *value_cache, const uint32_t *block_tables,
                                const uint32_t *context_lens, int32_t num_seqs, int32_t num_heads,
                                int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                int64_t num_blocks, int32_t max_num_blocks_per_seq,
                                int32_t max_context_len, float scale, float softcapping,
                                int64_t q_seq_stride, int32_t dtype, void *workspace,
                                size_t workspace_bytes, vasr_pa_stream_t stream) {
  return paged_attention_impl(out, query, key_cache, value_cache, block_tables, context_lens,
                              num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                              max_num_blocks_per_seq, max_context_len, scale, softcapping,
                              q_seq_stride, dtype, workspace, workspace_bytes, stream, 0);
}

int32_t vasr_pa_paged_attention_after_append(
    void *out, const void *query, const void *key_cache, const void *value_cache,
    const uint32_t *block_tables, const uint32_t *context_lens, int32_t num_seqs,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t num_blocks, int32_t max_num_blocks_per_seq, int32_t max_context_len, float scale,
    float softcapping, int64_t q_seq_stride, int32_t dtype, void *workspace,
    size_t workspace_bytes, vasr_pa_stream_t stream) {
  return paged_attention_impl(out, query, key_cache, value_cache, block_tables, context_lens,
                              num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                              max_num_blocks_per_seq, max_context_len, scale, softcapping,
                              q_seq_stride, dtype, workspace, workspace_bytes, stream, 1);
}

int32_t vasr_pa_gather_kv_cache(void *key_out, void *value_out, const void *key_cache,
                                const void *value_cache, const uint32_t *block_tables,
                                const uint32_t *cu_seqlens_kv, int32_t num_seqs,
                                int32_t max_num_blocks_per_seq, int64_t total_tokens,
                                int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                int64_t num_blocks, int32_t dtype, vasr_pa_stream_t stream) {
  const int g = check_geometry(dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (num_seqs < 0 || max_num_blocks_per_seq <= 0 || total_tokens < 0) return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0 || total_tokens == 0) return VASR_PA_OK;
  if (num_seqs > 65535) return VASR_PA_EINVAL_SHAPE;
  if (!key_out || !value_out || !key_cache || !value_cache || !block_tables || !cu_seqlens_kv)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(key_out) || !aligned16(value_out) || !aligned16(key_cache) ||
      !aligned16(value_cache) || !aligned(block_tables, 4) || !aligned(cu_seqlens_kv, 4))
    return VASR_PA_EINVAL_ALIGN;
  GatherArgs a{key_out, value_out, key_cache, value_cache, block_tables, cu_seqlens_kv, num_seqs,
               max_num_blocks_per_seq, total_tokens, num_kv_heads, head_dim, block_size,
               num_blocks, dtype};
  return vasr::launch_gather(a, to_stream(stream));
}

int32_t vasr_pa_gather_kv_cache_fp8(void *key_out, void *value_out, const void *key_cache,
                                    const void *value_cache, const uint32_t *block_tables,
                                    const uint32_t *cu_seqlens_kv, int32_t num_seqs,
                                    int32_t max_num_blocks_per_seq, int64_t total_tokens,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                    int64_t num_blocks, int32_t out_dtype, const float *k_scale,
                                    const float *v_scale, vasr_pa_stream_t stream) {
  const int g = check_geometry(out_dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (num_seqs < 0 || max_num_blocks_per_seq <= 0 || total_tokens < 0) return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0 || total_tokens == 0) return VASR_PA_OK;
  if (num_seqs > 65535) return VASR_PA_EINVAL_SHAPE;
  if (!key_out || !value_out || !key_cache || !value_cache || !block_tables || !cu_seqlens_kv ||
      !k_scale || !v_scale)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(key_out) || !aligned16(value_out) || !aligned16(key_cache) ||
      !aligned16(value_cache) || !aligned(block_tables, 4) || !aligned(cu_seqlens_kv, 4) ||
      !aligned(k_scale, 4) || !aligned(v_scale, 4))
    return VASR_PA_EINVAL_ALIGN;
  GatherArgs a{key_out, value_out, key_cache, value_cache, block_tables, cu_seqlens_kv, num_seqs,
               max_num_blocks_per_seq, total_tokens, num_kv_heads, head_dim, block_size,
               num_blocks, out_dtype};
  a.cache_dtype = VASR_PA_FP8_E4M3;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  return vasr::launch_gather(a, to_stream(stream));
}

int32_t vasr_pa_paged_attention_varlen_prefill(
    void *out, const void *query, const void *key_cache, const void *value_cache,
    const uint32_t *block_tables, const uint32_t *context_lens, const uint32_t *cu_seqlens_q,
    int32_t num_seqs, int64_t total_q_tokens, int32_t max_query_len, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int32_t max_num_blocks_per_seq, float scale, float softcapping, int64_t q_token_stride,
    int32_t dtype, vasr_pa_stream_t stream) {
  const int g = check_geometry(dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (num_seqs < 0 || total_q_tokens < 0 || max_query_len < 0 || num_heads <= 0 ||
      num_heads % num_kv_heads != 0 || max_num_blocks_per_seq <= 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0 || total_q_tokens == 0) return VASR_PA_OK;
  if (q_token_stride < (int64_t)num_heads * head_dim) return VASR_PA_EINVAL_SHAPE;
  if (!(softcapping > 0.f)) return VASR_PA_EINVAL_SHAPE;
  const int es = elem_size(dtype);
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens ||
      !cu_seqlens_q)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(query) || !aligned16(out) || !aligned16(key_cache) || !aligned16(value_cache) ||
      (q_token_stride * es) % 16 != 0 || !aligned(block_tables, 4) || !aligned(context_lens, 4) ||
      !aligned(cu_seqlens_q, 4))
    return VASR_PA_EINVAL_ALIGN;
  PrefillArgs a{out, query, key_cache, value_cache, block_tables, context_lens, cu_seqlens_q,
                num_seqs, total_q_tokens, max_query_len, num_heads, num_kv_heads, head_dim,
                block_size, num_blocks, max_num_blocks_per_seq, scale, softcapping,
                q_token_stride, dtype};
  return vasr::launch_prefill(a, to_stream(stream));
}

namespace {
struct PrefillFp8Layout {
  size_t off_k, off_v, off_table, total;
};
PrefillFp8Layout prefill_fp8_layout(int32_t num_seqs, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t block_size, int32_t cols) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t blocks = (size_t)num_seqs * (size_t)cols;
  const size_t pool = blocks * (size_t)num_kv_heads * head_dim * block_size * 2;
  PrefillFp8Layout l;
  l.off_k = 0;
  l.off_v = al(pool);
  l.off_table = al(l.off_v + pool);
  l.total = al(l.off_table + blocks * 4);
  return l;
}
}  // namespace

size_t vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size(int32_t num_seqs,
                                                                 int32_t num_kv_heads,
                                                                 int32_t head_dim,
                                                                 int32_t block_size,
                                                                 int32_t max_num_blocks_per_seq) {
  if (num_seqs <= 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      max_num_blocks_per_seq <= 0)
    return 0;
  return prefill_fp8_layout(num_seqs, num_kv_heads, head_dim, block_size, max_num_blocks_per_seq).total;
}

int32_t vasr_pa_paged_attention_varlen_prefill_fp8(
    void *out, const void *query, const void *key_cache, const void *value_cache,
    const uint32_t *block_tables, const uint32_t *context_lens, const uint32_t *cu_seqlens_q,
    int32_t num_seqs, int64_t total_q_tokens, int32_t max_query_len, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int32_t max_num_blocks_per_seq, float scale, float softcapping, int64_t q_token_stride,
    int32_t dtype, const float *k_scale, const float *v_scale, void *workspace,
    size_t workspace_bytes, vasr_pa_stream_t stream) {
  if (dtype != VASR_PA_BF16 && dtype != VASR_PA_F16) return VASR_PA_EINVAL_DTYPE;
  const int g = check_geometry(dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (num_seqs < 0 || total_q_tokens < 0 || max_query_len < 0 || num_heads <= 0 ||
      num_heads % num_kv_heads != 0 || max_num_blocks_per_seq <= 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0 || total_q_tokens == 0) return VASR_PA_OK;
  if (q_token_stride < (int64_t)num_heads * head_dim) return VASR_PA_EINVAL_SHAPE;
  if (!(softcapping > 0.f)) return VASR_PA_EINVAL_SHAPE;
  if (head_dim != 128 || num_seqs > 65535) return VASR_PA_ENOT_SUPPORTED;
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens ||
      !cu_seqlens_q || !k_scale || !v_scale)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned16(query) || !aligned16(out) || !aligned16(key_cache) || !aligned16(value_cache) ||
      (q_token_stride * 2) % 16 != 0 || !aligned(block_tables, 4) || !aligned(context_lens, 4) ||
      !aligned(cu_seqlens_q, 4) || !aligned(k_scale, 4) || !aligned(v_scale, 4))
    return VASR_PA_EINVAL_ALIGN;
  const PrefillFp8Layout l =
      prefill_fp8_layout(num_seqs, num_kv_heads, head_dim, block_size, max_num_blocks_per_seq);
  if (workspace == nullptr || workspace_bytes < l.total || !aligned16(workspace))
    return VASR_PA_EINVAL_WORKSPACE;
  const cudaStream_t st = to_stream(stream);
  // 16-token pages, head_dim 128, GQA 1 / 2 / 4: the tcgen05 prefill reads the
  // fp8 pages itself (converted to f16 on their way into shared memory); the
  // workspace is left untouched. Other shapes: dequantised pages in the
  // workspace, then the 16-bit prefill.
  {
    vasr::PrefillArgs f{out, query, key_cache, value_cache, block_tables, context_lens, cu_seqlens_q,
                        num_seqs, total_q_tokens, max_query_len, num_heads, num_kv_heads, head_dim,
                        block_size, num_blocks, max_num_blocks_per_seq, scale, softcapping,
                        q_token_stride, dtype};
    f.cache_dtype = VASR_PA_FP8_E4M3;
    f.k_scale = k_scale;
    f.v_scale = v_scale;
    const int32_t r = vasr::launch_prefill_umma(f, st);
    if (r != VASR_PA_ENOT_SUPPORTED) return r;
  }
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  vasr::DequantArgs d{key_cache, value_cache, block_tables, context_lens, num_seqs,
                      max_num_blocks_per_seq, num_kv_heads, head_dim, block_size, num_blocks,
                      dtype, k_scale, v_scale, ws + l.off_k, ws + l.off_v,
                      reinterpret_cast<uint32_t *>(ws + l.off_table)};
  const int32_t r = vasr::launch_dequant_pages(d, st);
  if (r != VASR_PA_OK) return r;
  vasr::PrefillArgs a{out, query, ws + l.off_k, ws + l.off_v,
                      reinterpret_cast<const uint32_t *>(ws + l.off_table), context_lens,
                      cu_seqlens_q, num_seqs, total_q_tokens, max_query_len, num_heads, num_kv_heads,
                      head_dim, block_size, (int64_t)num_seqs * max_num_blocks_per_seq,
                      max_num_blocks_per_seq, scale, softcapping, q_token_stride, dtype};
  return vasr::launch_prefill(a, st);
}

int32_t vasr_pa_copy_blocks(void *const *key_caches, void *const *value_caches,
                            int32_t num_layers, const int64_t *block_mapping, int64_t num_pairs,
                            int64_t num_blocks, int64_t block_bytes, vasr_pa_stream_t stream) {
  if (num_layers <= 0 || num_layers > 128 || num_pairs < 0 || num_blocks <= 0 ||
      block_bytes <= 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_pairs == 0) return VASR_PA_OK;
  if (num_pairs > 0x7fffffffLL) return VASR_PA_EINVAL_SHAPE;
  if (!key_caches || !value_caches || !block_mapping) return VASR_PA_EINVAL_POINTER;
  if (block_bytes % 16 != 0 || !aligned(block_mapping, 8)) return VASR_PA_EINVAL_ALIGN;
  for (int l = 0; l < num_layers; ++l) {
    if (!key_caches[l] || !value_caches[l]) return VASR_PA_EINVAL_POINTER;
    if (!aligned16(key_caches[l]) || !aligned16(value_caches[l])) return VASR_PA_EINVAL_ALIGN;
  }
  return vasr::launch_copy_blocks(key_caches, value_caches, num_layers, block_mapping, num_pairs,
                                  num_blocks, block_bytes, to_stream(stream));
}

int32_t vasr_pa_swap_blocks(void *dst, const void *src, const int64_t *block_mapping,
                            int64_t num_pairs, int64_t src_num_blocks, int64_t dst_num_blocks,
                            int64_t block_bytes, vasr_pa_stream_t stream) {
  if (num_pairs < 0 || src_num_blocks <= 0 || dst_num_blocks <= 0 || block_bytes <= 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_pairs == 0) return VASR_PA_OK;
  if (num_pairs > 0x7fffffffLL) return VASR_PA_EINVAL_SHAPE;
  if (!dst || !src || !block_mapping) return VASR_PA_EINVAL_POINTER;
  if (block_bytes % 16 != 0 || !aligned16(dst) || !aligned16(src) || !aligned(block_mapping, 8))
    return VASR_PA_EINVAL_ALIGN;
  // All three buffers must be reachable from the device: device memory or
  // page-locked host memory. Pageable host memory is rejected here.
  const void *ptrs[3] = {dst, src, block_mapping};
  for (const void *p : ptrs) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
      cudaGetLastError();
      return VASR_PA_EINVAL_POINTER;
    }
    if (attr.type == cudaMemoryTypeUnregistered) return VASR_PA_EINVAL_POINTER;
    if (attr.type == cudaMemoryTypeHost && attr.devicePointer != p) return VASR_PA_EINVAL_POINTER;
  }
  return vasr::launch_swap_blocks(dst, src, block_mapping, num_pairs, src_num_blocks,
                                  dst_num_blocks, block_bytes, to_stream(stream));
}

int32_t vasr_pa_fused_qk_norm_rope_append(
    void *q_out, const void *qkv, int64_t qkv_token_stride, const void *q_norm_weight,
    const void *k_norm_weight, float eps, const float *cos_table, const float *sin_table,
    int64_t max_position, const int64_t *positions, void *key_cache, void *value_cache,
    const int64_t *slot_mapping, int64_t num_tokens, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t block_size, int64_t num_blocks, int32_t dtype,
    vasr_pa_stream_t stream) {
  const int g = check_geometry(dtype, num_kv_heads, head_dim, block_size, num_blocks);
  if (g != VASR_PA_OK) return g;
  if (dtype == VASR_PA_F32 || head_dim != 128) return VASR_PA_ENOT_SUPPORTED;
  if (num_tokens < 0 || num_heads <= 0 || max_position <= 0) return VASR_PA_EINVAL_SHAPE;
  if (num_tokens == 0) return VASR_PA_OK;
  if (qkv_token_stride < (int64_t)(num_heads + 2 * num_kv_heads) * head_dim)
    return VASR_PA_EINVAL_SHAPE;
  if (!q_out || !qkv || !q_norm_weight || !k_norm_weight || !cos_table || !sin_table ||
      !positions || !key_cache || !value_cache || !slot_mapping)
    return VASR_PA_EINVAL_POINTER;
  if (!aligned(qkv, 4) || (qkv_token_stride % 2) != 0 || !aligned(q_out, 4) ||
      !aligned(q_norm_weight, 4) || !aligned(k_norm_weight, 4) || !aligned(cos_table, 8) ||
      !aligned(sin_table, 8) || !aligned(positions, 8) || !aligned(slot_mapping, 8) ||
      !aligned16(key_cache) || !aligned16(value_cache))
    return VASR_PA_EINVAL_ALIGN;
  vasr::FusedRopeArgs a{q_out, qkv, qkv_token_stride, q_norm_weight, k_norm_weight, eps,
                        cos_table, sin_table, max_position, positions, key_cache, value_cache,
                        slot_mapping, num_tokens, num_heads, num_kv_heads, head_dim, block_size,
                        num_blocks, dtype};
  return vasr::launch_fused_rope(a, to_stream(stream));
}

int32_t vasr_pa_decode_step_prepare(
    const uint32_t *next_ids, const uint32_t *eos_ids, int32_t num_eos,
    const uint32_t *prompt_lens, const uint32_t *step, const uint32_t *block_tables,
    const uint32_t *block_table_lens, int32_t max_num_blocks_per_seq, int32_t block_size,
    int64_t num_blocks, int32_t num_seqs, uint8_t *finished, uint32_t *generated,
    uint32_t *history, int32_t history_cols, int64_t *input_ids, int64_t *positions,
    int64_t *slot_mapping, uint32_t *context_lens, vasr_pa_stream_t stream) {
  if (num_seqs < 0 || num_eos < 0 || max_num_blocks_per_seq <= 0 || block_size <= 0 ||
      num_blocks <= 0 || history_cols < 0)
    return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0) return VASR_PA_OK;
  if (!next_ids || (num_eos > 0 && !eos_ids) || !prompt_lens || !step || !block_tables ||
      !finished || !input_ids || !positions || !slot_mapping || !context_lens ||
      (history && (!generated || history_cols == 0)))
    return VASR_PA_EINVAL_POINTER;
  if (!aligned(next_ids, 4) || !aligned(eos_ids, 4) || !aligned(prompt_lens, 4) ||
      !aligned(step, 4) || !aligned(block_tables, 4) || !aligned(block_table_lens, 4) ||
      !aligned(generated, 4) || !aligned(history, 4) || !aligned(input_ids, 8) ||
      !aligned(positions, 8) || !aligned(slot_mapping, 8) || !aligned(context_lens, 4))
    return VASR_PA_EINVAL_ALIGN;
  vasr::DecodeStepArgs a{next_ids,  eos_ids,   num_eos,      prompt_lens,  step,
                         block_tables, block_table_lens, max_num_blocks_per_seq, block_size,
                         num_blocks, num_seqs,  finished,     generated,    history,
                         history_cols, input_ids, positions,  slot_mapping, context_lens};
  return vasr::launch_decode_step_prepare(a, to_stream(stream));
}

size_t vasr_pa_greedy_argmax_workspace_size(int32_t num_seqs, int64_t vocab) {
  if (num_seqs <= 0 || vocab <= 0) return 0;
  return vasr::argmax_workspace_bytes(num_seqs, vocab);
}

int32_t vasr_pa_greedy_argmax(uint32_t *next_ids, const void *logits, int32_t num_seqs,
                              int64_t vocab, int64_t row_stride, int32_t dtype,
                              const uint8_t *finished, uint32_t *step, void *workspace,
                              size_t workspace_bytes, vasr_pa_stream_t stream) {
  if (dtype != VASR_PA_F32 && dtype != VASR_PA_BF16 && dtype != VASR_PA_F16)
    return VASR_PA_EINVAL_DTYPE;
  if (num_seqs < 0 || num_seqs > 65535 || vocab <= 0 || vocab > 0xfffffffeLL ||
      row_stride < vocab)
    return VASR_PA_EINVAL_SHAPE;
  if (num_seqs == 0) return VASR_PA_OK;
  if (!next_ids || !logits || !workspace) return VASR_PA_EINVAL_POINTER;
  if (workspace_bytes < vasr::argmax_workspace_bytes(num_seqs, vocab))
    return VASR_PA_EINVAL_WORKSPACE;
  if (!aligned(next_ids, 4) || !aligned(logits, elem_size(dtype)) || !aligned(step, 4) ||
      !aligned(workspace, 256))
    return VASR_PA_EINVAL_ALIGN;
  vasr::ArgmaxArgs a{};
  a.next_ids = next_ids;
  a.logits = logits;
  a.num_seqs = num_seqs;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.dtype = dtype;
  a.finished = finished;
  a.step = step;
  return vasr::launch_greedy_argmax(a, workspace, to_stream(stream));
}

int32_t vasr_pa_get_device_error(int32_t *out_bits, int32_t clear, vasr_pa_stream_t stream) {
  if (!out_bits) return VASR_PA_EINVAL_POINTER;
  uint32_t a = 0, b = 0, c = 0, d = 0, e = 0;
  int r;
  if ((r = vasr::read_error_kv_ops(&a, clear != 0, to_stream(stream))) != VASR_PA_OK) return r;
  if ((r = vasr::read_error_decode(&b, clear != 0, to_stream(stream))) != VASR_PA_OK) return r;
  if ((r = vasr::read_error_prefill(&c, clear != 0, to_stream(stream))) != VASR_PA_OK) return r;
  if ((r = vasr::read_error_fused(&d, clear != 0, to_stream(stream))) != VASR_PA_OK) return r;
  if ((r = vasr::read_error_prefill_umma(&e, clear != 0, to_stream(stream))) != VASR_PA_OK)
    return r;
  uint32_t f = 0;
  if ((r = vasr::read_error_decode_loop(&f, clear != 0, to_stream(stream))) != VASR_PA_OK) return r;
  *out_bits = (int32_t)(a | b | c | d | e | f);
  return VASR_PA_OK;
}

}  // extern "C"

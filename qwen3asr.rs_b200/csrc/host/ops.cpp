// ops.cpp — C++ mistralrs_paged_attn entry points over the C ABI.
// The argument order is the one thinker_text.rs uses (:1101-1139, :190-198);
// each function checks the tensor views like the Rust shim would and calls
// the matching vasr_pa_* function. Nothing here allocates.
#include <sstream>

#include "vasr_paged_attn.hpp"

namespace vasr_paged_attn {
namespace mistralrs_paged_attn {

namespace {
template <typename... A>
[[noreturn]] void bail(A &&...parts) {
  std::ostringstream os;
  (os << ... << parts);
  throw Error(os.str());
}
void check(int32_t st, const char *what) {
  if (st != VASR_PA_OK) bail(what, ": ", vasr_pa_status_string(st), " (status ", st, ")");
}
struct Geo {
  size_t nb, hkv, d, bs;
};
Geo geometry(const DeviceTensor &k, const DeviceTensor &v) {
  if (k.dims.size() != 5 || v.dims.size() != 4) bail("paged cache dims mismatch");
  if (k.dims[0] != v.dims[0] || k.dims[1] != v.dims[1] || k.dims[3] != v.dims[3] ||
      k.dims[2] * k.dims[4] != v.dims[2] || k.dtype != v.dtype)
    bail("paged cache shape mismatch for key/value caches");
  return {v.dims[0], v.dims[1], v.dims[2], v.dims[3]};
}
int32_t code(DType d) { return static_cast<int32_t>(d); }
}  // namespace

void reshape_and_cache(const DeviceTensor &key, const DeviceTensor &value,
                       const DeviceTensor *k_scale, const DeviceTensor *v_scale,
                       const DeviceTensor &key_cache, const DeviceTensor &value_cache,
                       const DeviceTensor &slot_mapping, vasr_pa_stream_t stream) {
  const Geo g = geometry(key_cache, value_cache);
  if (key.dims.size() != 3 || key.dims != value.dims || key.dims[1] != g.hkv || key.dims[2] != g.d)
    bail("reshape_and_cache: key/value must be [T, ", g.hkv, ", ", g.d, "]");
  if (slot_mapping.dims.size() != 1 || slot_mapping.dims[0] != key.dims[0])
    bail("reshape_and_cache: slot_mapping must be [T]");
  check(vasr_pa_reshape_and_cache(
            key.ptr, value.ptr, key_cache.ptr, value_cache.ptr,
            static_cast<const int64_t *>(slot_mapping.ptr), (int64_t)key.dims[0], (int32_t)g.hkv,
            (int32_t)g.d, (int32_t)g.bs, (int64_t)g.nb, (int64_t)(g.hkv * g.d),
            (int64_t)(g.hkv * g.d), code(key.dtype),
            k_scale ? static_cast<const float *>(k_scale->ptr) : nullptr,
            v_scale ? static_cast<const float *>(v_scale->ptr) : nullptr, stream),
        "reshape_and_cache");
}

size_t paged_attention_workspace_bytes(const DeviceTensor &q, const DeviceTensor &key_cache,
                                       size_t max_context_len) {
  if (q.dims.size() != 3 || key_cache.dims.size() != 5) bail("paged_attention: bad dims");
  return vasr_pa_paged_attention_workspace_size(
      (int32_t)q.dims[0], (int32_t)q.dims[1], (int32_t)key_cache.dims[1], (int32_t)q.dims[2],
      (int32_t)key_cache.dims[3], (int32_t)max_context_len, code(q.dtype));
}

void paged_attention(const DeviceTensor &out, const DeviceTensor &q, const DeviceTensor *k_scale,
                     const DeviceTensor *v_scale, const DeviceTensor &key_cache,
                     const DeviceTensor &value_cache, const DeviceTensor &block_tables,
                     const DeviceTensor &context_lens, const DeviceTensor *alibi,
                     size_t max_context_len, float softmax_scale, float softcapping,
                     const DeviceTensor *sinks, void *workspace, size_t workspace_bytes,
                     vasr_pa_stream_t stream) {
  (void)k_scale;
  (void)v_scale;
  if (alibi || sinks) bail("paged_attention: alibi / sinks are not supported");
  const Geo g = geometry(key_cache, value_cache);
  if (q.dims.size() != 3 || q.dims[2] != g.d || out.dims != q.dims)
    bail("paged_attention: q/out must be [B, Hq, ", g.d, "]");
  if (block_tables.dims.size() != 2 || block_tables.dims[0] != q.dims[0] ||
      context_lens.dims.size() != 1 || context_lens.dims[0] != q.dims[0])
    bail("paged_attention: block_tables [B, cols] / context_lens [B] mismatch");
  check(vasr_pa_paged_attention(
            out.ptr, q.ptr, key_cache.ptr, value_cache.ptr,
            static_cast<const uint32_t *>(block_tables.ptr),
            static_cast<const uint32_t *>(context_lens.ptr), (int32_t)q.dims[0],
            (int32_t)q.dims[1], (int32_t)g.hkv, (int32_t)g.d, (int32_t)g.bs, (int64_t)g.nb,
            (int32_t)block_tables.dims[1], (int32_t)max_context_len, softmax_scale, softcapping,
            (int64_t)(q.dims[1] * q.dims[2]), code(q.dtype), workspace, workspace_bytes, stream),
        "paged_attention");
}

void gather_kv_cache(const DeviceTensor &key_out, const DeviceTensor &value_out,
                     const DeviceTensor &key_cache, const DeviceTensor &value_cache,
                     const DeviceTensor *k_scale, const DeviceTensor *v_scale,
                     const DeviceTensor &block_tables, const DeviceTensor &cu_seqlens_kv,
                     vasr_pa_stream_t stream) {
  (void)k_scale;
  (void)v_scale;
  const Geo g = geometry(key_cache, value_cache);
  if (key_out.dims.size() != 3 || key_out.dims != value_out.dims)
    bail("gather_kv_cache: outputs must be [sum kv, Hkv, D]");
  if (block_tables.dims.size() != 2 || cu_seqlens_kv.dims.size() != 1 ||
      cu_seqlens_kv.dims[0] != block_tables.dims[0] + 1)
    bail("gather_kv_cache: cu_seqlens_kv must be [B + 1]");
  check(vasr_pa_gather_kv_cache(key_out.ptr, value_out.ptr, key_cache.ptr, value_cache.ptr,
                                static_cast<const uint32_t *>(block_tables.ptr),
                                static_cast<const uint32_t *>(cu_seqlens_kv.ptr),
                                (int32_t)block_tables.dims[0], (int32_t)block_tables.dims[1],
                                (int64_t)key_out.dims[0], (int32_t)g.hkv, (int32_t)g.d,
                                (int32_t)g.bs, (int64_t)g.nb, code(key_cache.dtype), stream),
        "gather_kv_cache");
}

void copy_blocks(const std::vector<DeviceTensor> &key_caches,
                 const std::vector<DeviceTensor> &value_caches, const DeviceTensor &block_mapping,
                 vasr_pa_stream_t stream) {
  if (key_caches.empty() || key_caches.size() != value_caches.size())
    bail("copy_blocks: one K and one V cache per layer");
  const Geo g = geometry(key_caches[0], value_caches[0]);
  std::vector<void *> k, v;
  for (size_t l = 0; l < key_caches.size(); ++l) {
    const Geo gl = geometry(key_caches[l], value_caches[l]);
    if (gl.nb != g.nb || gl.hkv != g.hkv || gl.d != g.d || gl.bs != g.bs)
      bail("copy_blocks: all layers must share one cache geometry");
    k.push_back(key_caches[l].ptr);
    v.push_back(value_caches[l].ptr);
  }
  if (block_mapping.dims.size() != 2 || block_mapping.dims[1] != 2)
    bail("copy_blocks: block_mapping must be [N, 2]");
  const size_t block_bytes = g.hkv * g.d * g.bs * dtype_size_in_bytes(key_caches[0].dtype);
  check(vasr_pa_copy_blocks(k.data(), v.data(), (int32_t)k.size(),
                            static_cast<const int64_t *>(block_mapping.ptr),
                            (int64_t)block_mapping.dims[0], (int64_t)g.nb, (int64_t)block_bytes,
                            stream),
        "copy_blocks");
}

void swap_blocks(const DeviceTensor &src, const DeviceTensor &dst,
                 const DeviceTensor &block_mapping, vasr_pa_stream_t stream) {
  if (src.dims.empty() || dst.dims.empty() || src.dtype != dst.dtype ||
      std::vector<size_t>(src.dims.begin() + 1, src.dims.end()) !=
          std::vector<size_t>(dst.dims.begin() + 1, dst.dims.end()))
    bail("swap_blocks: caches differ in geometry");
  const size_t block_bytes = src.elem_count() / src.dims[0] * dtype_size_in_bytes(src.dtype);
  check(vasr_pa_swap_blocks(dst.ptr, src.ptr, static_cast<const int64_t *>(block_mapping.ptr),
                            (int64_t)block_mapping.dims[0], (int64_t)src.dims[0],
                            (int64_t)dst.dims[0], (int64_t)block_bytes, stream),
        "swap_blocks");
}

}  // namespace mistralrs_paged_attn
}  // namespace vasr_paged_attn

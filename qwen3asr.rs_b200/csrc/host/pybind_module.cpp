// pybind_module.cpp — Python binding `_vasr_host` of the C++ host mirror.
// Exposes the vasr-paged-attn types with their Rust method names so the
// Python tests read like the reference's Rust tests.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "vasr_paged_attn.hpp"

namespace py = pybind11;
using namespace vasr_paged_attn;

namespace {

DType parse_dtype(const std::string &s) {
  if (s == "f32" || s == "float32") return DType::F32;
  if (s == "bf16" || s == "bfloat16") return DType::BF16;
  if (s == "f16" || s == "float16") return DType::F16;
  throw Error("unsupported paged kv cache dtype: " + s);
}

Device parse_device(int ordinal) { return ordinal < 0 ? Device::cpu() : Device::cuda(ordinal); }

py::list rows(const std::vector<uint32_t> &flat, size_t r, size_t c) {
  py::list out;
  for (size_t i = 0; i < r; ++i) {
    py::list row;
    for (size_t j = 0; j < c; ++j) row.append(flat[i * c + j]);
    out.append(row);
  }
  return out;
}

DeviceTensor tensor_view(uintptr_t ptr, std::vector<size_t> dims, const std::string &dtype,
                         int device) {
  DeviceTensor t;
  t.ptr = reinterpret_cast<void *>(ptr);
  t.dims = std::move(dims);
  t.dtype = parse_dtype(dtype);
  t.device = parse_device(device);
  return t;
}

}  // namespace

PYBIND11_MODULE(_vasr_host, m) {
  m.doc() = "C++ host mirror of the vasr-paged-attn crate (metadata, allocator, graph keys)";
  static py::exception<Error> exc(m, "VasrHostError", PyExc_ValueError);
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const Error &e) {
      exc(e.what());
    }
  });
  m.attr("PAD_SLOT_ID") = PAD_SLOT_ID;

  py::class_<FlashParams>(m, "FlashParams")
      .def_readonly("max_q", &FlashParams::max_q)
      .def_readonly("causal", &FlashParams::causal)
      .def_readonly("cumulative_seqlens_q", &FlashParams::cumulative_seqlens_q)
      .def_property_readonly("max_k", [](const FlashParams &f) { return f.logical_k.max; })
      .def_property_readonly("cumulative_seqlens_k",
                             [](const FlashParams &f) { return f.logical_k.cumulative_seqlens; });

  py::class_<PagedInputMetadata>(m, "PagedInputMetadata")
      .def_readonly("slot_mapping", &PagedInputMetadata::slot_mapping)
      .def_property_readonly("block_tables",
                             [](const PagedInputMetadata &x) {
                               return rows(x.block_tables, x.block_table_rows, x.block_table_cols);
                             })
      .def_readonly("block_tables_flat", &PagedInputMetadata::block_tables)
      .def_readonly("block_table_cols", &PagedInputMetadata::block_table_cols)
      .def_readonly("context_lens", &PagedInputMetadata::context_lens)
      .def_readonly("max_context_len", &PagedInputMetadata::max_context_len)
      .def_property_readonly("token_attention_mask",
                             [](const PagedInputMetadata &x) -> py::object {
                               if (!x.token_attention_mask) return py::none();
                               return rows(*x.token_attention_mask, x.block_table_rows,
                                           x.token_attention_mask_cols);
                             })
      .def_readonly("prefill_causal_only", &PagedInputMetadata::prefill_causal_only)
      .def_readonly("query_lens", &PagedInputMetadata::query_lens)
      .def_readonly("kv_lens", &PagedInputMetadata::kv_lens)
      .def_readonly("cu_seqlens_q", &PagedInputMetadata::cu_seqlens_q)
      .def_readonly("cu_seqlens_kv", &PagedInputMetadata::cu_seqlens_kv)
      .def_readonly("max_query_len", &PagedInputMetadata::max_query_len)
      .def_readonly("max_kv_len", &PagedInputMetadata::max_kv_len)
      .def("prefill_flash_params", &PagedInputMetadata::prefill_flash_params)
      .def("flash_params", &PagedInputMetadata::flash_params);

  py::class_<PagedKvCache>(m, "PagedKvCache")
      .def_static("new",
                  [](size_t l, size_t h, size_t d, size_t bs, size_t mt, const std::string &dt,
                     int dev) { return PagedKvCache::create(l, h, d, bs, mt, parse_dtype(dt), parse_device(dev)); },
                  py::arg("num_layers"), py::arg("num_kv_heads"), py::arg("head_dim"),
                  py::arg("block_size"), py::arg("max_tokens"), py::arg("dtype"), py::arg("device") = -1)
      .def_static("new_batched",
                  [](size_t l, size_t h, size_t d, size_t bs, size_t b, size_t mt,
                     const std::string &dt, int dev) {
                    return PagedKvCache::new_batched(l, h, d, bs, b, mt, parse_dtype(dt), parse_device(dev));
                  },
                  py::arg("num_layers"), py::arg("num_kv_heads"), py::arg("head_dim"),
                  py::arg("block_size"), py::arg("batch_size"), py::arg("max_tokens_per_sequence"),
                  py::arg("dtype"), py::arg("device") = -1)
      .def_static("new_pool",
                  [](size_t l, size_t h, size_t d, size_t bs, size_t nb, const std::string &dt,
                     int dev) { return PagedKvCache::new_pool(l, h, d, bs, nb, parse_dtype(dt), parse_device(dev)); },
                  py::arg("num_layers"), py::arg("num_kv_heads"), py::arg("head_dim"),
                  py::arg("block_size"), py::arg("num_blocks"), py::arg("dtype"), py::arg("device") = -1)
      .def_static("from_external",
                  [](const std::vector<uintptr_t> &kptrs, const std::vector<uintptr_t> &vptrs,
                     size_t num_blocks, size_t hkv, size_t d, size_t bs, const std::string &dt,
                     int dev) {
                    // Wrap caller-owned pages (e.g. torch tensors); null pointers give a
                    // geometry-only cache for the host metadata builders.
                    const DType t = parse_dtype(dt);
                    const size_t x = 16 / dtype_size_in_bytes(t);
                    std::vector<DeviceTensor> ks, vs;
                    for (size_t l = 0; l < kptrs.size(); ++l) {
                      ks.push_back(tensor_view(kptrs[l], {num_blocks, hkv, d / x, bs, x}, dt, dev));
                      vs.push_back(tensor_view(l < vptrs.size() ? vptrs[l] : 0, {num_blocks, hkv, d, bs}, dt, dev));
                    }
                    return PagedKvCache::from_external(std::move(ks), std::move(vs), bs);
                  },
                  py::arg("key_ptrs"), py::arg("value_ptrs"), py::arg("num_blocks"),
                  py::arg("num_kv_heads"), py::arg("head_dim"), py::arg("block_size"),
                  py::arg("dtype"), py::arg("device") = -1)
      .def_property_readonly("block_size", &PagedKvCache::block_size)
      .def_property_readonly("num_blocks", &PagedKvCache::num_blocks)
      .def_property_readonly("num_blocks_per_sequence", &PagedKvCache::num_blocks_per_sequence)
      .def_property_readonly("batch_size", &PagedKvCache::batch_size)
      .def_property_readonly("max_tokens_per_sequence", &PagedKvCache::max_tokens_per_sequence)
      .def_property_readonly("max_tokens", &PagedKvCache::max_tokens)
      .def_property_readonly("key_shape", &PagedKvCache::key_dims)
      .def_property_readonly("value_shape", &PagedKvCache::value_dims)
      .def("estimated_bytes", &PagedKvCache::estimated_bytes)
      .def("block_table_host", &PagedKvCache::block_table_host)
      .def("slot_for_position", &PagedKvCache::slot_for_position)
      .def("slot_for_sequence_position", &PagedKvCache::slot_for_sequence_position)
      .def("slot_mapping_for_range", &PagedKvCache::slot_mapping_for_range)
      .def("block_tables_tensor", &PagedKvCache::block_tables_tensor)
      .def("block_tables_tensor_for_batch", &PagedKvCache::block_tables_tensor_for_batch)
      .def("context_lens_tensor", &PagedKvCache::context_lens_tensor)
      .def("input_metadata_for_range", &PagedKvCache::input_metadata_for_range)
      .def("input_metadata_for_batch_ranges", &PagedKvCache::input_metadata_for_batch_ranges)
      .def("input_metadata_from_block_tables", &PagedKvCache::input_metadata_from_block_tables)
      .def("input_metadata_from_attention_masks", &PagedKvCache::input_metadata_from_attention_masks)
      .def("input_metadata_from_query_lens", &PagedKvCache::input_metadata_from_query_lens)
      .def("decode_metadata_for_steps", &PagedKvCache::decode_metadata_for_steps)
      .def("decode_metadata_for_batch_steps", &PagedKvCache::decode_metadata_for_batch_steps,
           py::arg("block_tables"), py::arg("prompt_lens"), py::arg("steps"), py::arg("cuda_graph") = false)
      .def("decode_metadata_for_batch_step", &PagedKvCache::decode_metadata_for_batch_step,
           py::arg("block_tables"), py::arg("prompt_lens"), py::arg("step"), py::arg("cuda_graph") = false)
      .def("key_value_cache_ptrs", [](const PagedKvCache &c, size_t layer) {
        auto kv = c.key_value_cache(layer);
        return py::make_tuple(reinterpret_cast<uintptr_t>(kv.first.ptr),
                              reinterpret_cast<uintptr_t>(kv.second.ptr));
      });

  py::class_<PagedBlockManager>(m, "PagedBlockManager")
      .def(py::init<size_t, size_t>(), py::arg("num_blocks"), py::arg("block_size"))
      .def_property_readonly("block_size", &PagedBlockManager::block_size)
      .def("free_blocks", &PagedBlockManager::free_blocks)
      .def("slots_available_for", &PagedBlockManager::slots_available_for)
      .def("blocks_for_request", &PagedBlockManager::blocks_for_request)
      .def("total_allocated_blocks", &PagedBlockManager::total_allocated_blocks)
      .def_static("allocatable_block_capacity", &PagedBlockManager::allocatable_block_capacity)
      .def("allocate_slots", &PagedBlockManager::allocate_slots)
      .def("try_allocate_slots", &PagedBlockManager::try_allocate_slots)
      .def("trim_request_to_num_tokens", &PagedBlockManager::trim_request_to_num_tokens)
      .def("block_ids", &PagedBlockManager::block_ids)
      .def("free_request", &PagedBlockManager::free_request)
      .def("free_many", &PagedBlockManager::free_many)
      .def("block_tables_for", &PagedBlockManager::block_tables_for);

  m.def("can_admit_with_projected_kv", &can_admit_with_projected_kv);
  m.def("bytes_per_paged_block",
        [](size_t l, size_t h, size_t d, size_t bs, size_t dtype_bytes) {
          return bytes_per_paged_block(l, h, d, bs, dtype_bytes == 4 ? DType::F32 : DType::BF16);
        });
  m.def("blocks_for_byte_budget", &blocks_for_byte_budget);
  m.def("cuda_graph_batch_bucket", &cuda_graph_batch_bucket);
  m.def("cuda_graph_batch_buckets", &cuda_graph_batch_buckets);
  m.def("cuda_graph_block_bucket", &cuda_graph_block_bucket);
  m.def("bucket_block_table_cols", &bucket_block_table_cols);
  m.def("cuda_graph_prewarm_batch_limit", &cuda_graph_prewarm_batch_limit);
  m.def("pad_decode_batch_to_max",
        [](size_t max_batch, const std::vector<int64_t> &ids, const std::vector<int64_t> &slots,
           const std::vector<uint32_t> &ctx, const std::vector<std::vector<uint32_t>> &tables,
           size_t cols) {
          PagedInputMetadata meta;
          meta.slot_mapping = slots;
          meta.context_lens = ctx;
          size_t mc = 0;
          for (const auto &r : tables) mc = std::max(mc, r.size());
          meta.block_table_rows = tables.size();
          meta.block_table_cols = mc;
          for (const auto &r : tables) {
            meta.block_tables.insert(meta.block_tables.end(), r.begin(), r.end());
            meta.block_tables.resize(meta.block_tables.size() + (mc - r.size()), r.empty() ? 0 : r.back());
          }
          auto p = pad_decode_batch_to_max(max_batch, ids, meta, cols);
          return py::make_tuple(p.input_ids, p.metadata.slot_mapping, p.metadata.context_lens,
                                rows(p.metadata.block_tables, p.metadata.block_table_rows,
                                     p.metadata.block_table_cols));
        });

  py::class_<DecodeGraphRegistry>(m, "DecodeGraphRegistry")
      .def(py::init<size_t, size_t>(), py::arg("block_size"), py::arg("max_batch"))
      .def("key",
           [](const DecodeGraphRegistry &r, size_t b, size_t c) {
             auto k = r.key(b, c);
             return py::make_tuple(k.batch, k.block_table_cols);
           })
      .def("enabled", &DecodeGraphRegistry::enabled)
      .def("enabled_for", &DecodeGraphRegistry::enabled_for)
      .def("disable_for", &DecodeGraphRegistry::disable_for)
      .def("disable_all", &DecodeGraphRegistry::disable_all);

  py::class_<PagedCacheStats>(m, "PagedCacheStats")
      .def_readonly("block_size", &PagedCacheStats::block_size)
      .def_readonly("num_blocks", &PagedCacheStats::num_blocks)
      .def_readonly("free_blocks", &PagedCacheStats::free_blocks)
      .def_readonly("max_context_tokens", &PagedCacheStats::max_context_tokens)
      .def_readonly("bytes", &PagedCacheStats::bytes);

  py::class_<PagedCacheRuntime>(m, "PagedCacheRuntime")
      .def(py::init([](size_t layers, size_t hkv, size_t d, const std::string &dt, int dev,
                       size_t block_size, const std::string &policy, double amount) {
             PagedCacheConfig cfg;
             cfg.block_size = block_size;
             if (policy == "blocks") cfg.memory = PagedCacheMemory::blocks((size_t)amount);
             else if (policy == "context") cfg.memory = PagedCacheMemory::context_size((size_t)amount);
             else if (policy == "fraction") cfg.memory = PagedCacheMemory::gpu_memory_fraction((float)amount);
             else throw Error("unknown paged cache memory policy: " + policy);
             return new PagedCacheRuntime(layers, hkv, d, parse_dtype(dt), parse_device(dev), cfg);
           }),
           py::arg("num_layers"), py::arg("num_kv_heads"), py::arg("head_dim"), py::arg("dtype"),
           py::arg("device"), py::arg("block_size"), py::arg("policy"), py::arg("amount"))
      .def_property_readonly("cache", &PagedCacheRuntime::cache, py::return_value_policy::reference_internal)
      .def("manager", &PagedCacheRuntime::manager_mut, py::return_value_policy::reference_internal)
      .def("block_tables_for", &PagedCacheRuntime::block_tables_for)
      .def("stats", &PagedCacheRuntime::stats)
      .def("graphs", &PagedCacheRuntime::graphs, py::return_value_policy::reference_internal)
      .def("set_cuda_graph_max_batch", &PagedCacheRuntime::set_cuda_graph_max_batch);

  // C++ mistralrs_paged_attn over raw pointers (stream = cudaStream_t as int).
  py::module_ ops = m.def_submodule("mistralrs_paged_attn", "C++ kernel entry points");
  ops.def("reshape_and_cache",
          [](uintptr_t k, uintptr_t v, uintptr_t kc, uintptr_t vc, uintptr_t slots,
             std::vector<size_t> kdims, std::vector<size_t> kcdims, std::vector<size_t> vcdims,
             const std::string &dt, int dev, uintptr_t stream) {
            auto K = tensor_view(k, kdims, dt, dev), V = tensor_view(v, kdims, dt, dev);
            auto KC = tensor_view(kc, kcdims, dt, dev), VC = tensor_view(vc, vcdims, dt, dev);
            auto S = tensor_view(slots, {kdims[0]}, "f32", dev);
            mistralrs_paged_attn::reshape_and_cache(K, V, nullptr, nullptr, KC, VC, S,
                                                    reinterpret_cast<vasr_pa_stream_t>(stream));
          });
  ops.def("paged_attention",
          [](uintptr_t out, uintptr_t q, uintptr_t kc, uintptr_t vc, uintptr_t bt, uintptr_t ctx,
             std::vector<size_t> qdims, std::vector<size_t> kcdims, std::vector<size_t> vcdims,
             size_t cols, size_t max_context_len, float scale, float softcap, const std::string &dt,
             int dev, uintptr_t ws, size_t ws_bytes, uintptr_t stream) {
            auto O = tensor_view(out, qdims, dt, dev), Q = tensor_view(q, qdims, dt, dev);
            auto KC = tensor_view(kc, kcdims, dt, dev), VC = tensor_view(vc, vcdims, dt, dev);
            auto BT = tensor_view(bt, {qdims[0], cols}, "f32", dev);
            auto CL = tensor_view(ctx, {qdims[0]}, "f32", dev);
            mistralrs_paged_attn::paged_attention(O, Q, nullptr, nullptr, KC, VC, BT, CL, nullptr,
                                                  max_context_len, scale, softcap, nullptr,
                                                  reinterpret_cast<void *>(ws), ws_bytes,
                                                  reinterpret_cast<vasr_pa_stream_t>(stream));
          });
}

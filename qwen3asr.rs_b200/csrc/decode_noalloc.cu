// decode_noalloc.cu — paged decode attention with library-owned scratch.
//
// Some callers cannot allocate device memory at the point where they run
// decode attention: an inference-server plugin's enqueue callback that must
// not touch the allocator, a host framework that owns a fixed device-memory
// budget and forbids allocations after start-up, or a real-time audio thread
// that must never block inside cudaMalloc. vasr_pa_paged_attention needs the
// caller to pass a split-K workspace; this entry point instead uses a scratch
// buffer compiled into the library as a file-scope device array, so the
// caller passes only inputs and outputs and nothing is allocated per call.
//
// The scratch is kNoAllocScratchBytes (16 MiB) per GPU and every GPU that
// loads the library holds it until the process exits. All calls on a device
// share it: calls that may overlap on the GPU (different streams without
// ordering, or concurrent host threads) race on the scratch and must not be
// issued that way.
#include <cuda_runtime.h>

#include <mutex>

#include "launch.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// Zero at module load. In host code this name is only a stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void *g_scratch_ptr[64] = {};

// Device address of the scratch on the current device. Outside stream
// capture every call looks it up again with that device current, so a module
// that the runtime reloaded (after cudaDeviceReset, for instance) is found at
// its new address; while `stream` is capturing, the address an earlier call
// resolved on this device is used, and the lookup runs only if there is none.
int32_t scratch_on_current_device(cudaStream_t stream, void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return VASR_PA_EDEVICE;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    cudaGetLastError();
    return VASR_PA_ELAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (cs == cudaStreamCaptureStatusNone || g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return VASR_PA_EDEVICE;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return VASR_PA_OK;
}

}  // namespace

extern "C" {

size_t vasr_pa_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int32_t vasr_pa_paged_attention_noalloc(void *out, const void *query, const void *key_cache,
                                        const void *value_cache, const uint32_t *block_tables,
                                        const uint32_t *context_lens, int32_t num_seqs,
                                        int32_t num_heads, int32_t num_kv_heads,
                                        int32_t head_dim, int32_t block_size, int64_t num_blocks,
                                        int32_t max_num_blocks_per_seq, int32_t max_context_len,
                                        float scale, float softcapping, int64_t q_seq_stride,
                                        int32_t dtype, vasr_pa_stream_t stream) {
  const size_t need = vasr_pa_paged_attention_workspace_size(
      num_seqs, num_heads, num_kv_heads, head_dim, block_size, max_context_len, dtype);
  if (need == 0 || num_seqs <= 0) {
    // Invalid sizes (or nothing to do): the regular entry point reports the
    // exact status without touching the scratch.
    return vasr_pa_paged_attention(out, query, key_cache, value_cache, block_tables,
                                   context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                                   block_size, num_blocks, max_num_blocks_per_seq,
                                   max_context_len, scale, softcapping, q_seq_stride, dtype,
                                   nullptr, 0, stream);
  }
  if (need > kNoAllocScratchBytes) return VASR_PA_ESCRATCH_LIMIT;
  void *scratch = nullptr;
  const int32_t st = scratch_on_current_device(reinterpret_cast<cudaStream_t>(stream), &scratch);
  if (st != VASR_PA_OK) return st;
  // The split-K arrival counters (the first num_seqs * num_kv_heads words of
  // the workspace layout) must start at zero. A completed decode launch leaves
  // the counters it used at zero; this clear guards against a previous launch
  // that stopped early (a bounded wait that gave up) and left some behind.
  const size_t counter_bytes = (size_t)num_seqs * (size_t)num_kv_heads * sizeof(uint32_t);
  if (cudaMemsetAsync(scratch, 0, counter_bytes, reinterpret_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    cudaGetLastError();
    return VASR_PA_ELAUNCH;
  }
  return vasr_pa_paged_attention(out, query, key_cache, value_cache, block_tables, context_lens,
                                 num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                 num_blocks, max_num_blocks_per_seq, max_context_len, scale,
                                 softcapping, q_seq_stride, dtype, scratch, kNoAllocScratchBytes,
                                 stream);
}

}  // extern "C"

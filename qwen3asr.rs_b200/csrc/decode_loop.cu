// decode_loop.cu — device-side decode-step bookkeeping, so that a captured
// decode step can be replayed step after step without a host round trip.
//
//  * decode_step_prepare_kernel: for every batch row, the token feedback and
//    EOS handling of paged_batch_decode_step
//    (vasr-models/src/model/paged_batch_engine.rs:634-676) and the decode
//    metadata of decode_metadata_for_batch_step
//    (vasr-paged-attn/src/paged_kv_cache.rs:924-1059, slot rule :74-103) for
//    the step held in a device counter. Finished rows become the padding rows
//    of pad_decode_batch_to_max (vasr-paged-attn/src/cuda_graph.rs:373-486):
//    token 0, position 0, slot 0 (the null block), context length 1.
//  * greedy_argmax_kernel: argmax_token_ids_from_logits
//    (vasr-models/src/model/generation.rs:443-460) on the device. A row is
//    split over several CTAs; each reduces its chunk to (max, first index),
//    and the last CTA of the row to finish (per-row counter, reset by that
//    CTA) merges the chunks in index order. The lowest index wins among equal
//    maxima; NaN never wins (an all-NaN row yields 0).
#include "common.cuh"
#include "launch.h"

namespace vasr {
namespace {

__global__ void __launch_bounds__(256) decode_step_prepare_kernel(const DecodeStepArgs a) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= a.num_seqs) return;
  const uint32_t step = *a.step;
  bool fin = a.finished[b] != 0;
  uint32_t tok = 0;
  if (!fin) {
    tok = a.next_ids[b];
    for (int e = 0; e < a.num_eos; ++e)
      if (a.eos_ids[e] == tok) fin = true;
    if (fin) a.finished[b] = 1;
  }
  if (fin) {  // padding row
    a.input_ids[b] = 0;
    a.positions[b] = 0;
    a.slot_mapping[b] = 0;
    a.context_lens[b] = 1;
    return;
  }
  if (a.generated) {
    const uint32_t g = a.generated[b];
    if (a.history && g < (uint32_t)a.history_cols)
      a.history[(int64_t)b * a.history_cols + g] = tok;
    a.generated[b] = g + 1;
  }
  const int64_t pos = (int64_t)a.prompt_lens[b] + step;
  const int64_t blk = pos / a.block_size;
  const int64_t len = a.block_table_lens ? (int64_t)a.block_table_lens[b] : a.max_num_blocks_per_seq;
  int64_t slot = -1;
  if (blk < len && blk < a.max_num_blocks_per_seq) {
    const uint32_t id = a.block_tables[(int64_t)b * a.max_num_blocks_per_seq + blk];
    if ((int64_t)id < a.num_blocks) slot = (int64_t)id * a.block_size + pos % a.block_size;
    else raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
  } else {
    raise_device_error(VASR_PA_DERR_SLOT_RANGE);  // table too short for this step
  }
  a.input_ids[b] = tok;
  a.positions[b] = pos;
  a.slot_mapping[b] = slot;
  a.context_lens[b] = (uint32_t)(pos + 1);
}

// (value, index) with "a before b" = larger value, or equal value and lower index.
struct Best {
  float v;
  uint32_t i;
};
__device__ __forceinline__ Best better(Best x, Best y) {
  if (y.v > x.v || (y.v == x.v && y.i < x.i)) return y;
  return x;
}
__device__ __forceinline__ Best warp_best(Best x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best y{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = better(x, y);
  }
  return x;
}

template <typename T>
__device__ __forceinline__ void scan_elem(Best &best, T raw, uint32_t idx) {
  const float v = Elem<T>::to_f32(raw);
  if (v > best.v) {  // strict: the first occurrence stays; NaN never passes
    best.v = v;
    best.i = idx;
  }
}

constexpr int kArgmaxThreads = 256;

template <typename T, bool kVec>
__global__ void __launch_bounds__(kArgmaxThreads) greedy_argmax_kernel(const ArgmaxArgs a) {
  const int b = blockIdx.y, chunk = blockIdx.x;
  if (a.step && b == 0 && chunk == 0 && threadIdx.x == 0) *a.step += 1;
  if (a.finished && a.finished[b]) return;
  const T *row = reinterpret_cast<const T *>(a.logits) + (int64_t)b * a.row_stride;
  const int64_t lo = (int64_t)chunk * a.chunk_elems;
  const int64_t hi = min(a.vocab, lo + a.chunk_elems);
  Best best{-INFINITY, 0xffffffffu};
  if (kVec) {
    // chunk_elems and the row start are multiples of 16 bytes
    constexpr int kPer = 16 / sizeof(T);
    const int64_t nvec = (hi - lo) / kPer;
    const uint4 *src = reinterpret_cast<const uint4 *>(row + lo);
    for (int64_t v = threadIdx.x; v < nvec; v += kArgmaxThreads) {
      const uint4 u = __ldcs(src + v);
      const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
      for (int k = 0; k < kPer; ++k) scan_elem(best, e[k], (uint32_t)(lo + v * kPer + k));
    }
    for (int64_t x = lo + nvec * kPer + threadIdx.x; x < hi; x += kArgmaxThreads)
      scan_elem(best, row[x], (uint32_t)x);
  } else {
    for (int64_t x = lo + threadIdx.x; x < hi; x += kArgmaxThreads) scan_elem(best, row[x], (uint32_t)x);
  }
  if (best.i == 0xffffffffu) best.i = (uint32_t)hi;  // nothing taken: loses every tie
  __shared__ Best part[kArgmaxThreads / 32];
  __shared__ bool last;
  best = warp_best(best);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    Best r = part[0];
    for (int w = 1; w < kArgmaxThreads / 32; ++w) r = better(r, part[w]);
    Best *slots = reinterpret_cast<Best *>(a.partials) + (int64_t)b * gridDim.x;
    slots[chunk] = r;
    __threadfence();
    const uint32_t done = atomicAdd(a.counters + b, 1u);
    last = (done == gridDim.x - 1);
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  const Best *slots = reinterpret_cast<const Best *>(a.partials) + (int64_t)b * gridDim.x;
  Best r{-INFINITY, 0xffffffffu};
  for (unsigned c = 0; c < gridDim.x; ++c) {
    const Best y{__ldcg(&slots[c].v), __ldcg(&slots[c].i)};
    r = better(r, y);
  }
  a.next_ids[b] = (r.v > -INFINITY) ? r.i : 0u;  // no finite maximum: index 0
  a.counters[b] = 0;  // ready for the next call
}

template <typename T>
int launch_argmax_t(const ArgmaxArgs &a, cudaStream_t s) {
  dim3 grid((unsigned)a.num_chunks, (unsigned)a.num_seqs);
  const bool vec = (reinterpret_cast<uintptr_t>(a.logits) % 16 == 0) &&
                   ((a.row_stride * (int64_t)sizeof(T)) % 16 == 0) &&
                   ((a.chunk_elems * (int64_t)sizeof(T)) % 16 == 0);
  if (vec) greedy_argmax_kernel<T, true><<<grid, kArgmaxThreads, 0, s>>>(a);
  else greedy_argmax_kernel<T, false><<<grid, kArgmaxThreads, 0, s>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

}  // namespace

// Chunk layout of a row: chunks of a multiple of 8 elements (16 bytes of bf16),
// about 8192 elements each, at most 64 per row.
void argmax_chunking(int64_t vocab, int *num_chunks, int64_t *chunk_elems) {
  int64_t n = (vocab + 8191) / 8192;
  if (n < 1) n = 1;
  if (n > 64) n = 64;
  int64_t per = (vocab + n - 1) / n;
  per = (per + 7) / 8 * 8;
  *num_chunks = (int)((vocab + per - 1) / per);
  *chunk_elems = per;
}

size_t argmax_workspace_bytes(int num_seqs, int64_t vocab) {
  int chunks;
  int64_t per;
  argmax_chunking(vocab, &chunks, &per);
  const size_t counters = ((size_t)num_seqs * 4 + 255) / 256 * 256;
  return counters + (size_t)num_seqs * chunks * sizeof(Best);
}

int launch_decode_step_prepare(const DecodeStepArgs &a, cudaStream_t s) {
  const int threads = 256;
  decode_step_prepare_kernel<<<(a.num_seqs + threads - 1) / threads, threads, 0, s>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

int launch_greedy_argmax(ArgmaxArgs a, void *workspace, cudaStream_t s) {
  argmax_chunking(a.vocab, &a.num_chunks, &a.chunk_elems);
  const size_t counters = ((size_t)a.num_seqs * 4 + 255) / 256 * 256;
  a.counters = reinterpret_cast<uint32_t *>(workspace);
  a.partials = reinterpret_cast<unsigned char *>(workspace) + counters;
  switch (a.dtype) {
    case VASR_PA_F32: return launch_argmax_t<float>(a, s);
    case VASR_PA_BF16: return launch_argmax_t<__nv_bfloat16>(a, s);
    case VASR_PA_F16: return launch_argmax_t<__half>(a, s);
    default: return VASR_PA_EINVAL_DTYPE;
  }
}

int read_error_decode_loop(uint32_t *bits, bool clear, cudaStream_t s) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s) !=
      cudaSuccess)
    return VASR_PA_ELAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return VASR_PA_ELAUNCH;
  if (clear) {
    const uint32_t z = 0;
    if (cudaMemcpyToSymbolAsync(g_device_error, &z, sizeof(z), 0, cudaMemcpyHostToDevice, s) !=
        cudaSuccess)
      return VASR_PA_ELAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return VASR_PA_ELAUNCH;
  }
  *bits = v;
  return VASR_PA_OK;
}

}  // namespace vasr

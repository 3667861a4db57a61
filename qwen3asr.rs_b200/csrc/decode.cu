// decode.cu — launchers and instantiations of the paged decode kernels.
//
// GQA group 2 (Qwen3-ASR: 16 query / 8 kv heads) runs paged_decode_g2_kernel
// (decode_g2.cuh); groups 1 and 4 run the generic paged_decode_kernel
// (decode.cuh). Both use the same split-K workspace layout.
#include <type_traits>

#include "decode_g2.cuh"
#include "decode_mma.cuh"
#include "launch.h"

// Launch-shape constants of the GQA-2 kernel (stages per CTA and resident
// CTAs per SM); chosen by measurement on B200, see the design notes.
#ifndef VASR_G2_NST
#define VASR_G2_NST 8
#endif
#ifndef VASR_G2_MINB
#define VASR_G2_MINB 3
#endif
// Launch shape of the tensor-core kernel over fp8 pages (stages per CTA,
// resident CTAs per SM)
#ifndef VASR_G2_NST_FP8
#define VASR_G2_NST_FP8 8
#endif
#ifndef VASR_G2_MINB_FP8
#define VASR_G2_MINB_FP8 5
#endif
// fp8 pages, grids of at least two waves at this occupancy: the same kernel
// at 6 CTAs per SM with the query fragments in shared memory (one wave: the
// extra CTA per SM slows the longest splits, which set the time)
#ifndef VASR_G2_MINB_FP8_WIDE
#define VASR_G2_MINB_FP8_WIDE 6
#endif
// GQA-2 bf16 / f16 pages: tensor-core score and P.V tiles (decode_mma.cuh)
#ifndef VASR_DECODE_MMA
#define VASR_DECODE_MMA 1
#endif
// honour DecodeArgs::overlap_append with a programmatic dependent launch
#ifndef VASR_DECODE_PDL
#define VASR_DECODE_PDL 1
#endif

namespace vasr {

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

DecodeWorkspace decode_workspace_layout(int num_seqs, int num_heads, int num_kv_heads,
                                        int head_dim, int block_size, int max_context_len) {
  DecodeWorkspace w;
  // GQA 2 (bf16 / f16 run the tensor-core kernel) takes longer splits
  const int split_tokens = (num_kv_heads > 0 && num_heads == 2 * num_kv_heads)
                               ? VASR_DECODE_SPLIT_TOKENS_G2
                               : VASR_DECODE_SPLIT_TOKENS;
  w.pages_per_split =
      decode_pages_per_split(num_seqs, num_kv_heads, block_size, max_context_len, split_tokens);
  const int P = w.pages_per_split * block_size;
  w.max_splits = (max_context_len + P - 1) / P;
  if (w.max_splits < 1) w.max_splits = 1;
  const size_t slots = (size_t)num_seqs * num_kv_heads * w.max_splits;
  const int G = num_heads / num_kv_heads;
  // The arrival counters sit in a fixed region at offset 0 that every call
  // returns to zero, so one zero-filled workspace stays valid across calls of
  // any shape (partials of an earlier call never overlap a later call's
  // counters).
  w.off_counters = 0;
  w.off_o = align256(kDecodeMaxCounters * sizeof(uint32_t));
  w.off_ml = align256(w.off_o + slots * G * head_dim * sizeof(float));
  w.total = align256(w.off_ml + slots * G * sizeof(float2));
  return w;
}

namespace {

DecodeParams make_decode_params(const DecodeArgs &a, const DecodeWorkspace &w) {
  DecodeParams p{};
  p.out = a.out;
  p.q = a.query;
  p.k_cache = a.key_cache;
  p.v_cache = a.value_cache;
  p.block_tables = a.block_tables;
  p.context_lens = a.context_lens;
  unsigned char *ws = static_cast<unsigned char *>(a.workspace);
  p.ws_o = reinterpret_cast<float *>(ws + w.off_o);
  p.ws_ml = reinterpret_cast<float2 *>(ws + w.off_ml);
  p.counters = reinterpret_cast<uint32_t *>(ws + w.off_counters);
  p.q_seq_stride = a.q_seq_stride;
  p.num_blocks = a.num_blocks;
  p.num_seqs = a.num_seqs;
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.cols = a.max_num_blocks_per_seq;
  p.pages_per_split = w.pages_per_split;
  p.max_splits = w.max_splits;
  p.scale = a.scale;
  p.softcap = a.softcapping;
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  return p;
}

// Host-side checks shared by both kernels; returns the workspace layout.
int check_workspace(const DecodeArgs &a, int max_pages_per_split, DecodeWorkspace *w) {
  *w = decode_workspace_layout(a.num_seqs, a.num_heads, a.num_kv_heads, a.head_dim,
                               a.block_size, a.max_context_len);
  if ((size_t)a.num_seqs * a.num_kv_heads > kDecodeMaxCounters) return VASR_PA_ENOT_SUPPORTED;
  if (a.workspace == nullptr || a.workspace_bytes < w->total) return VASR_PA_EINVAL_WORKSPACE;
  if (w->pages_per_split > max_pages_per_split) return VASR_PA_ENOT_SUPPORTED;
  return VASR_PA_OK;
}

// grid = (split, kv head, sequence): the splits of one (sequence, kv head)
// are adjacent, so its partials are merged soon after they are written.
template <typename T, int BS, int D, int G>
int launch_decode_generic(const DecodeArgs &a, cudaStream_t stream) {
  using C = DecodeCfg<T, BS, D, G>;
  DecodeWorkspace w;
  const int st = check_workspace(a, C::kMaxPagesPerSplit, &w);
  if (st != VASR_PA_OK) return st;
  const DecodeParams p = make_decode_params(a, w);
  static std::atomic<uint64_t> attr_done{0};
  if (!ensure_smem_attr(paged_decode_kernel<T, BS, D, G>, C::kSmemBytes, attr_done))
    return VASR_PA_ELAUNCH;
  dim3 grid((unsigned)w.max_splits, (unsigned)a.num_kv_heads, (unsigned)a.num_seqs);
  paged_decode_kernel<T, BS, D, G><<<grid, C::kThreads, C::kSmemBytes, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

template <typename T, int BS, int D, typename TC = T>
int launch_decode_g2(const DecodeArgs &a, cudaStream_t stream) {
  constexpr int kStageBytes = 2 * ((16 > BS) ? 16 / BS : 1) * D * BS * (int)sizeof(TC);
  // same bytes in flight per CTA for any page size: twice the stages for 4 KB stages
  constexpr bool kFp8Pages = std::is_same<TC, __nv_fp8_e4m3>::value;
  // fp8: the tuned stage count for 4 KB stages, half of it (a multiple of the
  // 4 warps) for the 8 KB stages of 32-token pages
  constexpr int kNST = kFp8Pages ? (kStageBytes <= 4096 ? VASR_G2_NST_FP8
                                    : ((VASR_G2_NST_FP8 / 2) / 4 * 4 < 4 ? 4 : (VASR_G2_NST_FP8 / 2) / 4 * 4))
                       : kStageBytes <= 4096 ? 2 * VASR_G2_NST : kStageBytes <= 8192 ? VASR_G2_NST : 4;
  constexpr int kMinB = kFp8Pages ? VASR_G2_MINB_FP8 : VASR_G2_MINB;
  using C = DecodeG2Cfg<TC, BS, D, kNST>;
  DecodeWorkspace w;
  const int st = check_workspace(a, C::kMaxPagesPerSplit, &w);
  if (st != VASR_PA_OK) return st;
  const DecodeParams p = make_decode_params(a, w);
  constexpr bool kMma = VASR_DECODE_MMA && !std::is_same<T, float>::value &&
                        (std::is_same<T, TC>::value || BS >= 16);
  if constexpr (kMma) {
    auto kern = paged_decode_mma_kernel<T, BS, D, kNST, kMinB, TC>;
    static std::atomic<uint64_t> attr_done{0};
    if (!ensure_smem_attr(kern, C::kSmemBytes, attr_done)) return VASR_PA_ELAUNCH;
    dim3 grid((unsigned)w.max_splits, (unsigned)a.num_kv_heads, (unsigned)a.num_seqs);
    if constexpr (kFp8Pages && VASR_G2_MINB_FP8_WIDE > kMinB) {
      auto wide = paged_decode_mma_kernel<T, BS, D, kNST, VASR_G2_MINB_FP8_WIDE, TC>;
      static std::atomic<uint64_t> attr_wide{0};
      static std::atomic<int64_t> resident[64];
      if (!ensure_smem_attr(wide, C::kSmemBytes, attr_wide)) return VASR_PA_ELAUNCH;
      const int64_t slots = resident_ctas(wide, C::kThreads, C::kSmemBytes, resident);
      if (slots > 0 && (int64_t)grid.x * grid.y * grid.z >= 2 * slots) kern = wide;
    }
    if (VASR_DECODE_PDL && a.overlap_append) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(C::kThreads);
      cfg.dynamicSmemBytes = C::kSmemBytes;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
    }
    kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(p);
    return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
  }
  auto kern = paged_decode_g2_kernel<T, BS, D, kNST, kMinB, TC>;
  static std::atomic<uint64_t> attr_done{0};
  if (!ensure_smem_attr(kern, C::kSmemBytes, attr_done)) return VASR_PA_ELAUNCH;
  dim3 grid((unsigned)w.max_splits, (unsigned)a.num_kv_heads, (unsigned)a.num_seqs);
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

template <typename T, int D, int G>
int dispatch_bs(const DecodeArgs &a, cudaStream_t s) {
  if constexpr (G == 2) {
    switch (a.block_size) {
      case 8: return launch_decode_g2<T, 8, D>(a, s);
      case 16: return launch_decode_g2<T, 16, D>(a, s);
      case 32: return launch_decode_g2<T, 32, D>(a, s);
      default: return VASR_PA_EINVAL_BLOCKSIZE;
    }
  }
  switch (a.block_size) {
    case 8: return launch_decode_generic<T, 8, D, G>(a, s);
    case 16: return launch_decode_generic<T, 16, D, G>(a, s);
    case 32: return launch_decode_generic<T, 32, D, G>(a, s);
    default: return VASR_PA_EINVAL_BLOCKSIZE;
  }
}

template <typename T>
int dispatch_g(const DecodeArgs &a, cudaStream_t s) {
  const int G = a.num_heads / a.num_kv_heads;
  if (a.head_dim != 128) return VASR_PA_ENOT_SUPPORTED;
  switch (G) {
    case 1: return dispatch_bs<T, 128, 1>(a, s);
    case 2: return dispatch_bs<T, 128, 2>(a, s);
    case 4: return dispatch_bs<T, 128, 4>(a, s);
    default: return VASR_PA_ENOT_SUPPORTED;
  }
}


template <typename T>
int dispatch_fp8(const DecodeArgs &a, cudaStream_t s) {
  if (a.head_dim != 128 || a.num_heads != 2 * a.num_kv_heads) return VASR_PA_ENOT_SUPPORTED;
  switch (a.block_size) {
    case 8: return VASR_PA_ENOT_SUPPORTED;  // an 8-byte V page row is under one 16-byte vector
    case 16: return launch_decode_g2<T, 16, 128, __nv_fp8_e4m3>(a, s);
    case 32: return launch_decode_g2<T, 32, 128, __nv_fp8_e4m3>(a, s);
    default: return VASR_PA_EINVAL_BLOCKSIZE;
  }
}

}  // namespace

int launch_decode(const DecodeArgs &a, cudaStream_t s) {
  if (a.cache_dtype == VASR_PA_FP8_E4M3) {
    switch (a.dtype) {
      case VASR_PA_BF16: return dispatch_fp8<__nv_bfloat16>(a, s);
      case VASR_PA_F16: return dispatch_fp8<__half>(a, s);
      default: return VASR_PA_EINVAL_DTYPE;
    }
  }
  switch (a.dtype) {
    case VASR_PA_F32: return dispatch_g<float>(a, s);
    case VASR_PA_BF16: return dispatch_g<__nv_bfloat16>(a, s);
    case VASR_PA_F16: return dispatch_g<__half>(a, s);
    default: return VASR_PA_EINVAL_DTYPE;
  }
}

int read_error_decode(uint32_t *bits, bool clear, cudaStream_t s) {
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

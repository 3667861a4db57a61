// kv_ops.cu — HBM-bound cache kernels for sm_100a: KV append
// (reshape_and_cache), gather_kv_cache, copy_blocks and swap_blocks.
//
// None of these does arithmetic on the values: every kernel is a byte-exact
// permutation of its input, moved in 16-byte vectors wherever the cache
// layout allows it.
#include <type_traits>

#include "common.cuh"
#include "launch.h"

namespace vasr {
namespace {

// ======================================================== reshape_and_cache
// Reference semantics: mistralrs_paged_attn::reshape_and_cache as called at
// vasr-models/src/model/thinker_text.rs:1101-1109 / :1324-1332; layout from
// vasr-paged-attn/src/paged_kv_cache.rs:285-294.
//
// A CTA stages a tile of up to 16 tokens x (up to 2 KB of heads) of K and V
// in shared memory with coalesced 16-byte loads, then
//  - writes K as 16-byte chunks K[blk, h, c, off, 0:x], threads ordered
//    token-fastest so consecutive offsets of one page form contiguous runs;
//  - writes V by runs: a run is up to 16/sizeof(T) tokens with consecutive
//    slots inside one aligned 16-byte group of a page row V[blk, h, d, :].
//    A full aligned run is one 16-byte store; anything else falls back to
//    element stores. Prefill chunks therefore store V in 16-byte vectors;
//    decode (one token per page) cannot, by the layout.
constexpr int kAppendThreads = 256;
constexpr int kAppendMaxTokens = 16;
constexpr int kAppendRowBytes = 2048;                 // bytes of heads per tile row

struct AppendParams {
  const unsigned char *key;
  const unsigned char *value;
  unsigned char *k_cache;
  unsigned char *v_cache;
  const int64_t *slots;
  int64_t num_tokens;
  int64_t k_stride_bytes;
  int64_t v_stride_bytes;
  int64_t num_blocks;
  int num_kv_heads;
  int tile_tokens;
  int heads_per_tile;
  int row_pitch;  // bytes of one staged token row: heads_per_tile * D * es + 16 (conflict-free columns)
  int tiles_per_cta;  // 16-token tiles: consecutive tiles one CTA handles in turn
};

template <typename T, int BS, int D>
__global__ void __launch_bounds__(kAppendThreads) kv_append_kernel(const AppendParams p) {
  constexpr int kX = Elem<T>::kX;
  constexpr int kCH = D / kX;          // 16-byte chunks per (token, head)
  constexpr int kTPS = kX;             // tokens per 16-byte V group
  constexpr int kES = (int)sizeof(T);
  extern __shared__ __align__(16) unsigned char sm[];
  const int pitch = p.row_pitch;
  unsigned char *kt = sm;
  unsigned char *vt = sm + p.tile_tokens * pitch;
  int64_t *s_slot = reinterpret_cast<int64_t *>(vt + p.tile_tokens * pitch);
  int *s_run_start = reinterpret_cast<int *>(s_slot + kAppendMaxTokens);
  int *s_run_len = s_run_start + kAppendMaxTokens;
  int *s_nruns = s_run_len + kAppendMaxTokens;

  const int TT = p.tile_tokens;
  const int64_t t0 = (int64_t)blockIdx.x * TT;
  const int h0 = blockIdx.y * p.heads_per_tile;
  const int HC = min(p.heads_per_tile, p.num_kv_heads - h0);
  const int ntok = (int)min((int64_t)TT, p.num_tokens - t0);
  const int64_t max_slot = p.num_blocks * BS;
  const int tid = threadIdx.x;

  if (tid < ntok) {
    int64_t s = p.slots[t0 + tid];
    if (s >= max_slot) {
      raise_device_error(VASR_PA_DERR_SLOT_RANGE);
      s = -1;
    }
    s_slot[tid] = s;
  }
  // coalesced 16-byte loads of the tile
  const int row_chunks = HC * kCH;
  for (int i = tid; i < ntok * row_chunks; i += kAppendThreads) {
    const int tt = i / row_chunks;
    const int r = i - tt * row_chunks;
    const int64_t col = (int64_t)h0 * D * kES + (int64_t)r * 16;
    const uint4 kv = __ldg(reinterpret_cast<const uint4 *>(p.key + (t0 + tt) * p.k_stride_bytes + col));
    const uint4 vv = __ldg(reinterpret_cast<const uint4 *>(p.value + (t0 + tt) * p.v_stride_bytes + col));
    *reinterpret_cast<uint4 *>(kt + tt * pitch + r * 16) = kv;
    *reinterpret_cast<uint4 *>(vt + tt * pitch + r * 16) = vv;
  }
  __syncthreads();
  if (tid == 0) {
    // split the tile into V runs (consecutive slots, same aligned group)
    int n = 0;
    int tt = 0;
    while (tt < ntok) {
      const int64_t s = s_slot[tt];
      if (s < 0) {
        ++tt;
        continue;
      }
      int len = 1;
      while (tt + len < ntok && len < kTPS && s_slot[tt + len] == s + len && ((s + len) % kTPS) != 0)
        ++len;
      s_run_start[n] = tt;
      s_run_len[n] = len;
      ++n;
      tt += len;
    }
    s_nruns[0] = n;
  }
  // K: (head, chunk, token) with token fastest
  for (int i = tid; i < ntok * row_chunks; i += kAppendThreads) {
    const int tt = i % ntok;
    const int r = i / ntok;
    const int64_t s = s_slot[tt];
    if (s < 0) continue;
    const int hc = r / kCH;
    const int c = r - hc * kCH;
    const int64_t blk = s / BS;
    const int off = (int)(s - blk * BS);
    const int64_t dst = ((((blk * p.num_kv_heads + h0 + hc) * kCH + c) * BS) + off) * 16;
    *reinterpret_cast<uint4 *>(p.k_cache + dst) =
        *reinterpret_cast<const uint4 *>(kt + tt * pitch + r * 16);
  }
  __syncthreads();
  // V: (head, dim, run) with run fastest
  const int nruns = s_nruns[0];
  const int nitems = nruns * HC * D;
  for (int i = tid; i < nitems; i += kAppendThreads) {
    const int j = i % nruns;
    const int hd = i / nruns;
    const int hc = hd / D;
    const int d = hd - hc * D;
    const int tt0 = s_run_start[j];
    const int len = s_run_len[j];
    const int64_t s = s_slot[tt0];
    const int64_t blk = s / BS;
    const int off = (int)(s - blk * BS);
    const int64_t row = ((blk * p.num_kv_heads + h0 + hc) * D + d) * BS;
    const unsigned char *src = vt + tt0 * pitch + (hc * D + d) * kES;
    T *dst = reinterpret_cast<T *>(p.v_cache) + row + off;
    if (len == kTPS && (off % kTPS) == 0) {
      T vals[kTPS];
#pragma unroll
      for (int e = 0; e < kTPS; ++e) vals[e] = *reinterpret_cast<const T *>(src + e * pitch);
      *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(vals);
    } else {
      for (int e = 0; e < len; ++e) dst[e] = *reinterpret_cast<const T *>(src + e * pitch);
    }
  }
}

// ---------------------------------------------- 16-token tiles (prefill)
// Prefill-sized appends: a CTA owns 16 consecutive tokens x HPT heads (512
// bytes of each token row). Every tile shape is a compile-time constant, so
// all index math is shifts and masks. Warp 0 reads the 16 slots and sorts the
// tokens into V groups of kTPS tokens (one 16-byte vector of a page row): a
// group whose slots are consecutive and start on a kTPS boundary leaves as
// one vector store per (head, dim); any other group (pads, a page change
// inside it, an unaligned start) stores its tokens element by element. K
// leaves as 16-byte chunks (16 bytes of one token's row), token fastest, so
// the tile's chunks of one page row form contiguous runs.
constexpr int kTile16 = 16;

// Tiles per CTA for `items` 16-token tiles over `resident` CTA slots: the
// fewest that fit every CTA into one wave, so that no CTA starts after
// another has finished (a second, partial wave of whole tiles left SMs idle
// for a quarter of the launch). 1 when the slots are unknown.
inline int tile16_per_cta(int64_t items, int64_t resident) {
  if (resident <= 0 || items <= resident) return 1;
  const int64_t t = (items + resident - 1) / resident;
  return t > 64 ? 64 : (int)t;
}

// Warp 0, lane l < ntok: the slot of token t0 + l (-1 for the other lanes).
__device__ __forceinline__ int64_t tile16_load_slot(const int64_t *slots, int64_t t0, int ntok) {
  const int lane = threadIdx.x;
  return lane < ntok ? slots[t0 + lane] : -1;
}

// Warp 0: the tile's slots (loaded by tile16_load_slot) into s_slot (out of
// range -> skipped and flagged) and, per V group of kTPS tokens, whether it
// is one aligned run of slots.
template <int BS, int kTPS, int kGroups>
__device__ __forceinline__ void tile16_slots(int64_t sl, int64_t num_blocks, int64_t *s_slot, int *s_gok) {
  const int lane = threadIdx.x;
  if (sl >= num_blocks * BS) {
    raise_device_error(VASR_PA_DERR_SLOT_RANGE);
    sl = -1;
  }
  if (lane < kTile16) s_slot[lane] = sl;
  const int g0 = lane & ~(kTPS - 1);
  const int64_t first = __shfl_sync(0xffffffffu, sl, g0);
  const bool ok = lane < kTile16 && sl >= 0 && (first & (kTPS - 1)) == 0 && sl == first + (lane - g0);
  const uint32_t ball = __ballot_sync(0xffffffffu, ok);
  constexpr uint32_t kAll = (1u << kTPS) - 1u;
  if (lane < kGroups) s_gok[lane] = ((ball >> (lane * kTPS)) & kAll) == kAll;
}

template <typename T, int BS, int D, int HPT>
__global__ void __launch_bounds__(kAppendThreads) kv_append_tile16_kernel(const AppendParams p) {
  constexpr int kES = (int)sizeof(T);
  constexpr int kX = 16 / kES;                     // elements per 16-byte chunk
  constexpr int kCH = D / kX;                      // chunks per (token, head)
  constexpr int kRow = HPT * kCH;                  // chunks per staged token row
  constexpr int kPitch = HPT * D * kES + 16;       // staged row bytes (+16 spreads banks)
  constexpr int kTPS = kX;                         // tokens per V vector
  constexpr int kGroups = kTile16 / kTPS;
  constexpr int kChunks = kTile16 * kRow;
  constexpr int kVItems = HPT * D * kGroups;
  static_assert(kTPS <= BS, "a V vector stays inside one page row");
  static_assert((kRow & (kRow - 1)) == 0 && (kCH & (kCH - 1)) == 0, "power-of-two tile shapes");
  __shared__ __align__(16) unsigned char kt[kTile16 * kPitch];
  __shared__ __align__(16) unsigned char vt[kTile16 * kPitch];
  __shared__ int64_t s_slot[kTile16];
  __shared__ int s_gok[kGroups];
  constexpr int kLd = (kChunks + kAppendThreads - 1) / kAppendThreads;  // 16-byte loads per thread
  const int tid = threadIdx.x;
  const int h0 = blockIdx.y * HPT;
  const int HC = min(HPT, p.num_kv_heads - h0);
  // The next tile's rows and slots are loaded into registers while this
  // tile's stores go out (software pipeline over the CTA's tiles).
  uint4 kr[kLd], vr[kLd];
  int64_t sl_next = -1;
  auto load_tile = [&](int64_t t0) {
    const int ntok = (int)min((int64_t)kTile16, p.num_tokens - t0);
    if (tid < 32) sl_next = tile16_load_slot(p.slots, t0, ntok);
#pragma unroll
    for (int k = 0; k < kLd; ++k) {
      const int i = tid + k * kAppendThreads;
      const int tt = i / kRow, r = i % kRow;
      if (i < kChunks && tt < ntok && r / kCH < HC) {
        const int64_t col = (int64_t)h0 * D * kES + r * 16;
        kr[k] = __ldg(reinterpret_cast<const uint4 *>(p.key + (t0 + tt) * p.k_stride_bytes + col));
        vr[k] = __ldg(reinterpret_cast<const uint4 *>(p.value + (t0 + tt) * p.v_stride_bytes + col));
      }
    }
  };
  const int64_t first = (int64_t)blockIdx.x * p.tiles_per_cta;
  if (first * kTile16 >= p.num_tokens) return;
  load_tile(first * kTile16);
  for (int it = 0; it < p.tiles_per_cta; ++it) {
    const int64_t t0 = (first + it) * kTile16;
    if (t0 >= p.num_tokens) break;
    if (it > 0) __syncthreads();  // the previous tile's staged rows and slots are read
    const int ntok = (int)min((int64_t)kTile16, p.num_tokens - t0);
    if (tid < 32) tile16_slots<BS, kTPS, kGroups>(sl_next, p.num_blocks, s_slot, s_gok);
#pragma unroll
    for (int k = 0; k < kLd; ++k) {
      const int i = tid + k * kAppendThreads;
      const int tt = i / kRow, r = i % kRow;
      if (i < kChunks && tt < ntok && r / kCH < HC) {
        *reinterpret_cast<uint4 *>(kt + tt * kPitch + r * 16) = kr[k];
        *reinterpret_cast<uint4 *>(vt + tt * kPitch + r * 16) = vr[k];
      }
    }
    __syncthreads();
    if (it + 1 < p.tiles_per_cta && t0 + kTile16 < p.num_tokens) load_tile(t0 + kTile16);
    // K: item i = (chunk r of the row, token tt), token fastest
#pragma unroll
    for (int k = 0; k < (kChunks + kAppendThreads - 1) / kAppendThreads; ++k) {
      const int i = tid + k * kAppendThreads;
      const int tt = i % kTile16, r = i / kTile16;
      const int hc = r / kCH, c = r % kCH;
      const int64_t sl = s_slot[tt];
      if (i < kChunks && sl >= 0 && hc < HC) {
        const uint64_t us = (uint64_t)sl, blk = us / BS, off = us % BS;
        const uint64_t dst = (((blk * (uint64_t)p.num_kv_heads + (uint64_t)(h0 + hc)) * kCH + c) * BS + off) * 16;
        *reinterpret_cast<uint4 *>(p.k_cache + dst) = *reinterpret_cast<const uint4 *>(kt + tt * kPitch + r * 16);
      }
    }
    // V: item i = (group g, dim d of head hc), group fastest: consecutive
    // threads fill consecutive 16-byte pieces of the page rows
#pragma unroll
    for (int k = 0; k < (kVItems + kAppendThreads - 1) / kAppendThreads; ++k) {
      const int i = tid + k * kAppendThreads;
      const int g = i % kGroups, hd = i / kGroups;
      const int hc = hd / D, d = hd % D;
      if (i >= kVItems || hc >= HC) continue;
      const unsigned char *src = vt + (g * kTPS) * kPitch + (hc * D + d) * kES;
      const uint64_t row = ((uint64_t)h0 + hc) * D + d;  // page row of (head, dim) within a block
      if (s_gok[g]) {
        const uint64_t us = (uint64_t)s_slot[g * kTPS], blk = us / BS, off = us % BS;
        T vals[kTPS];
#pragma unroll
        for (int e = 0; e < kTPS; ++e) vals[e] = *reinterpret_cast<const T *>(src + e * kPitch);
        T *dst = reinterpret_cast<T *>(p.v_cache) + (blk * (uint64_t)p.num_kv_heads * D + row) * BS + off;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(vals);
      } else {
#pragma unroll
        for (int e = 0; e < kTPS; ++e) {
          const int64_t sl = s_slot[g * kTPS + e];
          if (sl < 0) continue;
          const uint64_t us = (uint64_t)sl, blk = us / BS, off = us % BS;
          reinterpret_cast<T *>(p.v_cache)[(blk * (uint64_t)p.num_kv_heads * D + row) * BS + off] =
              *reinterpret_cast<const T *>(src + e * kPitch);
        }
      }
    }
  }
}

template <typename T, int BS, int D>
int launch_append_t(const AppendArgs &a, cudaStream_t stream) {
  AppendParams p{};
  p.key = static_cast<const unsigned char *>(a.key);
  p.value = static_cast<const unsigned char *>(a.value);
  p.k_cache = static_cast<unsigned char *>(a.key_cache);
  p.v_cache = static_cast<unsigned char *>(a.value_cache);
  p.slots = a.slot_mapping;
  p.num_tokens = a.num_tokens;
  p.k_stride_bytes = a.key_token_stride * (int64_t)sizeof(T);
  p.v_stride_bytes = a.value_token_stride * (int64_t)sizeof(T);
  p.num_blocks = a.num_blocks;
  p.num_kv_heads = a.num_kv_heads;
  // Decode-sized calls (one token per page) get one token per CTA for
  // parallelism; mid-sized calls 8-token tiles of up to 2 KB of heads, with
  // shared memory sized to the tile; prefill chunks (>= 4096 tokens) the
  // compile-time 16-token tiles of 512 bytes of heads above, so one CTA
  // writes whole 32-byte V page rows and small tiles keep many CTAs resident.
  if (a.num_tokens >= 4096) {  // prefill chunks: 16-token tiles of 512 bytes of heads
    constexpr int kHPT = 512 / (D * (int)sizeof(T)) > 0 ? 512 / (D * (int)sizeof(T)) : 1;
    static std::atomic<int64_t> resident[64];
    const int64_t tiles = (a.num_tokens + kTile16 - 1) / kTile16;
    const int hg = (a.num_kv_heads + kHPT - 1) / kHPT;
    p.tiles_per_cta = tile16_per_cta(tiles * hg, resident_ctas(kv_append_tile16_kernel<T, BS, D, kHPT>,
                                                                kAppendThreads, 0, resident));
    const int64_t gx = (tiles + p.tiles_per_cta - 1) / p.tiles_per_cta;
    if (gx > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
    dim3 grid((unsigned)gx, (unsigned)hg);
    kv_append_tile16_kernel<T, BS, D, kHPT><<<grid, kAppendThreads, 0, stream>>>(p);
    return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
  }
  const int tt = a.num_tokens >= 128 ? 8 : 1;
  const int row_bytes = kAppendRowBytes;
  p.tile_tokens = tt;
  p.heads_per_tile = row_bytes / (D * (int)sizeof(T)) > 0 ? row_bytes / (D * (int)sizeof(T)) : 1;
  p.row_pitch = p.heads_per_tile * D * (int)sizeof(T) + 16;
  // staged K and V rows of this tile, then the slot / run arrays (sized for 16 tokens)
  constexpr int kTail = kAppendMaxTokens * 8 + 2 * kAppendMaxTokens * 4 + 16;
  const int smem = 2 * tt * p.row_pitch + kTail;
  constexpr int kSmemMax = 2 * kAppendMaxTokens * (kAppendRowBytes + D * (int)sizeof(T) + 16) + kTail;
  static std::atomic<uint64_t> attr_done{0};
  if (!ensure_smem_attr(kv_append_kernel<T, BS, D>, kSmemMax, attr_done)) return VASR_PA_ELAUNCH;
  const int64_t tiles = (a.num_tokens + tt - 1) / tt;
  if (tiles > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
  dim3 grid((unsigned)tiles, (unsigned)((a.num_kv_heads + p.heads_per_tile - 1) / p.heads_per_tile));
  kv_append_kernel<T, BS, D><<<grid, kAppendThreads, smem, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

// ========================================================== gather_kv_cache
// Reference semantics: mistralrs_paged_attn::gather_kv_cache as called at
// thinker_text.rs:190-198 / :1344-1352: packed [sum kv, Hkv, D] K and V.
// One CTA per (page, sequence, kv head). Every thread first issues all of
// its 16-byte loads (K chunks into registers, V chunks too), so a CTA keeps
// its whole page pair in flight; K chunks are stored as they are (a K chunk
// is 16 bytes of one token's row), V rows [D][BS] are transposed through
// shared memory into 16-byte vectors of one token's row.
struct GatherParams {
  unsigned char *k_out;
  unsigned char *v_out;
  const unsigned char *k_cache;
  const unsigned char *v_cache;
  const uint32_t *block_tables;
  const uint32_t *cu;
  int64_t num_blocks;
  int cols;
  int num_kv_heads;
};

// threads per CTA for a page of `chunks` 16-byte chunks: about 4 chunks each
constexpr int gather_threads(int chunks) {
  return chunks / 4 < 32 ? 32 : (chunks / 4 > 256 ? 256 : chunks / 4);
}

// Locates (page, sequence, kv head) of this CTA; false when the page lies
// past the sequence. Block ids past the pool read block 0 and are flagged.
__device__ __forceinline__ bool gather_page(const GatherParams &p, int BS, int &n, int64_t &tok0,
                                            uint32_t &blk) {
  const int page = blockIdx.x, b = blockIdx.y;
  const int64_t start = p.cu[b];
  const int64_t len = (int64_t)p.cu[b + 1] - start;
  if ((int64_t)page * BS >= len) return false;
  n = (int)min((int64_t)BS, len - (int64_t)page * BS);
  tok0 = start + (int64_t)page * BS;
  blk = p.block_tables[(int64_t)b * p.cols + page];
  if ((int64_t)blk >= p.num_blocks) {
    if (threadIdx.x == 0) raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
    blk = 0;
  }
  return true;
}

// V page chunk e (16 bytes at byte e * 16 of the [D][row_bytes] page) into
// shared rows padded to row_bytes + 4 bytes (one 32-bit word each).
template <int kRowBytes>
__device__ __forceinline__ void stage_v_chunk(unsigned char *vsm, int e, const uint4 &v) {
  constexpr int kPad = kRowBytes + 4;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int off = e * 16 + 4 * i;
    *reinterpret_cast<uint32_t *>(vsm + (off / kRowBytes) * kPad + off % kRowBytes) = w[i];
  }
}

template <typename T, int BS, int D>
__global__ void __launch_bounds__(gather_threads(D * BS * (int)sizeof(T) / 16))
    gather_kernel(const GatherParams p) {
  constexpr int kES = (int)sizeof(T);
  constexpr int kVE = 16 / kES;                 // elements per 16-byte vector
  constexpr int kChunks = D * BS * kES / 16;    // 16-byte chunks of one head's K (or V) page
  constexpr int kThreads = gather_threads(kChunks);
  constexpr int kPer = kChunks / kThreads;
  static_assert(kChunks % kThreads == 0, "whole chunks per thread");
  constexpr int kRowBytes = BS * kES;           // one V row: one dim over the page's tokens
  constexpr int kPad = kRowBytes + 4;
  __shared__ __align__(16) unsigned char vsm[D * kPad];
  int n;
  int64_t tok0;
  uint32_t blk;
  if (!gather_page(p, BS, n, tok0, blk)) return;
  const int h = blockIdx.z, H = p.num_kv_heads;
  const int64_t page = ((int64_t)blk * H + h) * (D * BS * kES);
  const uint4 *ks = reinterpret_cast<const uint4 *>(p.k_cache + page);
  const uint4 *vs = reinterpret_cast<const uint4 *>(p.v_cache + page);
  uint4 kr[kPer], vr[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kThreads;  // K chunk e: dims (e / BS) * kVE.., token e % BS
    if (e % BS < n) kr[i] = __ldg(ks + e);
    vr[i] = __ldg(vs + e);
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) stage_v_chunk<kRowBytes>(vsm, threadIdx.x + i * kThreads, vr[i]);
  const int64_t row = (int64_t)D * kES;  // bytes of one (token, head) output row
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kThreads;
    const int t = e % BS;
    if (t < n)
      *reinterpret_cast<uint4 *>(p.k_out + ((tok0 + t) * H + h) * row + (e / BS) * 16) = kr[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int o = threadIdx.x + i * kThreads;  // output vector: token o % BS, dims (o / BS) * kVE..
    const int t = o % BS, d0 = (o / BS) * kVE;
    if (t >= n) continue;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (kES == 4) {
        w[j] = *reinterpret_cast<const uint32_t *>(vsm + (d0 + j) * kPad + t * 4);
      } else {
        const uint32_t lo = *reinterpret_cast<const uint16_t *>(vsm + (d0 + 2 * j) * kPad + t * 2);
        const uint32_t hi = *reinterpret_cast<const uint16_t *>(vsm + (d0 + 2 * j + 1) * kPad + t * 2);
        w[j] = lo | (hi << 16);
      }
    }
    *reinterpret_cast<uint4 *>(p.v_out + ((tok0 + t) * H + h) * row + d0 * kES) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename T, int BS, int D>
int launch_gather_t(const GatherArgs &a, cudaStream_t stream) {
  GatherParams p{};
  p.k_out = static_cast<unsigned char *>(a.key_out);
  p.v_out = static_cast<unsigned char *>(a.value_out);
  p.k_cache = static_cast<const unsigned char *>(a.key_cache);
  p.v_cache = static_cast<const unsigned char *>(a.value_cache);
  p.block_tables = a.block_tables;
  p.cu = a.cu_seqlens_kv;
  p.num_blocks = a.num_blocks;
  p.cols = a.max_num_blocks_per_seq;
  p.num_kv_heads = a.num_kv_heads;
  if (a.num_kv_heads > 65535) return VASR_PA_EINVAL_SHAPE;
  dim3 grid((unsigned)a.max_num_blocks_per_seq, (unsigned)a.num_seqs, (unsigned)a.num_kv_heads);
  gather_kernel<T, BS, D><<<grid, gather_threads(D * BS * (int)sizeof(T) / 16), 0, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

// ================================================ gather_kv_cache, fp8 pages
// The fp8 form of the same gather: the call site passes k_scale / v_scale
// and the model dtype as out_dtype, and the packed rows hold
// float(stored byte) * scale rounded to that dtype. Same decomposition as
// gather_kernel: one CTA per (page, sequence, kv head), all loads first; a
// 16-byte K chunk (16 dims of one token) becomes 16 outputs, V rows [D][BS]
// are transposed through shared memory.
struct GatherFp8Params {
  GatherParams g;
  const float *k_scale;
  const float *v_scale;
};

template <typename TO>
__device__ __forceinline__ void store16_scaled(TO *dst, const float (&f)[16], float scale) {
  if constexpr (std::is_same<TO, float>::value) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      reinterpret_cast<float4 *>(dst)[i] =
          make_float4(f[4 * i] * scale, f[4 * i + 1] * scale, f[4 * i + 2] * scale, f[4 * i + 3] * scale);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const TO lo = Elem<TO>::from_f32(f[2 * i] * scale), hi = Elem<TO>::from_f32(f[2 * i + 1] * scale);
      w[i] = (uint32_t)(*reinterpret_cast<const uint16_t *>(&lo)) |
             ((uint32_t)(*reinterpret_cast<const uint16_t *>(&hi)) << 16);
    }
    reinterpret_cast<uint4 *>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4 *>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

template <typename TO, int BS, int D>
__global__ void __launch_bounds__(gather_threads(2 * D * BS / 16))
    gather_fp8_kernel(const GatherFp8Params q) {
  const GatherParams &p = q.g;
  constexpr int kChunks = D * BS / 16;           // 16-byte chunks of one head's K (or V) page
  constexpr int kThreads = gather_threads(2 * kChunks);
  constexpr int kPer = kChunks / kThreads < 1 ? 1 : kChunks / kThreads;
  constexpr int kVE = 16 / (int)sizeof(TO);      // outputs per 16-byte vector
  constexpr int kOut = D * BS / kVE;             // output V vectors of the page
  constexpr int kOutPer = kOut / kThreads;
  static_assert(kChunks % kThreads == 0 || kChunks < kThreads, "whole chunks per thread");
  static_assert(kOut % kThreads == 0, "whole output vectors per thread");
  constexpr int kPad = BS + 4;
  __shared__ __align__(16) unsigned char vsm[D * kPad];
  int n;
  int64_t tok0;
  uint32_t blk;
  if (!gather_page(p, BS, n, tok0, blk)) return;
  const int h = blockIdx.z, H = p.num_kv_heads;
  const int64_t page = ((int64_t)blk * H + h) * (D * BS);
  const uint4 *ks = reinterpret_cast<const uint4 *>(p.k_cache + page);
  const uint4 *vs = reinterpret_cast<const uint4 *>(p.v_cache + page);
  uint4 kr[kPer], vr[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kThreads;  // K chunk e: dims (e / BS) * 16.., token e % BS
    if (e < kChunks) {
      if (e % BS < n) kr[i] = __ldg(ks + e);
      vr[i] = __ldg(vs + e);
    }
  }
  const float kscale = __ldg(q.k_scale), vscale = __ldg(q.v_scale);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kThreads;
    if (e < kChunks) stage_v_chunk<BS>(vsm, e, vr[i]);
  }
  TO *k_out = reinterpret_cast<TO *>(p.k_out);
  TO *v_out = reinterpret_cast<TO *>(p.v_out);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kThreads;
    const int t = e % BS;
    if (e < kChunks && t < n) {
      float f[16];
      unpack16_fp8(kr[i], f);
      store16_scaled<TO>(k_out + ((tok0 + t) * H + h) * (int64_t)D + (e / BS) * 16, f, kscale);
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kOutPer; ++i) {
    const int o = threadIdx.x + i * kThreads;  // output vector: token o % BS, dims (o / BS) * kVE..
    const int t = o % BS, d0 = (o / BS) * kVE;
    if (t >= n) continue;
    alignas(16) TO vals[kVE];
#pragma unroll
    for (int j = 0; j < kVE; ++j) {
      __nv_fp8_e4m3 b8;
      b8.__x = vsm[(d0 + j) * kPad + t];
      vals[j] = Elem<TO>::from_f32(static_cast<float>(b8) * vscale);
    }
    *reinterpret_cast<uint4 *>(v_out + ((tok0 + t) * H + h) * (int64_t)D + d0) =
        *reinterpret_cast<const uint4 *>(vals);
  }
}

template <typename TO, int BS, int D>
int launch_gather_fp8_t(const GatherArgs &a, cudaStream_t stream) {
  GatherFp8Params q{};
  q.g.k_out = static_cast<unsigned char *>(a.key_out);
  q.g.v_out = static_cast<unsigned char *>(a.value_out);
  q.g.k_cache = static_cast<const unsigned char *>(a.key_cache);
  q.g.v_cache = static_cast<const unsigned char *>(a.value_cache);
  q.g.block_tables = a.block_tables;
  q.g.cu = a.cu_seqlens_kv;
  q.g.num_blocks = a.num_blocks;
  q.g.cols = a.max_num_blocks_per_seq;
  q.g.num_kv_heads = a.num_kv_heads;
  q.k_scale = a.k_scale;
  q.v_scale = a.v_scale;
  if (a.num_kv_heads > 65535) return VASR_PA_EINVAL_SHAPE;
  dim3 grid((unsigned)a.max_num_blocks_per_seq, (unsigned)a.num_seqs, (unsigned)a.num_kv_heads);
  gather_fp8_kernel<TO, BS, D><<<grid, gather_threads(2 * D * BS / 16), 0, stream>>>(q);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

// ============================================ fp8 pages -> 16-bit scratch pool
// Prefill over fp8 pages runs the 16-bit kernels on a scratch pool: entry
// (b, i) of the block table (i < pages of sequence b) becomes block
// b * cols + i of the pool, holding the page's K and V as T(byte * scale) in
// the 16-bit page layouts (K [D/8][BS][8], V [D][BS]); the remapped table is
// written too. One CTA per (table entry, kv head).
constexpr int kDequantThreads = 128;

template <typename TO, int BS, int D>
__global__ void __launch_bounds__(kDequantThreads) dequant_pages_kernel(
    const unsigned char *k_cache, const unsigned char *v_cache, const uint32_t *block_tables,
    const uint32_t *context_lens, int cols, int num_kv_heads, int64_t num_blocks,
    const float *k_scale, const float *v_scale, TO *k_out, TO *v_out, uint32_t *table_out) {
  const int i = blockIdx.x, b = blockIdx.y, h = blockIdx.z;
  const int64_t dst = (int64_t)b * cols + i;
  if (h == 0 && threadIdx.x == 0) table_out[dst] = (uint32_t)dst;
  const int64_t ctx = min((int64_t)context_lens[b], (int64_t)cols * BS);
  if ((int64_t)i * BS >= ctx) return;
  uint32_t blk = block_tables[(int64_t)b * cols + i];
  if ((int64_t)blk >= num_blocks) {
    if (threadIdx.x == 0) raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
    blk = 0;
  }
  const float ks = __ldg(k_scale), vs = __ldg(v_scale);
  const int64_t src_page = ((int64_t)blk * num_kv_heads + h) * D * BS;  // bytes
  const int64_t dst_page = (dst * num_kv_heads + h) * D * BS;           // elements
  // K chunk e = fp8 dims 16c.. of token t (c = e / BS, t = e % BS) -> 16-bit
  // chunks 2c, 2c + 1 of token t; V chunk e = 16 bytes of the [D][BS] rows ->
  // 16 elements at the same place. Both loads of every chunk a thread owns
  // are issued before any store.
  constexpr int kChunks = D * BS / 16;  // per page, for K and for V alike
  constexpr int kPer = (kChunks + kDequantThreads - 1) / kDequantThreads;
  uint4 kr[kPer], vr[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kDequantThreads;
    if (e < kChunks) {
      kr[i] = __ldg(reinterpret_cast<const uint4 *>(k_cache + src_page + (int64_t)e * 16));
      vr[i] = __ldg(reinterpret_cast<const uint4 *>(v_cache + src_page + (int64_t)e * 16));
    }
  }
  auto pack = [](const float *f, float scale) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const TO lo = Elem<TO>::from_f32(f[2 * j] * scale), hi = Elem<TO>::from_f32(f[2 * j + 1] * scale);
      w[j] = (uint32_t)(*reinterpret_cast<const uint16_t *>(&lo)) |
             ((uint32_t)(*reinterpret_cast<const uint16_t *>(&hi)) << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  };
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x + i * kDequantThreads;
    if (e >= kChunks) continue;
    const int c = e / BS, t = e % BS;
    float f[16];
    unpack16_fp8(kr[i], f);
    *reinterpret_cast<uint4 *>(k_out + dst_page + ((int64_t)(2 * c) * BS + t) * 8) = pack(f, ks);
    *reinterpret_cast<uint4 *>(k_out + dst_page + ((int64_t)(2 * c + 1) * BS + t) * 8) = pack(f + 8, ks);
    unpack16_fp8(vr[i], f);
    uint4 *d4 = reinterpret_cast<uint4 *>(v_out + dst_page + (int64_t)e * 16);
    d4[0] = pack(f, vs);
    d4[1] = pack(f + 8, vs);
  }
}

template <typename TO, int BS>
int launch_dequant_t(const DequantArgs &a, cudaStream_t s) {
  dim3 grid((unsigned)a.cols, (unsigned)a.num_seqs, (unsigned)a.num_kv_heads);
  dequant_pages_kernel<TO, BS, 128><<<grid, kDequantThreads, 0, s>>>(
      static_cast<const unsigned char *>(a.key_cache), static_cast<const unsigned char *>(a.value_cache),
      a.block_tables, a.context_lens, a.cols, a.num_kv_heads, a.num_blocks, a.k_scale, a.v_scale,
      static_cast<TO *>(a.key_out), static_cast<TO *>(a.value_out), a.table_out);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

// ============================================================ block copies
// copy_blocks: one CTA per (pair, layer, K|V) moves one block with 16-byte
// loads; each thread keeps kCopyUnroll loads in flight.
constexpr int kMaxLayers = 128;
constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 8;

struct CopyBlocksParams {
  unsigned char *k[kMaxLayers];
  unsigned char *v[kMaxLayers];
  const int64_t *mapping;
  int64_t num_blocks;
  int64_t block_bytes;
};

__device__ __forceinline__ void copy_block_bytes(unsigned char *dst, const unsigned char *src,
                                                 int64_t bytes) {
  const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
  const int64_t n = bytes / 16;
  const int64_t step = (int64_t)kCopyThreads * kCopyUnroll;
  int64_t base = 0;
  for (; base + step <= n; base += step) {
    uint4 r[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) r[u] = __ldcs(s4 + base + u * kCopyThreads + threadIdx.x);
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) __stcs(d4 + base + u * kCopyThreads + threadIdx.x, r[u]);
  }
  for (int64_t i = base + threadIdx.x; i < n; i += kCopyThreads) __stcs(d4 + i, __ldcs(s4 + i));
}

__global__ void __launch_bounds__(kCopyThreads) copy_blocks_kernel(const CopyBlocksParams p) {
  const int64_t pair = blockIdx.x;
  const int layer = blockIdx.y;
  const int64_t src = p.mapping[2 * pair];
  const int64_t dst = p.mapping[2 * pair + 1];
  if (src < 0 || dst < 0 || src >= p.num_blocks || dst >= p.num_blocks) {
    if (threadIdx.x == 0) raise_device_error(VASR_PA_DERR_MAPPING_RANGE);
    return;
  }
  unsigned char *base = (blockIdx.z == 0) ? p.k[layer] : p.v[layer];
  copy_block_bytes(base + dst * p.block_bytes, base + src * p.block_bytes, p.block_bytes);
}

struct SwapParams {
  unsigned char *dst;
  const unsigned char *src;
  const int64_t *mapping;
  int64_t src_blocks;
  int64_t dst_blocks;
  int64_t block_bytes;
};

__global__ void __launch_bounds__(kCopyThreads) swap_blocks_kernel(const SwapParams p) {
  const int64_t pair = blockIdx.x;
  const int64_t src = p.mapping[2 * pair];
  const int64_t dst = p.mapping[2 * pair + 1];
  if (src < 0 || dst < 0 || src >= p.src_blocks || dst >= p.dst_blocks) {
    if (threadIdx.x == 0) raise_device_error(VASR_PA_DERR_MAPPING_RANGE);
    return;
  }
  copy_block_bytes(p.dst + dst * p.block_bytes, p.src + src * p.block_bytes, p.block_bytes);
}

// ====================================================== fp8 KV append
// Pages of one-byte E4M3 values with per-tensor scales: cache = value / scale
// (IEEE division), rounded to nearest even and saturated to +-448 by the
// cuda_fp8.h conversion. Calls of 4096 tokens or more use the ring kernel
// below; calls of 128-4095 tokens the tiling of kv_append_kernel: a tile of
// tokens (all kv heads) is quantised into shared memory as bytes; K goes out
// as 16-byte chunks (16 dims of one token), V by runs of consecutive slots
// of one page row, as one vector store when a run fills an aligned group of
// min(16, BS) tokens.
struct AppendFp8Params {
  const unsigned char *key;
  const unsigned char *value;
  unsigned char *k_cache;
  unsigned char *v_cache;
  const int64_t *slots;
  const float *k_scale;
  const float *v_scale;
  int64_t num_tokens;
  int64_t k_stride_bytes;
  int64_t v_stride_bytes;
  int64_t num_blocks;
  int num_kv_heads;
  int tile_tokens;
  int heads_per_tile;
  int row_pitch;  // bytes of one staged token row (one byte per element) + 16
};

// The quotient x / s as the IEEE division rounds it, RN(x / s), from a
// multiply by inv = RN(1 / s) and one correction step: Markstein's theorem
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990): when y is within
// half an ulp of 1 / b and q within one ulp of a / b, the remainder
// r = a - b q is exact (one fma) and RN(q + r y) = RN(a / b). Here t = RN(x
// inv) is within one ulp of x / s. Outside the range where those conditions
// hold (s or inv not normal, |x| small enough for r to underflow, |t| large
// enough for t s to overflow) the IEEE division runs instead; a |t| below
// 2^-12 converts to a signed E4M3 zero whatever its last bits, so t stands.
struct QuantScale {
  float s, inv;
  bool fast;
};
__device__ __forceinline__ QuantScale quant_scale(float s) {
  const float inv = __frcp_rn(s);
  const uint32_t ei = __float_as_uint(inv) & 0x7f800000u, es = __float_as_uint(s) & 0x7f800000u;
  return {s, inv, ei != 0u && ei != 0x7f800000u && es != 0u && es != 0x7f800000u};
}
__device__ __forceinline__ float quotient_rn(float x, const QuantScale &q) {
  const float t = x * q.inv;
  const float at = fabsf(t);
  if (at < 0x1p-12f) return t;
  if (q.fast && at < 0x1p100f && fabsf(x) >= 0x1p-90f) return fmaf(fmaf(-t, q.s, x), q.inv, t);
  return __fdiv_rn(x, q.s);
}
// Two quotients -> two E4M3 bytes (nearest even, saturating at 448), x0 low.
__device__ __forceinline__ uint32_t e4m3x2_quotients(float x0, float x1, const QuantScale &q) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(quotient_rn(x0, q), quotient_rn(x1, q)),
                                            __NV_SATFINITE, __NV_E4M3);
}

// 16 source elements at src (16-byte aligned) -> 16 E4M3 bytes of x / scale.
template <typename T>
__device__ __forceinline__ uint4 quantize16(const unsigned char *src, const QuantScale &q) {
  constexpr int kPer = Elem<T>::kX;  // elements per 16-byte load
  float f[16];
#pragma unroll
  for (int c = 0; c < 16 / kPer; ++c) {
    float g[kPer];
    unpack_chunk<T>(__ldg(reinterpret_cast<const uint4 *>(src) + c), g);
#pragma unroll
    for (int e = 0; e < kPer; ++e) f[c * kPer + e] = g[e];
  }
  uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i)
    w[i >> 1] |= e4m3x2_quotients(f[2 * i], f[2 * i + 1], q) << (16 * (i & 1));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T, int BS, int D>
__global__ void __launch_bounds__(kAppendThreads) kv_append_fp8_kernel(const AppendFp8Params p) {
  constexpr int kCH = D / 16;                 // 16-byte K chunks per (token, head)
  constexpr int kTPS = BS < 16 ? BS : 16;     // tokens per vector V store
  constexpr int kES = (int)sizeof(T);
  extern __shared__ __align__(16) unsigned char sm[];
  const int pitch = p.row_pitch;
  unsigned char *kt = sm;
  unsigned char *vt = sm + p.tile_tokens * pitch;
  int64_t *s_slot = reinterpret_cast<int64_t *>(vt + p.tile_tokens * pitch);
  int *s_run_start = reinterpret_cast<int *>(s_slot + kAppendMaxTokens);
  int *s_run_len = s_run_start + kAppendMaxTokens;
  int *s_nruns = s_run_len + kAppendMaxTokens;

  const int TT = p.tile_tokens;
  const int64_t t0 = (int64_t)blockIdx.x * TT;
  const int h0 = blockIdx.y * p.heads_per_tile;
  const int HC = min(p.heads_per_tile, p.num_kv_heads - h0);
  const int ntok = (int)min((int64_t)TT, p.num_tokens - t0);
  const int64_t max_slot = p.num_blocks * BS;
  const int tid = threadIdx.x;
  const QuantScale ks = quant_scale(__ldg(p.k_scale)), vs = quant_scale(__ldg(p.v_scale));

  if (tid < ntok) {
    int64_t s = p.slots[t0 + tid];
    if (s >= max_slot) {
      raise_device_error(VASR_PA_DERR_SLOT_RANGE);
      s = -1;
    }
    s_slot[tid] = s;
  }
  // quantise the tile: (token, 16-element chunk) -> 16 bytes
  const int row_chunks = HC * kCH;
  for (int i = tid; i < ntok * row_chunks; i += kAppendThreads) {
    const int tt = i / row_chunks;
    const int r = i - tt * row_chunks;
    const int64_t col = ((int64_t)h0 * D + (int64_t)r * 16) * kES;
    *reinterpret_cast<uint4 *>(kt + tt * pitch + r * 16) =
        quantize16<T>(p.key + (t0 + tt) * p.k_stride_bytes + col, ks);
    *reinterpret_cast<uint4 *>(vt + tt * pitch + r * 16) =
        quantize16<T>(p.value + (t0 + tt) * p.v_stride_bytes + col, vs);
  }
  __syncthreads();
  if (tid == 0) {
    // split the tile into V runs (consecutive slots, same aligned group)
    int n = 0;
    int tt = 0;
    while (tt < ntok) {
      const int64_t s = s_slot[tt];
      if (s < 0) {
        ++tt;
        continue;
      }
      int len = 1;
      while (tt + len < ntok && len < kTPS && s_slot[tt + len] == s + len && ((s + len) % kTPS) != 0)
        ++len;
      s_run_start[n] = tt;
      s_run_len[n] = len;
      ++n;
      tt += len;
    }
    s_nruns[0] = n;
  }
  // K: (head, chunk, token) with token fastest
  for (int i = tid; i < ntok * row_chunks; i += kAppendThreads) {
    const int tt = i % ntok;
    const int r = i / ntok;
    const int64_t s = s_slot[tt];
    if (s < 0) continue;
    const int hc = r / kCH;
    const int c = r - hc * kCH;
    const int64_t blk = s / BS;
    const int off = (int)(s - blk * BS);
    const int64_t dst = ((((blk * p.num_kv_heads + h0 + hc) * kCH + c) * BS) + off) * 16;
    *reinterpret_cast<uint4 *>(p.k_cache + dst) =
        *reinterpret_cast<const uint4 *>(kt + tt * pitch + r * 16);
  }
  __syncthreads();
  // V: (head, dim, run) with run fastest
  const int nruns = s_nruns[0];
  const int nitems = nruns * HC * D;
  for (int i = tid; i < nitems; i += kAppendThreads) {
    const int j = i % nruns;
    const int hd = i / nruns;
    const int hc = hd / D;
    const int d = hd - hc * D;
    const int tt0 = s_run_start[j];
    const int len = s_run_len[j];
    const int64_t s = s_slot[tt0];
    const int64_t blk = s / BS;
    const int off = (int)(s - blk * BS);
    const unsigned char *src = vt + tt0 * pitch + hc * D + d;
    unsigned char *dst = p.v_cache + ((blk * p.num_kv_heads + h0 + hc) * D + d) * BS + off;
    if (len == kTPS && (off % kTPS) == 0) {
      uint32_t w[kTPS / 4];
#pragma unroll
      for (int q = 0; q < kTPS / 4; ++q)
        w[q] = (uint32_t)src[(4 * q) * pitch] | ((uint32_t)src[(4 * q + 1) * pitch] << 8) |
               ((uint32_t)src[(4 * q + 2) * pitch] << 16) |
               ((uint32_t)src[(4 * q + 3) * pitch] << 24);
      if constexpr (kTPS == 16)
        *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      else
        *reinterpret_cast<uint2 *>(dst) = make_uint2(w[0], w[1]);
    } else {
      for (int e = 0; e < len; ++e) dst[e] = src[e * pitch];
    }
  }
}

// Quotients RN(x / s) without a division, two elements per packed f32x2
// instruction, for positive scales in a range where per-element range checks
// reduce to a clamp of the source (QuantScale2::fast): s in [2^-60, 2^60]
// (f16 sources: [2^-60, 2^7]). The source is clamped first to +-B, B the
// 16-bit value nearest s 2^15 (at most 65504 for f16); NaN stays NaN. Any
// |x| above B has |x / s| > 2^14 and saturates to +-448 like B itself, so the
// clamp moves no byte; after it |t| = |RN(x inv)| <= 2^15 (1 + 2^-8), t s
// stays finite, and
//  - |x / s| >= 2^-11: |x| >= 2^-71 keeps the remainder x - t s normal and
//    exact (s >= 2^-60), quotient_rn's conditions, and one correction step
//    gives RN(x / s);
//  - |x / s| < 2^-11: the byte is a signed zero; the corrected value stays
//    below 2^-10 in magnitude with t's sign.
// The remainder r = x - t s is computed rounding toward -inf: a nonzero r is
// exact either way, and an exact zero comes out as -0, so that t + r inv
// keeps the sign of a zero t (x = -0: -0 + -0; x = +0: -0 + +0 = +0), where a
// round-to-nearest remainder (+0) would turn t = -0 into +0.
// Other scales use quotient_rn element by element.
struct QuantScale2 {
  float2 inv;      // (1 / s, 1 / s) rounded
  float2 ns;       // (-s, -s)
  uint32_t bhi;    // (B, B) as packed 16-bit source values
  float bf;        // B for f32 sources
  QuantScale one;
  bool fast;
};
template <typename T>
__device__ __forceinline__ QuantScale2 quant_scale2(float s) {
  QuantScale2 q;
  q.one = quant_scale(s);
  q.inv = make_float2(q.one.inv, q.one.inv);
  q.ns = make_float2(-s, -s);
  const float top = std::is_same<T, __half>::value ? 0x1p7f : 0x1p60f;
  q.fast = s >= 0x1p-60f && s <= top;  // false for NaN and negative scales
  const float b = fminf(s * 0x1p15f, 65504.f * (std::is_same<T, __half>::value ? 1.f : 0x1p100f));
  q.bf = b;
  uint32_t h = 0;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    h = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b));
  else if constexpr (std::is_same<T, __half>::value)
    h = (uint32_t)__half_as_ushort(__float2half_rn(b));
  q.bhi = h | (h << 16);
  return q;
}
// Clamp a packed pair of 16-bit source values to [-B, B], NaN propagating:
// one min of magnitudes whose result takes sign(x) xor sign(B) = sign(x).
template <typename T>
__device__ __forceinline__ uint32_t clamp_pair(uint32_t w, const QuantScale2 &q) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("min.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(q.bhi));
  else
    asm("min.NaN.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(q.bhi));
  return r;
}
__device__ __forceinline__ float clamp_f32(float x, float b) {
  float y;
  asm("min.NaN.xorsign.abs.f32 %0, %1, %2;" : "=f"(y) : "f"(x), "f"(b));
  return y;
}
// Two clamped values -> RN(x / s) each (fast scales).
__device__ __forceinline__ float2 quot2_fast(float2 x, const QuantScale2 &q) {
  const float2 t = __fmul2_rn(x, q.inv);
  return __ffma2_rn(__ffma2_rd(t, q.ns, x), q.inv, t);
}
__device__ __forceinline__ uint32_t cvt_e4m3x2(float a, float b) {  // a -> low byte
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}
// One 32-bit source word (a pair of 16-bit values, or one f32 in .x with
// .y = next word) -> the pair's quotients in f32.
template <typename T, bool kFast>
__device__ __forceinline__ float2 quot_word(uint32_t w, const QuantScale2 &q) {
  float2 x;
  if constexpr (kFast) w = clamp_pair<T>(w, q);
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    unpack_bf16x2(w, x.x, x.y);
  else
    unpack_half2(w, x.x, x.y);
  if constexpr (kFast) return quot2_fast(x, q);
  return make_float2(quotient_rn(x.x, q.one), quotient_rn(x.y, q.one));
}
template <bool kFast>
__device__ __forceinline__ float2 quot_f32(float2 x, const QuantScale2 &q) {
  if constexpr (kFast) return quot2_fast(make_float2(clamp_f32(x.x, q.bf), clamp_f32(x.y, q.bf)), q);
  return make_float2(quotient_rn(x.x, q.one), quotient_rn(x.y, q.one));
}

// Prefill-sized fp8 appends (4096 tokens or more): a persistent grid of
// CTAs of 8 consumer warps and one producer warp over (16-token tile, pair
// of kv heads) items, dealt round-robin (item = tile * pairs + pair). The
// producer fills a ring of shared-memory stages: per token one bulk copy of
// its K row and one of its V row (the pair's 2 x D elements, contiguous in
// the source) and an 8-byte asynchronous copy of its slot, all completing on
// the stage's full barrier. A consumer warp reads its values of a stage,
// releases the stage (one arrive per warp on its empty barrier) and
// quantises from registers, 32 elements per thread:
//  warps 0-3 (K): head w >> 1, 16-dim chunk (lane >> 3) + 4 (w & 1), tokens
//     lane & 7 and (lane & 7) + 8: one 16-byte page chunk each, converted
//     in dim pairs;
//  warps 4-7 (V): head (w - 4) >> 1, dims 2 j and 2 j + 1 with j = 32
//     ((w - 4) & 1) + lane, all 16 tokens, converted in token pairs so that
//     each conversion yields two adjacent bytes of a dim's page row: a row
//     of min(16, BS) consecutive slots from an aligned start leaves as one
//     vector store, any other group byte by byte.
// Staged rows are kRow + 16 bytes apart, so the 8 K rows a quarter-warp
// reads at one offset fall in different bank groups. Every wait is bounded;
// a warp whose wait gave up stops, and the producer then waits (bounded) for
// the copies of its last stages before the CTA leaves.
constexpr int kRingConsumers = 256;
constexpr int kRingThreads = kRingConsumers + 32;
template <typename T, int D, int HPT>
struct RingLayout {
  static constexpr int kRow = HPT * D * (int)sizeof(T);  // one token's K (or V) row of the pair
  static constexpr int kPitch = kRow + 16;
  static constexpr int kSlots = 2 * kTile16 * kPitch;     // 16 int64 slots after the rows
  static constexpr int kStage = kSlots + kTile16 * 8;
  static constexpr int kStages = sizeof(T) == 4 ? 3 : 4;
  static constexpr int kBars = kStages * kStage;          // full[kStages], empty[kStages]
  static constexpr int kBytes = kBars + 2 * kStages * 8;
  static_assert(kPitch % 16 == 0 && kStage % 16 == 0, "bulk copy destinations 16-byte aligned");
};

template <typename T, int BS, int D, int HPT, bool kFast>
__device__ __forceinline__ void fp8_ring_body(const AppendFp8Params &p, const QuantScale2 &ks,
                                              const QuantScale2 &vs, const unsigned char *smem,
                                              uint32_t sbase) {
  static_assert(D == 128 && HPT == 2 && kRingConsumers == 256, "thread map: 2 heads x 128 dims x 16 tokens");
  using L = RingLayout<T, D, HPT>;
  constexpr int kES = (int)sizeof(T);
  constexpr int kTPS = BS < 16 ? BS : 16;  // tokens per V page-row vector
  constexpr int kGroups = kTile16 / kTPS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pairs = (p.num_kv_heads + HPT - 1) / HPT;
  const int tiles = (int)((p.num_tokens + kTile16 - 1) / kTile16);
  // items blockIdx.x, + gridDim.x, ... as (tile, pair), advanced without division
  const int step_t = (int)gridDim.x / pairs, step_p = (int)gridDim.x % pairs;
  auto full = [&](int st) { return sbase + (uint32_t)L::kBars + 8u * (uint32_t)st; };
  auto empty = [&](int st) { return sbase + (uint32_t)L::kBars + 8u * (uint32_t)(L::kStages + st); };
  int tile = (int)blockIdx.x / pairs, pair = (int)blockIdx.x % pairs;
  auto advance = [&]() {
    tile += step_t;
    pair += step_p;
    if (pair >= pairs) {
      pair -= pairs;
      ++tile;
    }
  };

  if (warp == kRingConsumers / 32) {
    // ------------------------------------------------------------ producer
    int k = 0;
    for (; tile < tiles; advance(), ++k) {
      const int st = k % L::kStages;
      if (k >= L::kStages) {
        const bool ok = mbar_wait_bounded(empty(st), (uint32_t)((k / L::kStages - 1) & 1));
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      const int64_t t0 = (int64_t)tile * kTile16;
      const int h0 = pair * HPT;
      const int hc = min(HPT, p.num_kv_heads - h0);
      const int ntok = (int)min((int64_t)kTile16, p.num_tokens - t0);
      const int pieces = hc * D * kES / 16;  // 16-byte pieces of a token's row
      const uint32_t base = sbase + (uint32_t)(st * L::kStage);
      const int64_t col = (int64_t)h0 * D * kES;
      const unsigned char *ksrc = p.key + t0 * p.k_stride_bytes + col;
      const unsigned char *vsrc = p.value + t0 * p.v_stride_bytes + col;
      for (int t = 0; t < ntok; ++t) {
#pragma unroll
        for (int c = lane; c < L::kRow / 16; c += 32) {
          if (c < pieces) {
            cp_async16(base + (uint32_t)(t * L::kPitch + c * 16), ksrc + t * p.k_stride_bytes + c * 16);
            cp_async16(base + (uint32_t)((kTile16 + t) * L::kPitch + c * 16), vsrc + t * p.v_stride_bytes + c * 16);
          }
        }
      }
      if (lane < ntok) cp_async8(base + (uint32_t)(L::kSlots + lane * 8), p.slots + t0 + lane);
      cp_async_arrive_noinc(full(st));  // one of the 32 lane arrivals of the phase
    }
    // the copies of the last stages issued land before shared memory is let go
    // (already waited for by the consumers in a healthy run)
    for (int j = max(0, k - L::kStages); j < k; ++j)
      mbar_wait_bounded(full(j % L::kStages), (uint32_t)((j / L::kStages) & 1));
    return;
  }

  // -------------------------------------------------------------- consumers
  const bool kwarp = warp < 4;
  const int hc = kwarp ? warp >> 1 : (warp - 4) >> 1;  // head of the pair (warp-uniform)
  const int kt = lane & 7, kc = (lane >> 3) + 4 * (warp & 1);  // K: tokens kt, kt + 8; 16-dim chunk
  const int jp = 32 * ((warp - 4) & 1) + lane;                // V: dims 2 jp, 2 jp + 1
  const int64_t max_slot = p.num_blocks * BS;
  // bytes of one block of the fp8 cache; the launcher keeps blocks and this below 2^32
  const uint32_t kpage = (uint32_t)(p.num_kv_heads * D * BS);
  auto block_base = [&](uint64_t slot) {  // byte offset of slot's block, and slot % BS
    return (uint64_t)(uint32_t)(slot / BS) * kpage;
  };
  int k = 0;
  for (; tile < tiles; advance(), ++k) {
    const int st = k % L::kStages;
    const bool ok = mbar_wait_bounded(full(st), (uint32_t)((k / L::kStages) & 1));
    if (!__all_sync(0xffffffffu, ok)) break;
    const int h = pair * HPT + hc;
    const bool live = h < p.num_kv_heads;
    const int ntok = (int)min((int64_t)kTile16, p.num_tokens - (int64_t)tile * kTile16);
    const unsigned char *stage = smem + st * L::kStage;
    const int64_t *sslot = reinterpret_cast<const int64_t *>(stage + L::kSlots);
    if (kwarp) {
      // ------------------------------------------------------------- K
      uint4 raw[2][kES];
      int64_t sl[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = kt + 8 * u;
        sl[u] = t < ntok ? sslot[t] : -1;
        const unsigned char *src = stage + t * L::kPitch + (hc * D + kc * 16) * kES;
#pragma unroll
        for (int i = 0; i < kES; ++i) raw[u][i] = *reinterpret_cast<const uint4 *>(src + 16 * i);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(st));  // this warp is done with the stage
      if (!live) continue;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (sl[u] >= max_slot) {
          raise_device_error(VASR_PA_DERR_SLOT_RANGE);
          continue;
        }
        if (sl[u] < 0) continue;
        const uint32_t *wd = reinterpret_cast<const uint32_t *>(raw[u]);
        uint32_t out[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // output word i = dims 4 i .. 4 i + 3
          float2 a, b;
          if constexpr (kES == 2) {
            a = quot_word<T, kFast>(wd[2 * i], ks);
            b = quot_word<T, kFast>(wd[2 * i + 1], ks);
          } else {
            a = quot_f32<kFast>(make_float2(__uint_as_float(wd[4 * i]), __uint_as_float(wd[4 * i + 1])), ks);
            b = quot_f32<kFast>(make_float2(__uint_as_float(wd[4 * i + 2]), __uint_as_float(wd[4 * i + 3])), ks);
          }
          out[i] = cvt_e4m3x2(a.x, a.y) | (cvt_e4m3x2(b.x, b.y) << 16);
        }
        const uint64_t us = (uint64_t)sl[u];
        const uint64_t dst = block_base(us) + (uint32_t)(((h * (D / 16) + kc) * BS + (int)(us % BS)) * 16);
        *reinterpret_cast<uint4 *>(p.k_cache + dst) = make_uint4(out[0], out[1], out[2], out[3]);
      }
      continue;
    }
    // --------------------------------------------------------------- V
    float2 v[kTile16];  // quotients of (dim 2 jp, dim 2 jp + 1) of each token
    const unsigned char *vsrc = stage + kTile16 * L::kPitch + (hc * D + 2 * jp) * kES;
    int64_t s = lane < ntok && lane < kTile16 ? sslot[lane] : -1;  // lanes 0-15: token lane's slot
    if constexpr (kES == 2) {
      uint32_t wv[kTile16];
#pragma unroll
      for (int t = 0; t < kTile16; ++t) wv[t] = *reinterpret_cast<const uint32_t *>(vsrc + t * L::kPitch);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(st));
      if (!live) continue;
#pragma unroll
      for (int t = 0; t < kTile16; ++t) v[t] = quot_word<T, kFast>(wv[t], vs);
    } else {
      float2 xv[kTile16];
#pragma unroll
      for (int t = 0; t < kTile16; ++t) xv[t] = *reinterpret_cast<const float2 *>(vsrc + t * L::kPitch);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(st));
      if (!live) continue;
#pragma unroll
      for (int t = 0; t < kTile16; ++t) v[t] = quot_f32<kFast>(xv[t], vs);
    }
    if (s >= max_slot) {
      raise_device_error(VASR_PA_DERR_SLOT_RANGE);
      s = -1;
    }
    // runs: kTPS consecutive slots from a multiple of kTPS
    const int idx = lane & 15;
    const int g0 = idx & ~(kTPS - 1);
    const int64_t gfirst = __shfl_sync(0xffffffffu, s, g0);
    const bool run = lane < kTile16 && s >= 0 && (gfirst & (kTPS - 1)) == 0 && s == gfirst + (idx - g0);
    const uint32_t ball = __ballot_sync(0xffffffffu, run);
    uint32_t row[2][4];  // [dim][tokens 4 i .. 4 i + 3], token 4 i in the low byte
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      row[0][i] = cvt_e4m3x2(v[4 * i].x, v[4 * i + 1].x) | (cvt_e4m3x2(v[4 * i + 2].x, v[4 * i + 3].x) << 16);
      row[1][i] = cvt_e4m3x2(v[4 * i].y, v[4 * i + 1].y) | (cvt_e4m3x2(v[4 * i + 2].y, v[4 * i + 3].y) << 16);
    }
    const uint32_t vrow = (uint32_t)(h * D + 2 * jp);
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      // the group's first slot (the run check already fetched it when one group spans the tile)
      const int64_t gs = kGroups == 1 ? gfirst : __shfl_sync(0xffffffffu, s, g * kTPS);
      if (((ball >> (g * kTPS)) & ((1u << kTPS) - 1u)) == (1u << kTPS) - 1u) {
        const uint64_t us = (uint64_t)gs;
        unsigned char *dst = p.v_cache + block_base(us) + (uint32_t)(vrow * BS + us % BS);
#pragma unroll
        for (int d = 0; d < 2; ++d) {
          if constexpr (kTPS == 16)
            *reinterpret_cast<uint4 *>(dst + d * BS) = make_uint4(row[d][0], row[d][1], row[d][2], row[d][3]);
          else
            *reinterpret_cast<uint2 *>(dst + d * BS) = make_uint2(row[d][2 * g], row[d][2 * g + 1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < kTPS; ++e) {
          const int t = g * kTPS + e;
          const int64_t ts = __shfl_sync(0xffffffffu, s, t);
          if (ts < 0) continue;
          const uint64_t us = (uint64_t)ts;
          unsigned char *dst = p.v_cache + block_base(us) + (uint32_t)(vrow * BS + us % BS);
#pragma unroll
          for (int d = 0; d < 2; ++d) dst[d * BS] = (unsigned char)(row[d][t >> 2] >> (8 * (t & 3)));
        }
      }
    }
  }
}

template <typename T, int BS, int D, int HPT>
__global__ void __launch_bounds__(kRingThreads) kv_append_fp8_ring_kernel(const AppendFp8Params p) {
  extern __shared__ __align__(128) unsigned char ring_smem[];
  using L = RingLayout<T, D, HPT>;
  const uint32_t sbase = smem_addr(ring_smem);
  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kStages; ++i) {
      mbar_init(sbase + L::kBars + 8 * i, 32);  // one arrival per producer lane, when its copies land
      mbar_init(sbase + L::kBars + 8 * (L::kStages + i), kRingConsumers / 32);
    }
    mbar_fence_init();
  }
  __syncthreads();
  const QuantScale2 ks = quant_scale2<T>(__ldg(p.k_scale)), vs = quant_scale2<T>(__ldg(p.v_scale));
  if (ks.fast && vs.fast)
    fp8_ring_body<T, BS, D, HPT, true>(p, ks, vs, ring_smem, sbase);
  else
    fp8_ring_body<T, BS, D, HPT, false>(p, ks, vs, ring_smem, sbase);
}

// Decode-sized fp8 appends (a few tokens, one per page row): one warp per
// (token, kv head), K as 16-byte chunks (lane c < D / 16 writes chunk c), V
// one byte per dim — the layout admits no wider V store for a lone token.
template <typename T, int BS, int D>
__global__ void __launch_bounds__(128) kv_append_fp8_token_kernel(const AppendFp8Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * 4 + warp;
  if (item >= p.num_tokens * p.num_kv_heads) return;
  const int64_t t = item / p.num_kv_heads;
  const int h = (int)(item % p.num_kv_heads);
  const int64_t slot = p.slots[t];
  if (slot < 0) return;
  const int64_t blk = slot / BS;
  const int off = (int)(slot % BS);
  if (blk >= p.num_blocks) {
    if (lane == 0) raise_device_error(VASR_PA_DERR_SLOT_RANGE);
    return;
  }
  const QuantScale ks = quant_scale(__ldg(p.k_scale)), vs = quant_scale(__ldg(p.v_scale));
  const unsigned char *k = p.key + t * p.k_stride_bytes + (int64_t)h * D * sizeof(T);
  const T *v = reinterpret_cast<const T *>(p.value + t * p.v_stride_bytes) + (int64_t)h * D;
  const int64_t page = (int64_t)blk * p.num_kv_heads + h;
  if (lane < D / 16)
    *reinterpret_cast<uint4 *>(p.k_cache + ((page * (D / 16) + lane) * BS + off) * 16) =
        quantize16<T>(k + lane * 16 * sizeof(T), ks);
  // lane covers dims lane and lane + 32 (a pair), then lane + 64 and lane + 96
#pragma unroll
  for (int d = lane; d < D; d += 64) {
    const uint32_t pr = e4m3x2_quotients(Elem<T>::to_f32(v[d]), Elem<T>::to_f32(v[d + 32]), vs);
    p.v_cache[(page * D + d) * BS + off] = (unsigned char)(pr & 0xffu);
    p.v_cache[(page * D + d + 32) * BS + off] = (unsigned char)(pr >> 8);
  }
}

template <typename T, int BS, int D>
int launch_append_fp8_t(const AppendArgs &a, cudaStream_t stream) {
  AppendFp8Params p{};
  p.key = static_cast<const unsigned char *>(a.key);
  p.value = static_cast<const unsigned char *>(a.value);
  p.k_cache = static_cast<unsigned char *>(a.key_cache);
  p.v_cache = static_cast<unsigned char *>(a.value_cache);
  p.slots = a.slot_mapping;
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  p.num_tokens = a.num_tokens;
  p.k_stride_bytes = a.key_token_stride * (int64_t)sizeof(T);
  p.v_stride_bytes = a.value_token_stride * (int64_t)sizeof(T);
  p.num_blocks = a.num_blocks;
  p.num_kv_heads = a.num_kv_heads;
  if (a.num_tokens < 128) {  // decode-sized: a warp per (token, kv head)
    const int64_t ctas = (a.num_tokens * a.num_kv_heads + 3) / 4;
    if (ctas > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
    kv_append_fp8_token_kernel<T, BS, D><<<(unsigned)ctas, 128, 0, stream>>>(p);
    return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
  }
  if (a.num_tokens >= 4096 && a.num_blocks <= 0xffffffffll &&
      (int64_t)a.num_kv_heads * D * BS <= 0xffffffffll) {  // prefill chunks: persistent ring CTAs
    using L = RingLayout<T, D, 2>;
    auto *kern = kv_append_fp8_ring_kernel<T, BS, D, 2>;
    static std::atomic<uint64_t> attr_done{0};
    static std::atomic<int64_t> resident[64];
    if (!ensure_smem_attr(kern, L::kBytes, attr_done)) return VASR_PA_ELAUNCH;
    const int64_t items = (a.num_tokens + kTile16 - 1) / kTile16 * ((a.num_kv_heads + 1) / 2);
    int64_t ctas = resident_ctas(kern, kRingThreads, L::kBytes, resident);
    if (ctas <= 0 || ctas > items) ctas = items;
    if (ctas > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
    kern<<<(unsigned)ctas, kRingThreads, L::kBytes, stream>>>(p);
    return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
  }
  const int tt = 8;  // mid-sized: 8-token tiles of up to 2 KB of heads (one byte per element)
  p.tile_tokens = tt;
  p.heads_per_tile = kAppendRowBytes / D;
  // staged rows hold the tile's heads only; shared memory sized to the tile
  p.row_pitch = (a.num_kv_heads < p.heads_per_tile ? a.num_kv_heads : p.heads_per_tile) * D + 16;
  constexpr int kTail = kAppendMaxTokens * 8 + (2 * kAppendMaxTokens + 1) * 4;
  const int smem = 2 * tt * p.row_pitch + kTail;
  constexpr int kSmemMax = 2 * kAppendMaxTokens * (kAppendRowBytes + 16) + kTail;
  static std::atomic<uint64_t> attr_done{0};
  if (!ensure_smem_attr(kv_append_fp8_kernel<T, BS, D>, kSmemMax, attr_done)) return VASR_PA_ELAUNCH;
  const int64_t tiles = (a.num_tokens + tt - 1) / tt;
  if (tiles > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
  dim3 grid((unsigned)tiles, (unsigned)((a.num_kv_heads + p.heads_per_tile - 1) / p.heads_per_tile));
  kv_append_fp8_kernel<T, BS, D><<<grid, kAppendThreads, smem, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

template <typename T>
int launch_append_fp8_bs(const AppendArgs &a, cudaStream_t s) {
  if (a.head_dim != 128) return VASR_PA_ENOT_SUPPORTED;
  switch (a.block_size) {
    case 8: return launch_append_fp8_t<T, 8, 128>(a, s);
    case 16: return launch_append_fp8_t<T, 16, 128>(a, s);
    case 32: return launch_append_fp8_t<T, 32, 128>(a, s);
    default: return VASR_PA_EINVAL_BLOCKSIZE;
  }
}

}  // namespace

// ------------------------------------------------------------- launchers
int launch_append(const AppendArgs &a, cudaStream_t s) {
  if (a.cache_dtype == VASR_PA_FP8_E4M3) {
    switch (a.dtype) {
      case VASR_PA_F32: return launch_append_fp8_bs<float>(a, s);
      case VASR_PA_BF16: return launch_append_fp8_bs<__nv_bfloat16>(a, s);
      case VASR_PA_F16: return launch_append_fp8_bs<__half>(a, s);
      default: return VASR_PA_EINVAL_DTYPE;
    }
  }
#define VASR_APPEND_CASE(T, BS_, D_) \
  if (a.block_size == BS_ && a.head_dim == D_) return launch_append_t<T, BS_, D_>(a, s);
#define VASR_APPEND_T(T)                                                            \
  VASR_APPEND_CASE(T, 8, 64) VASR_APPEND_CASE(T, 16, 64) VASR_APPEND_CASE(T, 32, 64) \
  VASR_APPEND_CASE(T, 8, 128) VASR_APPEND_CASE(T, 16, 128) VASR_APPEND_CASE(T, 32, 128) \
  VASR_APPEND_CASE(T, 8, 256) VASR_APPEND_CASE(T, 16, 256) VASR_APPEND_CASE(T, 32, 256)
  if (a.dtype == VASR_PA_F32) { VASR_APPEND_T(float) }
  if (a.dtype == VASR_PA_BF16) { VASR_APPEND_T(__nv_bfloat16) }
  if (a.dtype == VASR_PA_F16) { VASR_APPEND_T(__half) }
#undef VASR_APPEND_T
#undef VASR_APPEND_CASE
  return VASR_PA_ENOT_SUPPORTED;
}

int launch_dequant_pages(const DequantArgs &a, cudaStream_t s) {
  if (a.head_dim != 128 || a.num_seqs > 65535 || a.num_kv_heads > 65535) return VASR_PA_ENOT_SUPPORTED;
  const bool bf = a.dtype == VASR_PA_BF16;
  if (!bf && a.dtype != VASR_PA_F16) return VASR_PA_EINVAL_DTYPE;
  switch (a.block_size) {
    case 8: return bf ? launch_dequant_t<__nv_bfloat16, 8>(a, s) : launch_dequant_t<__half, 8>(a, s);
    case 16: return bf ? launch_dequant_t<__nv_bfloat16, 16>(a, s) : launch_dequant_t<__half, 16>(a, s);
    case 32: return bf ? launch_dequant_t<__nv_bfloat16, 32>(a, s) : launch_dequant_t<__half, 32>(a, s);
    default: return VASR_PA_EINVAL_BLOCKSIZE;
  }
}

int launch_gather(const GatherArgs &a, cudaStream_t s) {
  if (a.cache_dtype == VASR_PA_FP8_E4M3) {
    if (a.k_scale == nullptr || a.v_scale == nullptr) return VASR_PA_EINVAL_POINTER;
#define VASR_GATHER8_CASE(T, BS_, D_) \
  if (a.block_size == BS_ && a.head_dim == D_) return launch_gather_fp8_t<T, BS_, D_>(a, s);
#define VASR_GATHER8_T(T)                                                              \
  VASR_GATHER8_CASE(T, 8, 64) VASR_GATHER8_CASE(T, 16, 64) VASR_GATHER8_CASE(T, 32, 64) \
  VASR_GATHER8_CASE(T, 8, 128) VASR_GATHER8_CASE(T, 16, 128) VASR_GATHER8_CASE(T, 32, 128) \
  VASR_GATHER8_CASE(T, 8, 256) VASR_GATHER8_CASE(T, 16, 256) VASR_GATHER8_CASE(T, 32, 256)
    if (a.dtype == VASR_PA_F32) { VASR_GATHER8_T(float) }
    if (a.dtype == VASR_PA_BF16) { VASR_GATHER8_T(__nv_bfloat16) }
    if (a.dtype == VASR_PA_F16) { VASR_GATHER8_T(__half) }
#undef VASR_GATHER8_T
#undef VASR_GATHER8_CASE
    return VASR_PA_ENOT_SUPPORTED;
  }
#define VASR_GATHER_CASE(T, BS_, D_) \
  if (a.block_size == BS_ && a.head_dim == D_) return launch_gather_t<T, BS_, D_>(a, s);
#define VASR_GATHER_T(T)                                                             \
  VASR_GATHER_CASE(T, 8, 64) VASR_GATHER_CASE(T, 16, 64) VASR_GATHER_CASE(T, 32, 64) \
  VASR_GATHER_CASE(T, 8, 128) VASR_GATHER_CASE(T, 16, 128) VASR_GATHER_CASE(T, 32, 128) \
  VASR_GATHER_CASE(T, 8, 256) VASR_GATHER_CASE(T, 16, 256) VASR_GATHER_CASE(T, 32, 256)
  if (a.dtype == VASR_PA_F32) { VASR_GATHER_T(float) }
  if (a.dtype == VASR_PA_BF16) { VASR_GATHER_T(__nv_bfloat16) }
  if (a.dtype == VASR_PA_F16) { VASR_GATHER_T(__half) }
#undef VASR_GATHER_T
#undef VASR_GATHER_CASE
  return VASR_PA_ENOT_SUPPORTED;
}

int launch_copy_blocks(void *const *k, void *const *v, int layers, const int64_t *mapping,
                       int64_t pairs, int64_t num_blocks, int64_t block_bytes, cudaStream_t s) {
  if (layers > kMaxLayers) return VASR_PA_EINVAL_SHAPE;
  CopyBlocksParams p{};
  for (int l = 0; l < layers; ++l) {
    p.k[l] = static_cast<unsigned char *>(k[l]);
    p.v[l] = static_cast<unsigned char *>(v[l]);
  }
  for (int l = layers; l < kMaxLayers; ++l) p.k[l] = p.v[l] = nullptr;
  p.mapping = mapping;
  p.num_blocks = num_blocks;
  p.block_bytes = block_bytes;
  // pairs on x (up to 2^31-1), layers on y, K/V on z
  dim3 grid((unsigned)pairs, (unsigned)layers, 2);
  copy_blocks_kernel<<<grid, kCopyThreads, 0, s>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

int launch_swap_blocks(void *dst, const void *src, const int64_t *mapping, int64_t pairs,
                       int64_t src_blocks, int64_t dst_blocks, int64_t block_bytes,
                       cudaStream_t s) {
  SwapParams p{};
  p.dst = static_cast<unsigned char *>(dst);
  p.src = static_cast<const unsigned char *>(src);
  p.mapping = mapping;
  p.src_blocks = src_blocks;
  p.dst_blocks = dst_blocks;
  p.block_bytes = block_bytes;
  swap_blocks_kernel<<<(unsigned)pairs, kCopyThreads, 0, s>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

int read_error_kv_ops(uint32_t *bits, bool clear, cudaStream_t s) {
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

// prefill.cu — causal varlen (chunked) prefill attention over the pages.
//
// Semantics (see vasr_pa_paged_attention_varlen_prefill): sequence b owns
// query rows [cu_q[b], cu_q[b+1]); row i sits at absolute position
// ctx[b] - qlen_b + i and attends keys j <= position — the cached causal
// mask of vasr-models/src/model/attention.rs:86-149 applied to
// run_single_sequence_attention (:243-286). Keys are read straight from the
// pages, replacing gather_kv_cache + flash_attn_varlen
// (thinker_text.rs:1344-1365).
//
// bf16 / f16: tensor-core kernel (mma.sync m16n8k16, f32 accumulate),
// FlashAttention-2 style. A CTA of 8 warps owns 128 rows = (128 / G) query
// positions x the G query heads of one kv head, so each K/V tile staged in
// shared memory serves the whole GQA group and 128 rows. K pages
// [D/8][bs][8] and V pages [D][bs] are copied verbatim by 1-D CTA-local bulk
// copies into a 2-stage ring and both feed ldmatrix directly: a K page row
// (8 dims of one token) and a V page row (8 tokens of one dim) are each one
// 16-byte ldmatrix row. 64-key tiles are computed in two 32-key halves and
// the query fragments are re-read from shared memory per k-step, which keeps
// the kernel under 128 registers (2 CTAs = 16 warps per SM). Warps whose
// rows the causal mask hides from a whole half-tile skip it.
// f32: CUDA-core kernel, one CTA per (query row, kv head), online softmax.

#include "common.cuh"
#include "launch.h"

namespace vasr {
namespace {

struct PrefillParams {
  void *out;
  const void *q;
  const void *k_cache;
  const void *v_cache;
  const uint32_t *block_tables;
  const uint32_t *context_lens;
  const uint32_t *cu_q;
  int64_t q_stride;  // elements between query rows
  int64_t num_blocks;
  int num_seqs;
  int num_heads;
  int num_kv_heads;
  int cols;
  int tiles;  // position tiles per sequence (ceil(max_query_len / positions per CTA))
  float scale;
  float softcap;
};

// Find the sequence that owns query row t (cu_q is non-decreasing, B+1 long).
__device__ __forceinline__ int seq_of_row(const uint32_t *cu, int num_seqs, int64_t t) {
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((int64_t)cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// -------------------------------------------------- tensor-core kernel
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                            uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

template <typename T, int BS, int D, int G>
struct TcCfg {
  static constexpr int kWarps = 8;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kRows = 16 * kWarps;       // rows (position x head) per CTA
  static constexpr int kPos = kRows / G;          // query positions per CTA
  static constexpr int kBK = 64;                  // keys per staged tile
  static constexpr int kHK = 32;                  // keys per compute half
  static constexpr int kPagesPerTile = (kBK + BS - 1) / BS;
  static constexpr int kPB = D * BS * 2;          // bytes of one page (2-byte elements)
  static constexpr int kTileBytes = kPagesPerTile * kPB;
  static constexpr int kNST = 2;
  static constexpr int kQPitch = D * 2 + 16;      // padded Q row (conflict-free ldmatrix)
  static constexpr int kMaxIds = 512;             // block ids cached in shared memory
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kNST * kTileBytes;
  static constexpr int kOffQ = kOffV + kNST * kTileBytes;
  static constexpr int kOffIds = kOffQ + kRows * kQPitch;
  static constexpr int kOffBar = kOffIds + kMaxIds * 4;
  static constexpr int kSmemBytes = kOffBar + kNST * 8;
  static_assert(kBK % BS == 0, "tile/page mismatch");
  static_assert(kHK % 16 == 0 && kBK % kHK == 0, "halves");
  static_assert(D % 16 == 0, "head_dim multiple of 16");
};

template <typename T, int BS, int D, int G>
__global__ void __launch_bounds__(256, 2) prefill_tc_kernel(const PrefillParams p) {
  using C = TcCfg<T, BS, D, G>;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y;

  // ---- (sequence, position tile) of this CTA: blockIdx.x = b * tiles + tile
  const int b = (int)blockIdx.x / p.tiles, tile = (int)blockIdx.x % p.tiles;
  const int64_t q0 = p.cu_q[b];
  const int qlen = (int)(p.cu_q[b + 1] - q0);
  if (tile == p.tiles - 1 && qlen > p.tiles * C::kPos && tid == 0)
    raise_device_error(VASR_PA_DERR_QLEN_RANGE);
  if (tile * C::kPos >= qlen) return;
  int ctx = (int)p.context_lens[b];
  if (ctx > p.cols * BS) {
    if (tid == 0) raise_device_error(VASR_PA_DERR_CTX_RANGE);
    ctx = p.cols * BS;
  }
  const int i0 = tile * C::kPos;                        // first query index in the tile
  const int n_pos = min(C::kPos, qlen - i0);
  const int base_pos = ctx - qlen + i0;                 // absolute position of index i0
  const int kv_end = min(ctx, base_pos + n_pos);        // keys [0, kv_end) are visible to someone
  T *out = reinterpret_cast<T *>(p.out);
  if (kv_end <= 0) {
    // rows with no visible key (context shorter than the chunk): zeros
    for (int e = tid; e < n_pos * G * D; e += C::kThreads) {
      const int r = e / D, d = e % D;
      out[(q0 + i0 + r / G) * (int64_t)p.num_heads * D + (int64_t)(kvh * G + r % G) * D + d] =
          Elem<T>::from_f32(0.f);
    }
    return;
  }
  const int n_pages = (kv_end + BS - 1) / BS;
  const int n_kt = (kv_end + C::kBK - 1) / C::kBK;

  const uint32_t s_base = smem_addr(smem);
  uint32_t *ids = reinterpret_cast<uint32_t *>(smem + C::kOffIds);
  for (int i = tid; i < min(n_pages, C::kMaxIds); i += C::kThreads) {
    uint32_t id = __ldg(p.block_tables + (int64_t)b * p.cols + i);
    if ((int64_t)id >= p.num_blocks) {
      raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
      id = 0;
    }
    ids[i] = id;
  }
  if (tid < C::kNST) mbar_init(s_base + C::kOffBar + tid * 8, 1);
  if (tid == 0) mbar_fence_init();
  // Q tile -> shared memory (rows beyond the sequence are zero)
  {
    const T *qg = reinterpret_cast<const T *>(p.q);
    constexpr int kChunks = D * 2 / 16;
    for (int e = tid; e < C::kRows * kChunks; e += C::kThreads) {
      const int r = e / kChunks, c = e % kChunks;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r / G < n_pos) {
        const T *src = qg + (q0 + i0 + r / G) * p.q_stride + (int64_t)(kvh * G + r % G) * D;
        v = __ldg(reinterpret_cast<const uint4 *>(src) + c);
      }
      *reinterpret_cast<uint4 *>(smem + C::kOffQ + r * C::kQPitch + c * 16) = v;
    }
  }
  __syncthreads();

  const unsigned char *kc = reinterpret_cast<const unsigned char *>(p.k_cache);
  const unsigned char *vc = reinterpret_cast<const unsigned char *>(p.v_cache);
  auto page_id = [&](int pg) -> uint32_t {
    if (pg < C::kMaxIds) return ids[pg];
    uint32_t id = p.block_tables[(int64_t)b * p.cols + pg];
    return (int64_t)id < p.num_blocks ? id : 0u;
  };
  auto issue_tile = [&](int kt) {
    const int s = kt % C::kNST;
    const int pg0 = kt * C::kBK / BS;
    const int np = min(C::kPagesPerTile, n_pages - pg0);
    const uint32_t bar = s_base + C::kOffBar + s * 8;
    mbar_arrive_expect_tx(bar, (uint32_t)(2 * np * C::kPB));
    for (int i = 0; i < np; ++i) {
      const int64_t off = ((int64_t)page_id(pg0 + i) * p.num_kv_heads + kvh) * C::kPB;
      bulk_g2s(s_base + C::kOffK + s * C::kTileBytes + i * C::kPB, kc + off, C::kPB, bar);
      bulk_g2s(s_base + C::kOffV + s * C::kTileBytes + i * C::kPB, vc + off, C::kPB, bar);
    }
  };
  if (tid == 0)
    for (int kt = 0; kt < min(C::kNST, n_kt); ++kt) issue_tile(kt);

  const int grp = lane >> 2, tig = lane & 3;
  // ldmatrix row address of this lane inside the warp's 16 Q rows
  const uint32_t q_lane = s_base + C::kOffQ +
                          (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * C::kQPitch +
                          (lane >> 4) * 16;
  // rows of this thread: r_lo = warp*16 + grp, r_hi = r_lo + 8
  const int r_lo = warp * 16 + grp, r_hi = r_lo + 8;
  const int pos_lo = base_pos + r_lo / G, pos_hi = base_pos + r_hi / G;
  const bool val_lo = (r_lo / G) < n_pos, val_hi = (r_hi / G) < n_pos;
  // largest position among this warp's valid rows (-1: the warp has no valid row)
  const int warp_pos_max =
      (warp * 16) / G < n_pos ? base_pos + min((warp * 16 + 15) / G, n_pos - 1) : -1;

  constexpr int kNT = C::kHK / 8;  // n-tiles of 8 keys per half
  constexpr int kDT = D / 8;       // n-tiles of 8 dims
  float o[kDT][4];
#pragma unroll
  for (int j = 0; j < kDT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const bool use_softcap = (p.softcap != 1.0f) && (p.softcap > 0.f);

  for (int kt = 0; kt < n_kt; ++kt) {
    const int s = kt % C::kNST;
    const bool landed = mbar_wait_bounded(s_base + C::kOffBar + s * 8, (uint32_t)((kt / C::kNST) & 1));
    const int key0 = kt * C::kBK;
    const uint32_t sk = s_base + C::kOffK + s * C::kTileBytes;
    const uint32_t sv = s_base + C::kOffV + s * C::kTileBytes;
    // Partial tile: zero V for keys >= kv_end so masked keys (P = 0) cannot
    // bring stale or non-finite values into the P.V product.
    if (key0 + C::kBK > kv_end) {
      uint16_t *vtile = reinterpret_cast<uint16_t *>(smem + C::kOffV + s * C::kTileBytes);
      for (int e = tid; e < C::kPagesPerTile * D * BS; e += C::kThreads) {
        const int key = key0 + (e / (D * BS)) * BS + e % BS;
        if (key >= kv_end) vtile[e] = 0;
      }
      __syncthreads();
    }
#pragma unroll
    for (int h = 0; h < C::kBK / C::kHK; ++h) {
      const int hkey0 = key0 + h * C::kHK;
      if (hkey0 > warp_pos_max || hkey0 >= kv_end) continue;  // hidden from every row of this warp
      // ---- S = Q K^T for 16 rows x 32 keys
      float sacc[kNT][4];
#pragma unroll
      for (int j = 0; j < kNT; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t qa[4];
        ldmatrix_x4(q_lane + ks * 32, qa[0], qa[1], qa[2], qa[3]);
#pragma unroll
        for (int jp = 0; jp < kNT / 2; ++jp) {
          const int key = h * C::kHK + jp * 16 + (lane & 7) + (lane >> 4) * 8;
          const int chunk = 2 * ks + ((lane >> 3) & 1);
          const uint32_t addr = sk + (key / BS) * C::kPB + (chunk * BS + key % BS) * 16;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(addr, b0, b1, b2, b3);
          mma16816<T>(sacc[2 * jp], qa, b0, b1);
          mma16816<T>(sacc[2 * jp + 1], qa, b2, b3);
        }
      }
      // ---- scale, softcap, causal mask, online softmax (log2 domain)
      const bool need_mask = (hkey0 + C::kHK - 1 > base_pos) || (hkey0 + C::kHK > kv_end);
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int j = 0; j < kNT; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x = sacc[j][e] * p.scale;
          if (use_softcap) x = p.softcap * tanhf(x / p.softcap);
          x *= kLog2e;
          if (need_mask) {
            const int key = hkey0 + j * 8 + tig * 2 + (e & 1);
            const int pos = (e < 2) ? pos_lo : pos_hi;
            const bool ok = (e < 2 ? val_lo : val_hi) && key <= pos && key < kv_end;
            x = ok ? x : -INFINITY;
          }
          sacc[j][e] = x;
        }
        mx_lo = fmaxf(mx_lo, fmaxf(sacc[j][0], sacc[j][1]));
        mx_hi = fmaxf(mx_hi, fmaxf(sacc[j][2], sacc[j][3]));
      }
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
      const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
      // rows with nothing visible yet keep m = -inf; use 0 as the exp offset
      const float off_lo = (mn_lo == -INFINITY) ? 0.f : mn_lo;
      const float off_hi = (mn_hi == -INFINITY) ? 0.f : mn_hi;
      const float a_lo = exp2f(m_lo - off_lo), a_hi = exp2f(m_hi - off_hi);
      m_lo = mn_lo;
      m_hi = mn_hi;
      float ps_lo = 0.f, ps_hi = 0.f;
      uint32_t pa[kNT / 2][4];
#pragma unroll
      for (int j = 0; j < kNT; ++j) {
        const float p0 = exp2f(sacc[j][0] - off_lo), p1 = exp2f(sacc[j][1] - off_lo);
        const float p2 = exp2f(sacc[j][2] - off_hi), p3 = exp2f(sacc[j][3] - off_hi);
        ps_lo += p0 + p1;
        ps_hi += p2 + p3;
        // C fragment of n-tile j -> A fragment of key k-step j/2
        if ((j & 1) == 0) {
          pa[j / 2][0] = pack2<T>(p0, p1);
          pa[j / 2][1] = pack2<T>(p2, p3);
        } else {
          pa[j / 2][2] = pack2<T>(p0, p1);
          pa[j / 2][3] = pack2<T>(p2, p3);
        }
      }
      l_lo = l_lo * a_lo + ps_lo;
      l_hi = l_hi * a_hi + ps_hi;
#pragma unroll
      for (int j = 0; j < kDT; ++j) {
        o[j][0] *= a_lo;
        o[j][1] *= a_lo;
        o[j][2] *= a_hi;
        o[j][3] *= a_hi;
      }
      // ---- O += P V : k-steps of 16 keys, n-tiles of 8 dims
#pragma unroll
      for (int kk = 0; kk < C::kHK / 16; ++kk) {
#pragma unroll
        for (int dp = 0; dp < kDT / 2; ++dp) {
          const int d = dp * 16 + (lane & 7) + (lane >> 4) * 8;
          const int key = h * C::kHK + kk * 16 + ((lane >> 3) & 1) * 8;
          const uint32_t addr = sv + (key / BS) * C::kPB + (d * BS + key % BS) * 2;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(addr, b0, b1, b2, b3);
          mma16816<T>(o[2 * dp], pa[kk], b0, b1);
          mma16816<T>(o[2 * dp + 1], pa[kk], b2, b3);
        }
      }
    }
    // every warp is done with stage s; if any thread's wait gave up, issue
    // nothing more: the tiles still in flight (kt .. kt + kNST - 1) land
    // before the CTA retires (waited for once more, bounded), and the rows
    // stay unwritten (the device error word carries the timeout)
    if (!__syncthreads_and(landed)) {
      if (warp == 0)
        for (int t = kt; t < min(kt + C::kNST, n_kt); ++t)
          mbar_wait_bounded(s_base + C::kOffBar + (t % C::kNST) * 8, (uint32_t)((t / C::kNST) & 1));
      return;
    }
    if (tid == 0 && kt + C::kNST < n_kt) {
      fence_proxy_async_smem();
      issue_tile(kt + C::kNST);
    }
  }

  // ---- normalise and store
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f;
  const float inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  const int64_t row_stride = (int64_t)p.num_heads * D;
  if (val_lo) {
    T *dst = out + (q0 + i0 + r_lo / G) * row_stride + (int64_t)(kvh * G + r_lo % G) * D;
#pragma unroll
    for (int j = 0; j < kDT; ++j)
      *reinterpret_cast<uint32_t *>(dst + j * 8 + tig * 2) = pack2<T>(o[j][0] * inv_lo, o[j][1] * inv_lo);
  }
  if (val_hi) {
    T *dst = out + (q0 + i0 + r_hi / G) * row_stride + (int64_t)(kvh * G + r_hi % G) * D;
#pragma unroll
    for (int j = 0; j < kDT; ++j)
      *reinterpret_cast<uint32_t *>(dst + j * 8 + tig * 2) = pack2<T>(o[j][2] * inv_hi, o[j][3] * inv_hi);
  }
}

// ------------------------------------------------ CUDA-core kernel (f32)
// One CTA per (query row, kv head); 128 threads = 4 warps, warp w handles
// query head w % G of the group for keys w / G, w / G + 4 / G, ... (G <= 4).
// Keys are read with plain loads; online softmax per warp, merged at the end.
template <typename T, int BS, int D>
__global__ void __launch_bounds__(128) prefill_scalar_kernel(const PrefillParams p, int64_t row0,
                                                             int G) {
  constexpr int kX = Elem<T>::kX;
  __shared__ float sm_m[4], sm_l[4], sm_o[4][D];
  const int64_t t = row0 + blockIdx.x;
  const int kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = seq_of_row(p.cu_q, p.num_seqs, t);
  const int qlen = (int)(p.cu_q[b + 1] - p.cu_q[b]);
  int ctx = (int)p.context_lens[b];
  if (ctx > p.cols * BS) {
    if (threadIdx.x == 0) raise_device_error(VASR_PA_DERR_CTX_RANGE);
    ctx = p.cols * BS;
  }
  const int n_keys = min(ctx, ctx - qlen + (int)(t - p.cu_q[b]) + 1);
  const int g = warp % G;
  const int kstart = warp / G, kstep = 4 / G;
  const T *qp = reinterpret_cast<const T *>(p.q) + t * p.q_stride + (int64_t)(kvh * G + g) * D;
  // lane owns dims lane + 32 i
  float qv[D / 32], acc[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) {
    qv[i] = Elem<T>::to_f32(qp[lane + 32 * i]);
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const T *kc = reinterpret_cast<const T *>(p.k_cache);
  const T *vc = reinterpret_cast<const T *>(p.v_cache);
  const bool use_softcap = (p.softcap != 1.0f) && (p.softcap > 0.f);
  for (int j = kstart; j < n_keys; j += kstep) {
    uint32_t blk = p.block_tables[(int64_t)b * p.cols + j / BS];
    if ((int64_t)blk >= p.num_blocks) {
      raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
      blk = 0;
    }
    const int off = j % BS;
    const int64_t page = ((int64_t)blk * p.num_kv_heads + kvh) * D * BS;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
      const int d = lane + 32 * i;
      dot += qv[i] * Elem<T>::to_f32(kc[page + ((int64_t)(d / kX) * BS + off) * kX + d % kX]);
    }
    dot = warp_sum_xor(dot, 32);
    float s = dot * p.scale;
    if (use_softcap) s = p.softcap * tanhf(s / p.softcap);
    s *= kLog2e;
    const float mn = fmaxf(m, s);
    const float a = exp2f(m - mn), pj = exp2f(s - mn);
    l = l * a + pj;
#pragma unroll
    for (int i = 0; i < D / 32; ++i)
      acc[i] = acc[i] * a + pj * Elem<T>::to_f32(vc[page + (int64_t)(lane + 32 * i) * BS + off]);
    m = mn;
  }
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < D / 32; ++i) sm_o[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  // merge the warps of each head
  T *out = reinterpret_cast<T *>(p.out) + t * (int64_t)p.num_heads * D;
  for (int e = threadIdx.x; e < G * D; e += 128) {
    const int gg = e / D, d = e % D;
    float M = -INFINITY;
    for (int w = gg; w < 4; w += G) M = fmaxf(M, sm_m[w]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY)
      for (int w = gg; w < 4; w += G) {
        const float f = exp2f(sm_m[w] - M);
        L += sm_l[w] * f;
        O += sm_o[w][d] * f;
      }
    out[(int64_t)(kvh * G + gg) * D + d] = Elem<T>::from_f32(L > 0.f ? O / L : 0.f);
  }
}

template <typename T, int BS, int D, int G>
int launch_tc(const PrefillArgs &a, const PrefillParams &p, cudaStream_t s) {
  using C = TcCfg<T, BS, D, G>;
  static std::atomic<uint64_t> attr_done{0};
  if (!ensure_smem_attr(prefill_tc_kernel<T, BS, D, G>, C::kSmemBytes, attr_done))
    return VASR_PA_ELAUNCH;
  const int64_t tiles = prefill_tiles_per_seq(a, C::kPos);
  if (tiles <= 0 || tiles * a.num_seqs > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
  PrefillParams pt = p;
  pt.tiles = (int)tiles;
  dim3 grid((unsigned)(tiles * a.num_seqs), (unsigned)a.num_kv_heads);
  prefill_tc_kernel<T, BS, D, G><<<grid, C::kThreads, C::kSmemBytes, s>>>(pt);
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

template <typename T, int D, int G>
int tc_bs(const PrefillArgs &a, const PrefillParams &p, cudaStream_t s) {
  switch (a.block_size) {
    case 8: return launch_tc<T, 8, D, G>(a, p, s);
    case 16: return launch_tc<T, 16, D, G>(a, p, s);
    case 32: return launch_tc<T, 32, D, G>(a, p, s);
    default: return VASR_PA_EINVAL_BLOCKSIZE;
  }
}

template <typename T>
int tc_dispatch(const PrefillArgs &a, const PrefillParams &p, cudaStream_t s) {
  if (a.head_dim != 128) return VASR_PA_ENOT_SUPPORTED;
  switch (a.num_heads / a.num_kv_heads) {
    case 1: return tc_bs<T, 128, 1>(a, p, s);
    case 2: return tc_bs<T, 128, 2>(a, p, s);
    case 4: return tc_bs<T, 128, 4>(a, p, s);
    default: return VASR_PA_ENOT_SUPPORTED;
  }
}

// The tcgen05 kernel (prefill_umma.cu) serves the shapes it supports; an
// A/B build compiled with -DVASR_PREFILL_MMA_ONLY=1 sends every 16-bit call
// to this file's mma.sync kernel instead. The library reads no environment.
#ifndef VASR_PREFILL_MMA_ONLY
#define VASR_PREFILL_MMA_ONLY 0
#endif

template <int BS>
int scalar_launch(const PrefillArgs &a, const PrefillParams &p, cudaStream_t s) {
  const int G = a.num_heads / a.num_kv_heads;
  if (G > 4 || 4 % G != 0 || a.head_dim != 128) return VASR_PA_ENOT_SUPPORTED;
  for (int64_t r0 = 0; r0 < a.total_q_tokens; r0 += 0x7fffffff) {
    const int64_t n = a.total_q_tokens - r0 < 0x7fffffff ? a.total_q_tokens - r0 : 0x7fffffff;
    dim3 grid((unsigned)n, (unsigned)a.num_kv_heads);
    prefill_scalar_kernel<float, BS, 128><<<grid, 128, 0, s>>>(p, r0, G);
  }
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

}  // namespace

int launch_prefill(const PrefillArgs &a, cudaStream_t s) {
  if (a.num_kv_heads > 65535) return VASR_PA_EINVAL_SHAPE;
  PrefillParams p{};
  p.out = a.out;
  p.q = a.query;
  p.k_cache = a.key_cache;
  p.v_cache = a.value_cache;
  p.block_tables = a.block_tables;
  p.context_lens = a.context_lens;
  p.cu_q = a.cu_seqlens_q;
  p.q_stride = a.q_token_stride;
  p.num_blocks = a.num_blocks;
  p.num_seqs = a.num_seqs;
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.cols = a.max_num_blocks_per_seq;
  p.tiles = 1;
  p.scale = a.scale;
  p.softcap = a.softcapping;
  if ((a.dtype == VASR_PA_BF16 || a.dtype == VASR_PA_F16) && !VASR_PREFILL_MMA_ONLY) {
    const int r = launch_prefill_umma(a, s);
    if (r != VASR_PA_ENOT_SUPPORTED) return r;
  }
  switch (a.dtype) {
    case VASR_PA_BF16: return tc_dispatch<__nv_bfloat16>(a, p, s);
    case VASR_PA_F16: return tc_dispatch<__half>(a, p, s);
    case VASR_PA_F32:
      switch (a.block_size) {
        case 8: return scalar_launch<8>(a, p, s);
        case 16: return scalar_launch<16>(a, p, s);
        case 32: return scalar_launch<32>(a, p, s);
        default: return VASR_PA_EINVAL_BLOCKSIZE;
      }
    default: return VASR_PA_EINVAL_DTYPE;
  }
}

int read_error_prefill(uint32_t *bits, bool clear, cudaStream_t s) {
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

// decode_mma.cuh — paged decode attention for GQA group 2 with the dot
// products on the tensor cores (mma.sync m16n8k16, f32 accumulate).
//
// Same split-K decomposition, stage ring and merges as paged_decode_g2_kernel
// (decode_g2.cuh); what differs is the per-stage math. The g2 kernel spends
// ~400 instructions per warp on every 16 tokens (FMA dot products in f32 and
// the shuffles around them), which — not the bytes — limits it: fp8 pages
// (half the bytes) run no faster. Here a warp treats its 16 tokens as one
// MMA tile:
//   S[16 x 16] = Q[16 x 128] K^T   rows 0, 1 = the two query heads of the
//                                  kv head, rows 2-15 zero; 8 k-steps x 2
//                                  n-tiles, K read by ldmatrix straight from
//                                  the K page ([D/8][bs][8]: a row of 8 dims
//                                  of one token is one 16-byte ldmatrix row)
//   O^T[128 x 8] += V^T P^T        8 m-tiles of 16 dims, V^T (the V page,
//                                  [D][bs]: dim rows of the tile's tokens) as
//                                  the A operand by ldmatrix, P's score
//                                  fragments as the B operand (columns 0, 1
//                                  = the two heads)
// ~90 instructions per 16 tokens. Rows 0 and 1 of S live in lanes 0-7; O^T's
// columns 0 and 1 in lanes with tig = 0. The softmax keeps a per-row running maximum that moves only when
// a tile's maximum exceeds it by more than 2^8 (O is then rescaled), exact in
// real arithmetic because numerator and denominator share the offset.
// Tokens past the split's end are masked in S and their V entries zeroed in
// registers, so stale or non-finite page bytes never reach O.
#pragma once

#include <type_traits>

#include "decode_g2.cuh"

namespace vasr {

__device__ __forceinline__ void dec_ldmatrix_x4(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                                uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void dec_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void dec_mma<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                       uint32_t a2, uint32_t a3, uint32_t b0,
                                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void dec_mma<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t dec_pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t dec_pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t dec_pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ uint2 dec_lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// fp8 E4M3 pair -> f16 pair (exact), as one 32-bit A/B fragment register
__device__ __forceinline__ uint32_t fp8x2_to_h2(uint32_t v16) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v16 & 0xffffu), __NV_E4M3);
  return *reinterpret_cast<uint32_t *>(&h);
}

// One stage of a warp's tokens (n_valid of them, kNTT tiles of 16 at sk / sv
// in shared memory) through the tensor cores: per 16-token tile S = Q Kᵀ,
// the running-max softmax update of rows 0 / 1 (lanes 0-7) and O^T += V^T P^T.
// O is kept transposed, O^T[16 dims x 8 heads] += V^T P^T per 16-dim tile
// (V page rows as the A operand, P's score fragments as the B operand
// unchanged), so all four accumulators of a tile are real (lane (grp, 0):
// dims grp and grp + 8 of heads 0 and 1) and a tile takes half the MMAs and
// registers of O[16 x 8 dims] with rows 2-15 padding.
template <typename TC, int D>
constexpr int dec_o_tiles() { return D / 16; }

// kQSmem (fp8 pages, 6 CTAs per SM): the query fragments are read from
// shared memory per k-step instead of held in registers.
template <typename T, int BS, int D, typename TC, int kNTT, int kPB, bool kQSmem>
__device__ __forceinline__ void dec_mma_stage(uint32_t sk, uint32_t sv, int n_valid,
                                              const uint32_t (&qa)[D / 16][2], uint32_t sq, float c_log2,
                                              bool use_softcap, float scale, float softcap,
                                              float (&o)[dec_o_tiles<TC, D>()][4], float &m_used,
                                              float &l_part) {
  constexpr bool kFp8 = std::is_same<TC, __nv_fp8_e4m3>::value;
  using TM = typename std::conditional<kFp8, __half, T>::type;  // MMA operand type
  constexpr int kKS = D / 16;
  constexpr float kRescale = 8.f;
  const int lane = threadIdx.x & 31, grp = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int ti = 0; ti < kNTT; ++ti) {
    const int t0 = ti * 16;  // first token of this 16-token tile within the stage
    if (t0 >= n_valid) break;
    // ---- S = Q K^T (two 8-token n-tiles)
    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if constexpr (kFp8) {
      // matrices: (n-tile 0, chunk 2kp), (n-tile 1, 2kp), (n-tile 0, 2kp+1), (n-tile 1, 2kp+1)
      const int r = lane & 7;
      const int ktok = t0 + 4 * (r >> 1) + 2 * ((lane >> 3) & 1) + (r & 1);
      const uint32_t krow = sk + (ktok / BS) * kPB + ((lane >> 4) * BS + ktok % BS) * 16;
#pragma unroll
      for (int kp = 0; kp < kKS / 2; ++kp) {
        uint32_t r0, r1, r2, r3;
        dec_ldmatrix_x4(krow + kp * 2 * (BS * 16), r0, r1, r2, r3);
        uint2 q0 = make_uint2(qa[2 * kp][0], qa[2 * kp][1]), q1 = make_uint2(qa[2 * kp + 1][0], qa[2 * kp + 1][1]);
        if constexpr (kQSmem) {  // lanes 0-7 hold the two heads' rows; the other rows are zero
          q0 = q1 = make_uint2(0u, 0u);
          if (lane < 8) {
            q0 = dec_lds64(sq + (uint32_t)(((2 * kp) * 8 + lane) * 8));
            q1 = dec_lds64(sq + (uint32_t)(((2 * kp + 1) * 8 + lane) * 8));
          }
        }
        dec_mma<TM>(sacc[0], q0.x, 0u, q0.y, 0u, fp8x2_to_h2(r0), fp8x2_to_h2(r0 >> 16));
        dec_mma<TM>(sacc[1], q0.x, 0u, q0.y, 0u, fp8x2_to_h2(r1), fp8x2_to_h2(r1 >> 16));
        dec_mma<TM>(sacc[0], q1.x, 0u, q1.y, 0u, fp8x2_to_h2(r2), fp8x2_to_h2(r2 >> 16));
        dec_mma<TM>(sacc[1], q1.x, 0u, q1.y, 0u, fp8x2_to_h2(r3), fp8x2_to_h2(r3 >> 16));
      }
    } else {
      const int ktok = t0 + (lane & 7) + (lane >> 4) * 8;
      const uint32_t krow = sk + (ktok / BS) * kPB + (ktok % BS) * 16 + ((lane >> 3) & 1) * (BS * 16);
#pragma unroll
      for (int ks = 0; ks < kKS; ++ks) {
        uint32_t b0, b1, b2, b3;
        dec_ldmatrix_x4(krow + ks * 2 * (BS * 16), b0, b1, b2, b3);
        dec_mma<TM>(sacc[0], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
        dec_mma<TM>(sacc[1], qa[ks][0], 0u, qa[ks][1], 0u, b2, b3);
      }
    }
    // ---- scores of row grp: tokens t0 + n*8 + tig*2 + {0, 1}
    float x[4];
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = sacc[n][e];
        if (use_softcap) v = softcap * tanhf(v * scale / softcap) * kLog2e;
        else v *= c_log2;
        const int tok = kFp8 ? t0 + 4 * tig + 2 * n + e : t0 + n * 8 + tig * 2 + e;
        x[n * 2 + e] = (tok < n_valid) ? v : -INFINITY;
      }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (__any_sync(0xffffffffu, mx > m_used + kRescale)) {
      const float m_new = fmaxf(m_used, mx);
      const float alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
      m_used = m_new;
      l_part *= alpha;
      {  // O^T: heads 0 / 1 are the columns; their alphas live in lanes 0 / 4
        const float a0 = __shfl_sync(0xffffffffu, alpha, 0), a1 = __shfl_sync(0xffffffffu, alpha, 4);
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          o[j][0] *= a0;
          o[j][1] *= a1;
          o[j][2] *= a0;
          o[j][3] *= a1;
        }
      }
    }
    const float off = (m_used == -INFINITY) ? 0.f : m_used;
    float pv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      pv[e] = exp2f(x[e] - off);
      l_part += pv[e];
    }
    // P's fragments (rows = heads, k = tokens of the tile): the B operand of V^T P^T
    const uint32_t pa0 = dec_pack2<TM>(pv[0], pv[1]), pa2 = dec_pack2<TM>(pv[2], pv[3]);
    const bool tail = (t0 + 16 > n_valid);
    if constexpr (kFp8) {
      // ---- O^T += V^T P^T: one ldmatrix row = the tile's 16 tokens of one dim;
      // matrix j of an x4 = 8 dims, lane tig holds tokens 4 tig .. 4 tig + 3
      const int vd = (lane >> 3) * 8 + (lane & 7);
      const uint32_t vrow = sv + (t0 / BS) * kPB + vd * BS + t0 % BS;
      const int tk = t0 + 4 * tig;
      const uint32_t mlo = (tk < n_valid ? 0xffffu : 0u) | (tk + 1 < n_valid ? 0xffff0000u : 0u);
      const uint32_t mhi = (tk + 2 < n_valid ? 0xffffu : 0u) | (tk + 3 < n_valid ? 0xffff0000u : 0u);
      // O^T += V^T P^T: matrices 2 hf (dims 16 (2 dq + hf) + 0..7) and
      // 2 hf + 1 (+ 8..15) of the x4 are the A rows grp / grp + 8; the
      // token pairs (4 tig, 4 tig + 1) and (4 tig + 2, 4 tig + 3) are the
      // permuted k pairs of P's fragments (pa0, pa2), here the B operand
#pragma unroll
      for (int dq = 0; dq < D / 32; ++dq) {
        uint32_t r[4];
        dec_ldmatrix_x4(vrow + dq * 32 * BS, r[0], r[1], r[2], r[3]);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t a0 = fp8x2_to_h2(r[2 * hf]), a2 = fp8x2_to_h2(r[2 * hf] >> 16);
          uint32_t a1 = fp8x2_to_h2(r[2 * hf + 1]), a3 = fp8x2_to_h2(r[2 * hf + 1] >> 16);
          if (tail) {
            a0 &= mlo;
            a1 &= mlo;
            a2 &= mhi;
            a3 &= mhi;
          }
          dec_mma<TM>(o[dq * 2 + hf], a0, a1, a2, a3, pa0, pa2);
        }
      }
      continue;
    }
    // ---- O^T += V^T P^T: V rows = dims, 8 tokens per ldmatrix row
    const int vd = (lane & 7) + (lane >> 4) * 8;
    const int vtok = t0 + ((lane >> 3) & 1) * 8;
    const uint32_t vrow = sv + (vtok / BS) * kPB + (vd * BS + vtok % BS) * 2;
    const int tk0 = t0 + tig * 2;  // tokens of b0 / b2 halves; b1 / b3: +8
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t b0, b1, b2, b3;
      dec_ldmatrix_x4(vrow + dp * 16 * BS * 2, b0, b1, b2, b3);
      if (tail) {
        const uint32_t m0 = (tk0 < n_valid ? 0xffffu : 0u) | (tk0 + 1 < n_valid ? 0xffff0000u : 0u);
        const uint32_t m1 = (tk0 + 8 < n_valid ? 0xffffu : 0u) | (tk0 + 9 < n_valid ? 0xffff0000u : 0u);
        b0 &= m0;
        b2 &= m0;
        b1 &= m1;
        b3 &= m1;
      }
      // O^T += V^T P^T: the x4's matrices (dims 0-7 / 8-15 x tokens 0-7 /
      // 8-15) are the A fragments of the 16 x 16 V^T tile, P's score
      // fragments the B operand
      dec_mma<TM>(o[dp], b0, b2, b1, b3, pa0, pa2);
    }
  }
}

// TC = T: bf16 / f16 pages, the MMAs in T. TC = fp8 E4M3 (bs 16 or 32): the
// MMAs run in f16 on pages converted in registers, and the reduction index is
// permuted so one ldmatrix row of 16 fp8 bytes feeds one k-step: lane tig
// holds dims / tokens 4 tig .. 4 tig + 3 of its row, used as the logical
// k = 2 tig, 2 tig + 1 (low pair) and 2 tig + 8, 2 tig + 9 (high pair). Q
// fragments follow the same permutation over dims; the score tiles list their
// tokens as n-tile 0 = {0,1,4,5,8,9,12,13}, n-tile 1 = {2,3,6,7,...}, so that
// P's C fragments are already the A fragments of the P V product over the
// same permuted token order.
template <typename T, int BS, int D, int NST, int MINB, typename TC = T>
__global__ void __launch_bounds__(128, MINB) paged_decode_mma_kernel(const DecodeParams p) {
  constexpr bool kFp8 = std::is_same<TC, __nv_fp8_e4m3>::value;
  using TM = typename std::conditional<kFp8, __half, T>::type;  // MMA operand type
  using C = DecodeG2Cfg<TC, BS, D, NST>;
  constexpr int G = 2;
  constexpr int kKS = D / 16;  // k-steps of the score MMA
  constexpr float kRescale = 8.f;
  static_assert(!kFp8 || BS >= 16, "fp8 pages need 16-byte V rows");
  extern __shared__ __align__(128) unsigned char smem[];
  decode_g2_init_ring<TC, BS, D, NST>(smem);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane >> 2, tig = lane & 3;
  const int P = p.pages_per_split * BS;

  uint32_t spec_id = 0;
  const int spec_col = split * p.pages_per_split + tid;
  if (tid < p.pages_per_split && spec_col < p.cols)
    spec_id = __ldg(p.block_tables + (int64_t)b * p.cols + spec_col);
  int ctx = (int)p.context_lens[b];
  const int cap_tables = p.cols * BS;
  const int cap_splits = p.max_splits * P;
  if (ctx > cap_tables || ctx > cap_splits) {
    if (split == 0 && tid == 0) raise_device_error(VASR_PA_DERR_CTX_RANGE);
    ctx = min(ctx, min(cap_tables, cap_splits));
  }
  T *out = reinterpret_cast<T *>(p.out) + ((int64_t)b * p.num_heads + (int64_t)kvh * G) * D;
  if (ctx <= 0) {
    pdl_wait();  // no global write before the preceding kernel has completed
    if (split == 0)
      for (int e = tid; e < G * D; e += C::kThreads) out[e] = Elem<T>::from_f32(0.f);
    return;
  }
  const int n_splits = (ctx + P - 1) / P;
  if (split >= n_splits) return;
  const int seq_pages = (ctx + BS - 1) / BS;
  const int per = (seq_pages + n_splits - 1) / n_splits;  // pages shared evenly by the splits
  const int page_begin = split * per;
  const int tok_begin = page_begin * BS;
  const int tok_end = min(ctx, tok_begin + per * BS);
  const int n_pages = (tok_end - tok_begin + BS - 1) / BS;
  const int n_units = (n_pages + C::kSP - 1) / C::kSP;

  const uint32_t s_base = smem_addr(smem);
  uint32_t *blk = reinterpret_cast<uint32_t *>(smem + C::kOffBlk);
  if (tid < n_pages) {
    uint32_t id = spec_id;
    if (page_begin != split * p.pages_per_split)
      id = __ldg(p.block_tables + (int64_t)b * p.cols + page_begin + tid);
    if ((int64_t)id >= p.num_blocks) {
      raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
      id = 0;
    }
    blk[tid] = id;
  }
  __syncthreads();

  const TC *kc = reinterpret_cast<const TC *>(p.k_cache);
  const TC *vc = reinterpret_cast<const TC *>(p.v_cache);
  const int64_t page_elems = (int64_t)D * BS;
  auto issue_unit = [&](int u) {
    const int s = u % C::kNST;
    const int pg0 = u * C::kSP;
    const int np = min(C::kSP, n_pages - pg0);
    const uint32_t bar = s_base + C::kOffBar + s * 8;
    mbar_arrive_expect_tx(bar, (uint32_t)(2 * np * C::kPB));
    for (int i = 0; i < np; ++i) {
      const int64_t off = ((int64_t)blk[pg0 + i] * p.num_kv_heads + kvh) * page_elems;
      bulk_g2s(s_base + C::kOffK + (s * C::kSP + i) * C::kPB, kc + off, C::kPB, bar);
      bulk_g2s(s_base + C::kOffV + (s * C::kSP + i) * C::kPB, vc + off, C::kPB, bar);
    }
  };
  // Under a programmatic launch behind this step's KV append (which writes
  // q and each sequence's newest token only), everything read so far and
  // every page before the sequence's last one is already final: those stages
  // stream in while the append still runs. The stage holding the last page,
  // q, and every global write (bar the error word's atomic OR) wait for the
  // append to complete.
  const int last_in_split = seq_pages - 1 - page_begin;
  const int late_unit = (last_in_split >= 0 && last_in_split < n_pages) ? last_in_split / C::kSP : -1;
  if (lane == 0)
    for (int u = warp; u < min(C::kNST, n_units); u += C::kWarps)
      if (u != late_unit) issue_unit(u);
  pdl_wait();
  if (lane == 0 && late_unit >= 0 && late_unit < C::kNST && late_unit % C::kWarps == warp)
    issue_unit(late_unit);

  // query fragments (A operand, rows = heads): lanes 0-7 hold rows 0 / 1
  uint32_t qa[kKS][2];
  {
    const T *qp = reinterpret_cast<const T *>(p.q) + (int64_t)b * p.q_seq_stride +
                  (int64_t)(kvh * G + (grp & 1)) * D;
#pragma unroll
    for (int ks = 0; ks < kKS; ++ks) {
      if constexpr (kFp8) {  // dims 4 tig .. 4 tig + 3 of the k-step, as f16 pairs
        qa[ks][0] = qa[ks][1] = 0u;
        if (grp < G) {
          const T *q4 = qp + ks * 16 + tig * 4;
          qa[ks][0] = dec_pack2<__half>(Elem<T>::to_f32(q4[0]), Elem<T>::to_f32(q4[1]));
          qa[ks][1] = dec_pack2<__half>(Elem<T>::to_f32(q4[2]), Elem<T>::to_f32(q4[3]));
        }
      } else {
        qa[ks][0] = grp < G ? __ldg(reinterpret_cast<const uint32_t *>(qp + ks * 16 + tig * 2)) : 0u;
        qa[ks][1] = grp < G ? __ldg(reinterpret_cast<const uint32_t *>(qp + ks * 16 + 8 + tig * 2)) : 0u;
      }
    }
  }

  // fp8 pages at 6 CTAs per SM: lanes 0-7's query fragments go to shared
  // memory (the P staging area of the CUDA-core kernel, unused here) and are
  // read per k-step, which leaves the registers to the sixth CTA
  constexpr bool kQSmem = kFp8 && MINB >= 6;
  const uint32_t s_q = s_base + C::kOffP;
  if constexpr (kQSmem) {
    static_assert(C::kWarps * G * C::kST * 4 >= kKS * 8 * 8, "query fragments fit the P area");
    if (warp == 0 && lane < 8) {
#pragma unroll
      for (int ks = 0; ks < kKS; ++ks)
        asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(s_q + (uint32_t)((ks * 8 + lane) * 8)),
                     "r"(qa[ks][0]), "r"(qa[ks][1])
                     : "memory");
    }
    __syncthreads();
  }

  // fp8 pages hold K / k_scale and V / v_scale
  const float k_mul = p.k_scale ? p.scale * __ldg(p.k_scale) : p.scale;
  const float v_mul = p.v_scale ? __ldg(p.v_scale) : 1.f;
  const float c_log2 = k_mul * kLog2e;
  const bool use_softcap = (p.softcap != 1.0f) && (p.softcap > 0.f);
  float o[dec_o_tiles<TC, D>()][4];
#pragma unroll
  for (int j = 0; j < dec_o_tiles<TC, D>(); ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_used = -INFINITY, l_part = 0.f;  // row grp (lanes 0-7 meaningful)
  bool aborted = false;
  int u_abort = 0;

  for (int u = warp; u < n_units; u += C::kWarps) {
    const int s = u % C::kNST;
    if (!mbar_wait_bounded(s_base + C::kOffBar + s * 8, (uint32_t)((u / C::kNST) & 1))) {
      aborted = true;
      u_abort = u;
      break;
    }
    const int n_valid = min(C::kST, tok_end - (tok_begin + u * C::kST));
    const uint32_t sk = s_base + C::kOffK + s * C::kSP * C::kPB;
    const uint32_t sv = s_base + C::kOffV + s * C::kSP * C::kPB;
    dec_mma_stage<T, BS, D, TC, C::kNTT, C::kPB, kQSmem>(sk, sv, n_valid, qa, s_q, c_log2, use_softcap, p.scale,
                                                  p.softcap, o, m_used, l_part);
    __syncwarp();
    const int nu = u + C::kNST;
    if (nu < n_units && lane == 0) {
      fence_proxy_async_smem();
      issue_unit(nu);
    }
  }

  if (aborted) decode_drain_warp_stages<C>(s_base, u_abort, n_units, 0);

  // ---- warp results -> shared memory (rows 0 and 1 live in lanes 0-7)
  float l_row = l_part;
  l_row += __shfl_xor_sync(0xffffffffu, l_row, 1);
  l_row += __shfl_xor_sync(0xffffffffu, l_row, 2);
  float *co = reinterpret_cast<float *>(smem + C::kOffCO);
  float *cm = reinterpret_cast<float *>(smem + C::kOffCM);
  float *cl = reinterpret_cast<float *>(smem + C::kOffCL);
  if (aborted) {
    m_used = -INFINITY;
    l_row = 0.f;
  }
  if (grp < G && tig == 0) {
    cm[warp * G + grp] = m_used;
    cl[warp * G + grp] = l_row;
  }
  {  // O^T: lane (grp, 0) holds dims grp, grp + 8 of each 16-dim tile, both heads
    if (tig == 0) {
#pragma unroll
      for (int j = 0; j < D / 16; ++j) {
        co[(warp * G) * D + j * 16 + grp] = aborted ? 0.f : o[j][0];
        co[(warp * G + 1) * D + j * 16 + grp] = aborted ? 0.f : o[j][1];
        co[(warp * G) * D + j * 16 + grp + 8] = aborted ? 0.f : o[j][2];
        co[(warp * G + 1) * D + j * 16 + grp + 8] = aborted ? 0.f : o[j][3];
      }
    }
  }
  __syncthreads();

  const int64_t bk = (int64_t)b * p.num_kv_heads + kvh;
  const bool single = (n_splits == 1);
#pragma unroll
  for (int e0 = 0; e0 < G * D; e0 += C::kThreads) {
    const int e = e0 + tid;
    const int g = e / D;
    const int d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::kWarps; ++w) M = fmaxf(M, cm[w * G + g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < C::kWarps; ++w) {
        const float f = exp2f(cm[w * G + g] - M);
        L = fmaf(cl[w * G + g], f, L);
        O = fmaf(co[(w * G + g) * D + d], f, O);
      }
    }
    if (single) {
      out[g * D + d] = Elem<T>::from_f32(L > 0.f ? O / L * v_mul : 0.f);
    } else {
      const int64_t slot = bk * p.max_splits + split;
      p.ws_o[(slot * G + g) * D + d] = O;
      if (d == 0) p.ws_ml[slot * G + g] = make_float2(M, L);
    }
  }
  if (single) return;

  __syncthreads();
  uint32_t *flag = reinterpret_cast<uint32_t *>(smem + C::kOffFlag);
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.counters + bk, 1u);
    __threadfence();
    flag[0] = (prev == (uint32_t)(n_splits - 1)) ? 1u : 0u;
  }
  __syncthreads();
  if (flag[0] == 0u) return;
#pragma unroll
  for (int e0 = 0; e0 < G * D; e0 += C::kThreads) {
    const int e = e0 + tid;
    const int g = e / D;
    const int d = e % D;
    const int64_t slot0 = bk * p.max_splits;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_splits; ++s2) M = fmaxf(M, __ldcg(&p.ws_ml[(slot0 + s2) * G + g].x));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int s2 = 0; s2 < n_splits; ++s2) {
        const float2 ml = __ldcg(&p.ws_ml[(slot0 + s2) * G + g]);
        const float w = exp2f(ml.x - M);
        L = fmaf(ml.y, w, L);
        O = fmaf(__ldcg(&p.ws_o[((slot0 + s2) * G + g) * D + d]), w, O);
      }
    }
    out[g * D + d] = Elem<T>::from_f32(L > 0.f ? O / L * v_mul : 0.f);
  }
  if (tid == 0) p.counters[bk] = 0u;
}

}  // namespace vasr

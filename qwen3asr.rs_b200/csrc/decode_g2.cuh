// decode_g2.cuh — paged decode attention specialised for GQA group 2
// (Qwen3-ASR: 16 query heads over 8 kv heads).
//
// Same decomposition, pipeline and split-K merge as paged_decode_kernel
// (decode.cuh); what differs is the score computation. A warp takes 16
// tokens of a stage at a time and its 32 lanes split them as
// 8 tokens x 4 quarters of the head dimension: lane (t8, quarter) holds the
// two query heads' values for its quarter only (64 floats instead of 128),
// converts each K element once for both heads, and computes 2 tokens x 2
// heads partial dot products. A two-level transpose-reduce over the quarter
// lanes (xor 16, xor 8) leaves every lane with one complete score
// (token t8 + 8 * quarter_bit1, head quarter_bit0) after 3 shuffles.
#pragma once

#include "decode.cuh"

#ifndef VASR_DECODE_FFMA2
#define VASR_DECODE_FFMA2 1  // packed f32x2 FMAs (same rounding as two fmaf)
#endif
#ifndef VASR_DECODE_BALANCED
#define VASR_DECODE_BALANCED 1  // share a sequence's pages evenly among its splits
#endif

namespace vasr {

template <typename T, int BS, int D, int NST>
struct DecodeG2Cfg {
  static constexpr int G = 2;
  static constexpr int kThreads = 128;
  static constexpr int kWarps = 4;
  static constexpr int kX = Elem<T>::kX;                 // elements per 16-byte chunk
  static constexpr int kCH = D / kX;                     // chunks per token row
  static constexpr int kCQ = kCH / 4;                    // chunks per quarter
  static constexpr int kSP = (16 > BS) ? (16 / BS) : 1;  // pages per stage
  static constexpr int kST = kSP * BS;                   // tokens per stage
  static constexpr int kNTT = kST / 16;                  // 16-token sub-tiles per stage
  static constexpr int kPB = D * BS * (int)sizeof(T);
  static constexpr int kNST = NST;
  static constexpr int kTPS = 16 / (int)sizeof(T);
  static constexpr int kR = BS * (int)sizeof(T);
  static constexpr int kNSEG = kR / 16;
  static constexpr int kRPP = 8 / kNSEG;
  static constexpr int kNR = D / (4 * kRPP);
  static constexpr int kMaxPagesPerSplit = 64;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kNST * kSP * kPB;
  static constexpr int kOffP = kOffV + kNST * kSP * kPB;
  static constexpr int kOffCO = kOffP + kWarps * G * kST * 4;
  static constexpr int kOffCM = kOffCO + kWarps * G * D * 4;
  static constexpr int kOffCL = kOffCM + kWarps * G * 4;
  static constexpr int kOffBlk = kOffCL + kWarps * G * 4;
  static constexpr int kOffBar = (kOffBlk + kMaxPagesPerSplit * 4 + 15) & ~15;
  static constexpr int kOffFlag = kOffBar + kNST * 8;
  static constexpr int kSmemBytes = kOffFlag + 16;
  static_assert(kCH % 4 == 0, "head_dim must split into 4 chunk quarters");
  static_assert(kST % 16 == 0, "stage must hold whole 16-token sub-tiles");
  static_assert(kNST % kWarps == 0, "stages must split evenly over warps");
  static_assert(D % (4 * kRPP) == 0, "head_dim not covered by PV lanes");
};

// A warp whose wait on unit u_abort gave up issues no further stage. Its own
// copies still in flight are those of units u_abort, u_abort + kWarps, ...
// up to kNST units ahead (a warp refills only the stages it consumes, kNST
// units ahead); they must land before the CTA retires, since the hardware
// hands this shared memory to the next CTA. Each is waited for once more,
// again bounded; a copy that does not arrive within that second limit is the
// one case left that can outlive the CTA (recorded in the device error word).
template <typename C>
__device__ __forceinline__ void decode_drain_warp_stages(uint32_t s_base, int u_abort, int n_units,
                                                         uint32_t ubase) {
  for (int v = u_abort; v < min(u_abort + C::kNST, n_units); v += C::kWarps) {
    const uint32_t uu = ubase + (uint32_t)v;
    mbar_wait_bounded(s_base + C::kOffBar + (uu % C::kNST) * 8, (uu / C::kNST) & 1u);
  }
}

// One work item: (split, kv head, sequence). `ubase` = stage-ring units this
// CTA consumed before (the ring's barriers keep counting across items);
// returns the units consumed here. The barriers are initialised by the caller.
// T: query / output element; TC: cache element (T, or fp8 E4M3 with the
// per-tensor scales p.k_scale / p.v_scale).
template <typename T, int BS, int D, int NST, typename TC = T>
__device__ __forceinline__ uint32_t decode_g2_item(const DecodeParams &p, unsigned char *smem,
                                                   const int split, const int kvh, const int b,
                                                   const uint32_t ubase) {
  using C = DecodeG2Cfg<TC, BS, D, NST>;
  constexpr int G = 2;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int P = p.pages_per_split * BS;

  // The block ids of this split are loaded speculatively, in parallel with
  // the context length (only in-row entries; those past the length are
  // discarded below).
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
    if (split == 0)
      for (int e = tid; e < G * D; e += C::kThreads) out[e] = Elem<T>::from_f32(0.f);
    return 0;
  }
  const int n_splits = (ctx + P - 1) / P;
  if (split >= n_splits) return 0;
#if VASR_DECODE_BALANCED
  // Balanced splits: the sequence's pages are shared evenly by its splits
  // (every CTA of a sequence gets the same work), instead of full splits plus
  // a short last one; CTA durations vary less, which shortens the tail.
  const int seq_pages = (ctx + BS - 1) / BS;
  const int per = (seq_pages + n_splits - 1) / n_splits;
  const int page_begin = split * per;
#else
  const int per = p.pages_per_split;
  const int page_begin = split * p.pages_per_split;
#endif
  const int tok_begin = page_begin * BS;
  const int tok_end = min(ctx, tok_begin + per * BS);
  const int n_pages = (tok_end - tok_begin + BS - 1) / BS;
  const int n_units = (n_pages + C::kSP - 1) / C::kSP;

  const uint32_t s_base = smem_addr(smem);
  uint32_t *blk = reinterpret_cast<uint32_t *>(smem + C::kOffBlk);
  float *p_s = reinterpret_cast<float *>(smem + C::kOffP);

  if (tid < n_pages) {
    uint32_t id = spec_id;  // == block_tables[b * cols + tok_begin / BS + tid] when the starts agree
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
    const int s = (ubase + u) % C::kNST;
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
  if (lane == 0) {
    fence_proxy_async_smem();  // the previous item's generic reads of the ring come first
    for (int u = warp; u < min(C::kNST, n_units); u += C::kWarps) issue_unit(u);
  }

  // ---- query quarter of both heads: lane (t8, qtr) holds dims [qtr*D/4, +D/4)
  const int t8 = lane & 7;
  const int qtr = lane >> 3;
  const int qb0 = qtr & 1, qb1 = qtr >> 1;
  float q_reg[G][D / 4];
  {
    const T *qp = reinterpret_cast<const T *>(p.q) + (int64_t)b * p.q_seq_stride +
                  (int64_t)(kvh * G) * D + qtr * (D / 4);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint4 *q4 = reinterpret_cast<const uint4 *>(qp + g * D);
      constexpr int QX = Elem<T>::kX;
#pragma unroll
      for (int c = 0; c < D / 4 / QX; ++c) {
        float f[QX];
        unpack_chunk<T>(__ldg(q4 + c), f);
#pragma unroll
        for (int e = 0; e < QX; ++e) q_reg[g][c * QX + e] = f[e];
      }
    }
  }
  // fp8 caches hold K / k_scale and V / v_scale
  const float k_mul = p.k_scale ? p.scale * __ldg(p.k_scale) : p.scale;
  const float v_mul = p.v_scale ? __ldg(p.v_scale) : 1.f;
  // score lane identity after the reduce
  const int s_tok = qb1 * 8 + t8;  // token within a 16-token sub-tile
  const int s_head = qb0;

  const int rlo = lane % C::kRPP;
  const int sg = (lane / C::kRPP) % C::kNSEG;
  const int ph = lane / 8;

  float m_run[G] = {-INFINITY, -INFINITY};
  float acc[C::kNR][G];
#pragma unroll
  for (int i = 0; i < C::kNR; ++i) acc[i][0] = acc[i][1] = 0.f;
  float l_part = 0.f;
  const bool use_softcap = (p.softcap != 1.0f) && (p.softcap > 0.f);
  bool aborted = false;
  int u_abort = 0;
  float *p_w = p_s + warp * G * C::kST;

  for (int u = warp; u < n_units; u += C::kWarps) {
    const int s = (ubase + u) % C::kNST;
    const uint32_t bar = s_base + C::kOffBar + s * 8;
    if (!mbar_wait_bounded(bar, (uint32_t)(((ubase + u) / C::kNST) & 1))) {
      aborted = true;
      u_abort = u;
      break;
    }
    const int unit_tok0 = tok_begin + u * C::kST;
    const int n_valid = min(C::kST, tok_end - unit_tok0);
    const int np = min(C::kSP, n_pages - u * C::kSP);
    const uint32_t sk = s_base + C::kOffK + s * C::kSP * C::kPB;
    const uint32_t sv = s_base + C::kOffV + s * C::kSP * C::kPB;

    float sc[C::kNTT];
#pragma unroll
    for (int ti = 0; ti < C::kNTT; ++ti) {
      // partial dots v[r][g] for tokens ti*16 + r*8 + t8 over this lane's quarter
      float v0[2][G], v1[2][G];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int ts = ti * 16 + r * 8 + t8;
        const int pg = ts / BS;
        const int j = ts % BS;
#pragma unroll
        for (int g = 0; g < G; ++g) v0[r][g] = v1[r][g] = 0.f;
        if (pg < np) {
          const uint32_t row = sk + pg * C::kPB + (qtr * C::kCQ * BS + j) * 16;
#pragma unroll
          for (int c = 0; c < C::kCQ; ++c) {
            float kf[C::kX];
            unpack_chunk<TC>(lds128(row + c * BS * 16), kf);
#pragma unroll
            for (int e = 0; e < C::kX; e += 2) {
#pragma unroll
              for (int g = 0; g < G; ++g) {
#if VASR_DECODE_FFMA2
                fma2(v0[r][g], v1[r][g], q_reg[g][c * C::kX + e], q_reg[g][c * C::kX + e + 1],
                     kf[e], kf[e + 1]);
#else
                v0[r][g] = fmaf(q_reg[g][c * C::kX + e], kf[e], v0[r][g]);
                v1[r][g] = fmaf(q_reg[g][c * C::kX + e + 1], kf[e + 1], v1[r][g]);
#endif
              }
            }
          }
        }
      }
      // k = r * 2 + g
      const float v00 = v0[0][0] + v1[0][0], v01 = v0[0][1] + v1[0][1];
      const float v10 = v0[1][0] + v1[1][0], v11 = v0[1][1] + v1[1][1];
      // level 1 over quarter bit 1 (xor 16): keep round qb1
      const float send_a = qb1 ? v00 : v10, send_b = qb1 ? v01 : v11;
      const float ka = (qb1 ? v10 : v00) + __shfl_xor_sync(0xffffffffu, send_a, 16);
      const float kb = (qb1 ? v11 : v01) + __shfl_xor_sync(0xffffffffu, send_b, 16);
      // level 2 over quarter bit 0 (xor 8): keep head qb0
      const float send2 = qb0 ? ka : kb;
      const float dot = (qb0 ? kb : ka) + __shfl_xor_sync(0xffffffffu, send2, 8);
      float sv_ = dot * k_mul;
      if (use_softcap) sv_ = p.softcap * tanhf(sv_ / p.softcap);
      sc[ti] = (ti * 16 + s_tok < n_valid) ? sv_ * kLog2e : -INFINITY;
    }

    // ---- online softmax (lanes with qb0 = g hold head g's scores)
    float mloc = sc[0];
#pragma unroll
    for (int ti = 1; ti < C::kNTT; ++ti) mloc = fmaxf(mloc, sc[ti]);
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 1));
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 2));
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 4));
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 16));
    const float mother = __shfl_xor_sync(0xffffffffu, mloc, 8);
    const float mg0 = qb0 ? mother : mloc, mg1 = qb0 ? mloc : mother;
    const float mn0 = fmaxf(m_run[0], mg0), mn1 = fmaxf(m_run[1], mg1);
    const float a0 = exp2f(m_run[0] - mn0), a1 = exp2f(m_run[1] - mn1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    const float m_own = qb0 ? mn1 : mn0;
    const float a_own = qb0 ? a1 : a0;
    float psum = 0.f;
#pragma unroll
    for (int ti = 0; ti < C::kNTT; ++ti) {
      const float pv = exp2f(sc[ti] - m_own);
      psum += pv;
      p_w[s_head * C::kST + ti * 16 + s_tok] = pv;
    }
    l_part = fmaf(l_part, a_own, psum);
#pragma unroll
    for (int i = 0; i < C::kNR; ++i) {
      acc[i][0] *= a0;
      acc[i][1] *= a1;
    }
    __syncwarp();

    // ---- PV (as in paged_decode_kernel)
#pragma unroll
    for (int pg = 0; pg < C::kSP; ++pg) {
      if (pg < np) {
        float pw[G][C::kTPS];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float *src = p_w + g * C::kST + pg * BS + sg * C::kTPS;
#pragma unroll
          for (int e = 0; e < C::kTPS; e += 4) {
            const float4 v4 = *reinterpret_cast<const float4 *>(src + e);
            pw[g][e + 0] = v4.x;
            pw[g][e + 1] = v4.y;
            pw[g][e + 2] = v4.z;
            pw[g][e + 3] = v4.w;
          }
        }
        const int seg_tok0 = pg * BS + sg * C::kTPS;
        const bool tail = (seg_tok0 + C::kTPS > n_valid);
        const uint32_t vrow0 = sv + pg * C::kPB + sg * 16;
#pragma unroll
        for (int i = 0; i < C::kNR; ++i) {
          const int d = rlo + C::kRPP * ph + 4 * C::kRPP * i;
          float vf[C::kTPS];
          unpack_chunk<TC>(lds128(vrow0 + d * C::kR), vf);
          if (tail) {
#pragma unroll
            for (int e = 0; e < C::kTPS; ++e)
              if (seg_tok0 + e >= n_valid) vf[e] = 0.f;
          }
#if VASR_DECODE_FFMA2
#pragma unroll
          for (int e = 0; e < C::kTPS; ++e) fma2(acc[i][0], acc[i][1], pw[0][e], pw[1][e], vf[e], vf[e]);
#else
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < C::kTPS; ++e) acc[i][g] = fmaf(pw[g][e], vf[e], acc[i][g]);
#endif
        }
      }
    }
    __syncwarp();
    const int nu = u + C::kNST;
    if (nu < n_units && lane == 0) {
      fence_proxy_async_smem();
      issue_unit(nu);
    }
  }

  if (aborted) decode_drain_warp_stages<C>(s_base, u_abort, n_units, ubase);

  // ---- warp finalisation: l of head g lives in lanes with qb0 == g
  float l_g = l_part;
  l_g += __shfl_xor_sync(0xffffffffu, l_g, 1);
  l_g += __shfl_xor_sync(0xffffffffu, l_g, 2);
  l_g += __shfl_xor_sync(0xffffffffu, l_g, 4);
  l_g += __shfl_xor_sync(0xffffffffu, l_g, 16);
#pragma unroll
  for (int o = C::kRPP; o < C::kRPP * C::kNSEG; o <<= 1)
#pragma unroll
    for (int i = 0; i < C::kNR; ++i) {
      acc[i][0] += __shfl_xor_sync(0xffffffffu, acc[i][0], o);
      acc[i][1] += __shfl_xor_sync(0xffffffffu, acc[i][1], o);
    }
  float *co = reinterpret_cast<float *>(smem + C::kOffCO);
  float *cm = reinterpret_cast<float *>(smem + C::kOffCM);
  float *cl = reinterpret_cast<float *>(smem + C::kOffCL);
  if (aborted) {
    m_run[0] = m_run[1] = -INFINITY;
    l_g = 0.f;
#pragma unroll
    for (int i = 0; i < C::kNR; ++i) acc[i][0] = acc[i][1] = 0.f;
  }
  if (lane == 0 || lane == 8) {  // t8 == 0, qb1 == 0, qb0 = head
    cm[warp * G + qb0] = qb0 ? m_run[1] : m_run[0];
    cl[warp * G + qb0] = l_g;
  }
  if (sg == 0) {
#pragma unroll
    for (int i = 0; i < C::kNR; ++i) {
      const int d = rlo + C::kRPP * ph + 4 * C::kRPP * i;
      co[(warp * G + 0) * D + d] = acc[i][0];
      co[(warp * G + 1) * D + d] = acc[i][1];
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
  if (single) return (uint32_t)n_units;

  __syncthreads();
  uint32_t *flag = reinterpret_cast<uint32_t *>(smem + C::kOffFlag);
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.counters + bk, 1u);
    __threadfence();
    flag[0] = (prev == (uint32_t)(n_splits - 1)) ? 1u : 0u;
  }
  __syncthreads();
  if (flag[0] == 0u) return (uint32_t)n_units;
#pragma unroll
  for (int e0 = 0; e0 < G * D; e0 += C::kThreads) {
    const int e = e0 + tid;
    const int g = e / D;
    const int d = e % D;
    const int64_t slot0 = bk * p.max_splits;
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, __ldcg(&p.ws_ml[(slot0 + s) * G + g].x));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < n_splits; ++s) {
        const float2 ml = __ldcg(&p.ws_ml[(slot0 + s) * G + g]);
        const float w = exp2f(ml.x - M);
        L = fmaf(ml.y, w, L);
        O = fmaf(__ldcg(&p.ws_o[((slot0 + s) * G + g) * D + d]), w, O);
      }
    }
    out[g * D + d] = Elem<T>::from_f32(L > 0.f ? O / L * v_mul : 0.f);
  }
  if (tid == 0) p.counters[bk] = 0u;
  return (uint32_t)n_units;
}

template <typename TC, int BS, int D, int NST>
__device__ __forceinline__ void decode_g2_init_ring(unsigned char *smem) {
  using C = DecodeG2Cfg<TC, BS, D, NST>;
  if (threadIdx.x < C::kNST) mbar_init(smem_addr(smem) + C::kOffBar + threadIdx.x * 8, 1);
  if (threadIdx.x == 0) mbar_fence_init();
  __syncthreads();
}

// Grid form: one CTA per (split, kv head, sequence).
template <typename T, int BS, int D, int NST, int MINB, typename TC = T>
__global__ void __launch_bounds__(128, MINB) paged_decode_g2_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  decode_g2_init_ring<TC, BS, D, NST>(smem);
  decode_g2_item<T, BS, D, NST, TC>(p, smem, blockIdx.x, blockIdx.y, blockIdx.z, 0);
}

}  // namespace vasr

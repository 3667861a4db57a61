// decode.cuh — single-query paged decode attention for sm_100a.
//
// Semantics follow the reference's paged_attention call
// (vasr-models/src/model/thinker_text.rs:1126-1139) and its CPU oracle
// run_single_sequence_attention (vasr-models/src/model/attention.rs:243-286):
//   s_j = scale * (q . k_j)        (softcap s = c*tanh(s/c) when c != 1)
//   out = sum_j softmax(s)_j * v_j over the first context_len tokens.
//
// Work decomposition (one launch, no host sync, CUDA-graph safe):
//   grid  = (max_splits, num_kv_heads, num_seqs); 128 threads (4 warps).
//   A CTA owns one (sequence, kv head, split of P tokens). It computes all
//   G = num_heads / num_kv_heads query heads of the group, so every K/V byte
//   leaves HBM exactly once. Pages of the split are staged in shared memory
//   by 1-D bulk copies (cp.async.bulk, CTA-local destination) into NST
//   stages; stage s belongs to warp s % 4, which waits on the stage's
//   mbarrier, consumes it and immediately refills it with the page NST
//   stages ahead. Each warp keeps an online-softmax state; the 4 warp states
//   are merged in shared memory. Splits with no tokens exit at once.
//   Split-K reduce: a sequence with more than one split writes unnormalised
//   partials (o, m, l) to the workspace, bumps a per-(sequence, kv head)
//   counter, and the last CTA to arrive merges the partials in split order
//   (deterministic) and resets the counter to zero.
#pragma once

#include "common.cuh"

namespace vasr {

struct DecodeParams {
  void *out;
  const void *q;
  const void *k_cache;
  const void *v_cache;
  const uint32_t *block_tables;
  const uint32_t *context_lens;
  float *ws_o;        // [B * Hkv * S][G][D]
  float2 *ws_ml;      // [B * Hkv * S][G]  (m in log2 units, l)
  uint32_t *counters; // [B * Hkv]
  const float *k_scale;  // fp8 caches: per-tensor scales (device scalars), else null
  const float *v_scale;
  int64_t q_seq_stride;
  int64_t num_blocks;
  int num_seqs;
  int num_heads;
  int num_kv_heads;
  int cols;           // max_num_blocks_per_seq (block-table row width)
  int pages_per_split;
  int max_splits;
  float scale;
  float softcap;      // 1.0 = disabled
};

template <typename T, int BS, int D, int G>
struct DecodeCfg {
  static constexpr int kThreads = 128;
  static constexpr int kWarps = 4;
  static constexpr int kX = Elem<T>::kX;                // elements per 16 B
  static constexpr int kCH = D / kX;                    // 16-B chunks per K row
  static constexpr int kTT = 32 / G;                    // tokens per warp tile
  static constexpr int kSP = (kTT > BS) ? (kTT / BS) : 1;  // pages per stage
  static constexpr int kST = kSP * BS;                  // tokens per stage
  static constexpr int kNTT = kST / kTT;                // warp tiles per stage
  static constexpr int kPB = D * BS * (int)sizeof(T);   // bytes of one page
  static constexpr int kStageBytes = 2 * kSP * kPB;     // K + V pages
  static constexpr int kNST = (kStageBytes <= 8192) ? 8 : 4;
  // PV lane mapping: one V row (one dim, BS tokens) is kR bytes = kNSEG
  // 16-byte segments. An 8-lane phase covers kRPP rows x kNSEG segments so
  // that its 16-byte loads hit distinct bank groups.
  static constexpr int kTPS = 16 / (int)sizeof(T);      // tokens per segment
  static constexpr int kR = BS * (int)sizeof(T);
  static constexpr int kNSEG = kR / 16;
  static constexpr int kRPP = 8 / kNSEG;
  static constexpr int kNR = D / (4 * kRPP);            // rows per lane
  static constexpr int kMaxPagesPerSplit = 64;
  // shared memory layout (bytes)
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kNST * kSP * kPB;
  static constexpr int kOffP = kOffV + kNST * kSP * kPB;           // [W][G][ST] f32
  static constexpr int kOffCO = kOffP + kWarps * G * kST * 4;      // [W][G][D] f32
  static constexpr int kOffCM = kOffCO + kWarps * G * D * 4;       // [W][G] f32 m
  static constexpr int kOffCL = kOffCM + kWarps * G * 4;           // [W][G] f32 l
  static constexpr int kOffBlk = kOffCL + kWarps * G * 4;          // [64] u32
  static constexpr int kOffBar = (kOffBlk + kMaxPagesPerSplit * 4 + 15) & ~15;  // [NST] u64
  static constexpr int kOffFlag = kOffBar + kNST * 8;
  static constexpr int kSmemBytes = kOffFlag + 16;
  static_assert(D % (4 * kRPP) == 0, "head_dim not covered by PV lanes");
  static_assert(kNSEG >= 1 && kNSEG <= 8, "unsupported V row size");
  static_assert(kST % kTT == 0, "stage must hold whole warp tiles");
  static_assert(kNST % kWarps == 0, "stages must split evenly over warps");
};

template <typename T, int BS, int D, int G>
__global__ void __launch_bounds__(128, 2) paged_decode_kernel(const DecodeParams p) {
  using C = DecodeCfg<T, BS, D, G>;
  extern __shared__ __align__(128) unsigned char smem[];

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int P = p.pages_per_split * BS;

  // ---- context length and split range (true length read on the device)
  int ctx = (int)p.context_lens[b];
  const int ctx_cap_tables = p.cols * BS;
  const int ctx_cap_splits = p.max_splits * P;
  if (ctx > ctx_cap_tables || ctx > ctx_cap_splits) {
    if (split == 0 && tid == 0) raise_device_error(VASR_PA_DERR_CTX_RANGE);
    ctx = min(ctx, min(ctx_cap_tables, ctx_cap_splits));
  }
  T *out = reinterpret_cast<T *>(p.out) + ((int64_t)b * p.num_heads + (int64_t)kvh * G) * D;
  if (ctx <= 0) {
    if (split == 0) {
      for (int e = tid; e < G * D; e += C::kThreads) out[e] = Elem<T>::from_f32(0.f);
    }
    return;
  }
  const int n_splits = (ctx + P - 1) / P;
  if (split >= n_splits) return;
  const int tok_begin = split * P;
  const int tok_end = min(ctx, tok_begin + P);
  const int page_begin = tok_begin / BS;
  const int n_pages = (tok_end - tok_begin + BS - 1) / BS;
  const int n_units = (n_pages + C::kSP - 1) / C::kSP;

  const uint32_t s_base = smem_addr(smem);
  uint32_t *blk = reinterpret_cast<uint32_t *>(smem + C::kOffBlk);
  float *p_s = reinterpret_cast<float *>(smem + C::kOffP);

  // ---- block ids of this split; barrier init
  if (tid < n_pages) {
    uint32_t id = p.block_tables[(int64_t)b * p.cols + page_begin + tid];
    if ((int64_t)id >= p.num_blocks) {
      raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
      id = 0;
    }
    blk[tid] = id;
  }
  if (tid < C::kNST) mbar_init(s_base + C::kOffBar + tid * 8, 1);
  if (tid == 0) mbar_fence_init();
  __syncthreads();

  const T *kc = reinterpret_cast<const T *>(p.k_cache);
  const T *vc = reinterpret_cast<const T *>(p.v_cache);
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

  // Each warp primes its own stages.
  if (lane == 0) {
    for (int u = warp; u < min(C::kNST, n_units); u += C::kWarps) issue_unit(u);
  }

  // ---- per-lane query (head g of the group) in registers, f32
  const int t_lane = lane % C::kTT;
  const int g_lane = lane / C::kTT;
  float q_reg[D];
  {
    const T *qp = reinterpret_cast<const T *>(p.q) + (int64_t)b * p.q_seq_stride +
                  (int64_t)(kvh * G + g_lane) * D;
    const uint4 *q4 = reinterpret_cast<const uint4 *>(qp);
#pragma unroll
    for (int c = 0; c < C::kCH; ++c) {
      float f[C::kX];
      unpack_chunk<T>(__ldg(q4 + c), f);
#pragma unroll
      for (int e = 0; e < C::kX; ++e) q_reg[c * C::kX + e] = f[e];
    }
  }

  // PV lane mapping
  const int rlo = lane % C::kRPP;
  const int sg = (lane / C::kRPP) % C::kNSEG;
  const int ph = lane / 8;

  float m_run[G];
  float acc[C::kNR][G];
#pragma unroll
  for (int g = 0; g < G; ++g) m_run[g] = -INFINITY;
#pragma unroll
  for (int i = 0; i < C::kNR; ++i)
#pragma unroll
    for (int g = 0; g < G; ++g) acc[i][g] = 0.f;
  float l_part = 0.f;
  const float scale_l2 = p.scale;
  const bool use_softcap = (p.softcap != 1.0f) && (p.softcap > 0.f);
  bool aborted = false;
  int u_abort = 0;

  float *p_w = p_s + warp * G * C::kST;

  for (int u = warp; u < n_units; u += C::kWarps) {
    const int s = u % C::kNST;
    const uint32_t bar = s_base + C::kOffBar + s * 8;
    if (!mbar_wait_bounded(bar, (uint32_t)((u / C::kNST) & 1))) {
      aborted = true;
      u_abort = u;
      break;
    }
    const int unit_tok0 = tok_begin + u * C::kST;
    const int n_valid = min(C::kST, tok_end - unit_tok0);
    const int np = min(C::kSP, n_pages - u * C::kSP);
    const uint32_t sk = s_base + C::kOffK + s * C::kSP * C::kPB;
    const uint32_t sv = s_base + C::kOffV + s * C::kSP * C::kPB;

    // ---- scores: lane (t, g) computes q_g . k_t for each warp tile
    float sc[C::kNTT];
#pragma unroll
    for (int ti = 0; ti < C::kNTT; ++ti) {
      const int ts = ti * C::kTT + t_lane;
      const int pg = ts / BS;
      const int j = ts % BS;
      float part[C::kX];
#pragma unroll
      for (int e = 0; e < C::kX; ++e) part[e] = 0.f;
      if (pg < np) {
        const uint32_t row = sk + pg * C::kPB + j * 16;
#pragma unroll
        for (int c = 0; c < C::kCH; ++c) {
          float kf[C::kX];
          unpack_chunk<T>(lds128(row + c * BS * 16), kf);
#pragma unroll
          for (int e = 0; e < C::kX; ++e) part[e] = fmaf(q_reg[c * C::kX + e], kf[e], part[e]);
        }
      }
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < C::kX; ++e) dot += part[e];
      float sv_ = dot * scale_l2;
      if (use_softcap) sv_ = p.softcap * tanhf(sv_ / p.softcap);
      sc[ti] = (ts < n_valid) ? sv_ * kLog2e : -INFINITY;
    }

    // ---- online softmax update (log2 domain)
    float mloc = sc[0];
#pragma unroll
    for (int ti = 1; ti < C::kNTT; ++ti) mloc = fmaxf(mloc, sc[ti]);
    mloc = warp_max_xor(mloc, C::kTT);
    float alpha[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mg = __shfl_sync(0xffffffffu, mloc, g * C::kTT);
      const float mn = fmaxf(m_run[g], mg);
      alpha[g] = exp2f(m_run[g] - mn);
      m_run[g] = mn;
    }
    float m_own = m_run[0];
    float a_own = alpha[0];
#pragma unroll
    for (int g = 1; g < G; ++g) {
      if (g_lane == g) {
        m_own = m_run[g];
        a_own = alpha[g];
      }
    }
    float psum = 0.f;
#pragma unroll
    for (int ti = 0; ti < C::kNTT; ++ti) {
      const float pv = exp2f(sc[ti] - m_own);
      psum += pv;
      p_w[g_lane * C::kST + ti * C::kTT + t_lane] = pv;
    }
    l_part = fmaf(l_part, a_own, psum);
#pragma unroll
    for (int i = 0; i < C::kNR; ++i)
#pragma unroll
      for (int g = 0; g < G; ++g) acc[i][g] *= alpha[g];
    __syncwarp();

    // ---- PV: lane owns rows d = rlo + RPP*ph + 4*RPP*i, tokens of segment sg
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
          unpack_chunk<T>(lds128(vrow0 + d * C::kR), vf);
          if (tail) {
#pragma unroll
            for (int e = 0; e < C::kTPS; ++e)
              if (seg_tok0 + e >= n_valid) vf[e] = 0.f;
          }
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < C::kTPS; ++e) acc[i][g] = fmaf(pw[g][e], vf[e], acc[i][g]);
        }
      }
    }
    __syncwarp();

    // ---- refill this stage with the unit NST ahead
    const int nu = u + C::kNST;
    if (nu < n_units && lane == 0) {
      fence_proxy_async_smem();
      issue_unit(nu);
    }
  }

  // stages of this warp still in flight land before the CTA retires
  if (aborted) {
    for (int v = u_abort; v < min(u_abort + C::kNST, n_units); v += C::kWarps)
      mbar_wait_bounded(s_base + C::kOffBar + (v % C::kNST) * 8, (uint32_t)((v / C::kNST) & 1));
  }

  // ---- warp-level finalisation
  float l_g = warp_sum_xor(l_part, C::kTT);  // lanes of head g hold l_g
#pragma unroll
  for (int o = C::kRPP; o < C::kRPP * C::kNSEG; o <<= 1)
#pragma unroll
    for (int i = 0; i < C::kNR; ++i)
#pragma unroll
      for (int g = 0; g < G; ++g) acc[i][g] += __shfl_xor_sync(0xffffffffu, acc[i][g], o);

  float *co = reinterpret_cast<float *>(smem + C::kOffCO);
  float *cm = reinterpret_cast<float *>(smem + C::kOffCM);
  float *cl = reinterpret_cast<float *>(smem + C::kOffCL);
  if (aborted) {
    // A bounded wait gave up: contribute nothing (error already raised).
#pragma unroll
    for (int g = 0; g < G; ++g) m_run[g] = -INFINITY;
    l_g = 0.f;
#pragma unroll
    for (int i = 0; i < C::kNR; ++i)
#pragma unroll
      for (int g = 0; g < G; ++g) acc[i][g] = 0.f;
  }
  // m_run[g_lane] with a dynamic index would spill; pick it with selects.
  if (t_lane == 0) {
    float mo = m_run[0];
#pragma unroll
    for (int g = 1; g < G; ++g)
      if (g_lane == g) mo = m_run[g];
    cm[warp * G + g_lane] = mo;
    cl[warp * G + g_lane] = l_g;
  }
  if (sg == 0) {
#pragma unroll
    for (int i = 0; i < C::kNR; ++i) {
      const int d = rlo + C::kRPP * ph + 4 * C::kRPP * i;
#pragma unroll
      for (int g = 0; g < G; ++g) co[(warp * G + g) * D + d] = acc[i][g];
    }
  }
  __syncthreads();

  // ---- merge the 4 warp states; write final output or split partial
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
        const float sc_w = exp2f(cm[w * G + g] - M);
        L = fmaf(cl[w * G + g], sc_w, L);
        O = fmaf(co[(w * G + g) * D + d], sc_w, O);
      }
    }
    if (single) {
      out[g * D + d] = Elem<T>::from_f32(L > 0.f ? O / L : 0.f);
    } else {
      const int64_t slot = bk * p.max_splits + split;
      p.ws_o[(slot * G + g) * D + d] = O;
      if (d == 0) p.ws_ml[slot * G + g] = make_float2(M, L);
    }
  }
  if (single) return;

  // ---- split-K: the last CTA of this (sequence, kv head) merges partials.
  // The barrier orders every thread's partial stores before thread 0's
  // device-scope fence and arrival; the last arriver fences again before the
  // CTA reads the other splits' partials through L2.
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
    out[g * D + d] = Elem<T>::from_f32(L > 0.f ? O / L : 0.f);
  }
  if (tid == 0) p.counters[bk] = 0u;
}

// Split size chosen from host-visible arguments only, so that the workspace
// size and the launch always agree: `split_tokens` tokens per split, halved
// (down to 64) while fewer than 2 CTAs per B200 SM would be launched, and at
// most kDecodeMaxPagesPerSplit pages. Measured on B200 for config 2: the
// tensor-core GQA-2 kernel is fastest at 1024 (41.6 us vs 42.6 at 768 and
// 44.0 at 512), the CUDA-core kernels at 512 (46.8 us vs 50.7 at 256, 47.6 at
// 768, 49.8 at 1024).
#ifndef VASR_DECODE_SPLIT_TOKENS
#define VASR_DECODE_SPLIT_TOKENS 512
#endif
#ifndef VASR_DECODE_SPLIT_TOKENS_G2
#define VASR_DECODE_SPLIT_TOKENS_G2 1024
#endif
constexpr int kDecodeMaxPagesPerSplit = 64;
inline int decode_pages_per_split(int num_seqs, int num_kv_heads, int block_size,
                                  int max_context_len, int split_tokens) {
  const int kTargetCtas = 2 * 148;
  int tokens = split_tokens;
  auto ctas = [&](int t) {
    return (int64_t)num_seqs * num_kv_heads * ((max_context_len + t - 1) / t);
  };
  while (tokens > 64 && ctas(tokens) < kTargetCtas) tokens >>= 1;
  if (tokens < block_size) tokens = block_size;
  int pps = tokens / block_size;
  if (pps > kDecodeMaxPagesPerSplit) pps = kDecodeMaxPagesPerSplit;
  if (pps < 1) pps = 1;
  return pps;
}

}  // namespace vasr

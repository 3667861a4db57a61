/*
 * paged_oracle.c — CPU restatement of the reference's paged KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the parity tests and
 * bench.py's cpu_baseline / `--impl reference` arm compare against; nothing
 * in the product (libvasr_pa.so, the vasr_paged_attn package) links, loads
 * or calls it.
 *
 * What it restates (reference paths relative to di-osc/Qwen3ASR.rs):
 *  - cache layout K [nb, Hkv, D/x, bs, x], V [nb, Hkv, D, bs], x = 16/es:
 *    vasr-paged-attn/src/paged_kv_cache.rs:263-294;
 *  - reshape_and_cache scatter (slot = block*bs + pos%bs, -1 = skip):
 *    the call contract at vasr-models/src/model/thinker_text.rs:1101-1109,
 *    PAD_SLOT_ID at paged_kv_cache.rs:7;
 *  - gather_kv_cache (cu_seqlens_kv packing): thinker_text.rs:190-198;
 *  - attention: run_single_sequence_attention
 *    (vasr-models/src/model/attention.rs:243-286) after repeat_kv (:12-21):
 *    w = (q . k) * scale, optional softcap, masked entries = f32::MIN added
 *    (:68, :138-141), softmax over the last dim, then w . v;
 *  - the cached causal mask of make_causal_mask_cached (attention.rs:86-149)
 *    for chunked prefill: query at absolute position p sees keys j <= p.
 *  - copy/swap blocks as plain sequential block copies.
 * The attention entry points take f32 values laid out like a cache of any
 * element size (x = 16 / element size is passed in).
 * Arithmetic is f32 like Candle's CPU path, or f64 accumulation when
 * `use_double` is set (a tighter second check). OpenMP parallelises over
 * (sequence, head) for the timed CPU baseline.
 *
 * Parity pinning: the integer layout/slot math is pinned by the reference's
 * golden vectors (tests/test_oracle_golden.py); no test of the reference
 * executes reshape_and_cache / paged_attention / gather_kv_cache, so the
 * floating-point attention here is anchored only on attention.rs's own
 * packed-vs-unpacked equivalence test (<= 1e-4) and an independent
 * float64 restatement.
 */
#include <float.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_bits_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* byte offset of K element (blk, h, d, off) and of V element (blk, h, d, off) */
static inline int64_t k_index(int64_t blk, int h, int d, int off, int H, int D, int BS, int x) {
  return ((((blk * H + h) * (D / x) + d / x) * BS) + off) * x + d % x;
}
static inline int64_t v_index(int64_t blk, int h, int d, int off, int H, int D, int BS) {
  return (((blk * H + h) * (int64_t)D + d) * BS) + off;
}

/* reshape_and_cache on raw elements of size es (4 or 2). Strides in elements. */
void oracle_reshape_and_cache(const void *key, const void *value, void *key_cache,
                              void *value_cache, const int64_t *slots, int64_t T, int H, int D,
                              int BS, int64_t nb, int64_t k_stride, int64_t v_stride, int es) {
  const int x = 16 / es;
  const unsigned char *k = (const unsigned char *)key;
  const unsigned char *v = (const unsigned char *)value;
  unsigned char *kc = (unsigned char *)key_cache;
  unsigned char *vc = (unsigned char *)value_cache;
  for (int64_t t = 0; t < T; ++t) {
    const int64_t s = slots[t];
    if (s < 0 || s >= nb * BS) continue;
    const int64_t blk = s / BS;
    const int off = (int)(s % BS);
    for (int h = 0; h < H; ++h)
      for (int d = 0; d < D; ++d) {
        memcpy(kc + k_index(blk, h, d, off, H, D, BS, x) * es, k + (t * k_stride + h * D + d) * es, es);
        memcpy(vc + v_index(blk, h, d, off, H, D, BS) * es, v + (t * v_stride + h * D + d) * es, es);
      }
  }
}

void oracle_gather_kv_cache(void *k_out, void *v_out, const void *key_cache,
                            const void *value_cache, const uint32_t *block_tables,
                            const uint32_t *cu, int B, int cols, int H, int D, int BS, int es) {
  const int x = 16 / es;
  for (int b = 0; b < B; ++b) {
    const int64_t start = cu[b], len = (int64_t)cu[b + 1] - cu[b];
    for (int64_t t = 0; t < len; ++t) {
      const int64_t blk = block_tables[(int64_t)b * cols + t / BS];
      const int off = (int)(t % BS);
      for (int h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d) {
          memcpy((unsigned char *)k_out + (((start + t) * H + h) * D + d) * es,
                 (const unsigned char *)key_cache + k_index(blk, h, d, off, H, D, BS, x) * es, es);
          memcpy((unsigned char *)v_out + (((start + t) * H + h) * D + d) * es,
                 (const unsigned char *)value_cache + v_index(blk, h, d, off, H, D, BS) * es, es);
        }
    }
  }
}

/* copy_blocks over L layers: page dst <- page src, pairs applied in order. */
void oracle_copy_blocks(void **k_caches, void **v_caches, int L, const int64_t *pairs,
                        int64_t N, int64_t block_bytes) {
  for (int l = 0; l < L; ++l)
    for (int64_t i = 0; i < N; ++i) {
      const int64_t src = pairs[2 * i], dst = pairs[2 * i + 1];
      memmove((unsigned char *)k_caches[l] + dst * block_bytes,
              (unsigned char *)k_caches[l] + src * block_bytes, (size_t)block_bytes);
      memmove((unsigned char *)v_caches[l] + dst * block_bytes,
              (unsigned char *)v_caches[l] + src * block_bytes, (size_t)block_bytes);
    }
}

void oracle_swap_blocks(void *dst, const void *src, const int64_t *pairs, int64_t N,
                        int64_t block_bytes) {
  for (int64_t i = 0; i < N; ++i)
    memcpy((unsigned char *)dst + pairs[2 * i + 1] * block_bytes,
           (const unsigned char *)src + pairs[2 * i] * block_bytes, (size_t)block_bytes);
}

/* One query row against keys [0, n_keys) of one sequence / kv head.
 * Restates attention.rs:243-286 for a single (batch, head, query) row. */
static void attend_row(float *o, const float *q, const float *kc, const float *vc,
                       const uint32_t *table, int64_t n_keys, int kvh, int H, int D, int BS, int x,
                       float scale, float softcap, int use_double, float *w) {
  /* x = key pack of the cache layout the values came from (16 / element size). */
  for (int64_t j = 0; j < n_keys; ++j) {
    const int64_t blk = table[j / BS];
    const int off = (int)(j % BS);
    float s;
    if (use_double) {
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += (double)q[d] * (double)kc[k_index(blk, kvh, d, off, H, D, BS, x)];
      s = (float)acc;
    } else {
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc += q[d] * kc[k_index(blk, kvh, d, off, H, D, BS, x)];
      s = acc;
    }
    s *= scale;
    if (softcap != 1.0f && softcap > 0.f) s = softcap * tanhf(s / softcap);
    w[j] = s;
  }
  float m = -INFINITY;
  for (int64_t j = 0; j < n_keys; ++j) m = w[j] > m ? w[j] : m;
  if (use_double) {
    double sum = 0.0;
    double *od = (double *)calloc((size_t)D, sizeof(double));
    for (int64_t j = 0; j < n_keys; ++j) {
      const double e = exp((double)w[j] - (double)m);
      sum += e;
      const int64_t blk = table[j / BS];
      const int off = (int)(j % BS);
      for (int d = 0; d < D; ++d) od[d] += e * (double)vc[v_index(blk, kvh, d, off, H, D, BS)];
    }
    for (int d = 0; d < D; ++d) o[d] = n_keys > 0 ? (float)(od[d] / sum) : 0.f;
    free(od);
  } else {
    float sum = 0.f;
    for (int64_t j = 0; j < n_keys; ++j) {
      w[j] = expf(w[j] - m);
      sum += w[j];
    }
    for (int d = 0; d < D; ++d) o[d] = 0.f;
    for (int64_t j = 0; j < n_keys; ++j) {
      const float p = w[j] / sum;
      const int64_t blk = table[j / BS];
      const int off = (int)(j % BS);
      for (int d = 0; d < D; ++d) o[d] += p * vc[v_index(blk, kvh, d, off, H, D, BS)];
    }
  }
}

/* paged decode attention, f32 cache and q/out [B, Hq, D] contiguous. */
void oracle_paged_attention_f32(float *out, const float *q, const float *kc, const float *vc,
                                const uint32_t *block_tables, const uint32_t *ctx, int B, int Hq,
                                int Hkv, int D, int BS, int x, int cols, float scale,
                                float softcap, int use_double, int threads) {
  const int G = Hq / Hkv;
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h) {
      const int64_t n = ctx[b];
      float *w = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
      float *o = out + ((int64_t)b * Hq + h) * D;
      if (n == 0) {
        for (int d = 0; d < D; ++d) o[d] = 0.f;
      } else {
        attend_row(o, q + ((int64_t)b * Hq + h) * D, kc, vc, block_tables + (int64_t)b * cols, n,
                   h / G, Hkv, D, BS, x, scale, softcap, use_double, w);
      }
      free(w);
    }
}

/* causal chunked prefill: packed q/out [T, Hq, D]; sequence b has queries
 * cu_q[b]..cu_q[b+1] at absolute positions ctx[b]-qlen+i. */
void oracle_prefill_varlen_f32(float *out, const float *q, const float *kc, const float *vc,
                               const uint32_t *block_tables, const uint32_t *ctx,
                               const uint32_t *cu_q, int B, int Hq, int Hkv, int D, int BS, int x,
                               int cols, float scale, float softcap, int use_double, int threads) {
  const int G = Hq / Hkv;
  if (threads > 0) omp_set_num_threads(threads);
  const int64_t T = cu_q[B];
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t t = 0; t < T; ++t)
    for (int h = 0; h < Hq; ++h) {
      int b = 0;
      while (b + 1 < B && (int64_t)cu_q[b + 1] <= t) ++b;
      const int64_t qlen = (int64_t)cu_q[b + 1] - cu_q[b];
      const int64_t pos = (int64_t)ctx[b] - qlen + (t - cu_q[b]);
      const int64_t n = pos + 1; /* keys 0..pos visible */
      float *w = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
      float *o = out + (t * Hq + h) * D;
      if (n <= 0) {
        for (int d = 0; d < D; ++d) o[d] = 0.f;
      } else {
        attend_row(o, q + (t * Hq + h) * D, kc, vc, block_tables + (int64_t)b * cols, n, h / G, Hkv,
                   D, BS, x, scale, softcap, use_double, w);
      }
      free(w);
    }
}

int oracle_max_threads(void) { return omp_get_max_threads(); }

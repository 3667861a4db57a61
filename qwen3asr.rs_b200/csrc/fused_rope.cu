// fused_rope.cu — q/k RMSNorm + rotary embedding + KV append in one launch.
//
// Replaces, per decoder layer, the chain that precedes paged attention in
// vasr-models/src/model/thinker_text.rs:1041-1109: q_norm / k_norm (per-head
// RMSNorm with a learned weight), the rotary embedding of q and k (mRoPE,
// whose three position streams are equal for text and audio tokens, i.e.
// 1-D rotate-half RoPE), and reshape_and_cache of k and v.
//
// Numerics follow the unfused bf16 path step by step: RMSNorm in f32
// (x * rsqrt(mean(x^2) + eps) * w), result rounded to the element type;
// RoPE in f32 on the rounded values (x1 c - x2 s, x2 c + x1 s), result
// rounded again. One warp handles one (token, head); lane l owns dims
// 2l, 2l+1, 64+2l, 65+2l, so both rotate-half partners sit in one lane.
#include "common.cuh"
#include "launch.h"

namespace vasr {
namespace {

template <typename T>
struct Pair;
template <>
struct Pair<__nv_bfloat16> {
  using V = __nv_bfloat162;
  __device__ static float2 load(const __nv_bfloat16 *p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
  }
  __device__ static void store(__nv_bfloat16 *p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(a, b);
  }
  __device__ static float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <>
struct Pair<__half> {
  using V = __half2;
  __device__ static float2 load(const __half *p) {
    return __half22float2(*reinterpret_cast<const __half2 *>(p));
  }
  __device__ static void store(__half *p, float a, float b) {
    *reinterpret_cast<__half2 *>(p) = __floats2half2_rn(a, b);
  }
  __device__ static float round(float x) { return __half2float(__float2half_rn(x)); }
};

struct FusedRopeParams {
  void *q_out;
  const void *qkv;
  const void *q_norm_w;
  const void *k_norm_w;
  const float *cos_t;
  const float *sin_t;
  const int64_t *positions;
  void *k_cache;
  void *v_cache;
  const int64_t *slots;
  int64_t qkv_stride;   // elements between tokens of qkv
  int64_t num_tokens;
  int64_t num_blocks;
  int64_t max_position;
  int num_heads;
  int num_kv_heads;
  float eps;
};

constexpr int kWarpsPerCta = 8;

// D = 128, BS = block size. Warp task w of a token: [0, Hq) q heads,
// [Hq, Hq + Hkv) k heads, [Hq + Hkv, Hq + 2 Hkv) v heads.
template <typename T, int BS>
__global__ void __launch_bounds__(32 * kWarpsPerCta) fused_qk_norm_rope_append_kernel(
    const FusedRopeParams p) {
  // A decode launched behind this kernel as a programmatic dependent may
  // start now: it reads nothing this kernel writes before it waits.
  pdl_launch_dependents();
  constexpr int D = 128;
  constexpr int kX = Elem<T>::kX;
  const int tasks = p.num_heads + 2 * p.num_kv_heads;
  const int64_t gw = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (gw >= p.num_tokens * tasks) return;
  const int lane = threadIdx.x & 31;
  const int64_t t = gw / tasks;
  const int task = (int)(gw - t * tasks);
  const T *row = reinterpret_cast<const T *>(p.qkv) + t * p.qkv_stride + (int64_t)task * D;
  const int d0 = 2 * lane, d1 = 64 + 2 * lane;
  float2 a = Pair<T>::load(row + d0);  // dims d0, d0+1
  float2 c = Pair<T>::load(row + d1);  // dims d1, d1+1

  const bool is_v = task >= p.num_heads + p.num_kv_heads;
  const bool is_k = !is_v && task >= p.num_heads;
  int64_t slot = -1, blk = 0;
  int off = 0;
  if (is_k || is_v) {
    slot = p.slots[t];
    if (slot >= p.num_blocks * BS) {
      if (lane == 0) raise_device_error(VASR_PA_DERR_SLOT_RANGE);
      slot = -1;
    }
    blk = slot >= 0 ? slot / BS : 0;
    off = slot >= 0 ? (int)(slot - blk * BS) : 0;
  }
  if (is_v) {
    if (slot < 0) return;
    const int h = task - p.num_heads - p.num_kv_heads;
    T *vrow = reinterpret_cast<T *>(p.v_cache) + ((blk * p.num_kv_heads + h) * D) * BS + off;
    vrow[(int64_t)d0 * BS] = Elem<T>::from_f32(a.x);
    vrow[(int64_t)(d0 + 1) * BS] = Elem<T>::from_f32(a.y);
    vrow[(int64_t)d1 * BS] = Elem<T>::from_f32(c.x);
    vrow[(int64_t)(d1 + 1) * BS] = Elem<T>::from_f32(c.y);
    return;
  }
  // RMSNorm over the 128 dims of this head
  float ss = a.x * a.x + a.y * a.y + c.x * c.x + c.y * c.y;
  ss = warp_sum_xor(ss, 32);
  const float inv = rsqrtf(ss / (float)D + p.eps);
  const T *w = reinterpret_cast<const T *>(is_k ? p.k_norm_w : p.q_norm_w);
  const float2 wa = Pair<T>::load(w + d0), wc = Pair<T>::load(w + d1);
  const float n0 = Pair<T>::round(a.x * inv * wa.x), n1 = Pair<T>::round(a.y * inv * wa.y);
  const float n2 = Pair<T>::round(c.x * inv * wc.x), n3 = Pair<T>::round(c.y * inv * wc.y);
  // rotate-half RoPE: pairs (d0, d1) and (d0+1, d1+1) share frequencies 2l and 2l+1
  int64_t pos = p.positions[t];
  pos = pos < 0 ? 0 : (pos >= p.max_position ? p.max_position - 1 : pos);
  const float2 cs = *reinterpret_cast<const float2 *>(p.cos_t + pos * (D / 2) + d0);
  const float2 sn = *reinterpret_cast<const float2 *>(p.sin_t + pos * (D / 2) + d0);
  // Explicitly rounded products (no FMA contraction) so the rotation rounds
  // exactly like the unfused multiply-then-subtract path.
  const float r0 = __fsub_rn(__fmul_rn(n0, cs.x), __fmul_rn(n2, sn.x));
  const float r1 = __fsub_rn(__fmul_rn(n1, cs.y), __fmul_rn(n3, sn.y));
  const float r2 = __fadd_rn(__fmul_rn(n2, cs.x), __fmul_rn(n0, sn.x));
  const float r3 = __fadd_rn(__fmul_rn(n3, cs.y), __fmul_rn(n1, sn.y));
  if (!is_k) {
    T *q = reinterpret_cast<T *>(p.q_out) + (t * p.num_heads + task) * D;
    Pair<T>::store(q + d0, r0, r1);
    Pair<T>::store(q + d1, r2, r3);
    return;
  }
  if (slot < 0) return;
  const int h = task - p.num_heads;
  T *kpage = reinterpret_cast<T *>(p.k_cache) + ((blk * p.num_kv_heads + h) * D) * BS;
  // K layout [D/x][BS][x]: dims d, d+1 (d even) are adjacent inside one x-chunk
  Pair<T>::store(kpage + ((int64_t)(d0 / kX) * BS + off) * kX + d0 % kX, r0, r1);
  Pair<T>::store(kpage + ((int64_t)(d1 / kX) * BS + off) * kX + d1 % kX, r2, r3);
}

template <typename T>
int launch_t(const FusedRopeParams &p, int block_size, cudaStream_t s) {
  const int tasks = p.num_heads + 2 * p.num_kv_heads;
  const int64_t warps = p.num_tokens * tasks;
  const int64_t ctas = (warps + kWarpsPerCta - 1) / kWarpsPerCta;
  if (ctas > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
  switch (block_size) {
    case 8: fused_qk_norm_rope_append_kernel<T, 8><<<(unsigned)ctas, 32 * kWarpsPerCta, 0, s>>>(p); break;
    case 16: fused_qk_norm_rope_append_kernel<T, 16><<<(unsigned)ctas, 32 * kWarpsPerCta, 0, s>>>(p); break;
    case 32: fused_qk_norm_rope_append_kernel<T, 32><<<(unsigned)ctas, 32 * kWarpsPerCta, 0, s>>>(p); break;
    default: return VASR_PA_EINVAL_BLOCKSIZE;
  }
  return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
}

}  // namespace

int launch_fused_rope(const FusedRopeArgs &a, cudaStream_t s) {
  FusedRopeParams p{};
  p.q_out = a.q_out;
  p.qkv = a.qkv;
  p.q_norm_w = a.q_norm_weight;
  p.k_norm_w = a.k_norm_weight;
  p.cos_t = a.cos_table;
  p.sin_t = a.sin_table;
  p.positions = a.positions;
  p.k_cache = a.key_cache;
  p.v_cache = a.value_cache;
  p.slots = a.slot_mapping;
  p.qkv_stride = a.qkv_token_stride;
  p.num_tokens = a.num_tokens;
  p.num_blocks = a.num_blocks;
  p.max_position = a.max_position;
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.eps = a.eps;
  switch (a.dtype) {
    case VASR_PA_BF16: return launch_t<__nv_bfloat16>(p, a.block_size, s);
    case VASR_PA_F16: return launch_t<__half>(p, a.block_size, s);
    default: return VASR_PA_ENOT_SUPPORTED;
  }
}

int read_error_fused(uint32_t *bits, bool clear, cudaStream_t s) {
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

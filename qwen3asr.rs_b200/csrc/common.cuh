// common.cuh — shared device helpers for the sm_100a paged KV-cache kernels.
//
// Element types, 16-byte vector access, bf16 <-> f32 unpacking, the device
// error word, and the mbarrier + cp.async.bulk (CTA-local destination)
// primitives used to stage whole cache pages in shared memory.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vasr_pa.h"

namespace vasr {

// One error word per device and per translation unit (file-scope device
// variable with internal linkage, zero at load). Kernels OR VASR_PA_DERR_*
// bits into it; vasr_pa_get_device_error ORs the words of all units.
static __device__ uint32_t g_device_error;

__device__ __forceinline__ void raise_device_error(uint32_t bits) {
  atomicOr(&g_device_error, bits);
}

// ---------------------------------------------------------------- elements
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kX = 4;  // elements per 16-byte chunk
  __device__ static __forceinline__ float to_f32(float v) { return v; }
  __device__ static __forceinline__ float from_f32(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kX = 8;
  __device__ static __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static constexpr int kX = 8;
  __device__ static __forceinline__ float to_f32(__half v) { return __half2float(v); }
  __device__ static __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};

// Unpack one 16-byte chunk into f32 values (kX of them).
__device__ __forceinline__ void unpack16(const uint4 &u, float (&f)[4]) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}
// bf16 -> f32 is exact: the bf16 bits are the high half of the f32 bits.
__device__ __forceinline__ void unpack_bf16x2(uint32_t w, float &lo, float &hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xffff0000u);
}
__device__ __forceinline__ void unpack16_bf16(const uint4 &u, float (&f)[8]) {
  unpack_bf16x2(u.x, f[0], f[1]);
  unpack_bf16x2(u.y, f[2], f[3]);
  unpack_bf16x2(u.z, f[4], f[5]);
  unpack_bf16x2(u.w, f[6], f[7]);
}
__device__ __forceinline__ void unpack_half2(uint32_t w, float &lo, float &hi) {
  __half2 h = *reinterpret_cast<__half2 *>(&w);
  float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}
__device__ __forceinline__ void unpack16_f16(const uint4 &u, float (&f)[8]) {
  unpack_half2(u.x, f[0], f[1]);
  unpack_half2(u.y, f[2], f[3]);
  unpack_half2(u.z, f[4], f[5]);
  unpack_half2(u.w, f[6], f[7]);
}

// fp8 E4M3 (KV-cache storage only): 16 values per 16-byte chunk, converted
// through the cuda_fp8.h pair conversion to f16 (exact) and then to f32.
template <> struct Elem<__nv_fp8_e4m3> {
  static constexpr int kX = 16;
  __device__ static __forceinline__ float to_f32(__nv_fp8_e4m3 v) { return float(v); }
};
__device__ __forceinline__ void unpack16_fp8(const uint4 &u, float (&f)[16]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xffffu), __NV_E4M3);
    __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
    const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&lo));
    const float2 b = __half22float2(*reinterpret_cast<__half2 *>(&hi));
    f[4 * i + 0] = a.x;
    f[4 * i + 1] = a.y;
    f[4 * i + 2] = b.x;
    f[4 * i + 3] = b.y;
  }
}

template <typename T>
__device__ __forceinline__ void unpack_chunk(const uint4 &u, float (&f)[Elem<T>::kX]);
template <>
__device__ __forceinline__ void unpack_chunk<float>(const uint4 &u, float (&f)[4]) { unpack16(u, f); }
template <>
__device__ __forceinline__ void unpack_chunk<__nv_bfloat16>(const uint4 &u, float (&f)[8]) { unpack16_bf16(u, f); }
template <>
__device__ __forceinline__ void unpack_chunk<__half>(const uint4 &u, float (&f)[8]) { unpack16_f16(u, f); }
template <>
__device__ __forceinline__ void unpack_chunk<__nv_fp8_e4m3>(const uint4 &u, float (&f)[16]) {
  unpack16_fp8(u, f);
}

// ------------------------------------------------------- shared-memory I/O
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialisation may start while the kernel before it on the stream still
// runs; pdl_wait() returns once that kernel has completed and its memory
// operations are visible (at once when the launch was an ordinary one).
// pdl_launch_dependents() lets such a dependent start before this grid ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Global loads that bypass L1 (data written by other CTAs of this launch).
__device__ __forceinline__ float ldcg_f32(const float *p) { return __ldcg(p); }

// --------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after kMaxPolls polls (each try_wait suspends for a
// hardware-chosen interval), raises VASR_PA_DERR_WAIT_TIMEOUT and returns
// false so the caller can leave instead of spinning forever.
constexpr uint32_t kMaxPolls = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  raise_device_error(VASR_PA_DERR_WAIT_TIMEOUT);
  return false;
}
// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Destination is this CTA only; src and dst 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst_smem, const void *src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_smem),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 16-byte (L2 only) and 8-byte asynchronous copies global -> shared, and an
// arrive on `bar` once every such copy of this thread has landed (not
// counted up first: the barrier's expected count includes it).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// ------------------------------------------------------------ warp helpers
__device__ __forceinline__ float warp_max_xor(float v, int lanes) {
  for (int o = lanes >> 1; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_xor(float v, int lanes) {
  for (int o = lanes >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// d0 += a0 * b0, d1 += a1 * b1 as one sm_100 packed f32x2 FMA (each lane a
// fused multiply-add rounded to nearest, exactly as fmaf).
__device__ __forceinline__ void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rd, {%0, %1};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rd;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace vasr

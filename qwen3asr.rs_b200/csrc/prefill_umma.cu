// prefill_umma.cu — causal varlen (chunked) prefill attention on the
// 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// Same contract as the mma.sync kernel of prefill.cu (row i of sequence b
// sits at position ctx[b] - qlen_b + i and attends keys j <= position, the
// cached causal mask of vasr-models/src/model/attention.rs:86-149 applied
// to run_single_sequence_attention :243-286), for bf16 / f16 pages of 16
// tokens and head_dim 128.
//
// One CTA owns M = 128 rows = (128 / G) query positions x the G query heads
// of one kv head and walks the keys in 64-key tiles:
//   S  = Q K^T   one tcgen05.mma M128 N64 K16 per 16 head dims -> TMEM
//   P  = exp2(S * scale * log2e - m)   one thread per row; P (16-bit) is
//        stored back over the first half of its S buffer in TMEM
//   O += P V     one tcgen05.mma M128 N128 K16 per 16-token page, A = P read
//        from TMEM, accumulator O in TMEM
// Warp roles (256 threads): warps 0-3 own TMEM lanes 0-127 (one row per
// thread: softmax, O rescale, epilogue); warp 4 issues P V, warp 7 Q K^T
// (two issuers, so that neither kind of MMA waits behind the other's issue,
// which stalls while the tensor core is busy); warp 5 stages Q (TMA) and K,
// warp 6 stages V, both by 16-byte cp.async (a K page row is 16 bytes wide,
// so a K tile would cost 16 TMA gathers, and the SM's TMA unit serves both
// resident CTAs). S is double-buffered in TMEM, so Q K^T of tile j + 1 is
// ready while the softmax warps work on tile j, and the softmax of tile
// j + 1 does not wait for P V of tile j unless O needs a rescale.
//
// Launches with few items (a long context with few new tokens) use a
// second variant (224 threads, warp 4 issues both kinds of MMA): each item's
// key tiles are shared by a thread-block cluster of up to 8 CTAs whose
// partial O rows are combined through distributed shared memory.
//
// Shared-memory operand layouts (all "K-major", the reduction dim inside a
// 16-byte chunk):
//   Q  [2 dim halves][128 rows][128 B]   the 128-byte swizzle (SBO 1024),
//      the canonical SW128 K-major layout; one 3-D TMA load per half
//      (64 elements x head x token), 128-byte rows
//   K  [16 dim chunks][64 keys][16 B]    no swizzle, LBO 1024, SBO 128; the
//      K loader warp fills it with 16-byte cp.async copies (32 per lane)
//   V  one page = [128 dims][16 tokens] rows of 32 B in the 32-byte-swizzled
//      image (16-byte half h of dim d at h ^ ((d >> 2) & 1)), written by the
//      V loader's 16-byte cp.async copies = the canonical SW32 K-major layout
//      (SBO 256) that the page's 16 tokens feed as one K = 16 step
// Softmax keeps a per-row running max that only moves when a tile's max
// exceeds it by more than 2^8, so O in TMEM is rescaled rarely (exact in
// real arithmetic: numerator and denominator use the same offset).
// Every mbarrier wait is bounded (VASR_PA_DERR_WAIT_TIMEOUT). A warp whose
// wait gives up issues no further copy or MMA; the load warp then waits
// (bounded) for the last copy issued on each stage and the MMA warp for its
// last commit, so that no copy lands in shared memory and no MMA writes
// tensor memory after the CTA has let them go; the kernel always frees its
// tensor memory before returning.
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "launch.h"

namespace vasr {
namespace {

constexpr int kD = 128;
constexpr int kM = 128;                      // rows per CTA (UMMA M)
constexpr int kNT = 64;                      // keys per tile (UMMA N of S)
constexpr int kBS = 16;                      // tokens per page
constexpr int kPagesPerTile = kNT / kBS;     // 4
constexpr int kPageBytes = kD * kBS * 2;     // one head's K or V page (16-bit; the staged image)
constexpr int kPageBytesF8 = kD * kBS;       // one head's K or V page of fp8 bytes
constexpr int kStages = 2;
constexpr int kQBytes = kM * kD * 2;         // 32 KB
constexpr int kKVTile = kNT * kD * 2;        // 16 KB
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;
constexpr int kOffV = kOffK + kStages * kKVTile;
constexpr int kOffBar = kOffV + kStages * kKVTile;
// One commit per MMA group: "Q K^T j done" both fills S j and frees K
// stage j & 1; "P V j done" both frees V stage j & 1 and the S buffer of j.
// K and V stages are full after 32 cp.async arrivals (one per loader lane).
// kBarQ16: fp8 pages with bf16 queries — Q converted to f16 in place by the
// 128 softmax threads (the MMAs then run in f16, exact for every E4M3 value).
constexpr int kBarFullK = 0, kBarFullV = 2, kBarSFull = 4, kBarPFull = 6, kBarPvDone = 8,
              kBarQ = 10, kBarQ16 = 11;
constexpr int kBarEmptyK = kBarSFull, kBarEmptyV = kBarPvDone;
constexpr int kNumBars = 12;
__host__ __device__ constexpr uint32_t bar_count(int i) {
  return (i == kBarPFull || i == kBarPFull + 1 || i == kBarQ16) ? 128u : (i < kBarSFull ? 32u : 1u);
}
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemUsed = kOffTmemSlot + 16;
constexpr int kSmemAlign = 1024;             // SW128 Q tile: 1024-byte alignment
constexpr int kSmemBytes = kSmemUsed + kSmemAlign;
constexpr int kTmemCols = 256;               // S ring 2 x 64 columns + O 128 columns
constexpr int kTmemS = 0, kTmemO = 128;
// warps 0-3 rows, 4 P V MMAs, 5 Q + K loads, 6 V loads, 7 Q K^T MMAs; the
// split variant has no warp 7 (warp 4 issues both kinds of MMA there)
constexpr int kThreadsFor(bool split) { return split ? 224 : 256; }
constexpr int kMmaWarp = 4;
constexpr int kLoadWarp = 5;
constexpr int kVLoadWarp = 6;
constexpr int kSMmaWarp = 7;
constexpr int kIdRegs = 4;                 // block ids of pages 0..127 held in registers
constexpr float kRescaleLog2 = 8.f;          // rescale O only when the max grows > 2^8
constexpr uint64_t kWaitNs = 200000000ull;   // 200 ms per wait before giving up

static_assert(kSmemBytes + 1024 <= 233472 / 2, "two CTAs per SM must fit");

// ------------------------------------------------------------ tcgen05 helpers
// Shared-memory matrix descriptor: start, leading / stride byte offsets
// (16-byte units), descriptor version 1, layout type (0 none, 6 SW32).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                          uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
// Instruction descriptor of kind::f16: f32 accumulate, A and B of the same
// 16-bit type, both K-major, M = 128, N = n.
template <typename T>
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kM >> 4) << 24);
}
// The MMA helpers are called by a whole converged warp with warp-uniform
// operands; elect.sync picks the issuing lane inside the asm (always the
// same lane, so its commits track its own MMAs). Issued this way an MMA
// costs about half the issue time of one issued from a single-lane branch.
// A from tensor memory: row i in lane i, 16-bit K pairs packed per 32-bit column.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (count 1) on `bar` once every tcgen05 op issued so far by the
// elected lane completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
          bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   slot_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ float ex2_approx(float x) {  // PTX ex2.approx.ftz.f32
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// Warp-uniform bounded wait for the phase `parity` of `bar` (every lane of
// the warp calls it). After kWaitNs it raises VASR_PA_DERR_WAIT_TIMEOUT and
// sets `dead`; a dead warp skips all later waits, so the CTA runs straight
// to its end, drains its own copies and MMAs with bounded waits and frees
// its tensor memory.
__device__ __forceinline__ void wait_phase(uint32_t bar, uint32_t parity, bool &dead) {
  if (!dead && !mbar_try_wait(bar, parity)) {
    const uint64_t t0 = globaltimer_ns();
    bool ok = false;
    while (!ok) {
      for (int i = 0; i < 64 && !ok; ++i) ok = mbar_try_wait(bar, parity);
      if (!ok && globaltimer_ns() - t0 > kWaitNs) break;
    }
    if (!ok) {
      raise_device_error(VASR_PA_DERR_WAIT_TIMEOUT);
      dead = true;
    }
  }
  dead = __any_sync(0xffffffffu, dead);
}

// 3-D tiled TMA load (the Q tile: 64 elements x heads x tokens).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// Zero tokens >= valid of one V page in the SW32 layout (a 32-byte row per
// dim; the 16-byte half with tokens 8h..8h+7 of dim d sits at half
// h ^ ((d >> 2) & 1), token 8h + e at byte 2e). One warp, 16-byte accesses.
__device__ __forceinline__ void zero_v_page_tail(unsigned char *vp, int valid, int lane) {
#pragma unroll
  for (int i = 0; i < kD / 32; ++i) {
    const int d = lane + 32 * i;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int lo = valid - 8 * h;  // tokens 8h + e with e < lo stay
      if (lo >= 8) continue;
      uint4 *c = reinterpret_cast<uint4 *>(vp + d * 32 + ((h ^ ((d >> 2) & 1)) * 16));
      if (lo <= 0) {
        *c = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      uint4 v = *c;
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = (2 * e >= lo) ? 0u : (2 * e + 1 >= lo) ? (w[e] & 0xFFFFu) : w[e];
      *c = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2f(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2f<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2f<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
// 16 fp8 E4M3 bytes -> 16 f16 values (exact) as two 16-byte chunks: lo =
// bytes 0-7, hi = bytes 8-15, each byte's value at its own position.
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t v16) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v16 & 0xffffu), __NV_E4M3);
  return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ void e4m3x16_f16(const uint4 &v, uint4 &lo, uint4 &hi) {
  lo = make_uint4(e4m3x2_f16x2(v.x), e4m3x2_f16x2(v.x >> 16), e4m3x2_f16x2(v.y), e4m3x2_f16x2(v.y >> 16));
  hi = make_uint4(e4m3x2_f16x2(v.z), e4m3x2_f16x2(v.z >> 16), e4m3x2_f16x2(v.w), e4m3x2_f16x2(v.w >> 16));
}
// 8 bf16 values -> 8 f16 values (round to nearest; |x| above 65504 becomes inf)
__device__ __forceinline__ uint32_t bf16x2_f16x2(uint32_t w) {
  __half2 h = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  return *reinterpret_cast<uint32_t *>(&h);
}

// ---------------------------------------------- split items: cluster combine
// Every thread of every CTA of the cluster: a full cluster barrier (arrive has
// release, wait acquire semantics, so shared-memory writes before it are
// visible to the cluster's reads after it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the shared-memory address `addr` of this CTA, in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}
__device__ __forceinline__ float2 ld_cluster_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

constexpr int kMaxSplits = 8;             // CTAs per cluster (portable limit)
constexpr int kCPitch = kD + 4;           // floats per staged O row (rows 16 bytes apart mod 128)
constexpr int kOffRed = kOffQ + kM * kCPitch * 4;  // (m, l) per row
static_assert(kOffRed + kM * 8 <= kOffBar, "the combine staging fits in the Q, K and V buffers");

// The softmax threads (row r each) of one CTA of a split item. After the
// CTA's last barrier (which the loader and MMA warps meet before their two
// cluster barriers) the CTA's unnormalised O rows (f32) and (m, l) go to its
// own shared memory; after a cluster barrier each CTA reads every CTA's copy
// of its run of the rows that hold query positions, weights them by
// 2^(m_s - M) and writes O / L for those rows; a second cluster barrier keeps every CTA's
// shared memory alive until all reads are done. A CTA without key tiles (or
// whose waits gave up) contributes m = -inf and zeros.
template <typename T, int G>
__device__ void combine_splits(unsigned char *smem, uint32_t sbase, uint32_t t_o, int r, bool have,
                               float m, float l, int splits, int n_pos, T *out, int64_t row_stride,
                               float v_mul) {
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  float *stg = reinterpret_cast<float *>(smem + kOffQ) + r * kCPitch;
#pragma unroll 1
  for (int cc = 0; cc < kD; cc += 32) {
    uint32_t o[32];
    tmem_ld32(t_o + cc, o);  // warp-collective
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 8; ++i)
      *reinterpret_cast<float4 *>(stg + cc + 4 * i) =
          have ? make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                             __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]))
               : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  reinterpret_cast<float2 *>(smem + kOffRed)[r] = have ? make_float2(m, l) : make_float2(-INFINITY, 0.f);
  cluster_sync_all();
  // Rows of real query positions only, dealt to the cluster's CTAs in equal
  // runs and to the four warps row by row; lane i owns dims 4i .. 4i + 3, so
  // a warp reads each split's row as one contiguous 512-byte line.
  const uint32_t me = cluster_rank();
  const int rows = n_pos * G < kM ? n_pos * G : kM;
  const int r0 = (int)(me * rows / splits), r1 = (int)((me + 1) * rows / splits);
  const int lane = r & 31;
  for (int row = r0 + (r >> 5); row < r1; row += 4) {  // warp-uniform
    // lane s < splits holds split s's (m, l); max and weighted sum over lanes 0..7
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < splits) ml = ld_cluster_f2(cluster_map(sbase + kOffRed + row * 8, (uint32_t)lane));
    float M = ml.x;
#pragma unroll
    for (int x = kMaxSplits / 2; x > 0; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
    const float ws = (M == -INFINITY || ml.x == -INFINITY) ? 0.f : exp2f(ml.x - M);
    float L = ml.y * ws;
#pragma unroll
    for (int x = kMaxSplits / 2; x > 0; x >>= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
    L = __shfl_sync(0xffffffffu, L, 0);
    const uint32_t src = sbase + kOffQ + (uint32_t)(row * kCPitch + 4 * lane) * 4;
    float4 v[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      v[s] = s < splits ? ld_cluster_f4(cluster_map(src, (uint32_t)s)) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) {
      const float w = __shfl_sync(0xffffffffu, ws, s);
      acc.x = fmaf(v[s].x, w, acc.x);
      acc.y = fmaf(v[s].y, w, acc.y);
      acc.z = fmaf(v[s].z, w, acc.z);
      acc.w = fmaf(v[s].w, w, acc.w);
    }
    const float inv = L > 0.f ? v_mul / L : 0.f;
    T *orow = out + (int64_t)(row / G) * row_stride + (int64_t)(row % G) * kD;
    *reinterpret_cast<uint2 *>(orow + 4 * lane) =
        make_uint2(pack2f<T>(acc.x * inv, acc.y * inv), pack2f<T>(acc.z * inv, acc.w * inv));
  }
  cluster_sync_all();
}

// kSplit: launched as clusters of `splits` CTAs per item (else splits == 1
// and the split code compiles away). kF8: fp8 E4M3 pages with per-tensor
// scales; the loader warps convert each page to f16 on its way into shared
// memory (registers instead of cp.async), the MMAs run in f16 (P too), a
// bf16 Q is converted to f16 in place, k_scale joins the score scale and
// v_scale the output scale.
template <typename T, int G, bool kSplit, bool kF8>
__global__ void __launch_bounds__(kThreadsFor(kSplit), 2)
    prefill_umma_kernel(const PrefillArgs p, const int tiles, const int splits_arg,
                        const __grid_constant__ CUtensorMap q_map) {
  using TM = typename std::conditional<kF8, __half, T>::type;  // MMA operand type
  constexpr bool kQConv = kF8 && std::is_same<T, __nv_bfloat16>::value;
  const int splits = kSplit ? splits_arg : 1;
  constexpr int kPos = kM / G;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t sbase = (raw + kSmemAlign - 1) & ~(uint32_t)(kSmemAlign - 1);
  unsigned char *smem = smem_raw + (sbase - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ---- work item: blockIdx.x / splits = (r * num_seqs + b) * Hkv + kv head,
  // tile = tiles - 1 - r. The hardware hands out CTAs in index order, so
  // every sequence's last position tile (the one with the most keys) goes
  // first and the kv heads of one (sequence, tile) run side by side. With
  // splits > 1 the item's `splits` CTAs form a cluster, each takes an equal
  // share of its key tiles, and their partial results are combined through
  // distributed shared memory.
  const int citem = (int)(blockIdx.x / (unsigned)splits);
  const int kvh = (int)(citem % p.num_kv_heads);
  const int item = citem / p.num_kv_heads;
  const int b = item % p.num_seqs, tile = tiles - 1 - item / p.num_seqs;
  if (warp == kLoadWarp && lane == 0) prefetch_tensormap(&q_map);

  const int cols = p.max_num_blocks_per_seq;
  // The load warps fetch the sequence's first block ids (pages lane + 32 i)
  // together with its lengths, before they know how many they need.
  const uint32_t *table = p.block_tables + (int64_t)b * cols;
  uint32_t ids[kIdRegs];
#pragma unroll
  for (int i = 0; i < kIdRegs; ++i) ids[i] = 0u;
  if (warp == kLoadWarp || warp == kVLoadWarp) {
#pragma unroll
    for (int i = 0; i < kIdRegs; ++i)
      if (lane + 32 * i < cols) ids[i] = __ldg(table + lane + 32 * i);
  }
  // the lengths are read together (independent loads, one round trip)
  const int64_t q0 = p.cu_seqlens_q[b];
  const int64_t q1 = p.cu_seqlens_q[b + 1];
  int ctx = (int)p.context_lens[b];
  const int qlen = (int)(q1 - q0);
  if (tile == tiles - 1 && qlen > tiles * kPos && tid == 0)
    raise_device_error(VASR_PA_DERR_QLEN_RANGE);
  if (tile * kPos >= qlen) return;
  if (ctx > cols * kBS) {
    if (tid == 0) raise_device_error(VASR_PA_DERR_CTX_RANGE);
    ctx = cols * kBS;
  }
  const int i0 = tile * kPos;
  const int n_pos = min(kPos, qlen - i0);
  const int base_pos = ctx - qlen + i0;
  const int kv_end = min(ctx, base_pos + n_pos);
  T *out = reinterpret_cast<T *>(p.out);
  const int64_t row_stride = (int64_t)p.num_heads * kD;
  if (kv_end <= 0) {
    for (int e = tid; e < n_pos * G * kD; e += kThreadsFor(kSplit)) {
      const int r = e / kD, d = e % kD;
      out[(q0 + i0 + r / G) * row_stride + (int64_t)(kvh * G + r % G) * kD + d] =
          Elem<T>::from_f32(0.f);
    }
    return;
  }
  const int n_pages = (kv_end + kBS - 1) / kBS;
  const int n_kt = (kv_end + kNT - 1) / kNT;
  // this CTA's key tiles jb .. jb + n_loc - 1 (all of them without splits)
  const int split = (int)(blockIdx.x % (unsigned)splits);
  const int jb = (int)((int64_t)split * n_kt / splits);
  const int n_loc = (int)((int64_t)(split + 1) * n_kt / splits) - jb;
  // leaving: every warp passes the CTA's last barrier, then (with splits)
  // the two cluster barriers around the combine
  auto cluster_tail = [&]() {
    if constexpr (kSplit) {
      cluster_sync_all();
      cluster_sync_all();
    }
  };
  const uint32_t bar = sbase + kOffBar;
  auto B = [&](int i) { return bar + 8u * (uint32_t)i; };

  // page id of tile j for this lane (page lane & 3 of the tile; lanes past
  // the context get any valid page: its keys are masked). Lane l keeps the
  // block ids of pages l, l + 32, l + 64, l + 96 in registers.
  auto tile_page = [&](int j, int &np) -> uint32_t {
    const int pg0 = j * kPagesPerTile;
    np = min(kPagesPerTile, n_pages - pg0);
    const int grp = pg0 >> 5;  // warp-uniform: a tile's pages share one group of 32
    uint32_t v = ids[0];
#pragma unroll
    for (int i = 1; i < kIdRegs; ++i) v = grp == i ? ids[i] : v;
    uint32_t id = __shfl_sync(0xffffffffu, v, (pg0 & 31) + (lane & (kPagesPerTile - 1)));
    if (grp >= kIdRegs && lane < np) id = __ldg(table + pg0 + lane);
    if (lane < np && (int64_t)id >= p.num_blocks) {
      raise_device_error(VASR_PA_DERR_BLOCK_RANGE);
      id = 0;
    }
    const uint32_t id0 = __shfl_sync(0xffffffffu, id, 0);
    return (lane & (kPagesPerTile - 1)) < np ? id : id0;
  };

  if (warp == kLoadWarp) {
    // ------------------------------------------------------- Q and K loads
    // K tile j -> K stage j & 1 by 16-byte asynchronous copies (no TMA: a
    // page's key rows are 16 bytes wide, so a K tile would cost 16 TMA
    // gathers, and the SM's TMA unit is shared with the V loads of both
    // resident CTAs). K j + 2 waits for Q K^T j.
    if (lane == 0) {
      for (int i = 0; i < kNumBars; ++i) mbar_init(B(i), bar_count(i));
      mbar_fence_init();
      mbar_arrive_expect_tx(B(kBarQ), (uint32_t)kQBytes);
      tma_load_3d(sbase + kOffQ, &q_map, 0, kvh * G, (int)(q0 + i0), B(kBarQ));
      tma_load_3d(sbase + kOffQ + kQBytes / 2, &q_map, kD / 2, kvh * G, (int)(q0 + i0), B(kBarQ));
    }
    __syncwarp();
    auto load_k = [&](int j) {
      // 1024 16-byte pieces (dim chunk c, key k) of the tile, 32 per lane:
      // instruction i moves chunk i / 2 of keys (i & 1) * 32 + lane, i.e. 16
      // bytes at c * 256 + token * 16 of page (i & 1) * 2 + lane / 16
      int np;
      const uint32_t id = tile_page(jb + j, np);
      const int pga = lane >> 4, pgb = pga + 2, tok = lane & (kBS - 1);
      const uint32_t ida = __shfl_sync(0xffffffffu, id, pga), idb = __shfl_sync(0xffffffffu, id, pgb);
      const unsigned char *kc = static_cast<const unsigned char *>(p.key_cache);
      if constexpr (kF8) {
        // fp8 pages ([16-dim chunk][token][16 bytes]): 512 pieces per tile, 16
        // per lane; piece (h, c) = 16-dim chunk c of key h * 32 + lane becomes
        // the f16 chunks 2 c and 2 c + 1 of that key. All loads go out first.
        const uint4 *src_a =
            reinterpret_cast<const uint4 *>(kc + ((int64_t)ida * p.num_kv_heads + kvh) * kPageBytesF8) + tok;
        const uint4 *src_b =
            reinterpret_cast<const uint4 *>(kc + ((int64_t)idb * p.num_kv_heads + kvh) * kPageBytesF8) + tok;
        uint4 v[2][kD / 16];
#pragma unroll
        for (int c = 0; c < kD / 16; ++c) {
          v[0][c] = pga < np ? __ldg(src_a + c * kBS) : make_uint4(0u, 0u, 0u, 0u);
          v[1][c] = pgb < np ? __ldg(src_b + c * kBS) : make_uint4(0u, 0u, 0u, 0u);
        }
        unsigned char *dst = smem + kOffK + (j & 1) * kKVTile + lane * 16;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < kD / 16; ++c) {
            uint4 lo, hi;
            e4m3x16_f16(v[h][c], lo, hi);
            *reinterpret_cast<uint4 *>(dst + (2 * c) * (kNT * 16) + h * 32 * 16) = lo;
            *reinterpret_cast<uint4 *>(dst + (2 * c + 1) * (kNT * 16) + h * 32 * 16) = hi;
          }
        fence_proxy_async_smem();  // generic stores, read by the MMA through the async proxy
        mbar_arrive(B(kBarFullK + (j & 1)));  // one of 32 arrivals
      } else {
        const unsigned char *src_a = kc + ((int64_t)ida * p.num_kv_heads + kvh) * kPageBytes + tok * 16;
        const unsigned char *src_b = kc + ((int64_t)idb * p.num_kv_heads + kvh) * kPageBytes + tok * 16;
        const uint32_t dst = sbase + kOffK + (j & 1) * kKVTile + lane * 16;
#pragma unroll
        for (int c = 0; c < kD / 8; ++c) {
          if (pga < np) cp_async16(dst + c * (kNT * 16), src_a + c * (kBS * 16));
          if (pgb < np) cp_async16(dst + c * (kNT * 16) + 32 * 16, src_b + c * (kBS * 16));
        }
        cp_async_arrive_noinc(B(kBarFullK + (j & 1)));  // one of 32 arrivals, when this lane's copies land
      }
    };
    // (fp8 conversions wait for their loads: after the CTA-wide sync, so
    // that the other warps do not wait for them)
    if constexpr (kF8) __syncthreads();
    if (n_loc > 0) load_k(0);
    if (n_loc > 1) load_k(1);
    int k_issued = min(n_loc, 2);
    if constexpr (!kF8) __syncthreads();
    // Q K^T j completes in order; K j + 2 goes into its stage once it has.
    // Once a wait gives up, nothing more is issued: a stage whose reader has
    // not finished must not receive another copy.
    bool dead = false;
    for (int j = 2; j < n_loc && !dead; ++j) {
      wait_phase(B(kBarEmptyK + (j & 1)), ((j >> 1) - 1) & 1, dead);
      if (dead) break;
      load_k(j);
      k_issued = j + 1;
    }
    // copies still in flight must land before the CTA's shared memory goes
    // away: the last phase issued on each stage (in a healthy run every one
    // of them was already waited for); waited for once more, bounded
    dead = false;
    for (int j = max(0, k_issued - kStages); j < k_issued; ++j)
      wait_phase(B(kBarFullK + (j & 1)), (j >> 1) & 1, dead);
    __syncthreads();
    cluster_tail();
    return;
  }
  if (warp == kVLoadWarp) {
    // -------------------------------------------------------------- V loads
    // V tile j -> V stage j & 1 by 16-byte cp.async copies into the 32-byte
    // swizzled layout of each page (a TMA load of it runs in 32-byte pieces
    // and took ~1.4 us per tile); V j + 2 waits for P V j. The barriers are
    // initialised by the K loader before the CTA-wide sync.
    auto load_v = [&](int j) {
      // 1024 16-byte pieces of the tile, 32 per lane: instruction i moves
      // half h of dim row d of page i / 8, (d, h) = ((i % 8) * 32 + lane) /
      // 2, % 2, to its place in the 32-byte-swizzled page image
      int np;
      const uint32_t id = tile_page(jb + j, np);
      const unsigned char *vc = static_cast<const unsigned char *>(p.value_cache);
      if constexpr (kF8) {
        // fp8 pages ([dim][16 tokens]): 512 16-byte rows per tile, 16 per
        // lane; row (pg, q) = dim q * 32 + lane of page pg becomes the two
        // 16-byte halves of its 32-byte f16 row in the swizzled image
        uint4 v[kPagesPerTile][kD / 32];
#pragma unroll
        for (int pg = 0; pg < kPagesPerTile; ++pg) {
          const uint32_t idp = __shfl_sync(0xffffffffu, id, pg);
          const uint4 *src =
              reinterpret_cast<const uint4 *>(vc + ((int64_t)idp * p.num_kv_heads + kvh) * kPageBytesF8) + lane;
#pragma unroll
          for (int q = 0; q < kD / 32; ++q)
            v[pg][q] = pg < np ? __ldg(src + q * 32) : make_uint4(0u, 0u, 0u, 0u);
        }
        unsigned char *dst = smem + kOffV + (j & 1) * kKVTile;
#pragma unroll
        for (int pg = 0; pg < kPagesPerTile; ++pg)
#pragma unroll
          for (int q = 0; q < kD / 32; ++q) {
            const int d = q * 32 + lane, sw = (d >> 2) & 1;
            uint4 lo, hi;
            e4m3x16_f16(v[pg][q], lo, hi);
            *reinterpret_cast<uint4 *>(dst + pg * kPageBytes + d * 32 + (sw << 4)) = lo;
            *reinterpret_cast<uint4 *>(dst + pg * kPageBytes + d * 32 + ((sw ^ 1) << 4)) = hi;
          }
        fence_proxy_async_smem();
        mbar_arrive(B(kBarFullV + (j & 1)));  // one of 32 arrivals
        return;
      }
      const uint32_t dst = sbase + kOffV + (j & 1) * kKVTile;
#pragma unroll
      for (int pg = 0; pg < kPagesPerTile; ++pg) {
        const uint32_t idp = __shfl_sync(0xffffffffu, id, pg);
        if (pg >= np) continue;
        const unsigned char *src = vc + ((int64_t)idp * p.num_kv_heads + kvh) * kPageBytes;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = i * 32 + lane, d = r >> 1, h = r & 1;
          cp_async16(dst + pg * kPageBytes + d * 32 + ((h ^ ((d >> 2) & 1)) << 4), src + r * 16);
        }
      }
      cp_async_arrive_noinc(B(kBarFullV + (j & 1)));  // one of 32 arrivals
    };
    __syncthreads();
    if (n_loc > 0) load_v(0);
    if (n_loc > 1) load_v(1);
    int v_issued = min(n_loc, 2);
    bool dead = false;
    for (int j = 2; j < n_loc && !dead; ++j) {
      wait_phase(B(kBarEmptyV + (j & 1)), ((j >> 1) - 1) & 1, dead);
      if (dead) break;
      load_v(j);
      v_issued = j + 1;
    }
    dead = false;
    for (int j = max(0, v_issued - kStages); j < v_issued; ++j)
      wait_phase(B(kBarFullV + (j & 1)), (j >> 1) & 1, dead);
    __syncthreads();
    cluster_tail();
    return;
  }

  // ------------------------------------------------------ warps 0-4 and 7
  if (warp == 0) tmem_alloc(sbase + kOffTmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<const uint32_t *>(smem + kOffTmemSlot);
  bool dead = false;  // this warp gave up on a wait

  if (warp == kMmaWarp || warp == kSMmaWarp) {
    // ------------------------------------------------------- MMA issuers
    // Two issuing warps, so that neither kind of MMA waits behind the other's
    // issue (an MMA's issue stalls while the tensor core is busy): warp 7
    // issues Q K^T j into S buffer j & 1 once P V j - 2, the last reader of
    // that buffer (P j - 2 lives there), has completed; warp 4 issues P V j
    // once P j is stored. Each warp's commits track only its own MMAs. The
    // split variant (CTAs of one or two key tiles) issues both from warp 4,
    // which measured faster there.
    const uint32_t idesc_s = idesc_f16<TM>(kNT), idesc_o = idesc_f16<TM>(kD);
    // Descriptors are built once; a later operand differs only in its start
    // address, the low field of the descriptor (address / 16 < 2^14 for any
    // shared-memory address), so it is the base descriptor plus offset / 16.
    const uint64_t qd0 = sdesc(sbase + kOffQ, 16, 1024, 2);
    const uint64_t kd0 = sdesc(sbase + kOffK, kNT * 16, 128, 0);
    const uint64_t vd0 = sdesc(sbase + kOffV, 16, 256, 6);
    // last commit issued (barrier index, phase parity): once it arrives every
    // MMA this warp issued has completed
    int last_bar = -1;
    uint32_t last_par = 0;
    auto issue_s = [&](int j) {  // S(j & 1) = Q K_j^T
      wait_phase(B(kBarFullK + (j & 1)), (j >> 1) & 1, dead);
      if (dead) return;
      // the K copies are generic-proxy writes; the MMA reads through the
      // async proxy
      fence_proxy_async_smem();
      tc_fence_after();
      const uint64_t kd = kd0 + (uint64_t)(((j & 1) * kKVTile) >> 4);
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks)
        umma_f16(tmem + kTmemS + (j & 1) * kNT, qd0 + (uint64_t)(((ks >> 2) * (kQBytes / 2) + (ks & 3) * 32) >> 4),
                 kd + (uint64_t)((ks * 2 * (kNT * 16)) >> 4), idesc_s, ks > 0);
      umma_commit(B(kBarSFull + (j & 1)));  // = kBarEmptyK
      last_bar = kBarSFull + (j & 1);
      last_par = (j >> 1) & 1;
      __syncwarp();
    };
    auto issue_pv = [&](int j) {  // O += P_j V_j
      wait_phase(B(kBarFullV + (j & 1)), (j >> 1) & 1, dead);
      if (dead) return;
      fence_proxy_async_smem();  // the V copies are generic-proxy writes
      if (jb + j == n_kt - 1 && (kv_end % kBS) != 0) {
        // V of tokens >= kv_end in the last page holds other data (possibly
        // non-finite); zero it so that P = 0 there contributes exactly 0.
        const int pl = (kv_end - 1) / kBS - (jb + j) * kPagesPerTile;
        const int valid = kv_end - ((jb + j) * kPagesPerTile + pl) * kBS;
        zero_v_page_tail(smem + kOffV + (j & 1) * kKVTile + pl * kPageBytes, valid, lane);
        fence_proxy_async_smem();
        __syncwarp();
      }
      // P of tile j (a ring of two: the softmax warps may run one tile ahead)
      wait_phase(B(kBarPFull + (j & 1)), (j >> 1) & 1, dead);
      if (dead) return;
      tc_fence_after();
      const int np = min(kPagesPerTile, n_pages - (jb + j) * kPagesPerTile);
      const uint64_t vd = vd0 + (uint64_t)(((j & 1) * kKVTile) >> 4);
      for (int pg = 0; pg < np; ++pg)
        umma_f16_ts(tmem + kTmemO, tmem + kTmemS + (j & 1) * kNT + pg * (kBS / 2),
                    vd + (uint64_t)((pg * kPageBytes) >> 4), idesc_o, (j > 0 || pg > 0) ? 1u : 0u);
      umma_commit(B(kBarPvDone + (j & 1)));  // = kBarEmptyV
      last_bar = kBarPvDone + (j & 1);
      last_par = (j >> 1) & 1;
      __syncwarp();
    };
    // Q K^T j overwrites the S buffer that holds P j - 2: the tensor core does
    // not order a later MMA's D writes after an earlier MMA's TMEM A reads, so
    // P V j - 2 must have completed first.
    auto wait_pv_before_s = [&](int j) {
      wait_phase(B(kBarPvDone + (j & 1)), ((j - 2) >> 1) & 1, dead);
      if (!dead) tc_fence_after();
    };
    if constexpr (!kSplit) {  // two issuing warps
      if (warp == kSMmaWarp) {
        wait_phase(B(kQConv ? kBarQ16 : kBarQ), 0, dead);
        for (int j = 0; j < n_loc && !dead; ++j) {
          if (j >= 2) wait_pv_before_s(j);
          if (!dead) issue_s(j);
        }
      } else {
        for (int j = 0; j < n_loc && !dead; ++j) issue_pv(j);
      }
    } else if (warp == kMmaWarp) {  // split items (one or two key tiles per CTA): warp 4 issues both
      wait_phase(B(kQConv ? kBarQ16 : kBarQ), 0, dead);
      if (n_loc > 0 && !dead) issue_s(0);
      if (n_loc > 1 && !dead) issue_s(1);
      for (int j = 0; j < n_loc && !dead; ++j) {
        issue_pv(j);
        if (j + 2 < n_loc && !dead) {
          wait_pv_before_s(j + 2);
          if (!dead) issue_s(j + 2);
        }
      }
    }
    // In a healthy run the last P V commit (waited for by the epilogue)
    // covers every MMA (Q K^T j completed before the softmax read S j).
    // After a wait gave up, this warp issues nothing more and waits (bounded)
    // for its own last commit, so that no MMA still writes tensor memory when
    // it is freed.
    if (dead && last_bar >= 0) {
      bool d2 = false;
      wait_phase(B(last_bar), last_par, d2);
    }
    tc_fence_before();
    __syncthreads();
    cluster_tail();
    return;
  }

  // ------------------------------------------------- softmax, one row per thread
  const int r = tid;
  const bool row_ok = (r / G) < n_pos;
  const int lim = row_ok ? min(base_pos + r / G, kv_end - 1) : -1;  // last visible key
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const bool use_softcap = (p.softcapping != 1.0f) && (p.softcapping > 0.f);
  // fp8 pages hold K / k_scale: the scale of the scores takes k_scale
  const float qk_scale = kF8 ? p.scale * __ldg(p.k_scale) : p.scale;
  const float cx = use_softcap ? 1.f : qk_scale * kLog2e;
  if constexpr (kQConv) {
    // Q (bf16, landed by TMA) -> f16 in place, 256 bytes per thread; the
    // Q K^T issuer waits for all 128 threads
    wait_phase(B(kBarQ), 0, dead);
    if (!dead) {
      uint4 *qs = reinterpret_cast<uint4 *>(smem + kOffQ);
#pragma unroll 4
      for (int i = r; i < kQBytes / 16; i += 128) {
        const uint4 v = qs[i];
        qs[i] = make_uint4(bf16x2_f16x2(v.x), bf16x2_f16x2(v.y), bf16x2_f16x2(v.z), bf16x2_f16x2(v.w));
      }
      fence_proxy_async_smem();
    }
    mbar_arrive(B(kBarQ16));
  }
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j < n_loc; ++j) {
    wait_phase(B(kBarSFull + (j & 1)), (j >> 1) & 1, dead);
    tc_fence_after();
    uint32_t u[kNT];
    const uint32_t ts = tmem + lane_base + kTmemS + (j & 1) * kNT;
    tmem_ld32(ts, u);
    tmem_ld32(ts + 32, u + 32);
    tmem_wait_ld();
    const int kmax = lim - (jb + j) * kNT;  // elements k <= kmax are visible to this row
    // x holds raw scores (exponent x * c - m) or, with softcapping, log2-domain
    // capped logits (c = 1); m is kept in log2 units either way.
    float x[kNT];
#pragma unroll
    for (int k = 0; k < kNT; ++k) x[k] = __uint_as_float(u[k]);
    if (use_softcap) {
#pragma unroll
      for (int k = 0; k < kNT; ++k)
        x[k] = p.softcapping * tanhf(x[k] * qk_scale / p.softcapping) * kLog2e;
    }
    if (!__all_sync(0xffffffffu, kmax >= kNT - 1)) {  // diagonal / last tile: mask
#pragma unroll
      for (int k = 0; k < kNT; ++k) x[k] = (k <= kmax) ? x[k] : -INFINITY;
    }
    float m4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
    for (int k = 4; k < kNT; ++k) m4[k & 3] = fmaxf(m4[k & 3], x[k]);
    const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * cx;
    const float m_new = (mx > m + kRescaleLog2) ? mx : m;
    const float alpha = (m_new == m) ? 1.f : ex2_approx(m - m_new);
    const float off = (m_new == -INFINITY) ? 0.f : m_new;
    m = m_new;
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t pk[kNT / 2];
#pragma unroll
    for (int k = 0; k < kNT / 2; ++k) {
      const float p0 = ex2_approx(fmaf(x[2 * k], cx, -off));
      const float p1 = ex2_approx(fmaf(x[2 * k + 1], cx, -off));
      s4[k & 3] += p0 + p1;
      pk[k] = pack2f<TM>(p0, p1);
    }
    l = l * alpha + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
    if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
      // O moves to the new offset once P V of the previous tile is complete.
      // P V completion has one barrier per S buffer and this thread skips
      // the waits it does not need: the barrier of P V j - 1 is never two
      // phases away, since P V j - 3 completed before Q K^T j - 1 (whose S
      // this thread already read) and P V j + 1 needs this thread's P.
      wait_phase(B(kBarPvDone + ((j - 1) & 1)), ((j - 1) >> 1) & 1, dead);
      tc_fence_after();
      {
#pragma unroll 1
        for (int cc = 0; cc < kD; cc += 32) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kTmemO + cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tmem + lane_base + kTmemO + cc, o);
        }
        tmem_wait_st();
      }
    }
    // P (16-bit pairs) replaces the first 32 columns of its S buffer; P V of
    // the tile two back, which read them last, completed before this S did.
    // P V of the previous tile may still run: it reads the other buffer and
    // accumulates into O, which this store does not touch.
    tmem_st32(ts, pk);
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(B(kBarPFull + (j & 1)));
  }

  // ---- epilogue: O / l -> out (the last P V commit covers every MMA)
  if (n_loc > 0) wait_phase(B(kBarPvDone + ((n_loc - 1) & 1)), ((n_loc - 1) >> 1) & 1, dead);
  tc_fence_after();
  if constexpr (kSplit) {
    combine_splits<T, G>(smem, sbase, tmem + lane_base + kTmemO, r, n_loc > 0 && !dead, m, l, splits,
                         n_pos, out + (q0 + i0) * row_stride + (int64_t)kvh * G * kD, row_stride,
                         kF8 ? __ldg(p.v_scale) : 1.f);
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    return;
  }
  // fp8 pages hold V / v_scale
  const float inv = l > 0.f ? (kF8 ? __ldg(p.v_scale) : 1.f) / l : 0.f;
  // O / l (16-bit) is staged in the Q buffer, which no MMA reads any more:
  // row r at r * 256 bytes, its 16-byte chunk c at slot c ^ (r % 16), so a
  // warp's stores of one chunk of 32 rows and the later reads of one row
  // hit distinct banks. The rows then leave as whole token rows (the G
  // heads of a kv head are adjacent in out), 16 bytes per thread.
  unsigned char *stg = smem + kOffQ;
#pragma unroll 1
  for (int cc = 0; cc < kD; cc += 64) {
    uint32_t o[64];
    tmem_ld32(tmem + lane_base + kTmemO + cc, o);
    tmem_ld32(tmem + lane_base + kTmemO + cc + 32, o + 32);
    tmem_wait_ld();
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      w[i] = pack2f<T>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = cc / 8 + i;
      *reinterpret_cast<uint4 *>(stg + r * 256 + ((c ^ (r & 15)) << 4)) =
          make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");  // the four softmax warps
  const int chunks = n_pos * G * (kD * 2 / 16);
  for (int e = r; e < chunks; e += 128) {
    const int row = e >> 4, c = e & 15;  // row = position * G + head
    const uint4 v = *reinterpret_cast<const uint4 *>(stg + row * 256 + ((c ^ (row & 15)) << 4));
    *reinterpret_cast<uint4 *>(out + (q0 + i0 + row / G) * row_stride + (int64_t)(kvh * G + row % G) * kD +
                               c * 8) = v;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tensor_map_encoder() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Q viewed as [tokens][heads][128 elements]: a box of (64, G, 128 / G) at
// element offset 0 or 64 lands as 128 rows (row = position * G + head) of
// 128 bytes with the 128-byte swizzle, half of the CTA's Q in the canonical
// SW128 K-major layout. Rows past the last token read zeros.
bool make_q_map(CUtensorMap *map, const PrefillArgs &a, int g) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {kD, (cuuint64_t)a.num_heads, (cuuint64_t)a.total_q_tokens};
  const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)a.q_token_stride * 2};
  const cuuint32_t box[3] = {kD / 2, (cuuint32_t)g, (cuuint32_t)(kM / g)};
  const cuuint32_t estr[3] = {1, 1, 1};
  std::memset(map, 0, sizeof(*map));
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void *>(a.query), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int G, bool kF8>
int launch_g(const PrefillArgs &a, const CUtensorMap &qmap, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0}, attr_done_split{0};
  if (!ensure_smem_attr(prefill_umma_kernel<T, G, false, kF8>, kSmemBytes, attr_done) ||
      !ensure_smem_attr(prefill_umma_kernel<T, G, true, kF8>, kSmemBytes, attr_done_split))
    return VASR_PA_ELAUNCH;
  constexpr int kPos = kM / G;
  const int64_t tiles = prefill_tiles_per_seq(a, kPos);
  const int64_t items = tiles * a.num_seqs * a.num_kv_heads;
  if (tiles <= 0 || items * kMaxSplits > 0x7fffffff) return VASR_PA_EINVAL_SHAPE;
  // Few items (a long context with few new tokens: the last chunk rounds)
  // leave most SMs idle while each CTA walks its key tiles one by one: then
  // each item's tiles are shared by a cluster of CTAs, as many as fill about
  // one CTA per SM and leave at least one key tile each (bounded by the
  // block table's width), combined through distributed shared memory.
  static std::atomic<int64_t> sm_cache[64];
  int splits = 1;
  {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
      sms = (int)sm_cache[dev].load(std::memory_order_acquire);
      if (sms == 0 && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
        sm_cache[dev].store(sms, std::memory_order_release);
    }
    const int64_t kt_bound = ((int64_t)a.max_num_blocks_per_seq * kBS + kNT - 1) / kNT;
    if (sms > 0 && items * 2 <= sms) {
      int64_t sp = sms / items;
      if (sp > kMaxSplits) sp = kMaxSplits;
      if (sp > kt_bound) sp = kt_bound;
      splits = sp >= 2 ? (int)sp : 1;
    }
  }
  if (splits == 1) {
    prefill_umma_kernel<T, G, false, kF8><<<dim3((unsigned)items), kThreadsFor(false), kSmemBytes, s>>>(
        a, (int)tiles, 1, qmap);
    return cudaPeekAtLastError() == cudaSuccess ? VASR_PA_OK : VASR_PA_ELAUNCH;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(items * splits));
  cfg.blockDim = dim3(kThreadsFor(true));
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_umma_kernel<T, G, true, kF8>, a, (int)tiles, splits, qmap) == cudaSuccess
             ? VASR_PA_OK
             : VASR_PA_ELAUNCH;
}

template <int G>
int launch_dt(const PrefillArgs &a, const CUtensorMap &qmap, cudaStream_t s) {
  const bool bf = a.dtype == VASR_PA_BF16;
  if (a.cache_dtype == VASR_PA_FP8_E4M3)
    return bf ? launch_g<__nv_bfloat16, G, true>(a, qmap, s) : launch_g<__half, G, true>(a, qmap, s);
  return bf ? launch_g<__nv_bfloat16, G, false>(a, qmap, s) : launch_g<__half, G, false>(a, qmap, s);
}

}  // namespace

int launch_prefill_umma(const PrefillArgs &a, cudaStream_t s) {
  if (a.head_dim != kD || a.block_size != kBS) return VASR_PA_ENOT_SUPPORTED;
  if (a.dtype != VASR_PA_BF16 && a.dtype != VASR_PA_F16) return VASR_PA_ENOT_SUPPORTED;
  if (a.cache_dtype != -1 && a.cache_dtype != a.dtype &&
      (a.cache_dtype != VASR_PA_FP8_E4M3 || !a.k_scale || !a.v_scale))
    return VASR_PA_ENOT_SUPPORTED;
  const int g = a.num_heads / a.num_kv_heads;
  if (g != 1 && g != 2 && g != 4) return VASR_PA_ENOT_SUPPORTED;
  if (a.total_q_tokens >= (int64_t(1) << 31)) return VASR_PA_ENOT_SUPPORTED;
  // the Q tensor map and the 16-byte page copies want 16-byte aligned bases
  // and strides; other views take the mma.sync kernel
  if ((reinterpret_cast<uintptr_t>(a.query) | reinterpret_cast<uintptr_t>(a.key_cache) |
       reinterpret_cast<uintptr_t>(a.value_cache)) % 16 != 0 ||
      (a.q_token_stride * 2) % 16 != 0)
    return VASR_PA_ENOT_SUPPORTED;
  CUtensorMap qmap;
  if (!make_q_map(&qmap, a, g)) return VASR_PA_ELAUNCH;
  switch (g) {
    case 1: return launch_dt<1>(a, qmap, s);
    case 2: return launch_dt<2>(a, qmap, s);
    default: return launch_dt<4>(a, qmap, s);
  }
}

int read_error_prefill_umma(uint32_t *bits, bool clear, cudaStream_t s) {
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

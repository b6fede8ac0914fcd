// tcgen05 / TMEM helpers shared by the tensor-core trailing-update kernels
// (inline PTX for sm_100a): instruction and shared-memory matrix descriptors
// for kind::tf32 MMAs with K-major, no-swizzle operands, the MMA issue and its
// mbarrier commit, bounded mbarrier waits, the tcgen05 fences, a 32-column
// TMEM load, and the 3xTF32 operand split.
#pragma once

#include "qrb_common.cuh"

namespace qrb {
namespace tc {

constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 2 GHz
constexpr unsigned kFullMask = 0xffffffffu;

// Instruction descriptors (kind::tf32, FP32 accumulate, dense).
constexpr uint32_t idesc(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor, no swizzle (canonical interleaved core
// matrices of 8 x 16 bytes), sm_100 version field = 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Round to the nearest TF32 (10 explicit mantissa bits; ties away from zero
// on the magnitude), as a float with the 13 low mantissa bits cleared.
__device__ __forceinline__ float tf32_round(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ void split4(const float4& v, float4& hi, float4& lo) {
  hi.x = tf32_round(v.x); lo.x = tf32_round(v.x - hi.x);
  hi.y = tf32_round(v.y); lo.y = tf32_round(v.y - hi.y);
  hi.z = tf32_round(v.z); lo.z = tf32_round(v.z - hi.z);
  hi.w = tf32_round(v.w); lo.w = tf32_round(v.w - hi.w);
}

__device__ __forceinline__ float vmask(float x, int i, int a) {
  return i < a ? 0.f : (i == a ? 1.f : x);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Bounded wait on an mbarrier phase. Returns at once when *abort (a flag in
// shared memory) is set; on timeout records the device error and sets *abort,
// after which the block issues no further MMAs, reads no TMEM and writes no
// results, drains its issued MMAs (drain_mmas) and frees its TMEM.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t phase, int* err,
                                          volatile int* abort) {
  if (*abort != 0) return;
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) return;
    if (*abort != 0) return;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      atomicExch(err, 1);
      return;
    }
  }
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// After an abort: commit every tcgen05 operation this thread issued to a
// fresh mbarrier (count 1, never used before) and wait for it, bounded, so
// that no MMA still writes TMEM when it is freed.
__device__ __forceinline__ void drain_mmas(uint32_t fresh_bar) {
  mma_commit(fresh_bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(fresh_bar), "r"(0u)
        : "memory");
    if (done || clock64() - t0 > kWaitCycles) return;
  }
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]);
}


}  // namespace tc
}  // namespace qrb

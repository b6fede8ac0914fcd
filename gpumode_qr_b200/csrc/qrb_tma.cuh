// TMA (cp.async.bulk.tensor) and mbarrier helpers for sm_100a, plus the
// host-side tensor-map encoder. Inline PTX only; no multicast anywhere (every
// CTA loads its own tiles), so these helpers are safe in code that runs on
// several GPUs at once.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "qrb_common.cuh"

namespace qrb {
namespace tma {

// ---------------------------------------------------------------------------
// device side
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One plain arrival.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// One arrival that also announces `bytes` of incoming TMA transactions.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase of `bar` with the given parity to complete, for at most
// `limit` clock cycles. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  long long limit) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

// As mbar_wait_bounded, but also gives up at once when *abort (a flag in
// shared memory) is set, and sets it on a timeout, so that one timed-out role
// releases every other role of the block within a short time.
__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, long long limit,
                                                   volatile int* abort) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (*abort != 0) return false;
    if (clock64() - t0 > limit) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// Tiled loads of a box into shared memory, completing on an mbarrier.
__device__ __forceinline__ void load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                        int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                        int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// Element-wise FP32 add of a shared-memory box into global memory (the L2
// performs the read-modify-write); rows and columns outside the tensor are
// skipped. Tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void reduce_add_3d(const CUtensorMap* map, uint32_t src, int x, int y,
                                              int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group"
      " [%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until the issuing thread's bulk groups have finished reading shared
// memory (the source buffer may be rewritten), or have fully completed.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA stores, tensor-core operand reads).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link against libcuda); nullptr when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 encoder();

// A row-major FP32 tensor of `rank` dims (dims[0] innermost, element stride
// 1; strides[i] = byte stride of dims[i + 1]) seen through boxes of
// box[0] x box[1] x 1 x ... elements with a 128-byte swizzle (box[0] * 4 must
// be <= 128): 16-byte units permuted within each 128-byte row, or with atom32
// 32-byte units (the layout MN-major TF32 MMA operands need). Out-of-range
// elements of a load read as zero. Returns false if the driver rejects the
// description.
bool encode_f32_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides, uint32_t box0, uint32_t box1, bool atom32);

}  // namespace tma

// The tensor-core trailing update (qrb_larfb_tma.cu). Tensor maps over the
// whole batch of one qrb_geqrf_f32 call: H [batch][n][n] (C boxes for pass-1
// loads and pass-2 reduce-adds) and the panels' split reflectors,
// Vs [4][batch][n][kr] for blocks of kr = 32 or 64 (two panels) reflectors
// (plane 2 * buf + 0 = TF32 high part of V-buffer buf, + 1 = remainder).
struct LarfbMaps {
  CUtensorMap c1, c2, v1, v2;
  int kr = 32;
};
bool larfb_tma_supported(int n);
int make_larfb_maps(LarfbMaps* maps, const float* H, const float* Vs, int64_t batch, int n,
                    int kr);
// C <- C - V T^T V^T C for the columns [col0, col_end) of rows [j0, n) of
// matrices m0 .. m0 + count - 1 of the maps (T: kr x kr per matrix, stride
// sTb, pointing at matrix m0's factor), with the reflectors of V-buffer vbuf
// (0 or 1). col_end is n or col0 + a multiple of 32.
int launch_larfb_tma(const LarfbMaps& maps, const float* T, int64_t sTb, int64_t m0,
                     int64_t count, int j0, int col0, int col_end, int n, int vbuf,
                     cudaStream_t stream);

}  // namespace qrb

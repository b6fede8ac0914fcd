// Block-reflector trailing update C <- C - V (T^T (V^T C)) on the tcgen05
// tensor cores in 3xTF32, fed by TMA: the three batched GEMMs of the
// reference's trailing update (src/qrbench/variants.py:800-804) as one
// persistent kernel over (matrix, 128-column tile of C) work items.
//
// Operands (all row-major in HBM, read through swizzled TMA boxes):
//   C   the trailing block of H itself (rows j0.., the tile's columns);
//   V   the panel's unit-lower reflectors, already split by the panel kernel
//       into a TF32 high part and a TF32 remainder (Vs[hi|lo][matrix][row][KR]);
//   T   the panels' KR x KR compact-WY factor (KR = 32, or 64 for two-level
//       blocking).
// Each FP32 product a*b is formed as a_hi b_hi + a_hi b_lo + a_lo b_hi with
// FP32 accumulation in TMEM (the lo*lo term, ~2^-22 relative, is dropped);
// plain TF32 would not meet the FP32 accuracy gates.
//
// Per tile:
//   pass 1  W^T = C^T V over all rows: D1 in TMEM (128 lanes = tile columns x
//           KR columns = reflectors), as 256 / KR interleaved partial sums.
//           Both operands are MN-major (row-major C and V, contraction over
//           rows), which kind::tf32 takes straight from TMA boxes in the
//           32-byte-atom 128-byte swizzle. A ring of 32-row chunks; the worker
//           warps split each C chunk into hi (in place) and lo (a second
//           buffer) while earlier chunks' MMAs run.
//   T^T     W' = T^T W on the CUDA cores (each worker thread one column, read
//           from TMEM), split into hi / lo and stored as the K-major B operand
//           of pass 2.
//   pass 2  D2 = V W' per 128-row chunk (K-major V boxes from TMA); the
//           epilogue writes -D2 into a swizzled staging tile and a TMA
//           reduce-add adds it to C in place (the L2 does the
//           read-modify-write).
// Warp roles: warp 0 = TMA producer (one lane), warp 1 = MMA issuer (one
// lane; the warp owns the TMEM allocation), the rest = workers. The roles
// hand chunks to each other through mbarriers, so loads run ahead of the MMAs
// and the MMAs overlap the workers' splitting and epilogues.
// Three forms, chosen per launch, with the same FP32 operations in the same
// order (the same bits):
//   one CTA per SM    8 workers, 4 pass-1 stages, two pass-2 accumulators;
//   row-split pairs   (CS = 2; trailing blocks of 1024+ rows, 2 x tiles <=
//                     SMs) the rows in two halves, one per CTA of a 2-CTA
//                     cluster, the partial W swapped through distributed
//                     shared memory; a single CTA computes the same two half
//                     sums when the launch has more tiles;
//   two CTAs per SM   (DUAL; 32 reflectors, more tiles than SMs) 4 workers,
//                     2 pass-1 stages, one pass-2 accumulator, the epilogue in
//                     two column halves, so that one CTA's pass 1 runs beside
//                     the other's pass 2.
// Every wait is bounded: a timeout sets a block-wide abort flag and the device
// error flag; every role then skips its remaining work (its waits return at
// once), the block waits (bounded) for what it already issued, frees its TMEM
// and returns (a pair meets at a closing cluster barrier first). The test hook
// "test_skip_mma" withholds the pass-1 MMAs so that this path runs.
#include <mutex>

#include "qrb_tc.cuh"
#include "qrb_tma.cuh"

namespace qrb {

namespace tma {

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && p != nullptr)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      (void)cudaGetLastError();
  });
  return fn;
}

bool encode_f32_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides, uint32_t box0, uint32_t box1, bool atom32) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encoder();
  if (fn == nullptr || rank < 2 || rank > 5 || box0 * 4 > 128) return false;
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = i == 0 ? box0 : (i == 1 ? box1 : 1u);
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gs[i] = strides[i];
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base), gd,
            gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tma

namespace {

constexpr int TCOLS = 128;    // columns of C per tile
constexpr int R1 = 32;        // rows per pass-1 chunk
constexpr int S1MAX = 4;      // pass-1 ring stages (mbarrier slots)
constexpr int R2 = 128;       // rows per pass-2 chunk (MMA M)
constexpr uint32_t BOX1 = R1 * 128;   // one {32 x R1} FP32 box, 4 KiB
constexpr uint32_t CST = 4 * BOX1;    // C part of a pass-1 stage: 4 boxes = 128 columns
constexpr uint32_t BOX2 = R2 * 128;   // one {32 x 128} box, 16 KiB
// mbarriers
constexpr int B_FULL1 = 0, B_SPLIT1 = B_FULL1 + S1MAX, B_EMPTY1 = B_SPLIT1 + S1MAX,
              B_D1FULL = B_EMPTY1 + S1MAX, B_B2READY = B_D1FULL + 1, B_V2FULL = B_B2READY + 1,
              B_V2EMPTY = B_V2FULL + 2, B_ACCFULL = B_V2EMPTY + 2, B_ACCEMPTY = B_ACCFULL + 2,
              B_TILEDONE = B_ACCEMPTY + 2, B_FIN = B_TILEDONE + 1, B_XFULL = B_FIN + 1,
              B_XREAD = B_XFULL + 1, NBAR = B_XREAD + 1;

// Layout for a block of KR reflectors (32, or 64 for two-level blocking).
//   Shared memory (bytes from a 1024-aligned base): a pass-1 stage holds the
//   C chunk (hi after the split), the V hi and lo boxes (KR / 32 boxes each)
//   and the C lo buffer. Pass 2 reuses the pass-1 region once every pass-1
//   MMA of the tile is done: NV2 stages of V (hi and lo), NSTG staging boxes
//   for -V W', and W' hi / lo as the K-major B operand.
//   TMEM: pass 1 accumulates into NP1 = 256 / KR partial accumulators of KR
//   columns (chunk ch into partial ch % NP1), summed in FP32 afterwards: the
//   tensor core's accumulation inside an MMA is not rounded to nearest at
//   every add, so one accumulator over thousands of rows drifts ~5x further
//   from FP64 than FFMA; short chains keep it at FFMA's level. Pass 2
//   accumulates into NACC accumulators of 128 columns from column TM_D2. The
//   two may share columns: every partial is read (the W' step) before the
//   first pass-2 MMA of the tile, and the next tile's first pass-1 MMA waits
//   for the tile's last epilogue (through the staging tile and the producer).
// DUAL (32 reflectors only): two CTAs per SM, so that one CTA's pass 1 (bound
//   by issuing MMAs) runs beside the other's pass 2 (bound by the TMA
//   reduce-adds reading the staging tile): 4 worker warps, 2 pass-1 stages, one
//   pass-2 V stage and accumulator, 2 staging boxes (the epilogue in two
//   column halves), 256 TMEM columns. The FP32 operations are those of the
//   one-CTA-per-SM layout, in the same order: the same bits.
template <int KR, bool DUAL = false>
struct Lay {
  static constexpr int NWORK = DUAL ? 4 : 8;               // worker warps
  static constexpr int NTH = 32 * (2 + NWORK);
  static constexpr int S1 = DUAL ? 2 : 4;                  // pass-1 ring stages
  static constexpr int NA = KR / 32;                       // 32-wide atoms of V / of K
  static constexpr uint32_t VB1 = NA * BOX1;
  static constexpr uint32_t ST1 = CST + 2 * VB1 + CST;
  static constexpr uint32_t S1_VH = CST, S1_VL = CST + VB1, S1_CL = CST + 2 * VB1;
  static constexpr int NV2 = DUAL ? 1 : (KR == 32 ? 2 : 1);
  static constexpr uint32_t V2ST = 2 * NA * BOX2;
  static constexpr uint32_t OFF_STG = NV2 * V2ST;
  static constexpr int NSTG = DUAL ? 2 : 4;                // staging boxes of 32 columns
  static constexpr uint32_t B2B = NA * TCOLS * 128;
  static constexpr uint32_t OFF_BH = OFF_STG + NSTG * BOX2;
  static constexpr uint32_t OFF_BL = OFF_BH + B2B;
  static constexpr uint32_t P1END = S1 * ST1, P2END = OFF_BL + B2B;
  static constexpr uint32_t REGION = P1END > P2END ? P1END : P2END;
  static constexpr uint32_t OFF_T = REGION;
  static constexpr int T_LD = KR + 1;
  static constexpr uint32_t OFF_BAR = OFF_T + ((KR * T_LD * 4 + 127) / 128) * 128;
  static constexpr uint32_t OFF_TMEMV = OFF_BAR + NBAR * 8;
  static constexpr uint32_t OFF_ABORT = OFF_TMEMV + 4;
  static constexpr size_t SMEM_BYTES = OFF_ABORT + 12 + 1024;  // slack for aligning the base
  static constexpr int NP1 = 256 / KR;
  static constexpr int NACC = DUAL ? 1 : 2;
  static constexpr uint32_t TM_COLS = DUAL ? 256 : 512;
  static constexpr uint32_t TM_D2 = TM_COLS - 128 * NACC;
  static constexpr uint32_t IDESC1 = tc::idesc(TCOLS, KR, /*a_mn=*/true, /*b_mn=*/true);
  // row-split tiles: this CTA's partial W (TCOLS x KR) sits in the staging
  // boxes between the end of pass 1 and the first pass-2 epilogue
  static constexpr uint32_t OFF_X = OFF_STG;
  static_assert(!DUAL || KR == 32, "two CTAs per SM for 32 reflectors only");
  static_assert(S1 <= S1MAX, "pass-1 stages");
  // one CTA with two row halves keeps 2 x NP1 partials (never with DUAL)
  static_assert((DUAL ? 1 : 2) * NP1 * KR <= (int)TM_COLS, "pass-1 partials in TMEM");
  static_assert(TCOLS * KR * 4 <= NSTG * BOX2, "partial W must fit the staging boxes");
  static_assert(SMEM_BYTES <= (DUAL ? 113 * 1024 : 227 * 1024), "shared memory budget");
};
constexpr uint32_t IDESC2 = tc::idesc(R2, TCOLS, /*a_mn=*/false, /*b_mn=*/false);

// Shared-memory matrix descriptors (sm_100 version field 1) for the two
// swizzled layouts used here, both with 128-byte rows:
//  - K-major, 128-byte swizzle (layout type 2: 16-byte units of a row XORed
//    with the row index mod 8, 8-row atoms of 1024 bytes): sbo = distance
//    between 8-row M/N groups, lbo unused;
//  - MN-major 32-bit operands, 128-byte swizzle with 32-byte atoms (layout
//    type 1: 32-byte units XORed with the row index mod 4, 4-row atoms of 512
//    bytes; the only MN-major layout kind::tf32 accepts, written by TMA's
//    128B_ATOM_32B swizzle): lbo = distance between 32-element MN blocks,
//    sbo = between 4-row K groups.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                          uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t kLayoutSw128 = 2, kLayoutSw128Atom32 = 1;
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr) {
  return sdesc(saddr, 16, 1024, kLayoutSw128);
}
__device__ __forceinline__ uint64_t sdesc_mn32(uint32_t saddr, uint32_t lbo) {
  return sdesc(saddr, lbo, 512, kLayoutSw128Atom32);
}

// 32 consecutive TMEM columns of this warp's lane quarter (no wait).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float* v) {
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
#pragma unroll
  for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]);
}
// 16 consecutive TMEM columns of this warp's lane quarter (no wait).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int q = 0; q < 16; ++q) v[q] = __uint_as_float(r[q]);
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte unit u of row `row` in a 128-byte-swizzled region
// (rows of 128 bytes, 8-row atoms of 1024 bytes at a 1024-aligned base).
__device__ __forceinline__ uint32_t sw128(int row, int u) {
  return (uint32_t)(row * 128 + ((u ^ (row & 7)) << 4));
}

// Barrier among the worker warps only (named barrier 1), with an OR of a
// per-thread flag: every worker gets the same answer.
template <int NW>
__device__ __forceinline__ bool workers_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * NW)
      : "memory");
  return r != 0;
}

// ---- the two CTAs of a row-split cluster ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared-memory address of the same byte in cluster rank q.
__device__ __forceinline__ uint32_t peer_addr(uint32_t a, uint32_t q) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(q));
  return r;
}
__device__ __forceinline__ float4 ld_peer4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
// Arrive on an mbarrier of a peer CTA, releasing this thread's earlier
// shared-memory accesses at cluster scope.
__device__ __forceinline__ void mbar_arrive_peer(uint32_t peer_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(peer_bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded wait (acquire at cluster scope) for a phase the peer CTA completes;
// as tma::mbar_wait_or_abort for the abort flag.
__device__ __forceinline__ bool mbar_wait_cluster_or_abort(uint32_t bar, uint32_t parity,
                                                           long long limit,
                                                           volatile int* abort) {
  if (mbar_try_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_cluster(bar, parity)) {
    if (*abort != 0) return false;
    if (clock64() - t0 > limit) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// vw_hi / vw_lo: plane coordinates of the V hi / lo boxes in the V map.
// CS = 1: one CTA per tile. CS = 2: a cluster of two CTAs per tile, rank q
// taking rows [q * rsplit, (q + 1) * rsplit) of the trailing block (rsplit a
// multiple of 128): each forms the partial W^T of its rows, the two swap
// partials through distributed shared memory and add them (the same sum on
// both: a + b = b + a in FP32), and each applies the update to its own rows.
template <int KR, int CS, bool DUAL>
__global__ void __launch_bounds__(Lay<KR, DUAL>::NTH, DUAL ? 2 : 1)
k_larfb_tma(const __grid_constant__ CUtensorMap mC1, const __grid_constant__ CUtensorMap mC2,
            const __grid_constant__ CUtensorMap mV1, const __grid_constant__ CUtensorMap mV2,
            const float* __restrict__ T, int64_t sTb, int m0, int ntiles, int ntc, int j0,
            int col0, int col_end, int n, int vw_hi, int vw_lo, int rsplit,
            int* __restrict__ err, long long wait_limit, int skip_mma) {
  using L = Lay<KR, DUAL>;
  constexpr int NA = L::NA, NV2 = L::NV2, NP1 = L::NP1, S1 = L::S1, NWORK = L::NWORK;
  static_assert(!(DUAL && CS > 1), "row-split pairs use the one-CTA-per-SM layout");
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = tma::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  float* Ts = reinterpret_cast<float*>(sm + L::OFF_T);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L::OFF_TMEMV);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + L::OFF_ABORT);
  const uint32_t bar0 = base + L::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * (uint32_t)i; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // this CTA's rows of the trailing block: [y0, y0 + rq)
  const uint32_t rank = CS > 1 ? cluster_rank() : 0u, peer = rank ^ 1u;
  const int r = n - j0;
  const int y0 = j0 + (int)rank * rsplit;
  const int rq = CS > 1 ? min(r - (int)rank * rsplit, rsplit) : r;
  const int nch1 = (rq + R1 - 1) / R1;
  const int nch2 = (rq + R2 - 1) / R2;
  // Pass-1 partial accumulators. Without halves (rsplit >= r, one CTA): chunk
  // ch into partial ch % NP1. With halves (rsplit < r): rows [0, rsplit) and
  // [rsplit, r) each into NP1 interleaved partials and the two half sums
  // added last -- one CTA keeps both halves (partials NP1 and up for the
  // second), a 2-CTA cluster one half per CTA: the same FP32 operations in
  // the same order either way, so the bits do not depend on the CTA count.
  const bool halves = CS > 1 || rsplit < r;
  const int c1 = CS > 1 ? nch1 : (halves ? rsplit / R1 : nch1);  // chunks of the first half
  const int tfirst = (int)blockIdx.x / CS, tstep = (int)gridDim.x / CS;

  if (tid == 0) {
    const uint32_t counts[NBAR] = {1, 1, 1, 1,                          // full1
                                   NWORK, NWORK, NWORK, NWORK,          // split1
                                   1, 1, 1, 1,                          // empty1
                                   1,                                   // d1full
                                   NWORK,                               // b2ready
                                   1, 1, 1, 1, 1, 1,                    // v2full, v2empty, accfull
                                   NWORK, NWORK,                        // accempty
                                   1, 1,                                // tiledone, fin
                                   32 * NWORK, 32 * NWORK};             // xfull, xread
    for (int i = 0; i < NBAR; ++i) tma::mbar_init(BAR(i), counts[i]);
    tma::mbar_fence_init();
    *s_abort = 0;
    tma::prefetch_map(&mC1);
    tma::prefetch_map(&mV1);
    tma::prefetch_map(&mV2);
    tma::prefetch_map(&mC2);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     base + L::OFF_TMEMV),
                 "r"(L::TM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (CS > 1) cluster_sync_all();  // the peer's mbarriers are initialised
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      int g1 = 0, g2 = 0, it = 0;
      int last1[S1MAX] = {-1, -1, -1, -1}, last2[2] = {-1, -1};  // use index of the last load issued
      for (int t = tfirst; t < ntiles; t += tstep, ++it) {
        const int m = m0 + t / ntc;
        const int tc0 = col0 + (t % ntc) * TCOLS;
        const int nbox = min(4, (col_end - tc0 + 31) / 32);
        const uint32_t tx1 = (uint32_t)nbox * BOX1 + 2 * L::VB1;
        // the previous tile's pass 2 has released the shared buffers
        if (it > 0 && *s_abort == 0)
          tma::mbar_wait_or_abort(BAR(B_TILEDONE), (uint32_t)((it - 1) & 1), wait_limit, s_abort);
        for (int ch = 0; ch < nch1; ++ch, ++g1) {
          const int s = g1 % S1, u = g1 / S1;
          if (*s_abort != 0) continue;
          if (u > 0 &&
              !tma::mbar_wait_or_abort(BAR(B_EMPTY1 + s), (uint32_t)((u - 1) & 1), wait_limit,
                                       s_abort))
            continue;
          const uint32_t st = base + (uint32_t)s * L::ST1, fb = BAR(B_FULL1 + s);
          const int y = y0 + ch * R1;
          tma::mbar_expect_tx(fb, tx1);
          for (int bq = 0; bq < nbox; ++bq)
            tma::load_3d(st + bq * BOX1, &mC1, fb, tc0 + 32 * bq, y, m);
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            tma::load_4d(st + L::S1_VH + a * BOX1, &mV1, fb, 32 * a, y, m, vw_hi);
            tma::load_4d(st + L::S1_VL + a * BOX1, &mV1, fb, 32 * a, y, m, vw_lo);
          }
          last1[s] = u;
        }
        // pass 2 reuses the pass-1 region: wait until every pass-1 MMA is done
        if (*s_abort == 0)
          tma::mbar_wait_or_abort(BAR(B_D1FULL), (uint32_t)(it & 1), wait_limit, s_abort);
        for (int p = 0; p < nch2; ++p, ++g2) {
          const int v = g2 % NV2, u = g2 / NV2;
          if (*s_abort != 0) continue;
          if (u > 0 &&
              !tma::mbar_wait_or_abort(BAR(B_V2EMPTY + v), (uint32_t)((u - 1) & 1), wait_limit,
                                       s_abort))
            continue;
          const uint32_t st = base + (uint32_t)v * L::V2ST, fb = BAR(B_V2FULL + v);
          const int y = y0 + p * R2;
          tma::mbar_expect_tx(fb, L::V2ST);
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            tma::load_4d(st + a * BOX2, &mV2, fb, 32 * a, y, m, vw_hi);
            tma::load_4d(st + (NA + a) * BOX2, &mV2, fb, 32 * a, y, m, vw_lo);
          }
          last2[v] = u;
        }
      }
      if (*s_abort != 0) {
        // bounded wait for the last load issued into every stage
        for (int s = 0; s < S1; ++s)
          if (last1[s] >= 0)
            tma::mbar_wait_bounded(BAR(B_FULL1 + s), (uint32_t)(last1[s] & 1), wait_limit);
        for (int v = 0; v < NV2; ++v)
          if (last2[v] >= 0)
            tma::mbar_wait_bounded(BAR(B_V2FULL + v), (uint32_t)(last2[v] & 1), wait_limit);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      int g1 = 0, g2 = 0, it = 0;
      for (int t = tfirst; t < ntiles; t += tstep, ++it) {
        for (int ch = 0; ch < nch1; ++ch, ++g1) {
          const int s = g1 % S1, u = g1 / S1;
          if (*s_abort != 0 || skip_mma) continue;
          if (!tma::mbar_wait_or_abort(BAR(B_SPLIT1 + s), (uint32_t)(u & 1), wait_limit, s_abort))
            continue;
          tc::fence_after();
          const uint32_t st = base + (uint32_t)s * L::ST1;
          int slot;
          bool first;
          if (!halves) {
            slot = ch % NP1;
            first = ch < NP1;
          } else if (ch < c1) {
            slot = ch % NP1;
            first = ch < NP1;
          } else {
            slot = NP1 + (ch - c1) % NP1;
            first = ch - c1 < NP1;
          }
          const uint32_t d1 = tmem + (uint32_t)KR * (uint32_t)slot;
          // the k-step's operands are 1024 bytes further on: add to the
          // descriptors' address field (units of 16 bytes; no carry)
          const uint64_t ah0 = sdesc_mn32(st, BOX1), al0 = sdesc_mn32(st + L::S1_CL, BOX1);
          const uint64_t bh0 = sdesc_mn32(st + L::S1_VH, BOX1);
          const uint64_t bl0 = sdesc_mn32(st + L::S1_VL, BOX1);
#pragma unroll
          for (int ks = 0; ks < R1 / 8; ++ks) {
            const uint64_t dk = (uint64_t)(ks * (1024 >> 4));
            tc::mma_tf32(d1, ah0 + dk, bh0 + dk, L::IDESC1, (!first || ks != 0) ? 1u : 0u);
            tc::mma_tf32(d1, ah0 + dk, bl0 + dk, L::IDESC1, 1u);
            tc::mma_tf32(d1, al0 + dk, bh0 + dk, L::IDESC1, 1u);
          }
          tc::mma_commit(BAR(B_EMPTY1 + s));
        }
        if (*s_abort == 0 && !skip_mma) tc::mma_commit(BAR(B_D1FULL));
        // pass 2 once the workers have formed W'
        if (*s_abort == 0)
          tma::mbar_wait_or_abort(BAR(B_B2READY), (uint32_t)(it & 1), wait_limit, s_abort);
        for (int p = 0; p < nch2; ++p, ++g2) {
          const int v = g2 % NV2, u = g2 / NV2;
          const int ab = g2 % L::NACC, ua = g2 / L::NACC;  // TMEM accumulator
          if (*s_abort != 0) continue;
          if (!tma::mbar_wait_or_abort(BAR(B_V2FULL + v), (uint32_t)(u & 1), wait_limit, s_abort))
            continue;
          if (ua > 0 && !tma::mbar_wait_or_abort(BAR(B_ACCEMPTY + ab), (uint32_t)((ua - 1) & 1),
                                                 wait_limit, s_abort))
            continue;
          tc::fence_after();
          const uint32_t va = base + (uint32_t)v * L::V2ST;
          const uint32_t d = tmem + L::TM_D2 + 128u * (uint32_t)ab;
          const uint64_t ah0 = sdesc_kmajor(va), al0 = sdesc_kmajor(va + NA * BOX2);
          const uint64_t bh0 = sdesc_kmajor(base + L::OFF_BH);
          const uint64_t bl0 = sdesc_kmajor(base + L::OFF_BL);
#pragma unroll
          for (int ks = 0; ks < KR / 8; ++ks) {
            const uint32_t ka = (uint32_t)(ks >> 2), ko = 32u * (uint32_t)(ks & 3);
            const uint64_t da = (uint64_t)((ka * BOX2 + ko) >> 4);
            const uint64_t db = (uint64_t)((ka * TCOLS * 128 + ko) >> 4);
            tc::mma_tf32(d, ah0 + da, bh0 + db, IDESC2, ks != 0 ? 1u : 0u);
            tc::mma_tf32(d, ah0 + da, bl0 + db, IDESC2, 1u);
            tc::mma_tf32(d, al0 + da, bh0 + db, IDESC2, 1u);
          }
          tc::mma_commit(BAR(B_V2EMPTY + v));
          tc::mma_commit(BAR(B_ACCFULL + ab));
        }
      }
      if (*s_abort != 0) {  // every MMA issued so far has completed before TMEM is freed
        tc::mma_commit(BAR(B_FIN));
        tma::mbar_wait_bounded(BAR(B_FIN), 0u, wait_limit);
      }
    }
  } else {
    // ================= workers =================
    const int wt = tid - 64;               // 0 .. 32 * NWORK - 1
    const int q = warp & 3;                // TMEM lane quarter of this warp
    // half of the reflectors / columns (DUAL: each worker takes both)
    const int h = DUAL ? 0 : (warp - 2) >> 2;
    const int row = 32 * q + lane;         // TMEM lane = tile column (pass 1) / chunk row (pass 2)
    const bool issuer = wt == 0;
    int g1 = 0, g2 = 0, it = 0;
    for (int t = tfirst; t < ntiles; t += tstep, ++it) {
      const int ml = t / ntc, m = m0 + ml;
      const int tc0 = col0 + (t % ntc) * TCOLS;
      const int nbox = min(4, (col_end - tc0 + 31) / 32);
      if (it == 0) {  // later tiles' T is prefetched during the previous tile's pass 2
        const float* Tm = T + (int64_t)ml * sTb;
        for (int e = wt; e < KR * KR; e += 32 * NWORK)
          Ts[(e / KR) * L::T_LD + (e % KR)] = __ldg(Tm + e);
      }
      workers_sync_or<NWORK>(false);  // T in shared memory for the W' step below

      // ---- pass 1: split each chunk's C boxes into hi (in place) and lo ----
      const int units = nbox * (int)(BOX1 / 16);
      for (int ch = 0; ch < nch1; ++ch, ++g1) {
        const int s = g1 % S1, u = g1 / S1;
        if (*s_abort != 0) continue;
        // the chunk has landed (and, transitively, the MMAs of chunk g1 - S1
        // that last read this stage's lo buffer are done)
        if (!tma::mbar_wait_or_abort(BAR(B_FULL1 + s), (uint32_t)(u & 1), wait_limit, s_abort))
          continue;
        float4* c4 = reinterpret_cast<float4*>(sm + (uint32_t)s * L::ST1);
        float4* l4 = reinterpret_cast<float4*>(sm + (uint32_t)s * L::ST1 + L::S1_CL);
        for (int e = wt; e < units; e += 32 * NWORK) {
          float4 hi, lo;
          tc::split4(c4[e], hi, lo);
          c4[e] = hi;
          l4[e] = lo;
        }
        tma::fence_proxy_async();
        __syncwarp();
        if (lane == 0) tma::mbar_arrive(BAR(B_SPLIT1 + s));
      }

      // ---- W' = T^T W (this thread: tile column `row`, reflectors of half h) ----
      bool skip = *s_abort != 0 ||
                  !tma::mbar_wait_or_abort(BAR(B_D1FULL), (uint32_t)(it & 1), wait_limit, s_abort);
      skip = __any_sync(tc::kFullMask, skip);  // tcgen05.ld below is warp-collective
      float w[KR];
      if (!skip) {
        tc::fence_after();
        float wp[32];
        const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
#pragma unroll
        for (int a = 0; a < NA; ++a) tmem_ld32_nowait(tl + 32u * a, w + 32 * a);
        tmem_wait_ld();
        const int np = min(c1, NP1);
        for (int pp = 1; pp < np; ++pp) {
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            tmem_ld32_nowait(tl + (uint32_t)(KR * pp + 32 * a), wp);
            tmem_wait_ld();
#pragma unroll
            for (int b = 0; b < 32; ++b) w[32 * a + b] += wp[b];
          }
        }
        if (CS == 1 && halves) {  // the second half's sum (16 columns at a time), added
          const int np2 = min(nch1 - c1, NP1);
#pragma unroll
          for (int a = 0; a < KR / 16; ++a) {
            float ws2[16];
            tmem_ld16_nowait(tl + (uint32_t)(KR * NP1 + 16 * a), ws2);
            tmem_wait_ld();
            for (int pp = 1; pp < np2; ++pp) {
              tmem_ld16_nowait(tl + (uint32_t)(KR * (NP1 + pp) + 16 * a), wp);
              tmem_wait_ld();
#pragma unroll
              for (int b = 0; b < 16; ++b) ws2[b] += wp[b];
            }
#pragma unroll
            for (int b = 0; b < 16; ++b) w[16 * a + b] += ws2[b];
          }
        }
        constexpr int HALF = KR / 2;
        if (CS > 1) {
          // partial W of this CTA's rows -> X (16-byte unit (k / 4) * TCOLS +
          // column; half h writes reflectors [h * HALF, (h + 1) * HALF)), then
          // add the peer's (half 0 needs reflectors < HALF only)
          const uint32_t xl = base + L::OFF_X;
#pragma unroll
          for (int k4 = 0; k4 < KR / 4; ++k4)
            if ((k4 < HALF / 4) == (h == 0))
              *reinterpret_cast<float4*>(sm + L::OFF_X + ((uint32_t)k4 * TCOLS + row) * 16u) =
                  make_float4(w[4 * k4], w[4 * k4 + 1], w[4 * k4 + 2], w[4 * k4 + 3]);
          mbar_arrive_peer(peer_addr(BAR(B_XFULL), peer));
          bool ok = mbar_wait_cluster_or_abort(BAR(B_XFULL), (uint32_t)(it & 1), wait_limit,
                                               s_abort);
          ok = __all_sync(tc::kFullMask, ok);
          if (ok) {
            const uint32_t xp = peer_addr(xl, peer) + (uint32_t)row * 16u;
            // 8 loads in flight at a time (registers)
#pragma unroll
            for (int g = 0; g < KR / 32; ++g) {
              float4 pv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (h == 1 || 8 * g + i < HALF / 4)
                  pv[i] = ld_peer4(xp + (uint32_t)(8 * g + i) * TCOLS * 16u);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (h == 1 || 8 * g + i < HALF / 4) {
                  const int k = 4 * (8 * g + i);
                  w[k] += pv[i].x;
                  w[k + 1] += pv[i].y;
                  w[k + 2] += pv[i].z;
                  w[k + 3] += pv[i].w;
                }
            }
            // the peer may overwrite its X once all 256 workers are past here
            mbar_arrive_peer(peer_addr(BAR(B_XREAD), peer));
          }
          skip = !ok;
        }
      }
      if (!skip) {
        constexpr int HALF = KR / 2;
        for (int hh = h; hh < (DUAL ? 2 : h + 1); ++hh) {
          float o[HALF];
          if (hh == 0) {  // W'[a] for a < KR/2: T[b][a] = 0 for b > a
#pragma unroll
            for (int i = 0; i < HALF; ++i) {
              float acc = 0.f;
#pragma unroll
              for (int b = 0; b < HALF; ++b) acc = fmaf(Ts[b * L::T_LD + i], w[b], acc);
              o[i] = acc;
            }
          } else {
#pragma unroll
            for (int i = 0; i < HALF; ++i) {
              float acc = 0.f;
#pragma unroll
              for (int b = 0; b < KR; ++b) acc = fmaf(Ts[b * L::T_LD + HALF + i], w[b], acc);
              o[i] = acc;
            }
          }
          // B operand of pass 2, K-major: row = tile column, K atoms of 32
          // reflectors (128 bytes) each
#pragma unroll
          for (int j = 0; j < HALF / 4; ++j) {
            const int a0 = hh * HALF + 4 * j;
            float4 hi, lo;
            tc::split4(make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]), hi, lo);
            const uint32_t off = (uint32_t)(a0 >> 5) * TCOLS * 128 + sw128(row, (a0 & 31) >> 2);
            *reinterpret_cast<float4*>(sm + L::OFF_BH + off) = hi;
            *reinterpret_cast<float4*>(sm + L::OFF_BL + off) = lo;
          }
        }
        tma::fence_proxy_async();
        tc::fence_before();
        __syncwarp();
        if (lane == 0) tma::mbar_arrive(BAR(B_B2READY));
      }

      // the next tile's T, into registers now and into Ts once every worker
      // is past this tile's W' step (the first pass-2 barrier below)
      constexpr int TPT = KR * KR / (32 * NWORK);
      float tnext[TPT];
      const int tn = t + tstep;
      if (tn < ntiles) {
        const float* Tn = T + (int64_t)(tn / ntc) * sTb;
#pragma unroll
        for (int k = 0; k < TPT; ++k) tnext[k] = __ldg(Tn + wt + k * 32 * NWORK);
      }

      // ---- pass 2 epilogues: C += -(V W') by TMA reduce-add ----
      // 64-column pieces of each chunk: one per worker half (staging boxes 2h
      // and 2h + 1, all four reduced together), or with DUAL both, one after
      // the other through staging boxes 0 and 1
      constexpr int NPC = DUAL ? 2 : 1;
      for (int p = 0; p < nch2; ++p, ++g2) {
        const int ab = g2 % L::NACC, ua = g2 / L::NACC;
        bool sk = *s_abort != 0 ||
                  !tma::mbar_wait_or_abort(BAR(B_ACCFULL + ab), (uint32_t)(ua & 1), wait_limit,
                                           s_abort);
        sk = __any_sync(tc::kFullMask, sk);
        for (int pc = 0; pc < NPC; ++pc) {
          const int piece = DUAL ? pc : h;
          float d0[32], d1[32];
          if (!sk) {
            tc::fence_after();
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + L::TM_D2 +
                                128u * (uint32_t)ab + 64u * (uint32_t)piece;
            tmem_ld32_nowait(ta, d0);
            tmem_ld32_nowait(ta + 32, d1);
            tmem_wait_ld();
            if (pc == NPC - 1) {
              tc::fence_before();
              __syncwarp();
              if (lane == 0) tma::mbar_arrive(BAR(B_ACCEMPTY + ab));
            }
          }
          if (issuer) tma::bulk_wait_read_all();  // the previous reduce has read the staging tile
          // row-split tiles: the staging boxes hold X until the peer has read it
          if (CS > 1 && p == 0 && issuer && *s_abort == 0)
            mbar_wait_cluster_or_abort(BAR(B_XREAD), (uint32_t)(it & 1), wait_limit, s_abort);
          if (workers_sync_or<NWORK>(sk || *s_abort != 0)) break;
          if (p == 0 && pc == 0 && tn < ntiles) {
#pragma unroll
            for (int k = 0; k < TPT; ++k) {
              const int e = wt + k * 32 * NWORK;
              Ts[(e / KR) * L::T_LD + (e % KR)] = tnext[k];
            }
          }
          const uint32_t sb = L::OFF_STG + (DUAL ? 0u : 2u * (uint32_t)h) * BOX2;
#pragma unroll
          for (int uu = 0; uu < 8; ++uu) {
            *reinterpret_cast<float4*>(sm + sb + sw128(row, uu)) =
                make_float4(-d0[4 * uu], -d0[4 * uu + 1], -d0[4 * uu + 2], -d0[4 * uu + 3]);
            *reinterpret_cast<float4*>(sm + sb + BOX2 + sw128(row, uu)) =
                make_float4(-d1[4 * uu], -d1[4 * uu + 1], -d1[4 * uu + 2], -d1[4 * uu + 3]);
          }
          tma::fence_proxy_async();
          workers_sync_or<NWORK>(false);
          if (issuer) {
            for (int bq = 0; bq < L::NSTG; ++bq) {
              const int box = (DUAL ? 2 * pc : 0) + bq;
              if (box < nbox)
                tma::reduce_add_3d(&mC2, base + L::OFF_STG + bq * BOX2, tc0 + 32 * box,
                                   y0 + R2 * p, m);
            }
            tma::bulk_commit();
          }
        }
      }
      if (issuer) {  // the tile's buffers are free once the last reduce has read its staging
        tma::bulk_wait_read_all();
        tma::mbar_arrive(BAR(B_TILEDONE));
      }
    }
    if (issuer) tma::bulk_wait_all();  // every reduce-add has completed
  }

  // ---------------- teardown ----------------
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  // the peer reads this CTA's shared memory and arrives on its mbarriers
  // until it is past its last exchange (every wait before here is bounded)
  if (CS > 1) cluster_sync_all();
  if (tid == 0 && *s_abort != 0) atomicExch(err, 1);
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TM_COLS)
                 : "memory");
}

// Test probe of the bounded wait: one thread waits on an mbarrier phase that
// nothing completes, for `limit` cycles, then records the timeout in the
// device error flag and returns.
__global__ void k_wait_probe(int* __restrict__ err, long long limit) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = tma::smem_addr(&bar);
  tma::mbar_init(b, 1);
  tma::mbar_fence_init();
  if (!tma::mbar_wait_bounded(b, 0u, limit)) atomicExch(err, 1);
}

}  // namespace

int launch_wait_probe(long long limit, cudaStream_t stream) {
  int* err = nullptr;
  if (device_error_ptr(&err) != QRB_OK) return QRB_ERR_DEVICE;
  k_wait_probe<<<1, 1, 0, stream>>>(err, limit);
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

bool larfb_tma_supported(int n) { return n % 4 == 0 && n > 32 && tma::encoder() != nullptr; }

int make_larfb_maps(LarfbMaps* maps, const float* H, const float* Vs, int64_t batch, int n,
                    int kr) {
  if (maps == nullptr || H == nullptr || Vs == nullptr || batch <= 0 || n % 4 != 0 ||
      batch > 0x7fffffffLL || (kr != 32 && kr != 64))
    return QRB_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(H) & 15) != 0 || (reinterpret_cast<uintptr_t>(Vs) & 15) != 0)
    return QRB_ERR_UNSUPPORTED;
  const uint64_t nn = (uint64_t)n, k = (uint64_t)kr;
  const uint64_t cdims[3] = {nn, nn, (uint64_t)batch};
  const uint64_t cstr[2] = {nn * 4, nn * nn * 4};
  // the split reflectors: 4 planes (two V buffers x hi / lo) of
  // [batch][n][kr]
  const uint64_t vdims[4] = {k, nn, (uint64_t)batch, 4u};
  const uint64_t vstr[3] = {k * 4, nn * k * 4, (uint64_t)batch * nn * k * 4};
  // pass-1 boxes are MN-major operands (32-byte-atom swizzle); pass-2 V boxes
  // are K-major operands and the C boxes take the staged reduce-add (plain
  // 128-byte swizzle)
  const bool ok = tma::encode_f32_sw128(&maps->c1, H, 3, cdims, cstr, 32, R1, true) &&
                  tma::encode_f32_sw128(&maps->c2, H, 3, cdims, cstr, 32, R2, false) &&
                  tma::encode_f32_sw128(&maps->v1, Vs, 4, vdims, vstr, 32, R1, true) &&
                  tma::encode_f32_sw128(&maps->v2, Vs, 4, vdims, vstr, 32, R2, false);
  maps->kr = kr;
  return ok ? QRB_OK : QRB_ERR_UNSUPPORTED;
}

namespace {
// Row split of a tile across a 2-CTA cluster: rank 0 takes the first rsplit
// rows of the trailing block (a multiple of the pass-2 chunk), rank 1 the rest.
int split_rows_of(int r) { return (((r + 1) / 2 + R2 - 1) / R2) * R2; }

template <int KR>
int launch_tma_t(const LarfbMaps& maps, const float* T, int64_t sTb, int64_t m0, int64_t count,
                 int j0, int col0, int col_end, int n, int vw_hi, int vw_lo,
                 cudaStream_t stream) {
  static bool attr_set[64] = {};
  static int* err_ptr[64] = {};
  static int sms[64] = {};
  static int max_pairs[64] = {};  // co-resident 2-CTA clusters
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k_larfb_tma<KR, 1, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Lay<KR>::SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(k_larfb_tma<KR, 2, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Lay<KR>::SMEM_BYTES) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    if constexpr (KR == 32) {
      if (cudaFuncSetAttribute(k_larfb_tma<KR, 1, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)Lay<KR, true>::SMEM_BYTES) != cudaSuccess)
        return QRB_ERR_LAUNCH;
    }
    if (device_error_ptr(&err_ptr[dev]) != QRB_OK) return QRB_ERR_DEVICE;
    if (cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms[dev] <= 0)
      return QRB_ERR_DEVICE;
    cudaLaunchConfig_t qc = {};
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    qc.gridDim = dim3(2 * (unsigned)sms[dev]);
    qc.blockDim = dim3(Lay<KR>::NTH);
    qc.dynamicSmemBytes = Lay<KR>::SMEM_BYTES;
    qc.attrs = qa;
    qc.numAttrs = 1;
    int pairs = 0;
    if (cudaOccupancyMaxActiveClusters(&pairs, k_larfb_tma<KR, 2, false>, &qc) != cudaSuccess) {
      (void)cudaGetLastError();
      pairs = 0;  // no row split on this device
    }
    max_pairs[dev] = pairs;
    attr_set[dev] = true;
  }
  const int64_t ntc = (col_end - col0 + TCOLS - 1) / TCOLS;
  const int64_t tiles = ntc * count;
  if (tiles > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  int most = sms[dev];  // persistent: at most one CTA per SM
  const int cap = tma_cta_cap();
  if (cap > 0 && cap < most) most = cap;
  const int r = n - j0;
  const int split_min = tma_split_rows();
  // The arithmetic (two row halves or not) is a pure function of the trailing
  // block's height and the hooks, never of the batch, so results do not depend
  // on how a batch is grouped. One CTA or a CTA pair per tile computes the
  // same bits: a pair when the launch's tiles fit the SMs twice over (the
  // batch groups and the look-ahead kernels beside it fill the SMs left).
  const bool halves = split_min > 0 && r >= split_min && r > R2;
  const int rs = halves ? split_rows_of(r) : r;
  const int mode = tma_pair_mode();
  const bool pair = halves && max_pairs[dev] > 0 &&
                    (mode == 2 || (mode == 0 && 2 * tiles <= sms[dev]));
  // Two CTAs per SM (32 reflectors, no row halves; the same bits as one CTA
  // per SM) when one CTA per SM would take more than one wave of tiles.
  const int dmode = tma_dual_mode();
  const bool dual = KR == 32 && !halves &&
                    (dmode == 2 || (dmode == 0 && tiles > (int64_t)sms[dev]));
  if (dual) {
    if constexpr (KR == 32) {
      int most2 = 2 * sms[dev];
      if (cap > 0 && cap < most2) most2 = cap;
      const int grid = (int)(tiles < most2 ? tiles : most2);
      k_larfb_tma<KR, 1, true><<<grid, Lay<KR, true>::NTH, Lay<KR, true>::SMEM_BYTES, stream>>>(
          maps.c1, maps.c2, maps.v1, maps.v2, T, sTb, (int)m0, (int)tiles, (int)ntc, j0, col0,
          col_end, n, vw_hi, vw_lo, rs, err_ptr[dev], device_wait_limit(),
          test_skip_mma() ? 1 : 0);
    }
  } else if (!pair) {
    const int grid = (int)(tiles < most ? tiles : most);
    k_larfb_tma<KR, 1, false><<<grid, Lay<KR>::NTH, Lay<KR>::SMEM_BYTES, stream>>>(
        maps.c1, maps.c2, maps.v1, maps.v2, T, sTb, (int)m0, (int)tiles, (int)ntc, j0, col0,
        col_end, n, vw_hi, vw_lo, rs, err_ptr[dev], device_wait_limit(),
        test_skip_mma() ? 1 : 0);
  } else {
    int pairs = most / 2 > 0 ? most / 2 : 1;
    if (pairs > max_pairs[dev]) pairs = max_pairs[dev];
    if (tiles < pairs) pairs = (int)tiles;
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeClusterDimension;
    la[0].val.clusterDim.x = 2;
    la[0].val.clusterDim.y = 1;
    la[0].val.clusterDim.z = 1;
    lc.gridDim = dim3(2 * (unsigned)pairs);
    lc.blockDim = dim3(Lay<KR>::NTH);
    lc.dynamicSmemBytes = Lay<KR>::SMEM_BYTES;
    lc.stream = stream;
    lc.attrs = la;
    lc.numAttrs = 1;
    if (cudaLaunchKernelEx(&lc, k_larfb_tma<KR, 2, false>, maps.c1, maps.c2, maps.v1, maps.v2, T, sTb,
                           (int)m0, (int)tiles, (int)ntc, j0, col0, col_end, n, vw_hi, vw_lo,
                           rs, err_ptr[dev], device_wait_limit(),
                           test_skip_mma() ? 1 : 0) != cudaSuccess)
      return QRB_ERR_LAUNCH;
  }
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}
}  // namespace

int launch_larfb_tma(const LarfbMaps& maps, const float* T, int64_t sTb, int64_t m0,
                     int64_t count, int j0, int col0, int col_end, int n, int vbuf,
                     cudaStream_t stream) {
  if (count <= 0 || col_end <= col0) return QRB_OK;
  const int kr = maps.kr;
  if (j0 < 0 || j0 + kr > n || col0 % 4 != 0 || m0 < 0 || m0 + count > 0x7fffffffLL ||
      vbuf < 0 || vbuf > 1)
    return QRB_ERR_UNSUPPORTED;
  if (col_end != n && (col_end - col0) % 32 != 0) return QRB_ERR_UNSUPPORTED;
  if (kr == 32)
    return launch_tma_t<32>(maps, T, sTb, m0, count, j0, col0, col_end, n, 2 * vbuf, 2 * vbuf + 1,
                            stream);
  if (kr == 64)
    return launch_tma_t<64>(maps, T, sTb, m0, count, j0, col0, col_end, n, 2 * vbuf,
                            2 * vbuf + 1, stream);
  return QRB_ERR_UNSUPPORTED;
}

}  // namespace qrb

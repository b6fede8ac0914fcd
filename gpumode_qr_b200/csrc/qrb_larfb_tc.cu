// Block-reflector trailing update C <- C - V (T^T (V^T C)) on the 5th-gen
// tensor cores (tcgen05), in 3xTF32: every FP32 operand x is split into
// hi = tf32(x) and lo = tf32(x - hi), and each product is formed as
// hi*hi + hi*lo + lo*hi with FP32 accumulation in tensor memory (TMEM); the
// dropped lo*lo term is below FP32 rounding. Plain TF32 is never used.
//
// One CTA (256 threads, one per SM) owns one matrix's r x 128 column tile of C:
//   G1   W^T (128 x 32) = C^T V over all r rows. A = C^T and B = V are staged
//        K-major (transposed while staging: four rows of one column become
//        one 16-byte chunk of a canonical 8 x 16-byte core matrix). 32-row
//        chunks are staged (loaded, split, stored) into one of two
//        shared-memory buffers while the MMAs of the previous chunk run.
//   mid  thread m (TMEM lane m) reads row m of W^T, forms W'[:,m] = T^T W[:,m]
//        and writes it (split) as the K-major A operand of G2.
//   G2   D (128 x 128) = W'^T V^T for 128-row chunks of V: D[m][i] is the
//        update of C[i][c0+m]. Both operands are K-major in their natural
//        layout. Two TMEM accumulators alternate so the MMAs of one chunk run
//        while the epilogue of the previous one (TMEM -> registers, C - D,
//        coalesced: a warp covers 32 consecutive columns of a row) is done.
// The k = 32 reflector block, the unit-lower masking of V's top rows and the
// row-major layouts are those of the FFMA kernel in qrb_larfb.cu.
//
// Synchronisation: the single MMA-issuing thread commits each chunk's MMAs to
// an mbarrier; waits on mbarriers are bounded by a clock limit after which the
// kernel records an error (qrb_device_error) and carries on, so it always
// reaches the TMEM release at the end.
#include "qrb_common.cuh"
#include "qrb_tc.cuh"

namespace qrb {

namespace {

using namespace tc;

constexpr int KR = 32;     // reflectors per block
constexpr int TCN = 128;   // C columns per CTA (G1 M, G2 M)
constexpr int R1 = 32;     // rows per G1 chunk (4 MMA k-steps of 8)
constexpr int R2 = 128;    // rows per G2 chunk (G2 N)
constexpr int NT = 256;

// Shared memory carve-up (bytes).
constexpr int G1_A = TCN * R1 * 4;           // 16 KiB: C^T chunk, one of hi/lo
constexpr int G1_B = R1 * KR * 4;            // 4 KiB: V chunk, one of hi/lo
constexpr int G1_STAGE = 2 * G1_A + 2 * G1_B;  // 40 KiB
constexpr int G2_B = R2 * KR * 4;            // 16 KiB: V^T chunk, one of hi/lo
constexpr int G2_STAGE = 2 * G2_B;           // 32 KiB
constexpr int STAGES_BYTES = 2 * G1_STAGE;   // 80 KiB (G2 stages alias them)
constexpr int A2_BYTES = TCN * KR * 4;       // 16 KiB: W'^T, one of hi/lo
constexpr int OFF_A2 = STAGES_BYTES;
constexpr int OFF_T = OFF_A2 + 2 * A2_BYTES;
constexpr int T_LD = KR + 1;
constexpr int OFF_BAR = OFF_T + KR * T_LD * 4 + 64;
constexpr int SMEM_BYTES = OFF_BAR + 64 + 16;

// TMEM columns: two G2 accumulators (128 columns each) and eight partial G1
// accumulators (32 columns each). G1 chunks go round-robin to the partials,
// which are summed in FP32 afterwards: the tensor core's accumulating add is
// not an IEEE round-to-nearest FP32 add, so a single accumulator over all r
// rows loses accuracy in proportion to the number of accumulation steps.
constexpr uint32_t TM_D2_0 = 0, TM_D2_1 = 128, TM_D1 = 256, TM_COLS = 512;
constexpr int kG1Parts = 8;

constexpr uint32_t IDESC_G1 = idesc(TCN, KR, false, false);
constexpr uint32_t IDESC_G2 = idesc(TCN, R2, false, false);

__global__ void __launch_bounds__(NT, 1)
k_larfb_tc(const float* __restrict__ V, int64_t sVb, int64_t ldv,
           const float* __restrict__ T, int64_t sTb, int t_ld,
           const float* __restrict__ Csrc, int64_t sCsb, int64_t ldcs,
           float* __restrict__ Cdst, int64_t sCdb, int64_t ldcd, int r, int c,
           int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int64_t m = blockIdx.y;
  const int c0 = blockIdx.x * TCN;
  const float* __restrict__ Vm = V + m * sVb;
  const float* __restrict__ Cm = Csrc + m * sCsb;
  float* __restrict__ Dm = Cdst + m * sCdb;

  float* Ts = reinterpret_cast<float*>(smem + OFF_T);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // [0,1] G1, [2,3] G2, [4] drain
  __shared__ int s_abort_word;
  volatile int* s_abort = &s_abort_word;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 64);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
#pragma unroll
    for (int b = 0; b < 5; ++b)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar0 + 8 * b), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *s_abort = 0;
  }
  for (int e = tid; e < KR * KR; e += NT) {
    const int q = e / KR, k = e % KR;
    Ts[q * T_LD + k] = __ldg(T + m * sTb + (int64_t)q * t_ld + k);
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  uint32_t ph[4] = {0u, 0u, 0u, 0u};

  // ---------------- G1: W^T = C^T V ----------------
  const int nch1 = (r + R1 - 1) / R1;
  for (int ch = 0; ch < nch1; ++ch) {
    const int s = ch & 1;
    if (ch >= 2) {  // the MMAs of chunk ch-2 have finished reading buffer s
      mbar_wait(bar0 + 8 * s, ph[s], err, s_abort);
      ph[s] ^= 1u;
    }
    unsigned char* st = smem + s * G1_STAGE;
    const int i0 = ch * R1;
    // K-major staging (the transpose happens here): unit (kq, m) = rows
    // 4kq..4kq+3 of column m, loaded element-wise (a warp reads 128 contiguous
    // bytes of a row per load) and stored as one 16-byte chunk at
    // (kq * 16 + m / 8) * 128 + (m % 8) * 16 = kq * 2048 + m * 16, so
    // consecutive lanes store consecutive chunks.
#pragma unroll
    for (int e = 0; e < (R1 / 4) * TCN / NT; ++e) {  // C^T: 8 k-quads x 128 columns
      const int u = tid + e * NT;
      const int kq = u >> 7, mc = u & 127;
      const int col = c0 + mc;
      float4 v;
      float* vp = reinterpret_cast<float*>(&v);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int i = i0 + 4 * kq + t;
        vp[t] = (i < r && col < c) ? __ldg(Cm + (int64_t)i * ldcs + col) : 0.f;
      }
      float4 hi, lo;
      split4(v, hi, lo);
      const int off = u * 16;
      *reinterpret_cast<float4*>(st + off) = hi;
      *reinterpret_cast<float4*>(st + G1_A + off) = lo;
    }
    {  // V: 8 k-quads x 32 reflectors, chunk at kq * 512 + n * 16
      const int kq = tid >> 5, n = tid & 31;
      float4 v;
      float* vp = reinterpret_cast<float*>(&v);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int i = i0 + 4 * kq + t;
        vp[t] = (i < r) ? vmask(__ldg(Vm + (int64_t)i * ldv + n), i, n) : 0.f;
      }
      float4 hi, lo;
      split4(v, hi, lo);
      const int off = tid * 16;
      *reinterpret_cast<float4*>(st + 2 * G1_A + off) = hi;
      *reinterpret_cast<float4*>(st + 2 * G1_A + G1_B + off) = lo;
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0 && *s_abort == 0) {
      fence_after();
      const uint32_t a_hi = sbase + s * G1_STAGE, a_lo = a_hi + G1_A;
      const uint32_t b_hi = a_hi + 2 * G1_A, b_lo = b_hi + G1_B;
#pragma unroll
      for (int ks = 0; ks < R1 / 8; ++ks) {
        const uint64_t ah = sdesc(a_hi + ks * 4096, 2048, 128);
        const uint64_t al = sdesc(a_lo + ks * 4096, 2048, 128);
        const uint64_t bh = sdesc(b_hi + ks * 1024, 512, 128);
        const uint64_t bl = sdesc(b_lo + ks * 1024, 512, 128);
        const uint32_t d1 = tmem + TM_D1 + 32 * (ch % kG1Parts);
        mma_tf32(d1, ah, bh, IDESC_G1, (ch >= kG1Parts || ks != 0) ? 1u : 0u);
        mma_tf32(d1, ah, bl, IDESC_G1, 1u);
        mma_tf32(d1, al, bh, IDESC_G1, 1u);
      }
      mma_commit(bar0 + 8 * s);
    }
  }
  // Drain the last (up to two) commits: G1 is complete.
  for (int ch = (nch1 >= 2 ? nch1 - 2 : 0); ch < nch1; ++ch) {
    const int s = ch & 1;
    mbar_wait(bar0 + 8 * s, ph[s], err, s_abort);
    ph[s] ^= 1u;
  }
  fence_after();

  // ---------------- mid: W' = T^T W, written as G2's A operand ----------------
  if (warp < 4 && !__any_sync(kFullMask, *s_abort != 0)) {
    float w[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + TM_D1, w);
    const int parts = nch1 < kG1Parts ? nch1 : kG1Parts;
    for (int p = 1; p < parts; ++p) {
      float t[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + TM_D1 + 32 * p, t);
#pragma unroll
      for (int q = 0; q < 32; ++q) w[q] += t[q];
    }
    float o[32];
#pragma unroll
    for (int k = 0; k < KR; ++k) {
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q <= k; ++q) acc = fmaf(Ts[q * T_LD + k], w[q], acc);
      o[k] = acc;
    }
    const int mcol = tid;  // 0..127
    unsigned char* a2 = smem + OFF_A2;
#pragma unroll
    for (int kq = 0; kq < KR / 4; ++kq) {
      float4 hi, lo;
      split4(make_float4(o[4 * kq], o[4 * kq + 1], o[4 * kq + 2], o[4 * kq + 3]), hi, lo);
      const int off = (kq * 16 + (mcol >> 3)) * 128 + (mcol & 7) * 16;
      *reinterpret_cast<float4*>(a2 + off) = hi;
      *reinterpret_cast<float4*>(a2 + A2_BYTES + off) = lo;
    }
  }
  fence_before();
  fence_async_smem();
  __syncthreads();

  // ---------------- G2: D = W'^T V^T per 128-row chunk, C -= D^T ----------------
  const int nch2 = (r + R2 - 1) / R2;
  auto epilogue = [&](int cp) {
    const int s = cp & 1;
    mbar_wait(bar0 + 8 * (2 + s), ph[2 + s], err, s_abort);
    ph[2 + s] ^= 1u;
    if (__any_sync(kFullMask, *s_abort != 0)) return;  // no TMEM reads, no stores
    fence_after();
    const int q = warp & 3, h = warp >> 2;
    const int col = c0 + 32 * q + lane;
#pragma unroll 1
    for (int part = 0; part < 2; ++part) {
      const int rbase = cp * R2 + 64 * h + 32 * part;
      float d[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (s ? TM_D2_1 : TM_D2_0) + 64 * h + 32 * part, d);
      if (col < c) {
#pragma unroll 8
        for (int rr = 0; rr < 32; ++rr) {
          const int i = rbase + rr;
          if (i < r) Dm[(int64_t)i * ldcd + col] = Cm[(int64_t)i * ldcs + col] - d[rr];
        }
      }
    }
    fence_before();
  };
  for (int ch = 0; ch < nch2; ++ch) {
    const int s = ch & 1;
    // Buffer s and accumulator s were last used by chunk ch-2, whose epilogue
    // (in the previous iteration) waited for its MMAs and read its results.
    unsigned char* st = smem + s * G2_STAGE;
    const int i0 = ch * R2;
#pragma unroll
    for (int e = 0; e < (R2 * KR) / (4 * NT); ++e) {  // V: 128 rows x 32
      const int idx = tid + e * NT;
      const int row = idx & 127, k4 = (idx >> 7) << 2;
      const int i = i0 + row;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < r) v = __ldg(reinterpret_cast<const float4*>(Vm + (int64_t)i * ldv + k4));
      v.x = vmask(v.x, i, k4 + 0);
      v.y = vmask(v.y, i, k4 + 1);
      v.z = vmask(v.z, i, k4 + 2);
      v.w = vmask(v.w, i, k4 + 3);
      float4 hi, lo;
      split4(v, hi, lo);
      const int off = idx * 16;  // == ((k4 >> 2) * 16 + (row >> 3)) * 128 + (row & 7) * 16
      *reinterpret_cast<float4*>(st + off) = hi;
      *reinterpret_cast<float4*>(st + G2_B + off) = lo;
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0 && *s_abort == 0) {
      fence_after();
      const uint32_t a_hi = sbase + OFF_A2, a_lo = a_hi + A2_BYTES;
      const uint32_t b_hi = sbase + s * G2_STAGE, b_lo = b_hi + G2_B;
      const uint32_t d = tmem + (s ? TM_D2_1 : TM_D2_0);
#pragma unroll
      for (int ks = 0; ks < KR / 8; ++ks) {
        const uint64_t ah = sdesc(a_hi + ks * 4096, 2048, 128);
        const uint64_t al = sdesc(a_lo + ks * 4096, 2048, 128);
        const uint64_t bh = sdesc(b_hi + ks * 4096, 2048, 128);
        const uint64_t bl = sdesc(b_lo + ks * 4096, 2048, 128);
        mma_tf32(d, ah, bh, IDESC_G2, ks != 0);
        mma_tf32(d, ah, bl, IDESC_G2, 1u);
        mma_tf32(d, al, bh, IDESC_G2, 1u);
      }
      mma_commit(bar0 + 8 * (2 + s));
    }
    if (ch >= 1) epilogue(ch - 1);
  }
  epilogue(nch2 - 1);

  __syncthreads();
  if (tid == 0 && *s_abort != 0) drain_mmas(bar0 + 8 * 4);
  __syncthreads();
  fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TM_COLS)
                 : "memory");
}

}  // namespace

__device__ int g_qrb_device_error = 0;

int device_error_flag(int* value, bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_qrb_device_error, sizeof(int)) != cudaSuccess) return QRB_ERR_DEVICE;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_qrb_device_error, &zero, sizeof(int)) != cudaSuccess)
      return QRB_ERR_DEVICE;
  }
  *value = v;
  return QRB_OK;
}

int device_error_ptr(int** p) {
  void* q = nullptr;
  if (cudaGetSymbolAddress(&q, g_qrb_device_error) != cudaSuccess) return QRB_ERR_DEVICE;
  *p = static_cast<int*>(q);
  return QRB_OK;
}

bool larfb_tc_supported(const float* V, int64_t sVb, int64_t ldv, const float* Csrc,
                        int64_t sCsb, int64_t ldcs, const float* Cdst, int64_t sCdb,
                        int64_t ldcd, int k, int c) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return k == KR && c % 4 == 0 && ldv % 4 == 0 && sVb % 4 == 0 && ldcs % 4 == 0 &&
         sCsb % 4 == 0 && ldcd % 4 == 0 && sCdb % 4 == 0 && al(V) && al(Csrc) && al(Cdst);
}

int launch_larfb_tc(const float* V, int64_t sVb, int64_t ldv, const float* T,
                    int64_t sTb, int t_ld, const float* Csrc, int64_t sCsb,
                    int64_t ldcs, float* Cdst, int64_t sCdb, int64_t ldcd,
                    int64_t batch, int r, int c, cudaStream_t stream) {
  static bool attr_set[64] = {};
  static int* err_ptr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k_larfb_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qrb_device_error) != cudaSuccess) return QRB_ERR_DEVICE;
    err_ptr[dev] = static_cast<int*>(p);
    attr_set[dev] = true;
  }
  constexpr int64_t kMaxGridY = 65535;
  for (int64_t b0 = 0; b0 < batch; b0 += kMaxGridY) {
    const int64_t nb = batch - b0 < kMaxGridY ? batch - b0 : kMaxGridY;
    const dim3 grid((unsigned)((c + TCN - 1) / TCN), (unsigned)nb, 1);
    k_larfb_tc<<<grid, NT, SMEM_BYTES, stream>>>(V + b0 * sVb, sVb, ldv, T + b0 * sTb, sTb, t_ld,
                                                 Csrc + b0 * sCsb, sCsb, ldcs, Cdst + b0 * sCdb,
                                                 sCdb, ldcd, r, c, err_ptr[dev]);
    note_launches(1);
    if (cudaGetLastError() != cudaSuccess) return QRB_ERR_LAUNCH;
  }
  return QRB_OK;
}

}  // namespace qrb

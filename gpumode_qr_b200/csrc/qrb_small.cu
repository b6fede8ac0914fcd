// Fused whole-matrix Householder QR for n <= 32: LPM = 16 (or 8) lanes per
// matrix, two (or four) matrices per warp.
//
// Mapping: lane l of a matrix's lane group owns columns l, l + LPM, ... (CPL =
// 32 / LPM columns, "slots"), each in 32 registers held as 16 row pairs (rows
// and columns beyond n are zero). The lane groups of a warp factor their
// matrices with the same instructions, so the per-column work that does not
// scale with the matrix (the two shuffles, the reflector coefficients,
// publishing the column) is paid once for two (four) matrices. The updates run
// on the packed FP32x2 FMA of sm_100 (two IEEE FMAs per instruction).
//
// The column loop is unrolled (j, the owner lane j mod LPM and the owner's
// slot j / LPM are compile-time constants, so every row index is a register
// name and only rows below j are touched). With n == 32 every bound is a
// constant as well.
//
// Memory: every lane loads and stores its own columns element by element
// (a lane group touches 64 (32) contiguous bytes of a row per access). The host
// instantiations serve host-resident batches: A and/or H and tau are
// page-locked host memory mapped into the device address space, read and
// written once with streaming (evict-first) loads and stores.
//
// Step j: the owner lane publishes its unscaled column x through a per-group
// shared-memory line, every lane reads it back as row pairs, and each column
// k > j gets H_j = I - tau v v^T with v = scale * x below the diagonal:
//     d = a_j + scale * sum_{i>j} x_i a_i,  a_j -= tau d,  a_i -= (tau d scale) x_i.
// A slot is skipped once all its columns are finished. The sum of squares
// that step j+1 needs is accumulated during the update, only for the slot that
// holds column j+1. A finished column keeps
// its unscaled x below the diagonal; it is scaled once at the end (deferred
// scaling) and beta is stored on the diagonal.
//
// Semantics follow the reference's fused kernel step for step
// (src/qrbench/triton_kernels.py:676-715): slarfg coefficients (:691-700),
// rank-1 trailing update (:703-708), geqrf packing (:710-715); the last column
// has nothing below the diagonal and gets tau = 0.
#include "qrb_common.cuh"

namespace qrb {

namespace {

constexpr int NP = kFusedMaxN;  // padded matrix size (32 rows/columns)
constexpr int NQ = NP / 2;      // row pairs
constexpr int kWarpsPerBlock = 4;
constexpr int64_t kFusedQuadMaxBatch = 148 * 2 * kWarpsPerBlock * 4;

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

__device__ __forceinline__ float get_row(const float2 (&a)[NQ], int i) {
  return (i & 1) ? a[i >> 1].y : a[i >> 1].x;
}

__device__ __forceinline__ float2 xpair(const float* xb, int q) {
  return reinterpret_cast<const float2*>(xb)[q];
}

// Apply step J's reflector to one column (registers a) given the published
// column x (in shared memory at xb, rows > J valid) and the coefficients; with
// WANT_S, return in *s the sum of squares of rows > J+1 of the updated column.
template <int J, bool WANT_S>
__device__ __forceinline__ void apply_step(float2 (&a)[NQ], const float* xb, bool active,
                                           float tau, float scale, float* s) {
  constexpr int qf = (J + 2) / 2;  // first full row pair strictly below row J
  float dsum = 0.f;
  if ((J & 1) == 0) dsum = xb[J + 1] * a[J >> 1].y;
  float2 dA = make_float2(0.f, 0.f), dB = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = qf; q < NQ; ++q) {
    if (((q - qf) & 1) == 0)
      dA = __ffma2_rn(xpair(xb, q), a[q], dA);
    else
      dB = __ffma2_rn(xpair(xb, q), a[q], dB);
  }
  dsum += (dA.x + dA.y) + (dB.x + dB.y);
  const float aj = get_row(a, J);
  const float d = fmaf(scale, dsum, aj);
  const float f = active ? tau * d : 0.f;
  const float g = f * scale;
  const float2 ng = f2(-g);
  if (J & 1) {
    a[J >> 1].y -= f;
  } else {
    a[J >> 1].x -= f;
    a[J >> 1].y = fmaf(-g, xb[J + 1], a[J >> 1].y);
  }
  float2 sA = make_float2(0.f, 0.f), sB = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = qf; q < NQ; ++q) {
    a[q] = __ffma2_rn(ng, xpair(xb, q), a[q]);
    if (WANT_S) {
      // rows strictly below J+1: for odd J pair qf starts at row J+1.
      if (q == qf && (J & 1))
        sA.y = fmaf(a[q].y, a[q].y, sA.y);
      else if (((q - qf) & 1) == 0)
        sA = __ffma2_rn(a[q], a[q], sA);
      else
        sB = __ffma2_rn(a[q], a[q], sB);
    }
  }
  if (WANT_S) *s = (sA.x + sA.y) + (sB.x + sB.y);
}

// Per-lane state: CPL columns of one matrix (column l + k * LPM in slot k,
// LPM = 32 / CPL lanes per matrix), as row pairs.
template <int CPL>
struct LaneState {
  float2 a[CPL][NQ];
  float s[CPL];                    // sum of squares below the diagonal, per slot
  float mt[CPL], mb[CPL], ms[CPL];  // tau, beta, scale of the columns this lane owns
};

template <int J, int CPL, int K>
__device__ __forceinline__ void apply_slots(LaneState<CPL>& st, const float* xb, int l,
                                            float tau, float scale) {
  constexpr int LPM = NP / CPL;
  if constexpr (K < CPL) {
    if constexpr ((K + 1) * LPM > J + 1) {  // slot K still has a column > J
      constexpr int next_slot = (J + 1) / LPM;
      apply_step<J, K == next_slot>(st.a[K], xb, l + K * LPM > J, tau, scale, &st.s[K]);
    }
    apply_slots<J, CPL, K + 1>(st, xb, l, tau, scale);
  }
}

template <int J, int CPL, bool FULL>
__device__ __forceinline__ void step(LaneState<CPL>& st, float* xb0, float* xb1, int l,
                                     int grp, int n) {
  if constexpr (J < NP - 1) {
    if (!FULL && J >= n - 1) return;  // uniform: the last column gets tau = 0
    constexpr int LPM = NP / CPL;
    constexpr int owner = J % LPM;
    constexpr int slot = J / LPM;
    float* xb = (J & 1) ? xb1 : xb0;
    const float2(&ac)[NQ] = st.a[slot];
    const int src = grp * LPM + owner;
    const float alpha = __shfl_sync(kFull, get_row(ac, J), src);
    const float sigma = __shfl_sync(kFull, st.s[slot], src);
    const Reflector h = make_reflector(alpha, sigma);
    if (l == owner) {
      // rows > J are read back (and row J + 1 individually): publish from the
      // float4 holding row J + 1 on
#pragma unroll
      for (int q4 = (J + 1) / 4; q4 < NQ / 2; ++q4)
        reinterpret_cast<float4*>(xb)[q4] =
            make_float4(ac[2 * q4].x, ac[2 * q4].y, ac[2 * q4 + 1].x, ac[2 * q4 + 1].y);
      st.mt[slot] = h.tau;
      st.mb[slot] = h.beta;
      st.ms[slot] = h.scale;
    }
    __syncwarp();
    apply_slots<J, CPL, 0>(st, xb, l, h.tau, h.scale);
    step<J + 1, CPL, FULL>(st, xb0, xb1, l, grp, n);
  }
}

template <bool SYS>
__device__ __forceinline__ float load_a(const float* p) {
  if constexpr (SYS) return __ldcs(p);
  else return __ldg(p);
}

template <bool SYS>
__device__ __forceinline__ void store_h(float* p, float v) {
  if constexpr (SYS) __stcs(p, v);
  else *p = v;
}

// Factor matrices m0 .. m0 + CPL - 1 (those < batch) with this warp; lane
// group grp (LPM lanes) takes matrix m0 + grp. FULL: n == 32, so no row or
// column is padding and every bound below is a constant.
template <int CPL, bool IN_SYS, bool H_SYS, bool TAU_SYS, bool FULL>
__device__ __forceinline__ void factor_group(const float* __restrict__ A, int64_t sAb,
                                             int64_t sAr, float* __restrict__ H,
                                             float* __restrict__ tau, int64_t batch, int n,
                                             int64_t m0, float* xb0, float* xb1, int grp,
                                             int l) {
  constexpr int LPM = NP / CPL;
  const int64_t m = m0 + grp;
  const bool mat_ok = m < batch;  // a short last group leaves lanes idle

  LaneState<CPL> st;
  {
    const float* __restrict__ Am = A + (mat_ok ? m : m0) * sAb;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = l + k * LPM;
      const bool kc = FULL || c < n;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int i = 2 * q;
        const bool r0 = mat_ok && kc && (FULL || i < n);
        const bool r1 = mat_ok && kc && (FULL || i + 1 < n);
        st.a[k][q].x = r0 ? load_a<IN_SYS>(Am + (int64_t)i * sAr + c) : 0.f;
        st.a[k][q].y = r1 ? load_a<IN_SYS>(Am + (int64_t)(i + 1) * sAr + c) : 0.f;
      }
    }
  }
  {
    float2 s2 = make_float2(st.a[0][0].y * st.a[0][0].y, 0.f);
#pragma unroll
    for (int q = 1; q < NQ; ++q) s2 = __ffma2_rn(st.a[0][q], st.a[0][q], s2);
    st.s[0] = s2.x + s2.y;
  }
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    if (k > 0) st.s[k] = 0.f;
    st.mt[k] = st.mb[k] = st.ms[k] = 0.f;
  }

  step<0, CPL, FULL>(st, xb0, xb1, l, grp, n);

  // Final columns: deferred scaling below the diagonal, beta on it.
  float* __restrict__ Hm = H + (mat_ok ? m : 0) * (int64_t)n * n;
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    const int c = l + k * LPM;
    const bool refl = c < n - 1;  // columns 0 .. n-2 were factored
    const float sc = st.ms[k], be = st.mb[k];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * q + e;
        float v = e ? st.a[k][q].y : st.a[k][q].x;
        if (refl) v = i > c ? v * sc : (i == c ? be : v);
        if (mat_ok && (FULL || (c < n && i < n))) store_h<H_SYS>(Hm + (int64_t)i * n + c, v);
      }
    }
    if (mat_ok && (FULL || c < n)) store_h<TAU_SYS>(tau + m * n + c, st.mt[k]);
  }
}

// CPL = 2: 128 registers per thread (4 blocks of 4 warps per SM), two matrices
// per warp; config 2's 2048 warps fit in one wave of 148 SMs. CPL = 4: four
// matrices per warp (8 lanes x 4 columns each), up to 255 registers (2 blocks
// per SM); the per-column work that does not scale with the matrix is then
// shared by four matrices. With device memory the grid covers every group and
// each warp factors one. IN_SYS / H_SYS / TAU_SYS: A / H / tau are mapped host
// memory; with IN_SYS or H_SYS each warp factors the groups p, p + P,
// p + 2P, ... (P = warps in the grid), and the grid is kept small on purpose so
// that the first groups of every warp are written back over PCIe while later
// groups are still being read.
template <int CPL, bool IN_SYS, bool H_SYS, bool TAU_SYS, bool FULL>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, CPL == 2 ? 4 : 2)
k_fused(const float* __restrict__ A, int64_t sAb, int64_t sAr, float* __restrict__ H,
        float* __restrict__ tau, int64_t batch, int n) {
  constexpr int LPM = NP / CPL;
  __shared__ __align__(16) float xbuf[kWarpsPerBlock][CPL][2][NP];  // [warp][grp][parity][row]
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grp = lane / LPM;
  const int l = lane % LPM;
  const int64_t groups = (batch + CPL - 1) / CPL;
  const int64_t first = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if constexpr (!IN_SYS && !H_SYS) {  // device matrices: the grid covers every group
    if (first < groups)
      factor_group<CPL, false, false, TAU_SYS, FULL>(A, sAb, sAr, H, tau, batch, n, CPL * first,
                                                     xbuf[warp][grp][0], xbuf[warp][grp][1],
                                                     grp, l);
  } else {
    const int64_t stride = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = first; p < groups; p += stride) {
      __syncwarp();  // the previous group's readers are done with xbuf
      factor_group<CPL, IN_SYS, H_SYS, TAU_SYS, FULL>(A, sAb, sAr, H, tau, batch, n, CPL * p,
                                                      xbuf[warp][grp][0], xbuf[warp][grp][1],
                                                      grp, l);
    }
  }
}

template <int CPL, bool FULL>
void launch_variant(HostMem where, dim3 grid, dim3 block, cudaStream_t stream, const float* A,
                    int64_t sAb, int64_t sAr, float* H, float* tau, int64_t batch, int n) {
  switch (where) {
    case HostMem::kNone:
      k_fused<CPL, false, false, false, FULL><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau,
                                                                          batch, n);
      break;
    case HostMem::kTau:
      k_fused<CPL, false, false, true, FULL><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau,
                                                                         batch, n);
      break;
    case HostMem::kOutputs:
      k_fused<CPL, false, true, true, FULL><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau,
                                                                        batch, n);
      break;
    case HostMem::kAll:
      k_fused<CPL, true, true, true, FULL><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau,
                                                                       batch, n);
      break;
  }
}

template <int CPL>
int launch_cpl(const float* A, int64_t sAb, int64_t sAr, float* H, float* tau, int64_t batch,
               int n, cudaStream_t stream, HostMem where, int64_t max_blocks) {
  constexpr int64_t kPerBlock = CPL * kWarpsPerBlock;
  const bool looped = where == HostMem::kAll || where == HostMem::kOutputs;
  int64_t blocks = (batch + kPerBlock - 1) / kPerBlock;
  if (!looped && blocks > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  if (looped && max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
  if (blocks > 0x7fffffffLL) blocks = 0x7fffffffLL;  // host matrices: the kernel loops
  const dim3 grid((unsigned)blocks), block(kWarpsPerBlock * 32);
  if (n == NP)
    launch_variant<CPL, true>(where, grid, block, stream, A, sAb, sAr, H, tau, batch, n);
  else
    launch_variant<CPL, false>(where, grid, block, stream, A, sAb, sAr, H, tau, batch, n);
  return QRB_OK;
}

}  // namespace

int launch_fused_small(const float* A, int64_t sAb, int64_t sAr, float* H,
                       float* tau, int64_t batch, int n, cudaStream_t stream, HostMem where,
                       int64_t max_blocks) {
  if (n < 1 || n > kFusedMaxN) return QRB_ERR_UNSUPPORTED;
  // Per-element loads and stores: staging whole matrices through shared memory
  // with 16-byte copies measured slower here (more registers, no overlap).
  // Four matrices per warp while the batch fits about one wave of 2 blocks x 4
  // warps x 4 matrices per SM on 148 SMs; beyond that two per warp (measured on
  // B200: 22.5 vs 24.5 us at 4096 x 32x32, 69.5 vs 66.4 us at 16384).
  int cpl = fused_cpl();
  if (cpl == 0) cpl = batch <= kFusedQuadMaxBatch ? 4 : 2;
  const int rc = cpl == 4
                     ? launch_cpl<4>(A, sAb, sAr, H, tau, batch, n, stream, where, max_blocks)
                     : launch_cpl<2>(A, sAb, sAr, H, tau, batch, n, stream, where, max_blocks);
  if (rc != QRB_OK) return rc;
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace qrb

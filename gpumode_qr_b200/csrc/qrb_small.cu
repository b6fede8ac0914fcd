// Fused whole-matrix Householder QR for n <= 32: one half-warp per matrix,
// two matrices per warp.
//
// Mapping: in each half-warp (16 lanes) lane l owns columns l and l + 16 of its
// matrix, each in 32 registers held as 16 row pairs (rows and columns beyond n
// are zero). The two halves of a warp factor two matrices with the same
// instructions, so the per-column work that does not scale with the matrix
// (the two shuffles, the reflector coefficients, publishing the column) is
// paid once for two matrices. The updates run on the packed FP32x2 FMA of
// sm_100 (two IEEE FMAs per instruction).
//
// The column loop is unrolled (j, the owner lane j mod 16 and the owner's
// column slot j / 16 are compile-time constants, so every row index is a
// register name and only rows below j are touched).
//
// Memory: every lane loads and stores its own columns element by element
// (a half-warp touches 64 contiguous bytes of a row per access). The host
// instantiations serve host-resident batches: A and/or H and tau are
// page-locked host memory mapped into the device address space, read and
// written once with streaming (evict-first) loads and stores.
//
// Step j: the owner lane publishes its unscaled column x through a per-half
// shared-memory line, every lane reads it back as row pairs (once for the dot
// product, once for the update, to keep register pressure down), and each column
// k > j gets H_j = I - tau v v^T with v = scale * x below the diagonal:
//     d = a_j + scale * sum_{i>j} x_i a_i,  a_j -= tau d,  a_i -= (tau d scale) x_i.
// Column slot 0 (columns 0..15) is skipped once j >= 15, when all its columns
// are finished. The sum of squares that step j+1 needs is accumulated during
// the update, only for the slot that holds column j+1. A finished column keeps
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

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

__device__ __forceinline__ float get_row(const float2 (&a)[NQ], int i) {
  return (i & 1) ? a[i >> 1].y : a[i >> 1].x;
}

// Apply step J's reflector to one column (registers a) given the published
// column x (in shared memory at xb, rows > J valid) and the coefficients; with
// WANT_S, return in *s the sum of squares of rows > J+1 of the updated
// column. x is read twice (dot product, then update) instead of being held in
// registers across both loops.
template <int J>
__device__ __forceinline__ float2 xpair(const float* xb, int q) {
  return reinterpret_cast<const float2*>(xb)[q];
}

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
      dA = __ffma2_rn(xpair<J>(xb, q), a[q], dA);
    else
      dB = __ffma2_rn(xpair<J>(xb, q), a[q], dB);
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
    a[q] = __ffma2_rn(ng, xpair<J>(xb, q), a[q]);
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

struct PairState {
  float2 a0[NQ], a1[NQ];  // columns l and l + 16
  float s[2];             // sum of squares below the diagonal, per column slot
  float mt[2], mb[2], ms[2];  // tau, beta, scale of the columns this lane owns
};

template <int J>
__device__ __forceinline__ void step(PairState& st, float* xb0, float* xb1, int l,
                                     int half, int n) {
  if constexpr (J < NP - 1) {
    if (J >= n - 1) return;  // uniform: the last column gets tau = 0
    constexpr int owner = J & 15;
    constexpr int slot = J >> 4;
    float* xb = (J & 1) ? xb1 : xb0;
    const float2(&ac)[NQ] = slot ? st.a1 : st.a0;
    const int src = (half << 4) | owner;
    const float alpha = __shfl_sync(kFull, get_row(ac, J), src);
    const float sigma = __shfl_sync(kFull, st.s[slot], src);
    const Reflector h = make_reflector(alpha, sigma);
    if (l == owner) {
#pragma unroll
      for (int q4 = 0; q4 < NQ / 2; ++q4)
        reinterpret_cast<float4*>(xb)[q4] =
            make_float4(ac[2 * q4].x, ac[2 * q4].y, ac[2 * q4 + 1].x, ac[2 * q4 + 1].y);
      st.mt[slot] = h.tau;
      st.mb[slot] = h.beta;
      st.ms[slot] = h.scale;
    }
    __syncwarp();
    constexpr int next_slot = (J + 1) >> 4;
    if constexpr (J < 15)
      apply_step<J, next_slot == 0>(st.a0, xb, l > J, h.tau, h.scale, &st.s[0]);
    apply_step<J, next_slot == 1>(st.a1, xb, l + 16 > J, h.tau, h.scale, &st.s[1]);
    step<J + 1>(st, xb0, xb1, l, half, n);
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

// Factor matrices m0 and m0 + 1 (when < batch) with this warp.
template <bool IN_SYS, bool H_SYS, bool TAU_SYS>
__device__ __forceinline__ void factor_pair(const float* __restrict__ A, int64_t sAb, int64_t sAr,
                                            float* __restrict__ H, float* __restrict__ tau,
                                            int64_t batch, int n, int64_t m0, float* xb0,
                                            float* xb1, int half, int l) {
  const int64_t m = m0 + half;
  const bool mat_ok = m < batch;  // the odd last matrix leaves one half idle
  const int c0 = l, c1 = l + 16;

  PairState st;
  {
    const float* __restrict__ Am = A + (mat_ok ? m : m0) * sAb;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int i = 2 * q;
      const bool r0 = mat_ok && i < n, r1 = mat_ok && i + 1 < n;
      st.a0[q].x = (r0 && c0 < n) ? load_a<IN_SYS>(Am + (int64_t)i * sAr + c0) : 0.f;
      st.a0[q].y = (r1 && c0 < n) ? load_a<IN_SYS>(Am + (int64_t)(i + 1) * sAr + c0) : 0.f;
      st.a1[q].x = (r0 && c1 < n) ? load_a<IN_SYS>(Am + (int64_t)i * sAr + c1) : 0.f;
      st.a1[q].y = (r1 && c1 < n) ? load_a<IN_SYS>(Am + (int64_t)(i + 1) * sAr + c1) : 0.f;
    }
  }
  {
    float2 s2 = make_float2(st.a0[0].y * st.a0[0].y, 0.f);
#pragma unroll
    for (int q = 1; q < NQ; ++q) s2 = __ffma2_rn(st.a0[q], st.a0[q], s2);
    st.s[0] = s2.x + s2.y;
    st.s[1] = 0.f;
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) st.mt[e] = st.mb[e] = st.ms[e] = 0.f;

  step<0>(st, xb0, xb1, l, half, n);

  // Final columns: deferred scaling below the diagonal, beta on it.
  float* __restrict__ Hm = H + (mat_ok ? m : 0) * (int64_t)n * n;
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int c = slot ? c1 : c0;
    const float2(&ac)[NQ] = slot ? st.a1 : st.a0;
    const bool refl = c < n - 1;  // columns 0 .. n-2 were factored
    const float sc = st.ms[slot], be = st.mb[slot];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * q + e;
        float v = e ? ac[q].y : ac[q].x;
        if (refl) v = i > c ? v * sc : (i == c ? be : v);
        if (mat_ok && c < n && i < n) store_h<H_SYS>(Hm + (int64_t)i * n + c, v);
      }
    }
    if (mat_ok && c < n) store_h<TAU_SYS>(tau + m * n + c, st.mt[slot]);
  }
}

// 128 registers per thread (4 blocks of 4 warps per SM): config 2's 2048 warps
// fit in one wave of 148 SMs. With device memory the grid covers every pair
// and each warp factors one. IN_SYS / H_SYS / TAU_SYS: A / H / tau are mapped
// host memory; with IN_SYS or H_SYS each warp factors the pairs p, p + P,
// p + 2P, ... (P = warps in the grid), and the grid is kept small on purpose so
// that the first pairs of every warp are written back over PCIe while later
// pairs are still being read.
template <bool IN_SYS, bool H_SYS, bool TAU_SYS>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 4)
k_fused_pair(const float* __restrict__ A, int64_t sAb, int64_t sAr,
             float* __restrict__ H, float* __restrict__ tau, int64_t batch,
             int n) {
  __shared__ __align__(16) float xbuf[kWarpsPerBlock][2][2][NP];  // [warp][half][parity][row]
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;
  const int l = lane & 15;
  const int64_t pairs = (batch + 1) / 2;
  const int64_t first = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if constexpr (!IN_SYS && !H_SYS) {  // device matrices: the grid covers every pair
    if (first < pairs)
      factor_pair<false, false, TAU_SYS>(A, sAb, sAr, H, tau, batch, n, 2 * first,
                                         xbuf[warp][half][0], xbuf[warp][half][1], half, l);
  } else {
    const int64_t stride = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t p = first; p < pairs; p += stride) {
      __syncwarp();  // the previous pair's readers are done with xbuf
      factor_pair<IN_SYS, H_SYS, TAU_SYS>(A, sAb, sAr, H, tau, batch, n, 2 * p,
                                          xbuf[warp][half][0], xbuf[warp][half][1], half, l);
    }
  }
}

}  // namespace

int launch_fused_small(const float* A, int64_t sAb, int64_t sAr, float* H,
                       float* tau, int64_t batch, int n, cudaStream_t stream, HostMem where,
                       int64_t max_blocks) {
  if (n < 1 || n > kFusedMaxN) return QRB_ERR_UNSUPPORTED;
  constexpr int64_t kPerBlock = 2 * kWarpsPerBlock;
  const bool looped = where == HostMem::kAll || where == HostMem::kOutputs;
  int64_t blocks = (batch + kPerBlock - 1) / kPerBlock;
  if (!looped && blocks > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  if (looped && max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
  if (blocks > 0x7fffffffLL) blocks = 0x7fffffffLL;  // host matrices: the kernel loops
  // Per-element loads and stores: staging whole matrices through shared memory
  // with 16-byte copies measured slower here (more registers, no overlap).
  const dim3 grid((unsigned)blocks), block(kWarpsPerBlock * 32);
  switch (where) {
    case HostMem::kNone:
      k_fused_pair<false, false, false><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau, batch, n);
      break;
    case HostMem::kTau:
      k_fused_pair<false, false, true><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau, batch, n);
      break;
    case HostMem::kOutputs:
      k_fused_pair<false, true, true><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau, batch, n);
      break;
    case HostMem::kAll:
      k_fused_pair<true, true, true><<<grid, block, 0, stream>>>(A, sAb, sAr, H, tau, batch, n);
      break;
  }
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace qrb

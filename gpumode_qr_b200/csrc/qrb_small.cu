// Fused whole-matrix Householder QR for n <= 32: one warp per matrix.
//
// Mapping: lane k owns column k of its matrix in 32 registers (rows 0..31,
// zero padded beyond n). At step j lane j turns its column into the reflector
// (slarfg, coefficients computed redundantly by every lane from two shuffles),
// publishes v through a per-warp shared-memory line, and every lane k > j
// applies H_j to its own column: d = v . a_k, a_k -= tau * d * v. The sum of
// squares that step j+1 needs (rows below j+1 of column j+1) is accumulated
// while the update is applied, so each step carries no separate reduction.
//
// Semantics follow the reference's fused kernel step for step
// (src/qrbench/triton_kernels.py:676-715): slarfg coefficients (:691-700),
// rank-1 trailing update (:703-708), geqrf packing (:710-715); the last column
// has nothing below the diagonal and gets tau = 0.
#include "qrb_common.cuh"

namespace qrb {

namespace {

constexpr int NP = kFusedMaxN;  // padded matrix size (32 rows/columns)

template <int WPB>
__global__ void __launch_bounds__(WPB * 32)
k_fused_warp(const float* __restrict__ A, int64_t sAb, int64_t sAr,
             float* __restrict__ H, float* __restrict__ tau, int64_t batch,
             int n) {
  __shared__ __align__(16) float vbuf[WPB][2][NP];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t m = (int64_t)blockIdx.x * WPB + warp;
  if (m >= batch) return;  // warp-uniform

  const float* __restrict__ Am = A + m * sAb;
  const bool col_ok = lane < n;
  float a[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i)
    a[i] = (col_ok && i < n) ? __ldg(Am + (int64_t)i * sAr + lane) : 0.f;

  // Sum of squares below the diagonal for the step that consumes this column.
  float s = 0.f;
#pragma unroll
  for (int i = 1; i < NP; ++i) s = fmaf(a[i], a[i], s);

  float my_tau = 0.f;
#pragma unroll
  for (int j = 0; j < NP - 1; ++j) {
    if (j >= n - 1) break;  // uniform: the last column gets tau = 0
    float* vb = vbuf[warp][j & 1];
    const float alpha = __shfl_sync(kFull, a[j], j);
    const float sigma = __shfl_sync(kFull, s, j);
    const Reflector h = make_reflector(alpha, sigma);
    if (lane == j) {
#pragma unroll
      for (int i = j + 1; i < NP; ++i) {
        const float v = a[i] * h.scale;
        vb[i] = v;
        a[i] = v;
      }
      a[j] = h.beta;
      my_tau = h.tau;
    }
    __syncwarp();
    float v[NP];
#pragma unroll
    for (int q = (j + 1) / 4; q < NP / 4; ++q) {
      const float4 t = reinterpret_cast<const float4*>(vb)[q];
      v[4 * q + 0] = t.x;
      v[4 * q + 1] = t.y;
      v[4 * q + 2] = t.z;
      v[4 * q + 3] = t.w;
    }
    float d = a[j];
#pragma unroll
    for (int i = j + 1; i < NP; ++i) d = fmaf(v[i], a[i], d);
    const float f = (lane > j) ? h.tau * d : 0.f;
    a[j] -= f;
    s = 0.f;
#pragma unroll
    for (int i = j + 1; i < NP; ++i) {
      a[i] = fmaf(-f, v[i], a[i]);
      if (i > j + 1) s = fmaf(a[i], a[i], s);
    }
  }

  if (col_ok) {
    float* __restrict__ Hm = H + m * (int64_t)n * n;
#pragma unroll
    for (int i = 0; i < NP; ++i)
      if (i < n) Hm[(int64_t)i * n + lane] = a[i];
    tau[m * n + lane] = my_tau;
  }
}

constexpr int kWarpsPerBlock = 4;

}  // namespace

int launch_fused_small(const float* A, int64_t sAb, int64_t sAr, float* H,
                       float* tau, int64_t batch, int n, cudaStream_t stream) {
  if (n < 1 || n > kFusedMaxN) return QRB_ERR_UNSUPPORTED;
  const int64_t blocks = (batch + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  k_fused_warp<kWarpsPerBlock><<<(unsigned)blocks, kWarpsPerBlock * 32, 0, stream>>>(
      A, sAb, sAr, H, tau, batch, n);
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace qrb

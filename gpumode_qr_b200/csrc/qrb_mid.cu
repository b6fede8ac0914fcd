// Fused whole-matrix Householder QR for 32 < n <= 128: one CTA per matrix,
// one thread per column (NP = 64 or 128 threads; columns and rows beyond n are
// zero padding). The reference's champion routes n <= 128 to its fused
// one-program-per-matrix kernel (src/qrbench/variants.py:898, cap=128;
// src/qrbench/triton_kernels.py:641-720); this is that path, not the blocked
// one, so a mid-size factorization is one launch instead of 2 n / 32.
//
// Thread t keeps column t in registers as NP / 2 row pairs, plus copies of its
// diagonal element a_tt and sub-diagonal element a_(t+1)t in scalars (updated
// alongside, bit for bit). The column steps run as runtime loops in phases of
// 16 (J in [16 P, 16 P + 16)), each phase compiled with its own static row
// range (rows from 16 P: above them u is zero), so the work per step shrinks
// as the factorization proceeds. Column step J (one block barrier):
//   owner t = J  forms the reflector from alpha = a_JJ and sigma (its
//                look-ahead sum), and publishes u with u_i = 0 above J,
//                u_J = alpha - beta and u_i = x_i below J (so v = scale * u)
//                into one of two shared buffers, plus tau and scale;
//   all t > J    d = scale * sum_i u_i a_i,  a_i -= (tau d scale) u_i over the
//                whole padded row range (rows above J see u_i = 0, row J
//                loses tau d), with the packed FP32x2 FMA;
//   thread J+1   keeps sigma_(J+1) = sum_{i > J+1} a_i^2 for the next step,
//                accumulated (by every thread, for its own column) inside
//                the update loop.
// The owner writes u with 16-byte stores of its row pairs from the group that
// holds row J + 1 on, then fixes rows J-3 .. J with scalar stores (zeros and
// alpha - beta), so the buffer holds zeros above J without a runtime index
// into the register array. A finished column keeps x unscaled; it is scaled
// once when H is stored (deferred scaling), with beta on the diagonal.
#include <type_traits>

#include "qrb_common.cuh"

namespace qrb {

namespace {

template <int NP>
__global__ void __launch_bounds__(NP)
k_fused_cta(const float* __restrict__ A, int64_t sAb, int64_t sAr, float* __restrict__ H,
            float* __restrict__ tau_out, int n) {
  constexpr int NQ = NP / 2;
  __shared__ __align__(16) float ubuf[2][NP];
  __shared__ float coef[2][2];  // [parity][tau, scale]
  __shared__ float mt[NP], mb[NP], ms[NP];
  const int t = threadIdx.x;
  const int64_t m = blockIdx.x;
  const float* __restrict__ Am = A + m * sAb;

  // zero both u buffers (the owner only rewrites what changes, see above)
  for (int e = t; e < 2 * NP; e += NP) (&ubuf[0][0])[e] = 0.f;
  mt[t] = 0.f;
  mb[t] = 0.f;
  ms[t] = 0.f;

  float2 a[NQ];
  const bool col = t < n;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int i = 2 * q;
    a[q].x = (col && i < n) ? __ldg(Am + (int64_t)i * sAr + t) : 0.f;
    a[q].y = (col && i + 1 < n) ? __ldg(Am + (int64_t)(i + 1) * sAr + t) : 0.f;
  }
  float diag = (col && t < n) ? __ldg(Am + (int64_t)t * sAr + t) : 0.f;
  float sub = (col && t + 1 < n) ? __ldg(Am + (int64_t)(t + 1) * sAr + t) : 0.f;

  // sigma of this thread's column below its diagonal: pairs past the one
  // holding row t, plus row t + 1 when it shares that pair with row t.
  // (pairs before QS are known to lie at or above the diagonal: t >= 2 QS)
  auto below_diag_sumsq = [&](auto qs) {
    constexpr int QS = decltype(qs)::value;
    const int q0 = t >> 1;
    float2 s2 = make_float2(0.f, 0.f), s3 = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = QS; q < NQ; ++q) {
      if (q > q0) {
        if (q & 1)
          s3 = __ffma2_rn(a[q], a[q], s3);
        else
          s2 = __ffma2_rn(a[q], a[q], s2);
      }
    }
    float s = (s2.x + s2.y) + (s3.x + s3.y);
    if ((t & 1) == 0) s = fmaf(sub, sub, s);
    return s;
  };
  float sig = (t == 0) ? below_diag_sumsq(std::integral_constant<int, 0>{}) : 0.f;
  __syncthreads();  // buffers zeroed before the first owner writes

  // Column steps in phases of 16: in phase P every step has J >= 16 P, so rows
  // above 16 P hold u = 0 and are skipped at compile time (row pairs from 8 P,
  // 16-byte groups from 4 P); the skipped terms were exact zeros.
  auto phase = [&](auto pc) {
    constexpr int P = decltype(pc)::value;
    if constexpr (P < NP / 16) {
      constexpr int QS = 8 * P;  // first row pair
      constexpr int GS = 4 * P;  // first 4-row group
      const int j_end = min(16 * (P + 1), n - 1);
#pragma unroll 1
      for (int J = 16 * P; J < j_end; ++J) {
        const int par = J & 1;
        float* ub = ubuf[par];
        if (t == J) {
          const Reflector h = make_reflector(diag, sig);
          const float ujj = diag - h.beta;
          const unsigned us = (unsigned)__cvta_generic_to_shared(ub);
          // rows from the 4-group holding row J + 1 on (the group may include
          // rows <= J; they are fixed below)
#pragma unroll
          for (int g = GS; g < NP / 4; ++g) {
            const unsigned on = (4 * g + 3 > J) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %0, 0;\n\t"
                "@p st.shared.v4.f32 [%1], {%2, %3, %4, %5};\n\t}\n" ::"r"(on),
                "r"(us + 16u * g), "f"(a[2 * g].x), "f"(a[2 * g].y), "f"(a[2 * g + 1].x),
                "f"(a[2 * g + 1].y)
                : "memory");
          }
          // rows J-3 .. J-1 to zero (stale from two steps ago or written
          // above), row J to alpha - beta
#pragma unroll
          for (int d = 3; d >= 1; --d)
            if (J - d >= 0) ub[J - d] = 0.f;
          ub[J] = ujj;
          coef[par][0] = h.tau;
          coef[par][1] = h.scale;
          mt[J] = h.tau;
          mb[J] = h.beta;
          ms[J] = h.scale;
        }
        __syncthreads();
        const float tau = coef[par][0];
        const float scale = coef[par][1];
        float2 d0 = make_float2(0.f, 0.f), d1 = d0, d2 = d0, d3 = d0;
#pragma unroll
        for (int g = GS; g < NQ / 2; ++g) {
          const float4 u = reinterpret_cast<const float4*>(ub)[g];
          if (g & 1) {
            d2 = __ffma2_rn(make_float2(u.x, u.y), a[2 * g], d2);
            d3 = __ffma2_rn(make_float2(u.z, u.w), a[2 * g + 1], d3);
          } else {
            d0 = __ffma2_rn(make_float2(u.x, u.y), a[2 * g], d0);
            d1 = __ffma2_rn(make_float2(u.z, u.w), a[2 * g + 1], d1);
          }
        }
        const float dsum = ((d0.x + d0.y) + (d1.x + d1.y)) + ((d2.x + d2.y) + (d3.x + d3.y));
        const float f = (t > J && col) ? tau * (scale * dsum) : 0.f;
        const float ng = -(f * scale);
        const float2 ng2 = make_float2(ng, ng);
        // the next owner's norm below its diagonal (pairs past t / 2, plus
        // row t + 1 for even t), accumulated as the pairs are updated, in the
        // order of below_diag_sumsq; every thread computes it, thread J + 1
        // keeps it
        const int q0 = t >> 1;
        float2 s2 = make_float2(0.f, 0.f), s3 = make_float2(0.f, 0.f);
#pragma unroll
        for (int g = GS; g < NQ / 2; ++g) {
          const float4 u = reinterpret_cast<const float4*>(ub)[g];
          a[2 * g] = __ffma2_rn(ng2, make_float2(u.x, u.y), a[2 * g]);
          a[2 * g + 1] = __ffma2_rn(ng2, make_float2(u.z, u.w), a[2 * g + 1]);
          if (2 * g > q0) s2 = __ffma2_rn(a[2 * g], a[2 * g], s2);
          if (2 * g + 1 > q0) s3 = __ffma2_rn(a[2 * g + 1], a[2 * g + 1], s3);
        }
        diag = fmaf(ng, ub[t], diag);
        if (t + 1 < NP) sub = fmaf(ng, ub[t + 1], sub);
        if (t == J + 1) {
          float sq = (s2.x + s2.y) + (s3.x + s3.y);
          if ((t & 1) == 0) sq = fmaf(sub, sub, sq);
          sig = sq;
        }
      }
    }
  };
  phase(std::integral_constant<int, 0>{});
  phase(std::integral_constant<int, 1>{});
  phase(std::integral_constant<int, 2>{});
  phase(std::integral_constant<int, 3>{});
  phase(std::integral_constant<int, 4>{});
  phase(std::integral_constant<int, 5>{});
  phase(std::integral_constant<int, 6>{});
  phase(std::integral_constant<int, 7>{});
  __syncthreads();

  // H: R above the diagonal, beta on it, v = scale * x below; tau.
  if (col) {
    float* __restrict__ Hm = H + m * (int64_t)n * n;
    const bool refl = t < n - 1;
    const float sc = ms[t], be = mb[t];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * q + e;
        if (i < n) {
          float v = e ? a[q].y : a[q].x;
          if (refl) v = i > t ? v * sc : (i == t ? be : v);
          Hm[(int64_t)i * n + t] = v;
        }
      }
    }
    tau_out[m * n + t] = mt[t];
  }
}

}  // namespace

int launch_fused_mid(const float* A, int64_t sAb, int64_t sAr, float* H, float* tau,
                     int64_t batch, int n, cudaStream_t stream) {
  if (n <= kFusedMaxN || n > kFusedMidMaxN) return QRB_ERR_UNSUPPORTED;
  constexpr int64_t kMaxGrid = 0x7fffffffLL;
  for (int64_t b0 = 0; b0 < batch; b0 += kMaxGrid) {
    const int64_t nb = batch - b0 < kMaxGrid ? batch - b0 : kMaxGrid;
    if (n <= 64)
      k_fused_cta<64><<<(unsigned)nb, 64, 0, stream>>>(A + b0 * sAb, sAb, sAr,
                                                         H + b0 * (int64_t)n * n, tau + b0 * n, n);
    else
      k_fused_cta<128><<<(unsigned)nb, 128, 0, stream>>>(A + b0 * sAb, sAb, sAr,
                                                           H + b0 * (int64_t)n * n, tau + b0 * n,
                                                           n);
    note_launches(1);
    if (cudaGetLastError() != cudaSuccess) return QRB_ERR_LAUNCH;
  }
  return QRB_OK;
}

}  // namespace qrb

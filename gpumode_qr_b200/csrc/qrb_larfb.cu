// Block-reflector trailing update C <- C - V (T^T (V^T C)), FP32 FFMA.
//
// One CTA (256 threads) owns one matrix's r x 64 column tile of C and runs the
// three products of the reference's trailing update (src/qrbench/variants.py
// :800-804, W1 = V^T C, W2 = T^T W1, C -= V W2) without writing the k x 64
// intermediate to global memory:
//   pass 1  W = V^T C over all r rows: 96-row chunks of V and C double-buffered
//           into shared memory with cp.async; each warp takes every 8th row
//           and each lane accumulates an 8 x 8 register block of W (32 packed
//           FP32x2 FMAs per four 16-byte shared loads); the eight warp
//           partials are summed, then W <- T^T W is formed;
//   pass 2  C -= V W over 256-row chunks: each thread updates an 8-row x
//           8-column block of C in registers with packed FMAs (columns c, c+1,
//           c+2, c+3 and c+32..c+35, so that a warp's global loads and stores
//           cover whole 128-byte rows). With 16-byte aligned operands V is
//           staged row-major by cp.async (double-buffered, the first chunk
//           requested before W <- T^T W; 16-byte units swizzled by row group)
//           and W is stored negated; otherwise V is staged transposed and
//           negated through registers.
// V is read through its strictly lower part only: the diagonal is taken as 1
// and everything above it as 0 (so V can point into a packed H), columns at or
// beyond k as 0.
#include "qrb_common.cuh"
#include "qrb_tc.cuh"

#include <type_traits>

namespace qrb {

namespace {

constexpr int K = 32;        // reflectors per block (padded)
constexpr int TC = 64;       // columns of C per CTA
constexpr int NT = 256;      // threads per CTA (8 warps)
constexpr int NW = NT / 32;
constexpr int RC1 = 96;      // rows per pass-1 chunk
constexpr int RC2 = 256;     // rows per pass-2 chunk
constexpr int VS_LD = K + 4;     // pass-1 V chunk row stride (floats)
constexpr int CS_LD = TC + 4;    // pass-1 C chunk row stride
constexpr int VT_LD = RC2 + 4;   // pass-2 transposed V row stride
constexpr int WS_LD = TC + 4;    // W row stride
constexpr int T_LD = K + 1;

struct __align__(16) Stage {
  float Vs[2][RC1 * VS_LD];
  float Cs[2][RC1 * CS_LD];
};
struct __align__(16) Smem {
  union {
    Stage st;                 // pass 1 staging
    float Wp[NW][K * TC];     // per-warp partial W (after pass 1)
    float Vt[K * VT_LD];      // pass 2 transposed V chunk (unaligned operands)
    float Vr[2][RC2 * K];     // pass 2 V chunks as loaded, 16-byte units swizzled
  } u;
  float Ws[K * WS_LD];
  float Ts[K * T_LD];
};

// Tensor-core pass 2 (TCP2): D (128 rows x 64 columns, TMEM) = V_chunk W' as
// kind::tf32 MMAs in 3xTF32, both operands K-major without swizzle: A = the
// V chunk, 16-byte units (k-quad kq, row m) at kq * 2048 + m * 16; B = W'^T,
// units (kq, column n) at kq * 1024 + n * 16.
constexpr int R2T = 128;                    // rows per tensor-core chunk (MMA M)
constexpr int A2T_BYTES = R2T * K * 4;      // 16 KiB per hi / lo part
constexpr int B2T_BYTES = TC * K * 4;       // 8 KiB per hi / lo part
constexpr uint32_t IDESC_P2 = tc::idesc(R2T, TC, false, false);
constexpr uint32_t TM_COLS_P2 = 2 * TC;     // two 64-column accumulators
struct __align__(1024) SmemTc {
  union {
    Stage st;
    float Wp[NW][K * TC];
    unsigned char A[2][2][A2T_BYTES];       // [buffer][hi, lo]
    float Vr[2][RC2 * K];                   // (FFMA pass 2 only; keeps one code path)
  } u;
  unsigned char B[2][B2T_BYTES];            // [hi, lo]
  float Ws[K * WS_LD];
  float Ts[K * T_LD];
  uint64_t bar[3];                          // [0,1] accumulators, [2] drain after an abort
  int abort;
  uint32_t tmem;
};

__device__ __forceinline__ void cp_async16(void* s, const void* g, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(g), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* s, const void* g, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  const int sz = valid ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(g), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Value of the implicit reflector matrix at (row i, column a) given the stored
// element x: unit diagonal, zero above, zero for columns >= k.
__device__ __forceinline__ float vmask(float x, int i, int a, int k) {
  return (a >= k || i < a) ? 0.f : (i == a ? 1.f : x);
}

// Pass 2 on the tensor cores: W' (in Ws, 32 x 64) becomes the B operand; per
// 128-row chunk of V (staged, masked, split) one elected thread issues 4
// k-steps x 3 MMAs into one of two TMEM accumulators and commits them to an
// mbarrier; the previous chunk's accumulator is read back (warp w: TMEM lanes
// 32 (w % 4) .., columns 32 (w / 4) ..) and subtracted from C.
__device__ __forceinline__ void pass2_tc(SmemTc& sm, const float* __restrict__ Vm, int64_t ldv,
                                         const float* __restrict__ Cm, int64_t ldcs,
                                         float* __restrict__ Dm, int64_t ldcd, int r, int c,
                                         int c0, int tid, int warp, int lane,
                                         int* __restrict__ err) {
  __syncthreads();  // W' complete in Ws; the pass-1 partials (aliased by A) consumed
  // B = W'^T, K-major, split
#pragma unroll
  for (int e = 0; e < (K / 4) * TC / NT; ++e) {
    const int u = tid + e * NT;
    const int kq = u / TC, n = u % TC;
    const float4 w = make_float4(sm.Ws[(4 * kq + 0) * WS_LD + n], sm.Ws[(4 * kq + 1) * WS_LD + n],
                                 sm.Ws[(4 * kq + 2) * WS_LD + n], sm.Ws[(4 * kq + 3) * WS_LD + n]);
    float4 hi, lo;
    tc::split4(w, hi, lo);
    *reinterpret_cast<float4*>(sm.B[0] + u * 16) = hi;
    *reinterpret_cast<float4*>(sm.B[1] + u * 16) = lo;
  }
  const uint32_t tmem = sm.tmem;
  uint32_t ph[2] = {0u, 0u};
  const uint32_t bar0 = tc::smem_u32(&sm.bar[0]);
  volatile int* abort = &sm.abort;
  const int nch = (r + R2T - 1) / R2T;

  // The previous chunk's C rows are loaded before waiting for its MMAs, and
  // the next chunk's V rows while the epilogue runs (register prefetch).
  auto epilogue = [&](int cp) {
    const int s = cp & 1;
    const int q = warp & 3, h = warp >> 2;
    const int i = cp * R2T + 32 * q + lane;
    const bool row_ok = i < r;
    const float* src = Cm + (int64_t)(row_ok ? i : 0) * ldcs + c0 + 32 * h;
    float4 cv[8];
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4)
      cv[j4] = (row_ok && c0 + 32 * h + 4 * j4 < c) ? *reinterpret_cast<const float4*>(src + 4 * j4)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    tc::mbar_wait(bar0 + 8 * s, ph[s], err, abort);
    ph[s] ^= 1u;
    if (__any_sync(tc::kFullMask, *abort != 0)) return;  // no TMEM reads, no stores
    tc::fence_after();
    float d[32];
    tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + s * TC + 32 * h, d);
    if (row_ok) {
      float* dst = Dm + (int64_t)i * ldcd + c0 + 32 * h;
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        if (c0 + 32 * h + 4 * j4 < c) {
          float4 v = cv[j4];
          v.x -= d[4 * j4 + 0];
          v.y -= d[4 * j4 + 1];
          v.z -= d[4 * j4 + 2];
          v.w -= d[4 * j4 + 3];
          *reinterpret_cast<float4*>(dst + 4 * j4) = v;
        }
      }
    }
    tc::fence_before();
  };

  constexpr int kUnits = (R2T * K / 4) / NT;  // 16-byte V units per thread per chunk
  float4 vpre[kUnits];
  auto load_v = [&](int ch) {
#pragma unroll
    for (int e = 0; e < kUnits; ++e) {
      const int u = tid + e * NT;
      const int i = ch * R2T + (u & (R2T - 1));
      vpre[e] = i < r ? __ldg(reinterpret_cast<const float4*>(Vm + (int64_t)i * ldv + 4 * (u >> 7)))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  load_v(0);
  for (int ch = 0; ch < nch; ++ch) {
    const int s = ch & 1;
    // A = V rows ch*128 .., masked (unit diagonal, zero above) and split. The
    // buffer was last read by the MMAs of chunk ch - 2, which the epilogue of
    // the previous iteration waited for.
#pragma unroll
    for (int e = 0; e < kUnits; ++e) {
      const int u = tid + e * NT;
      const int i = ch * R2T + (u & (R2T - 1)), kq = u >> 7;
      float4 v = vpre[e];
      v.x = tc::vmask(v.x, i, 4 * kq + 0);
      v.y = tc::vmask(v.y, i, 4 * kq + 1);
      v.z = tc::vmask(v.z, i, 4 * kq + 2);
      v.w = tc::vmask(v.w, i, 4 * kq + 3);
      float4 hi, lo;
      tc::split4(v, hi, lo);
      *reinterpret_cast<float4*>(sm.u.A[s][0] + u * 16) = hi;
      *reinterpret_cast<float4*>(sm.u.A[s][1] + u * 16) = lo;
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    if (tid == 0 && *abort == 0) {
      tc::fence_after();
      const uint32_t a_hi = tc::smem_u32(sm.u.A[s][0]), a_lo = tc::smem_u32(sm.u.A[s][1]);
      const uint32_t b_hi = tc::smem_u32(sm.B[0]), b_lo = tc::smem_u32(sm.B[1]);
      const uint32_t dacc = tmem + s * TC;
#pragma unroll
      for (int ks = 0; ks < K / 8; ++ks) {
        const uint64_t ah = tc::sdesc(a_hi + ks * 4096, 2048, 128);
        const uint64_t al = tc::sdesc(a_lo + ks * 4096, 2048, 128);
        const uint64_t bh = tc::sdesc(b_hi + ks * 2048, 1024, 128);
        const uint64_t bl = tc::sdesc(b_lo + ks * 2048, 1024, 128);
        tc::mma_tf32(dacc, ah, bh, IDESC_P2, ks != 0 ? 1u : 0u);
        tc::mma_tf32(dacc, ah, bl, IDESC_P2, 1u);
        tc::mma_tf32(dacc, al, bh, IDESC_P2, 1u);
      }
      tc::mma_commit(bar0 + 8 * s);
    }
    if (ch + 1 < nch) load_v(ch + 1);
    if (ch >= 1) epilogue(ch - 1);
  }
  epilogue(nch - 1);
  __syncthreads();
  if (tid == 0 && *abort != 0) tc::drain_mmas(bar0 + 8 * 2);
  __syncthreads();
  tc::fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TM_COLS_P2)
                 : "memory");
}

// TCP2 (with VEC): pass 2 on the tensor cores (tcgen05, 3xTF32) instead of
// FFMA; err receives a bounded mbarrier wait's timeout.
template <bool VEC, bool TCP2>
__global__ void __launch_bounds__(NT, 2)
k_larfb(const float* __restrict__ V, int64_t sVb, int64_t ldv,
        const float* __restrict__ T, int64_t sTb, int t_ld,
        const float* __restrict__ Csrc, int64_t sCsb, int64_t ldcs,
        float* __restrict__ Cdst, int64_t sCdb, int64_t ldcd, int r, int k,
        int c, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  using SM = typename std::conditional<TCP2, SmemTc, Smem>::type;
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t m = blockIdx.y;
  const int c0 = blockIdx.x * TC;
  const float* __restrict__ Vm = V + m * sVb;
  const float* __restrict__ Cm = Csrc + m * sCsb;
  float* __restrict__ Dm = Cdst + m * sCdb;

  for (int e = tid; e < K * K; e += NT) {
    const int i = e / K, a = e % K;
    sm.Ts[i * T_LD + a] = (i < k && a < k) ? __ldg(T + m * sTb + (int64_t)i * t_ld + a) : 0.f;
  }
  if constexpr (TCP2) {
    if (warp == 0) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       tc::smem_u32(&sm.tmem)),
                   "r"(TM_COLS_P2)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
      for (int b = 0; b < 3; ++b)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc::smem_u32(&sm.bar[b])),
                     "r"(1)
                     : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      sm.abort = 0;
    }
  }

  // ---------------- pass 1: W = V^T C ----------------
  const int wa = (lane >> 3) << 3;  // W rows wa..wa+7
  const int wc = (lane & 7) << 2;   // W cols wc..wc+3 and wc+32..wc+35
  // acc[x][j]: W(wa + x, column pair j) with pairs (wc, wc+1), (wc+2, wc+3),
  // (wc+32, wc+33), (wc+34, wc+35), updated with the packed FP32x2 FMA.
  float2 acc[8][4];
#pragma unroll
  for (int x = 0; x < 8; ++x)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[x][j] = make_float2(0.f, 0.f);

  const int nch = (r + RC1 - 1) / RC1;
  auto load_chunk = [&](int ch, int buf) {
    const int i0 = ch * RC1;
    if (VEC) {
#pragma unroll
      for (int e = 0; e < (RC1 * K) / (4 * NT); ++e) {  // V: 64 x 32 = 512 float4
        const int idx = tid + e * NT;
        const int row = idx >> 3, c4 = (idx & 7) << 2;
        const int i = i0 + row;
        const bool ok = i < r;
        const float* g = ok ? Vm + (int64_t)i * ldv + c4 : Vm;
        cp_async16(&sm.u.st.Vs[buf][row * VS_LD + c4], g, ok);
      }
#pragma unroll
      for (int e = 0; e < (RC1 * TC) / (4 * NT); ++e) {  // C: 64 x 64 = 1024 float4
        const int idx = tid + e * NT;
        const int row = idx >> 4, c4 = (idx & 15) << 2;
        const int i = i0 + row, col = c0 + c4;
        const bool ok = i < r && col < c;
        const float* g = ok ? Cm + (int64_t)i * ldcs + col : Cm;
        cp_async16(&sm.u.st.Cs[buf][row * CS_LD + c4], g, ok);
      }
    } else {
#pragma unroll 4
      for (int e = 0; e < (RC1 * K) / NT; ++e) {
        const int idx = tid + e * NT;
        const int row = idx >> 5, col = idx & 31;
        const int i = i0 + row;
        const bool ok = i < r && col < k;
        const float* g = ok ? Vm + (int64_t)i * ldv + col : Vm;
        cp_async4(&sm.u.st.Vs[buf][row * VS_LD + col], g, ok);
      }
#pragma unroll 4
      for (int e = 0; e < (RC1 * TC) / NT; ++e) {
        const int idx = tid + e * NT;
        const int row = idx >> 6, cc = idx & 63;
        const int i = i0 + row, col = c0 + cc;
        const bool ok = i < r && col < c;
        const float* g = ok ? Cm + (int64_t)i * ldcs + col : Cm;
        cp_async4(&sm.u.st.Cs[buf][row * CS_LD + cc], g, ok);
      }
    }
    cp_async_commit();
  };

  load_chunk(0, 0);
  for (int ch = 0; ch < nch; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < nch) {
      load_chunk(ch + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (ch == 0 || k < K) {  // unit-lower mask on the top rows, zero cols >= k
      const int i0 = ch * RC1;
      for (int e = tid; e < RC1 * K; e += NT) {
        const int row = e / K, a = e % K;
        const int i = i0 + row;
        if (a >= k || i <= a) {
          float& s = sm.u.st.Vs[buf][row * VS_LD + a];
          s = vmask(s, i, a, k);
        }
      }
      __syncthreads();
    }
    const float* vb = sm.u.st.Vs[buf];
    const float* cb = sm.u.st.Cs[buf];
#pragma unroll 2
    for (int rr = warp; rr < RC1; rr += NW) {
      const float4 v0 = *reinterpret_cast<const float4*>(vb + rr * VS_LD + wa);
      const float4 v1 = *reinterpret_cast<const float4*>(vb + rr * VS_LD + wa + 4);
      const float4 ca = *reinterpret_cast<const float4*>(cb + rr * CS_LD + wc);
      const float4 cbv = *reinterpret_cast<const float4*>(cb + rr * CS_LD + wc + 32);
      const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      const float2 cp[4] = {make_float2(ca.x, ca.y), make_float2(ca.z, ca.w),
                            make_float2(cbv.x, cbv.y), make_float2(cbv.z, cbv.w)};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const float2 vx = make_float2(vv[x], vv[x]);
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[x][j] = __ffma2_rn(vx, cp[j], acc[x][j]);
      }
    }
    __syncthreads();
  }

  // per-warp partials of W (the staging area is free now)
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    float* row = &sm.u.Wp[warp][(wa + x) * TC];
    *reinterpret_cast<float4*>(row + wc) =
        make_float4(acc[x][0].x, acc[x][0].y, acc[x][1].x, acc[x][1].y);
    *reinterpret_cast<float4*>(row + wc + 32) =
        make_float4(acc[x][2].x, acc[x][2].y, acc[x][3].x, acc[x][3].y);
  }
  __syncthreads();

  // ---------------- W <- T^T (sum of partials) ----------------
  // Sum the eight warp partials (8 consecutive W entries per thread, 16-byte
  // loads), into Ws; then each thread forms 8 rows of one column of T^T W.
  {
    const int e0 = tid * 8;  // W entries e0..e0+7 (row e0 / TC)
    float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
#pragma unroll
    for (int w2 = 0; w2 < NW; ++w2) {
      const float4 p0 = *reinterpret_cast<const float4*>(&sm.u.Wp[w2][e0]);
      const float4 p1 = *reinterpret_cast<const float4*>(&sm.u.Wp[w2][e0 + 4]);
      s0.x += p0.x; s0.y += p0.y; s0.z += p0.z; s0.w += p0.w;
      s1.x += p1.x; s1.y += p1.y; s1.z += p1.z; s1.w += p1.w;
    }
    float* ws = &sm.Ws[(e0 / TC) * WS_LD + (e0 % TC)];
    *reinterpret_cast<float4*>(ws) = s0;
    *reinterpret_cast<float4*>(ws + 4) = s1;
  }
  __syncthreads();
  // Pass 2 (FFMA, aligned operands) stages V row-major with cp.async: row i of
  // a chunk keeps its eight 16-byte units at positions u ^ ((i / 8) % 8), so
  // that the eight-row groups a warp reads at once fall on distinct banks.
  // The first chunk is requested here, before T^T W (the partials are summed).
  auto issue_v2 = [&](int i0, int buf) {
#pragma unroll
    for (int e = 0; e < (RC2 * K) / (4 * NT); ++e) {
      const int idx = tid + e * NT;
      const int row = idx >> 3, u = idx & 7;
      const int i = i0 + row;
      const bool ok = i < r;
      const float* g = ok ? Vm + (int64_t)i * ldv + 4 * u : Vm;
      cp_async16(&sm.u.Vr[buf][row * K + ((u ^ ((row >> 3) & 7)) << 2)], g, ok);
    }
    cp_async_commit();
  };
  constexpr bool kRowMajorP2 = VEC && !TCP2;
  if constexpr (kRowMajorP2) issue_v2(0, 0);
  {
    const int cc = tid & 63;
    const int ab = (tid >> 6) << 3;
    float o[8];
#pragma unroll
    for (int x = 0; x < 8; ++x) o[x] = 0.f;
#pragma unroll 4
    for (int q = 0; q < K; ++q) {
      const float wq = sm.Ws[q * WS_LD + cc];
#pragma unroll
      for (int x = 0; x < 8; ++x) o[x] = fmaf(sm.Ts[q * T_LD + ab + x], wq, o[x]);
    }
    __syncthreads();  // every thread has read the sums in Ws
    // stored negated for the row-major pass 2 (C += V (-W') is a plain FMA)
    const float sg = kRowMajorP2 ? -1.f : 1.f;
#pragma unroll
    for (int x = 0; x < 8; ++x) sm.Ws[(ab + x) * WS_LD + cc] = sg * o[x];
  }

  if constexpr (TCP2) {
    pass2_tc(sm, Vm, ldv, Cm, ldcs, Dm, ldcd, r, c, c0, tid, warp, lane, err);
  } else if constexpr (kRowMajorP2) {
  // ---------------- pass 2: C += V (-W'), V row-major ----------------
  const int rg = (tid >> 3) << 3;   // chunk rows rg..rg+7
  const int cq = (tid & 7) << 2;    // tile cols cq..cq+3 and cq+32..cq+35
  const int sw = (tid >> 3) & 7;    // swizzle of rows rg..rg+7
  const int colA = c0 + cq, colB = c0 + cq + 32;
  int it = 0;
  for (int i0 = 0; i0 < r; i0 += RC2, ++it) {
    const int buf = it & 1;
    __syncthreads();  // W' ready (first) / the other V buffer consumed (later)
    if (i0 + RC2 < r) {
      issue_v2(i0 + RC2, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    float2 cv[8][4];
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      const int i = i0 + rg + x;
      const float* g = Cm + (int64_t)i * ldcs;
      float4 ta = make_float4(0.f, 0.f, 0.f, 0.f), tb = ta;
      if (i < r && colA < c) ta = *reinterpret_cast<const float4*>(g + colA);
      if (i < r && colB < c) tb = *reinterpret_cast<const float4*>(g + colB);
      cv[x][0] = make_float2(ta.x, ta.y); cv[x][1] = make_float2(ta.z, ta.w);
      cv[x][2] = make_float2(tb.x, tb.y); cv[x][3] = make_float2(tb.z, tb.w);
    }
    __syncthreads();  // this chunk of V has landed for every thread
    if (i0 == 0) {  // unit-lower mask on the top rows (k == 32 here)
      for (int e = tid; e < K * K; e += NT) {
        const int row = e >> 5, a = e & 31;
        if (row <= a)
          sm.u.Vr[buf][row * K + (((a >> 2) ^ ((row >> 3) & 7)) << 2) + (a & 3)] =
              row == a ? 1.f : 0.f;
      }
      __syncthreads();
    }
    const float* vb = sm.u.Vr[buf];
#pragma unroll 2
    for (int a4 = 0; a4 < K / 4; ++a4) {
      float4 vq[8];
#pragma unroll
      for (int x = 0; x < 8; ++x)
        vq[x] = *reinterpret_cast<const float4*>(vb + (rg + x) * K + ((a4 ^ sw) << 2));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int a = 4 * a4 + u;
        const float4 wA = *reinterpret_cast<const float4*>(&sm.Ws[a * WS_LD + cq]);
        const float4 wB = *reinterpret_cast<const float4*>(&sm.Ws[a * WS_LD + cq + 32]);
        const float2 wp[4] = {make_float2(wA.x, wA.y), make_float2(wA.z, wA.w),
                              make_float2(wB.x, wB.y), make_float2(wB.z, wB.w)};
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const float v = u == 0 ? vq[x].x : u == 1 ? vq[x].y : u == 2 ? vq[x].z : vq[x].w;
          const float2 vx = make_float2(v, v);
#pragma unroll
          for (int j = 0; j < 4; ++j) cv[x][j] = __ffma2_rn(vx, wp[j], cv[x][j]);
        }
      }
    }
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      const int i = i0 + rg + x;
      if (i >= r) continue;
      float* g = Dm + (int64_t)i * ldcd;
      if (colA < c)
        *reinterpret_cast<float4*>(g + colA) =
            make_float4(cv[x][0].x, cv[x][0].y, cv[x][1].x, cv[x][1].y);
      if (colB < c)
        *reinterpret_cast<float4*>(g + colB) =
            make_float4(cv[x][2].x, cv[x][2].y, cv[x][3].x, cv[x][3].y);
    }
  }
  } else {
  // ---------------- pass 2: C -= V W ----------------
  const int rg = (tid >> 3) << 3;   // chunk rows rg..rg+7
  const int cq = (tid & 7) << 2;    // tile cols cq..cq+3 and cq+32..cq+35
  const int colA = c0 + cq, colB = c0 + cq + 32;
  for (int i0 = 0; i0 < r; i0 += RC2) {
    __syncthreads();  // Ws ready and partials consumed (first) / Vt free (later)
    // Stage V rows i0..i0+255 transposed: Vt[a][row].
#pragma unroll 2
    for (int e = 0; e < (RC2 * K) / (4 * NT); ++e) {
      const int idx = tid + e * NT;
      const int row = idx & (RC2 - 1), c4 = (idx / RC2) << 2;
      const int i = i0 + row;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < r) {
        const float* g = Vm + (int64_t)i * ldv + c4;
        if (VEC) {
          t = __ldg(reinterpret_cast<const float4*>(g));
        } else {
          t.x = c4 + 0 < k ? __ldg(g + 0) : 0.f;
          t.y = c4 + 1 < k ? __ldg(g + 1) : 0.f;
          t.z = c4 + 2 < k ? __ldg(g + 2) : 0.f;
          t.w = c4 + 3 < k ? __ldg(g + 3) : 0.f;
        }
      }
      // stored negated: the update below is then a plain FMA
      sm.u.Vt[(c4 + 0) * VT_LD + row] = -vmask(t.x, i, c4 + 0, k);
      sm.u.Vt[(c4 + 1) * VT_LD + row] = -vmask(t.y, i, c4 + 1, k);
      sm.u.Vt[(c4 + 2) * VT_LD + row] = -vmask(t.z, i, c4 + 2, k);
      sm.u.Vt[(c4 + 3) * VT_LD + row] = -vmask(t.w, i, c4 + 3, k);
    }
    // cv[x][j]: C(i0 + rg + x, column pair j), pairs as for pass 1
    float2 cv[8][4];
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      const int i = i0 + rg + x;
      const float* g = Cm + (int64_t)i * ldcs;
      if (VEC) {
        float4 ta = make_float4(0.f, 0.f, 0.f, 0.f), tb = ta;
        if (i < r && colA < c) ta = *reinterpret_cast<const float4*>(g + colA);
        if (i < r && colB < c) tb = *reinterpret_cast<const float4*>(g + colB);
        cv[x][0] = make_float2(ta.x, ta.y); cv[x][1] = make_float2(ta.z, ta.w);
        cv[x][2] = make_float2(tb.x, tb.y); cv[x][3] = make_float2(tb.z, tb.w);
      } else {
        float t8[8];
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          t8[y] = (i < r && colA + y < c) ? g[colA + y] : 0.f;
          t8[4 + y] = (i < r && colB + y < c) ? g[colB + y] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) cv[x][j] = make_float2(t8[2 * j], t8[2 * j + 1]);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int a = 0; a < K; ++a) {
      const float4 wA = *reinterpret_cast<const float4*>(&sm.Ws[a * WS_LD + cq]);
      const float4 wB = *reinterpret_cast<const float4*>(&sm.Ws[a * WS_LD + cq + 32]);
      const float4 v0 = *reinterpret_cast<const float4*>(&sm.u.Vt[a * VT_LD + rg]);
      const float4 v1 = *reinterpret_cast<const float4*>(&sm.u.Vt[a * VT_LD + rg + 4]);
      const float nv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      const float2 wp[4] = {make_float2(wA.x, wA.y), make_float2(wA.z, wA.w),
                            make_float2(wB.x, wB.y), make_float2(wB.z, wB.w)};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const float2 vx = make_float2(nv[x], nv[x]);
#pragma unroll
        for (int j = 0; j < 4; ++j) cv[x][j] = __ffma2_rn(vx, wp[j], cv[x][j]);
      }
    }
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      const int i = i0 + rg + x;
      if (i >= r) continue;
      float* g = Dm + (int64_t)i * ldcd;
      if (VEC) {
        if (colA < c)
          *reinterpret_cast<float4*>(g + colA) =
              make_float4(cv[x][0].x, cv[x][0].y, cv[x][1].x, cv[x][1].y);
        if (colB < c)
          *reinterpret_cast<float4*>(g + colB) =
              make_float4(cv[x][2].x, cv[x][2].y, cv[x][3].x, cv[x][3].y);
      } else {
        const float t8[8] = {cv[x][0].x, cv[x][0].y, cv[x][1].x, cv[x][1].y,
                             cv[x][2].x, cv[x][2].y, cv[x][3].x, cv[x][3].y};
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          if (colA + y < c) g[colA + y] = t8[y];
          if (colB + y < c) g[colB + y] = t8[4 + y];
        }
      }
    }
  }
  }  // FFMA pass 2
}

template <bool VEC, bool TCP2>
int launch_larfb_t(const float* V, int64_t sVb, int64_t ldv, const float* T,
                   int64_t sTb, int t_ld, const float* Csrc, int64_t sCsb,
                   int64_t ldcs, float* Cdst, int64_t sCdb, int64_t ldcd,
                   int64_t batch, int r, int k, int c, cudaStream_t stream) {
  static bool attr_set[64] = {};  // per device ordinal
  static int* err_ptr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  const size_t smem = TCP2 ? sizeof(SmemTc) : sizeof(Smem);
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k_larfb<VEC, TCP2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    if (TCP2 && device_error_ptr(&err_ptr[dev]) != QRB_OK) return QRB_ERR_DEVICE;
    attr_set[dev] = true;
  }
  const dim3 grid((unsigned)((c + TC - 1) / TC), (unsigned)batch, 1);
  k_larfb<VEC, TCP2><<<grid, NT, smem, stream>>>(V, sVb, ldv, T, sTb, t_ld, Csrc, sCsb, ldcs,
                                                 Cdst, sCdb, ldcd, r, k, c, err_ptr[dev]);
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int launch_larfb(const float* V, int64_t sVb, int64_t ldv, const float* T,
                 int64_t sTb, int t_ld, const float* Csrc, int64_t sCsb,
                 int64_t ldcs, float* Cdst, int64_t sCdb, int64_t ldcd,
                 int64_t batch, int r, int k, int c, bool tc_pass2,
                 cudaStream_t stream) {
  if (r < 1 || k < 1 || k > K || c < 1) return QRB_ERR_UNSUPPORTED;
  const bool vec = k == K && c % 4 == 0 && ldv % 4 == 0 && sVb % 4 == 0 &&
                   ldcs % 4 == 0 && sCsb % 4 == 0 && ldcd % 4 == 0 &&
                   sCdb % 4 == 0 && aligned16(V) && aligned16(Csrc) && aligned16(Cdst);
  constexpr int64_t kMaxGridY = 65535;
  for (int64_t b0 = 0; b0 < batch; b0 += kMaxGridY) {
    const int64_t nb = batch - b0 < kMaxGridY ? batch - b0 : kMaxGridY;
    const int rc = vec && tc_pass2
                       ? launch_larfb_t<true, true>(V + b0 * sVb, sVb, ldv, T + b0 * sTb, sTb,
                                                    t_ld, Csrc + b0 * sCsb, sCsb, ldcs,
                                                    Cdst + b0 * sCdb, sCdb, ldcd, nb, r, k, c,
                                                    stream)
                   : vec ? launch_larfb_t<true, false>(V + b0 * sVb, sVb, ldv, T + b0 * sTb, sTb, t_ld,
                                              Csrc + b0 * sCsb, sCsb, ldcs, Cdst + b0 * sCdb,
                                              sCdb, ldcd, nb, r, k, c, stream)
                       : launch_larfb_t<false, false>(V + b0 * sVb, sVb, ldv, T + b0 * sTb, sTb, t_ld,
                                               Csrc + b0 * sCsb, sCsb, ldcs, Cdst + b0 * sCdb,
                                               sCdb, ldcd, nb, r, k, c, stream);
    if (rc != QRB_OK) return rc;
  }
  return QRB_OK;
}

}  // namespace qrb

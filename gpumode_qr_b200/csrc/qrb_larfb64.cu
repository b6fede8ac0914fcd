// Two-level blocking: the trailing update for a block of 64 reflectors (two
// 32-column panels), C <- C - V (T^T (V^T C)) with V r x 64 and T 64 x 64,
// and the T of such a block from the two panels' factors.
//
// With 32-reflector blocks every reflector pair costs two reads and one write
// of the trailing matrix per 32 reflectors; with 64 the same traffic covers
// twice the reflectors and the per-launch work that does not scale with k
// (staging, partial sums, the T product) is amortised over twice the FLOPs.
//
//   k_larfb64  one 256-thread CTA per (matrix, 64-column tile), FFMA with the
//              packed FP32x2 FMA, 16-byte aligned operands only:
//                pass 1  W = V^T C (64 x 64) over 32-row chunks staged with
//                        cp.async (double-buffered); warps 2p and 2p+1 take
//                        rows p, p+4, ... of each chunk for W rows 0..31 and
//                        32..63; each lane an 8 x 8 register tile;
//                        the four row partitions are summed in shared memory;
//                mid     W' = T^T W (thread: one column, 16 rows);
//                pass 2  C -= V W' over 256-row chunks (V staged transposed
//                        and negated; 8 x 8 register tiles, 64 k-steps).
//   k_t64      the cross block of that T, in place: the two panels write
//              T1 and T2 on the diagonal of the 64 x 64 factor, this kernel
//              X = -T1 (V1^T V2) T2 above it and zeros below, giving
//              T = [[T1, X], [0, T2]] (LARFT of the combined block; the
//              reference's forward recurrence gives the same matrix,
//              src/qrbench/triton_kernels.py:886-909). The Gram block V1^T V2
//              is split by rows over a cluster of up to 8 CTAs (about 256
//              rows each), staged in 128-row chunks by double-buffered
//              cp.async.
// V is read through its strictly lower part: the diagonal is 1, everything
// above it 0 (so V points into a packed H; panel 2's first 32 rows, which hold
// R entries, read as 0).
#include <cooperative_groups.h>

#include "qrb_common.cuh"

namespace cg = cooperative_groups;

namespace qrb {

namespace {

constexpr int K = 64;
constexpr int TC = 64;
constexpr int NT = 256;
constexpr int NPART = 4;         // row partitions of pass 1
constexpr int RC1 = 32;          // rows per pass-1 chunk
constexpr int RC2 = 256;         // rows per pass-2 chunk
constexpr int VS_LD = K + 4;
constexpr int CS_LD = TC + 4;
constexpr int VT_LD = RC2 + 4;
constexpr int WS_LD = TC + 4;
constexpr int T_LD = K + 1;

struct __align__(16) Stage64 {
  float Vs[2][RC1 * VS_LD];
  float Cs[2][RC1 * CS_LD];
};
struct __align__(16) Smem64 {
  union {
    Stage64 st;
    float Wp[NPART][K * TC];
    float Vt[K * VT_LD];
  } u;
  float Ws[K * WS_LD];
  float Ts[K * T_LD];
};

__device__ __forceinline__ void cp_async16(void* s, const void* g, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(g), "r"(sz)
               : "memory");
}

__device__ __forceinline__ float vmask(float x, int i, int a) {
  return i < a ? 0.f : (i == a ? 1.f : x);
}

__global__ void __launch_bounds__(NT, 2)
k_larfb64(const float* __restrict__ V, int64_t sVb, int64_t ldv, const float* __restrict__ T,
          int64_t sTb, const float* __restrict__ Csrc, int64_t sCsb, int64_t ldcs,
          float* __restrict__ Cdst, int64_t sCdb, int64_t ldcd, int r, int c) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem64& sm = *reinterpret_cast<Smem64*>(smem_raw);
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
    sm.Ts[i * T_LD + a] = __ldg(T + m * sTb + e);
  }

  // ---------------- pass 1: W = V^T C ----------------
  const int hw = warp & 1;                      // W rows 32 hw .. 32 hw + 31
  const int part = warp >> 1;                   // chunk rows part, part + 4, ...
  const int wa = 32 * hw + ((lane >> 3) << 3);  // W rows wa .. wa + 7
  const int wc = (lane & 7) << 2;               // W cols wc..wc+3, wc+32..wc+35
  float2 acc[8][4];
#pragma unroll
  for (int x = 0; x < 8; ++x)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[x][j] = make_float2(0.f, 0.f);

  const int nch = (r + RC1 - 1) / RC1;
  auto load_chunk = [&](int ch, int buf) {
    const int i0 = ch * RC1;
#pragma unroll
    for (int e = 0; e < (RC1 * K) / (4 * NT); ++e) {  // V: 32 x 64 = 512 float4
      const int idx = tid + e * NT;
      const int row = idx >> 4, c4 = (idx & 15) << 2;
      const int i = i0 + row;
      const bool ok = i < r;
      cp_async16(&sm.u.st.Vs[buf][row * VS_LD + c4], ok ? Vm + (int64_t)i * ldv + c4 : Vm, ok);
    }
#pragma unroll
    for (int e = 0; e < (RC1 * TC) / (4 * NT); ++e) {  // C: 32 x 64 = 512 float4
      const int idx = tid + e * NT;
      const int row = idx >> 4, c4 = (idx & 15) << 2;
      const int i = i0 + row, col = c0 + c4;
      const bool ok = i < r && col < c;
      cp_async16(&sm.u.st.Cs[buf][row * CS_LD + c4], ok ? Cm + (int64_t)i * ldcs + col : Cm, ok);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  load_chunk(0, 0);
  for (int ch = 0; ch < nch; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < nch) {
      load_chunk(ch + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const int i0 = ch * RC1;
    if (i0 < K) {  // unit-lower mask on the top rows
      for (int e = tid; e < RC1 * K; e += NT) {
        const int row = e / K, a = e % K;
        const int i = i0 + row;
        if (i <= a) {
          float& v = sm.u.st.Vs[buf][row * VS_LD + a];
          v = vmask(v, i, a);
        }
      }
      __syncthreads();
    }
    const float* vb = sm.u.st.Vs[buf];
    const float* cb = sm.u.st.Cs[buf];
#pragma unroll 2
    for (int rr = part; rr < RC1; rr += NPART) {
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

#pragma unroll
  for (int x = 0; x < 8; ++x) {
    float* row = &sm.u.Wp[part][(wa + x) * TC];
    *reinterpret_cast<float4*>(row + wc) =
        make_float4(acc[x][0].x, acc[x][0].y, acc[x][1].x, acc[x][1].y);
    *reinterpret_cast<float4*>(row + wc + 32) =
        make_float4(acc[x][2].x, acc[x][2].y, acc[x][3].x, acc[x][3].y);
  }
  __syncthreads();
  {  // sum the partitions into Ws: 16 consecutive entries per thread
    const int e0 = tid * 16;
#pragma unroll
    for (int h4 = 0; h4 < 4; ++h4) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < NPART; ++p) {
        const float4 q = *reinterpret_cast<const float4*>(&sm.u.Wp[p][e0 + 4 * h4]);
        s4.x += q.x; s4.y += q.y; s4.z += q.z; s4.w += q.w;
      }
      const int e = e0 + 4 * h4;
      *reinterpret_cast<float4*>(&sm.Ws[(e / TC) * WS_LD + (e % TC)]) = s4;
    }
  }
  __syncthreads();
  {  // W' = T^T W: thread = column cc, rows ab .. ab + 15
    const int cc = tid & 63;
    const int ab = (tid >> 6) << 4;
    float o[16];
#pragma unroll
    for (int x = 0; x < 16; ++x) o[x] = 0.f;
#pragma unroll 4
    for (int q = 0; q < K; ++q) {
      const float wq = sm.Ws[q * WS_LD + cc];
#pragma unroll
      for (int x = 0; x < 16; ++x) o[x] = fmaf(sm.Ts[q * T_LD + ab + x], wq, o[x]);
    }
    __syncthreads();
#pragma unroll
    for (int x = 0; x < 16; ++x) sm.Ws[(ab + x) * WS_LD + cc] = o[x];
  }

  // ---------------- pass 2: C -= V W' ----------------
  const int rg = (tid >> 3) << 3;
  const int cq = (tid & 7) << 2;
  const int colA = c0 + cq, colB = c0 + cq + 32;
  for (int i0 = 0; i0 < r; i0 += RC2) {
    __syncthreads();  // W' ready / the previous chunk's Vt consumed
#pragma unroll 2
    for (int e = 0; e < (RC2 * K) / (4 * NT); ++e) {  // 256 rows x 64 = 4096 float4
      const int idx = tid + e * NT;
      const int row = idx & (RC2 - 1), c4 = (idx / RC2) << 2;
      const int i = i0 + row;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < r) t = __ldg(reinterpret_cast<const float4*>(Vm + (int64_t)i * ldv + c4));
      sm.u.Vt[(c4 + 0) * VT_LD + row] = -vmask(t.x, i, c4 + 0);
      sm.u.Vt[(c4 + 1) * VT_LD + row] = -vmask(t.y, i, c4 + 1);
      sm.u.Vt[(c4 + 2) * VT_LD + row] = -vmask(t.z, i, c4 + 2);
      sm.u.Vt[(c4 + 3) * VT_LD + row] = -vmask(t.w, i, c4 + 3);
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
      if (colA < c)
        *reinterpret_cast<float4*>(g + colA) =
            make_float4(cv[x][0].x, cv[x][0].y, cv[x][1].x, cv[x][1].y);
      if (colB < c)
        *reinterpret_cast<float4*>(g + colB) =
            make_float4(cv[x][2].x, cv[x][2].y, cv[x][3].x, cv[x][3].y);
    }
  }
}

// T of a 64-reflector block, in place: the two panels have written T1 into
// rows/columns 0..31 and T2 into rows/columns 32..63 of the 64 x 64 factor
// (row stride 64); this fills the cross block X = -T1 (V1^T V2) T2 and zeroes
// the lower-left block. The Gram block G = V1^T V2 is split over a cluster of
// cs CTAs by rows (each CTA a contiguous slice of rows_per rows); rank 0 sums
// the slices through distributed shared memory and forms X.
constexpr int T64_CH = 128;  // rows per staged chunk of k_t64
constexpr size_t T64_SMEM = 2 * (size_t)T64_CH * K * sizeof(float);  // double buffer

__global__ void __launch_bounds__(NT)
k_t64(const float* __restrict__ V, int64_t sVb, int64_t ldv, float* __restrict__ T,
      int64_t sTb, int r, int cs, int rows_per) {
  constexpr int W = 32;
  constexpr int NG = NT / W;  // 8 row groups
  extern __shared__ __align__(16) float vbuf[];  // [2][T64_CH][K]
  __shared__ float red[NG / 2][W][W + 1];
  __shared__ float Gs[W][W + 1];
  __shared__ float t1[W][W + 1], t2[W][W + 1], y[W][W + 1];
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x;
  const int a = tid & (W - 1);
  const int g = tid >> 5;
  const int rank = cs > 1 ? (int)cluster.block_rank() : 0;
  const int64_t m = blockIdx.x / cs;
  const float* __restrict__ Vm = V + m * sVb;
  float* __restrict__ Tm = T + m * sTb;
  if (rank == 0) {
    for (int e = tid; e < W * W; e += NT) {
      const int i = e / W, j = e % W;
      t1[i][j] = Tm[i * K + j];
      t2[i][j] = Tm[(W + i) * K + W + j];
    }
  }
  // rows below 32 + b only contribute to G[a][b]; rows < 32 contribute nothing
  int lo = rank * rows_per;
  const int hi = min(r, lo + rows_per);
  if (lo < W) lo = W;
  const int nchunk = hi > lo ? (hi - lo + T64_CH - 1) / T64_CH : 0;
  // stage chunk c (rows lo + c * T64_CH ..) into buffer c & 1: 16-byte cp.async,
  // all of a chunk's requests in flight, the next chunk loading while this
  // one is multiplied
  auto stage = [&](int c) {
    float* dst = vbuf + (size_t)(c & 1) * T64_CH * K;
    const int i0 = lo + c * T64_CH;
    const int nr = min(T64_CH, hi - i0);
    for (int e = tid; e < nr * (K / 4); e += NT) {
      const int row = e >> 4, c4 = (e & 15) << 2;
      cp_async16(dst + row * K + c4, Vm + (int64_t)(i0 + row) * ldv + c4, true);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[W];
#pragma unroll
  for (int b = 0; b < W; ++b) acc[b] = 0.f;
  if (nchunk > 0) stage(0);
  for (int c = 0; c < nchunk; ++c) {
    if (c + 1 < nchunk) {
      stage(c + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    float* Vs = vbuf + (size_t)(c & 1) * T64_CH * K;
    const int i0 = lo + c * T64_CH;
    const int nr = min(T64_CH, hi - i0);
    if (i0 < K) {  // panel 2's diagonal block: unit diagonal, zero above it
      for (int e = tid; e < nr * W; e += NT) {
        const int row = e >> 5, b = e & (W - 1);
        const int i = i0 + row;
        if (i < K) Vs[row * K + W + b] = vmask(Vs[row * K + W + b], i, W + b);
      }
      __syncthreads();
    }
#pragma unroll 4
    for (int row = g; row < nr; row += NG) {
      const float xa = Vs[row * K + a];
#pragma unroll
      for (int b4 = 0; b4 < W / 4; ++b4) {
        const float4 xb = *reinterpret_cast<const float4*>(&Vs[row * K + W + 4 * b4]);
        acc[4 * b4 + 0] = fmaf(xa, xb.x, acc[4 * b4 + 0]);
        acc[4 * b4 + 1] = fmaf(xa, xb.y, acc[4 * b4 + 1]);
        acc[4 * b4 + 2] = fmaf(xa, xb.z, acc[4 * b4 + 2]);
        acc[4 * b4 + 3] = fmaf(xa, xb.w, acc[4 * b4 + 3]);
      }
    }
    __syncthreads();  // the buffer is restaged two chunks on
  }
  // tree-sum the 8 row groups: 4..7 -> 0..3, 2..3 -> 0..1, 1 -> 0
#pragma unroll
  for (int half = NG / 2; half >= 1; half >>= 1) {
    __syncthreads();
    if (g >= half && g < 2 * half) {
#pragma unroll
      for (int b = 0; b < W; ++b) red[g - half][a][b] = acc[b];
    }
    __syncthreads();
    if (g < half) {
#pragma unroll
      for (int b = 0; b < W; ++b) acc[b] += red[g][a][b];
    }
  }
  if (g == 0) {
#pragma unroll
    for (int b = 0; b < W; ++b) Gs[a][b] = acc[b];
  }
  if (cs > 1) {
    cluster.sync();  // every slice in shared memory
    if (rank == 0) {
      for (int e = tid; e < W * W; e += NT) {
        const int i = e / W, j = e % W;
        float s = Gs[i][j];
        for (int q = 1; q < cs; ++q) s += cluster.map_shared_rank(&Gs[0][0], q)[i * (W + 1) + j];
        red[0][i][j] = s;
      }
    }
    cluster.sync();  // peers stay resident until rank 0 has read them
    if (rank != 0) return;
    __syncthreads();
    for (int e = tid; e < W * W; e += NT) Gs[e / W][e % W] = red[0][e / W][e % W];
  }
  __syncthreads();
  // y = G T2, then X = -T1 y
  for (int e = tid; e < W * W; e += NT) {
    const int i = e / W, j = e % W;
    float s = 0.f;
#pragma unroll 8
    for (int q = 0; q < W; ++q) s = fmaf(Gs[i][q], t2[q][j], s);
    y[i][j] = s;
  }
  __syncthreads();
  for (int e = tid; e < W * W; e += NT) {
    const int i = e / W, j = e % W;
    float s = 0.f;
#pragma unroll 8
    for (int q = 0; q < W; ++q) s = fmaf(t1[i][q], y[q][j], s);
    Tm[i * K + W + j] = -s;
    Tm[(W + i) * K + j] = 0.f;
  }
}

size_t smem64() { return sizeof(Smem64); }

}  // namespace

bool larfb64_supported(const float* V, int64_t sVb, int64_t ldv, const float* Csrc, int64_t sCsb,
                       int64_t ldcs, const float* Cdst, int64_t sCdb, int64_t ldcd, int c) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return c % 4 == 0 && ldv % 4 == 0 && sVb % 4 == 0 && ldcs % 4 == 0 && sCsb % 4 == 0 &&
         ldcd % 4 == 0 && sCdb % 4 == 0 && al(V) && al(Csrc) && al(Cdst);
}

int launch_larfb64(const float* V, int64_t sVb, int64_t ldv, const float* T, int64_t sTb,
                   const float* Csrc, int64_t sCsb, int64_t ldcs, float* Cdst, int64_t sCdb,
                   int64_t ldcd, int64_t batch, int r, int c, cudaStream_t stream) {
  if (r < K || c < 1) return QRB_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k_larfb64, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem64()) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  constexpr int64_t kMaxGridY = 65535;
  for (int64_t b0 = 0; b0 < batch; b0 += kMaxGridY) {
    const int64_t nb = batch - b0 < kMaxGridY ? batch - b0 : kMaxGridY;
    const dim3 grid((unsigned)((c + TC - 1) / TC), (unsigned)nb, 1);
    k_larfb64<<<grid, NT, smem64(), stream>>>(V + b0 * sVb, sVb, ldv, T + b0 * sTb, sTb,
                                              Csrc + b0 * sCsb, sCsb, ldcs, Cdst + b0 * sCdb,
                                              sCdb, ldcd, r, c);
    note_launches(1);
    if (cudaGetLastError() != cudaSuccess) return QRB_ERR_LAUNCH;
  }
  return QRB_OK;
}

int launch_t64(const float* V, int64_t sVb, int64_t ldv, float* T64, int64_t sT64b,
               int64_t batch, int r, cudaStream_t stream) {
  if (r <= K) return QRB_ERR_UNSUPPORTED;
  if (ldv % 4 != 0 || sVb % 4 != 0 || (reinterpret_cast<uintptr_t>(V) & 15) != 0)
    return QRB_ERR_UNSUPPORTED;
  // about 256 rows per cluster rank (up to 8 ranks)
  int cs = (r + 255) / 256;
  if (cs > kMaxCluster) cs = kMaxCluster;
  if (batch * cs > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k_t64, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)T64_SMEM) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  const int rows_per = ((r + cs - 1) / cs + 31) / 32 * 32;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(batch * cs), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = T64_SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cs > 1 ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_t64, V, sVb, ldv, T64, sT64b, r, cs, rows_per);
  note_launches(1);
  return e == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace qrb

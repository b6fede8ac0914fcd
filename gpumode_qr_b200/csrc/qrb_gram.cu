// Gram matrix S = G G^T of a batch of n x k row-major matrices, and the
// factorization of S: the optimizer-statistics step that the reference's
// workload puts in front of the QR (gradients viewed as [basis_dim,
// contracted_dim], statistics G @ G.T, QR of the square basis_dim x basis_dim
// result; the task statement in AGENTS.md:27 of the reference).
//
//   k_gram<VEC>  one 256-thread CTA per (matrix, 64 x 64 tile of S on or above
//                the diagonal); the tile below the diagonal is written as its
//                mirror, so S is exactly symmetric. Per 32-column chunk of G,
//                rows p0.. and q0.. of the chunk land row-major in shared
//                memory by cp.async while the previous chunk is multiplied,
//                then are transposed into a second buffer; warps 2p and
//                2p+1 take chunk columns p, p+4, ... for tile rows 0..31 and
//                32..63, each lane an 8 x 8 register tile updated with the
//                packed FP32x2 FMA (32 FMAs per four 16-byte shared loads).
//                The four partitions are summed in shared memory, then the
//                tile and its mirror are stored with coalesced rows.
//
// FP32 throughout (products and sums in FP32 with FMA), the same arithmetic as
// an FP32 G @ G.T without TF32.
#include "qrb_common.cuh"

namespace qrb {

namespace {

constexpr int TS = 64;       // S tile (rows and columns)
constexpr int KC = 32;       // columns of G per chunk
constexpr int NT = 256;
constexpr int NPART = 4;
constexpr int GT_LD = TS + 4;  // transposed staging row stride
constexpr int TL_LD = TS + 1;  // summed tile row stride (conflict-free mirror reads)

constexpr int RAW_LD = KC + 4;  // row-major landing buffer row stride
constexpr int kGramBigTileMinN = 64;  // 128 x 128 tiles above this n

struct __align__(16) SmemGram {
  union {
    struct {
      float rawP[TS * RAW_LD];  // chunk as loaded: [row][column]
      float rawQ[TS * RAW_LD];
      float P[2][KC * GT_LD];   // transposed: [column][row]
      float Q[2][KC * GT_LD];
    } st;
    float Wp[NPART][TS * TS];
  } u;
  float tile[TS * TL_LD];
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

// Tile (ti, tj), ti <= tj, of the id-th upper-triangle tile in row order.
__device__ __forceinline__ void tile_of(int id, int nt, int* ti, int* tj) {
  int i = 0;
  while (id >= nt - i) {
    id -= nt - i;
    ++i;
  }
  *ti = i;
  *tj = i + id;
}

template <bool VEC>
__global__ void __launch_bounds__(NT, 2)
k_gram(const float* __restrict__ G, int64_t sGb, int64_t ldg, float* __restrict__ S,
       int n, int k, int nt) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SmemGram& sm = *reinterpret_cast<SmemGram*>(smem_raw);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t m = blockIdx.y;
  int ti, tj;
  tile_of((int)blockIdx.x, nt, &ti, &tj);
  const int p0 = ti * TS, q0 = tj * TS;
  const bool diag = ti == tj;
  const float* __restrict__ Gm = G + m * sGb;

  // Chunk staging: cp.async lands rows p0.. and q0.. of the chunk row-major
  // (no registers held across the multiply), then the threads transpose them
  // into P / Q [column][row].
  auto issue_chunk = [&](int t0) {
    if (VEC) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int idx = tid + e * NT;
        const int row = idx >> 3, c4 = (idx & 7) << 2;
        const int t = t0 + c4;
        const int ip = p0 + row, iq = q0 + row;
        const bool okp = ip < n && t < k, okq = !diag && iq < n && t < k;
        cp_async16(&sm.u.st.rawP[row * RAW_LD + c4], okp ? Gm + (int64_t)ip * ldg + t : Gm, okp);
        if (!diag)
          cp_async16(&sm.u.st.rawQ[row * RAW_LD + c4], okq ? Gm + (int64_t)iq * ldg + t : Gm, okq);
      }
    } else {
#pragma unroll 4
      for (int e = 0; e < (TS * KC) / NT; ++e) {
        const int idx = tid + e * NT;
        const int row = idx >> 5, c = idx & 31;
        const int t = t0 + c;
        const int ip = p0 + row, iq = q0 + row;
        const bool okp = ip < n && t < k, okq = !diag && iq < n && t < k;
        cp_async4(&sm.u.st.rawP[row * RAW_LD + c], okp ? Gm + (int64_t)ip * ldg + t : Gm, okp);
        if (!diag)
          cp_async4(&sm.u.st.rawQ[row * RAW_LD + c], okq ? Gm + (int64_t)iq * ldg + t : Gm, okq);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  auto transpose_chunk = [&](int buf) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int idx = tid + e * NT;
      const int row = idx >> 3, c4 = (idx & 7) << 2;
      const float4 a = *reinterpret_cast<const float4*>(&sm.u.st.rawP[row * RAW_LD + c4]);
      float* P = sm.u.st.P[buf];
      P[(c4 + 0) * GT_LD + row] = a.x;
      P[(c4 + 1) * GT_LD + row] = a.y;
      P[(c4 + 2) * GT_LD + row] = a.z;
      P[(c4 + 3) * GT_LD + row] = a.w;
      if (!diag) {
        const float4 b = *reinterpret_cast<const float4*>(&sm.u.st.rawQ[row * RAW_LD + c4]);
        float* Q = sm.u.st.Q[buf];
        Q[(c4 + 0) * GT_LD + row] = b.x;
        Q[(c4 + 1) * GT_LD + row] = b.y;
        Q[(c4 + 2) * GT_LD + row] = b.z;
        Q[(c4 + 3) * GT_LD + row] = b.w;
      }
    }
  };

  const int hw = warp & 1;                      // tile rows 32 hw .. 32 hw + 31
  const int part = warp >> 1;                   // chunk columns part, part + 4, ...
  const int wa = 32 * hw + ((lane >> 3) << 3);  // tile rows wa .. wa + 7
  const int wc = (lane & 7) << 2;               // tile cols wc..wc+3, wc+32..wc+35
  float2 acc[8][4];
#pragma unroll
  for (int x = 0; x < 8; ++x)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[x][j] = make_float2(0.f, 0.f);

  const int nch = (k + KC - 1) / KC;
  issue_chunk(0);
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  transpose_chunk(0);
  __syncthreads();
  for (int ch = 0; ch < nch; ++ch) {
    const int buf = ch & 1;
    const bool more = ch + 1 < nch;
    if (more) issue_chunk((ch + 1) * KC);  // the landing buffer was consumed before the last barrier
    const float* pb = sm.u.st.P[buf];
    const float* qb = diag ? pb : sm.u.st.Q[buf];
#pragma unroll 2
    for (int t = part; t < KC; t += NPART) {
      const float4 v0 = *reinterpret_cast<const float4*>(pb + t * GT_LD + wa);
      const float4 v1 = *reinterpret_cast<const float4*>(pb + t * GT_LD + wa + 4);
      const float4 ca = *reinterpret_cast<const float4*>(qb + t * GT_LD + wc);
      const float4 cb = *reinterpret_cast<const float4*>(qb + t * GT_LD + wc + 32);
      const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      const float2 cp[4] = {make_float2(ca.x, ca.y), make_float2(ca.z, ca.w),
                            make_float2(cb.x, cb.y), make_float2(cb.z, cb.w)};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const float2 vx = make_float2(vv[x], vv[x]);
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[x][j] = __ffma2_rn(vx, cp[j], acc[x][j]);
      }
    }
    if (more) {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      __syncthreads();  // the next chunk has landed for every thread
      transpose_chunk(buf ^ 1);
    }
    __syncthreads();  // transposed chunk complete; this chunk's buffers free
  }

  // partitions -> shared memory (the staging area is free after the last barrier)
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    float* row = &sm.u.Wp[part][(wa + x) * TS];
    *reinterpret_cast<float4*>(row + wc) =
        make_float4(acc[x][0].x, acc[x][0].y, acc[x][1].x, acc[x][1].y);
    *reinterpret_cast<float4*>(row + wc + 32) =
        make_float4(acc[x][2].x, acc[x][2].y, acc[x][3].x, acc[x][3].y);
  }
  __syncthreads();
  {  // sum the partitions: 16 consecutive entries per thread
    const int e0 = tid * 16;
    const int i = e0 / TS, j0 = e0 % TS;
#pragma unroll
    for (int h4 = 0; h4 < 4; ++h4) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < NPART; ++p) {
        const float4 q = *reinterpret_cast<const float4*>(&sm.u.Wp[p][e0 + 4 * h4]);
        s4.x += q.x; s4.y += q.y; s4.z += q.z; s4.w += q.w;
      }
      float* tl = &sm.tile[i * TL_LD + j0 + 4 * h4];
      tl[0] = s4.x; tl[1] = s4.y; tl[2] = s4.z; tl[3] = s4.w;
    }
  }
  __syncthreads();
  float* __restrict__ Sm = S + m * (int64_t)n * n;
  for (int e = tid; e < TS * TS; e += NT) {  // the tile: S[p0 + i][q0 + j]
    const int i = e / TS, j = e % TS;
    if (p0 + i < n && q0 + j < n) Sm[(int64_t)(p0 + i) * n + q0 + j] = sm.tile[i * TL_LD + j];
  }
  if (!diag) {
    for (int e = tid; e < TS * TS; e += NT) {  // its mirror: S[q0 + i][p0 + j] = tile[j][i]
      const int i = e / TS, j = e % TS;
      if (q0 + i < n && p0 + j < n) Sm[(int64_t)(q0 + i) * n + p0 + j] = sm.tile[j * TL_LD + i];
    }
  }
}

// 128 x 128 tiles without the split over chunk columns: thread (ty, tx) of
// 16 x 16 owns tile rows {4 ty .. 4 ty + 3, 64 + 4 ty ..} and columns
// {4 tx .., 64 + 4 tx ..} (8 x 8 outputs, 32 packed FMAs per four 16-byte
// shared loads, no partial sums to reduce); chunks of 32 columns of G land
// row-major by cp.async while the previous chunk is multiplied and are then
// transposed into the second of two [column][row] buffers.
constexpr int TB = 128;
constexpr int TB_LD = TB + 4;
struct __align__(16) SmemGram128 {
  float rawP[TB * RAW_LD];
  float rawQ[TB * RAW_LD];
  float P[2][KC * TB_LD];
  float Q[2][KC * TB_LD];
};

template <bool VEC>
__global__ void __launch_bounds__(NT, 2)
k_gram128(const float* __restrict__ G, int64_t sGb, int64_t ldg, float* __restrict__ S,
          int n, int k, int nt) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SmemGram128& sm = *reinterpret_cast<SmemGram128*>(smem_raw);
  const int tid = threadIdx.x;
  const int64_t m = blockIdx.y;
  int ti, tj;
  tile_of((int)blockIdx.x, nt, &ti, &tj);
  const int p0 = ti * TB, q0 = tj * TB;
  const bool diag = ti == tj;
  const float* __restrict__ Gm = G + m * sGb;

  auto issue_chunk = [&](int t0) {
    if (VEC) {
#pragma unroll
      for (int e = 0; e < (TB * KC) / (4 * NT); ++e) {
        const int idx = tid + e * NT;
        const int row = idx >> 3, c4 = (idx & 7) << 2;
        const int t = t0 + c4;
        const int ip = p0 + row, iq = q0 + row;
        const bool okp = ip < n && t < k, okq = !diag && iq < n && t < k;
        cp_async16(&sm.rawP[row * RAW_LD + c4], okp ? Gm + (int64_t)ip * ldg + t : Gm, okp);
        if (!diag)
          cp_async16(&sm.rawQ[row * RAW_LD + c4], okq ? Gm + (int64_t)iq * ldg + t : Gm, okq);
      }
    } else {
#pragma unroll 4
      for (int e = 0; e < (TB * KC) / NT; ++e) {
        const int idx = tid + e * NT;
        const int row = idx >> 5, c = idx & 31;
        const int t = t0 + c;
        const int ip = p0 + row, iq = q0 + row;
        const bool okp = ip < n && t < k, okq = !diag && iq < n && t < k;
        cp_async4(&sm.rawP[row * RAW_LD + c], okp ? Gm + (int64_t)ip * ldg + t : Gm, okp);
        if (!diag)
          cp_async4(&sm.rawQ[row * RAW_LD + c], okq ? Gm + (int64_t)iq * ldg + t : Gm, okq);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  // consecutive threads take consecutive rows of one 4-column group, so the
  // 16-byte reads and the transposed scalar stores are both conflict-free
  auto transpose_chunk = [&](int buf) {
#pragma unroll
    for (int e = 0; e < (TB * KC) / (4 * NT); ++e) {
      const int idx = tid + e * NT;
      const int row = idx & (TB - 1), c4 = (idx >> 7) << 2;
      const float4 a = *reinterpret_cast<const float4*>(&sm.rawP[row * RAW_LD + c4]);
      float* P = sm.P[buf];
      P[(c4 + 0) * TB_LD + row] = a.x;
      P[(c4 + 1) * TB_LD + row] = a.y;
      P[(c4 + 2) * TB_LD + row] = a.z;
      P[(c4 + 3) * TB_LD + row] = a.w;
      if (!diag) {
        const float4 b = *reinterpret_cast<const float4*>(&sm.rawQ[row * RAW_LD + c4]);
        float* Q = sm.Q[buf];
        Q[(c4 + 0) * TB_LD + row] = b.x;
        Q[(c4 + 1) * TB_LD + row] = b.y;
        Q[(c4 + 2) * TB_LD + row] = b.z;
        Q[(c4 + 3) * TB_LD + row] = b.w;
      }
    }
  };

  const int ty = tid >> 4, tx = tid & 15;
  const int ra = 4 * ty, ca = 4 * tx;  // row groups ra, 64 + ra; column groups ca, 64 + ca
  float2 acc[8][4];  // rows ra..ra+3, 64+ra..; column pairs (ca, ca+1), (ca+2, ca+3), (64+ca, ..)
#pragma unroll
  for (int x = 0; x < 8; ++x)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[x][j] = make_float2(0.f, 0.f);

  const int nch = (k + KC - 1) / KC;
  issue_chunk(0);
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  transpose_chunk(0);
  __syncthreads();
  for (int ch = 0; ch < nch; ++ch) {
    const int buf = ch & 1;
    const bool more = ch + 1 < nch;
    if (more) issue_chunk((ch + 1) * KC);
    const float* pb = sm.P[buf];
    const float* qb = diag ? pb : sm.Q[buf];
#pragma unroll 4
    for (int t = 0; t < KC; ++t) {
      const float4 a0 = *reinterpret_cast<const float4*>(pb + t * TB_LD + ra);
      const float4 a1 = *reinterpret_cast<const float4*>(pb + t * TB_LD + 64 + ra);
      const float4 b0 = *reinterpret_cast<const float4*>(qb + t * TB_LD + ca);
      const float4 b1 = *reinterpret_cast<const float4*>(qb + t * TB_LD + 64 + ca);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float2 bp[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                            make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const float2 ax = make_float2(av[x], av[x]);
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[x][j] = __ffma2_rn(ax, bp[j], acc[x][j]);
      }
    }
    if (more) {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      __syncthreads();
      transpose_chunk(buf ^ 1);
    }
    __syncthreads();
  }

  float* __restrict__ Sm = S + m * (int64_t)n * n;
  const bool vst = (n & 3) == 0;  // 16-byte row stores stay aligned
#pragma unroll
  for (int x = 0; x < 8; ++x) {  // the tile: rows p0 + (x < 4 ? ra + x : 64 + ra + x - 4)
    const int i = p0 + (x < 4 ? ra + x : 60 + ra + x);
    if (i >= n) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = q0 + h * 64 + ca;
      const float v[4] = {acc[x][2 * h].x, acc[x][2 * h].y, acc[x][2 * h + 1].x,
                          acc[x][2 * h + 1].y};
      float* g = Sm + (int64_t)i * n + j;
      if (vst && j + 3 < n) {
        *reinterpret_cast<float4*>(g) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int y = 0; y < 4; ++y)
          if (j + y < n) g[y] = v[y];
      }
    }
  }
  if (!diag) {  // the mirror: S[q0 + col][p0 + row]
#pragma unroll
    for (int y = 0; y < 8; ++y) {  // tile column y of this thread
      const int jc = q0 + (y < 4 ? ca + y : 60 + ca + y);
      if (jc >= n) continue;
      const int pair = (y < 4 ? 0 : 2) + ((y & 3) >> 1);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i0 = p0 + h * 64 + ra;
        float v[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float2 a = acc[4 * h + x][pair];
          v[x] = (y & 1) ? a.y : a.x;
        }
        float* g = Sm + (int64_t)jc * n + i0;
        if (vst && i0 + 3 < n) {
          *reinterpret_cast<float4*>(g) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
          for (int x = 0; x < 4; ++x)
            if (i0 + x < n) g[x] = v[x];
        }
      }
    }
  }
}

template <bool VEC, bool BIG>
int launch_gram_t(const float* G, int64_t sGb, int64_t ldg, float* S, int64_t batch, int n, int k,
                  cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  auto kern = BIG ? k_gram128<VEC> : k_gram<VEC>;
  const size_t smem = BIG ? sizeof(SmemGram128) : sizeof(SmemGram);
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return QRB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  const int tile = BIG ? TB : TS;
  const int nt = (n + tile - 1) / tile;
  const unsigned tiles = (unsigned)(nt * (nt + 1) / 2);
  constexpr int64_t kMaxGridY = 65535;
  for (int64_t b0 = 0; b0 < batch; b0 += kMaxGridY) {
    const int64_t nb = batch - b0 < kMaxGridY ? batch - b0 : kMaxGridY;
    kern<<<dim3(tiles, (unsigned)nb, 1), NT, smem, stream>>>(G + b0 * sGb, sGb, ldg,
                                                             S + b0 * (int64_t)n * n, n, k, nt);
    note_launches(1);
    if (cudaGetLastError() != cudaSuccess) return QRB_ERR_LAUNCH;
  }
  return QRB_OK;
}

int launch_gram(const float* G, int64_t sGb, int64_t ldg, float* S, int64_t batch, int n, int k,
                cudaStream_t stream) {
  const bool vec = (reinterpret_cast<uintptr_t>(G) & 15) == 0 && ldg % 4 == 0 &&
                   (batch == 1 || sGb % 4 == 0) && k % 4 == 0;
  const int pref = gram_tile();
  const bool big = pref == 128 || (pref == 0 && n > kGramBigTileMinN);
  if (big)
    return vec ? launch_gram_t<true, true>(G, sGb, ldg, S, batch, n, k, stream)
               : launch_gram_t<false, true>(G, sGb, ldg, S, batch, n, k, stream);
  return vec ? launch_gram_t<true, false>(G, sGb, ldg, S, batch, n, k, stream)
             : launch_gram_t<false, false>(G, sGb, ldg, S, batch, n, k, stream);
}

bool bad_gram_args(const float* G, int64_t sGb, int64_t ldg, const void* out, int64_t batch,
                   int n, int k) {
  if (!G || !out) return true;
  if (ldg < k) return true;
  if (batch > 1 && sGb < (int64_t)(n - 1) * ldg + k) return true;
  return false;
}

}  // namespace

}  // namespace qrb

extern "C" {

int qrb_gram_f32(const float* G, int64_t strideG_b, int64_t strideG_row, float* S, int64_t batch,
                 int32_t n, int32_t k, void* stream) {
  if (batch < 0 || n < 0 || k < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB_OK;
  if (n > qrb::kMaxN) return QRB_ERR_UNSUPPORTED;
  if (k == 0) {  // an empty contraction: S = 0
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!S) return QRB_ERR_INVALID_ARG;
    if (qrb::take_injected_failure_any()) return QRB_ERR_INJECTED;
    if (cudaMemsetAsync(S, 0, (size_t)batch * n * n * sizeof(float), s) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    return qrb::finish_call(QRB_OK, s);
  }
  if (qrb::bad_gram_args(G, strideG_b, strideG_row, S, batch, n, k)) return QRB_ERR_INVALID_ARG;
  if (qrb::take_injected_failure_any()) return QRB_ERR_INJECTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return qrb::finish_call(qrb::launch_gram(G, strideG_b, strideG_row, S, batch, n, k, s), s);
}

int qrb_gram_geqrf_f32(const float* G, int64_t strideG_b, int64_t strideG_row, float* H,
                       float* tau, int64_t batch, int32_t n, int32_t k, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (batch < 0 || n < 0 || k < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB_OK;
  if (n > qrb::kMaxN) return QRB_ERR_UNSUPPORTED;
  if (!tau) return QRB_ERR_INVALID_ARG;
  if (k > 0 && qrb::bad_gram_args(G, strideG_b, strideG_row, H, batch, n, k))
    return QRB_ERR_INVALID_ARG;
  if (!H) return QRB_ERR_INVALID_ARG;
  qrb::FactorScratch fs;
  if (n > qrb::kFusedMaxN) {
    const size_t one = qrb::min_workspace_bytes(batch);
    if (workspace == nullptr || workspace_bytes < one) return QRB_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return QRB_ERR_INVALID_ARG;
    fs = qrb::factor_scratch(workspace, workspace_bytes, batch, n);
  }
  if (qrb::take_injected_failure_any()) return QRB_ERR_INJECTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (k == 0)
    rc = cudaMemsetAsync(H, 0, (size_t)batch * n * n * sizeof(float), s) == cudaSuccess
             ? QRB_OK
             : QRB_ERR_LAUNCH;
  else
    rc = qrb::launch_gram(G, strideG_b, strideG_row, H, batch, n, k, s);
  if (rc == QRB_OK) {
    const int64_t nn = (int64_t)n * n;
    rc = qrb::geqrf_enqueue(H, nn, n, H, tau, fs, batch, n, s);
  }
  return qrb::finish_call(rc, s);
}

}  // extern "C"

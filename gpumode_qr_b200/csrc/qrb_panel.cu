// Householder factorization of an r x w panel (w <= 32) plus its compact-WY
// factor T, one thread-block cluster per matrix.
//
// Layout: thread t of cluster rank q owns panel rows q*rows_per_cta + t +
// p*blockDim.x (p < RPT), all 32 columns of each, in registers. Nothing of the
// panel lives in shared memory; shared memory carries only reductions.
//
// One column step j is one 32-slot reduction over the rows below j:
//     slot[m] = sum_{i>j} x_i * a_im,   x = column j
// which yields, at once, sigma = slot[j] (the norm below the diagonal), the
// trailing dot products d_k = a_jk + scale * slot[k] (k > j), and the Gram
// column G[m][j] (m < j) used by the T recurrence. The reduction is a warp
// reduce-scatter (31 shuffles), a cross-warp sum in shared memory, and for
// clusters a cross-CTA sum over distributed shared memory. Every warp forms
// the reflector coefficients itself from the summed slots, so a step costs one
// block barrier (plus one cluster barrier for clusters); the partial-sum
// buffers alternate by step parity so no second barrier is needed.
//
// The column loop is a runtime loop with a compact body (the register array is
// indexed only by compile-time constants; the current column is picked with a
// select tree), which keeps the kernel inside the instruction cache. Reflector
// scaling is deferred: below the diagonal a finished column keeps its unscaled
// values x_m during the loop and is multiplied by scale_m = 1/(alpha_m-beta_m)
// only when the panel is written back; the Gram entries are scaled to match:
//     G[m][j] = scale_m * (x_m(j) + scale_j * sum_{i>j} x_j(i) x_m(i)).
//
// Semantics follow the reference panel kernel (src/qrbench/triton_kernels.py
// :839-871 reflectors and packing, :873-884 unit-lower V, :886-909 forward
// LARFT recurrence T[i,i] = tau_i, T[:i,i] = -tau_i T[:i,:i] (V[:,:i]^T v_i)).
#include <cooperative_groups.h>

#include "qrb_common.cuh"
#include "qrb_tc.cuh"

namespace cg = cooperative_groups;

namespace qrb {

namespace {

constexpr int W = kPanelW;
constexpr int kMaxThreads = 512;        // upper bound the shared buffers are sized for
constexpr int kPanelCtaThreads = 256;   // threads per CTA used by panel_shape

// Reduce 32 per-lane slot values across a warp; afterwards lane l holds the
// warp total of slot l in v[0]. 16+8+4+2+1 shuffles.
__device__ __forceinline__ void reduce_scatter32(float (&v)[W], int lane) {
#pragma unroll
  for (int half = 16; half >= 1; half >>= 1) {
    const bool upper = (lane & half) != 0;
#pragma unroll
    for (int q = 0; q < half; ++q) {
      const float keep = upper ? v[q + half] : v[q];
      const float send = upper ? v[q] : v[q + half];
      v[q] = keep + __shfl_xor_sync(kFull, send, half);
    }
  }
}

// v[j] for a runtime j in [0, 32): a five-level select tree (31 selects).
__device__ __forceinline__ float pick32(const float (&v)[W], int j) {
  float t16[16], t8[8], t4[4], t2[2];
#pragma unroll
  for (int q = 0; q < 16; ++q) t16[q] = (j & 16) ? v[q + 16] : v[q];
#pragma unroll
  for (int q = 0; q < 8; ++q) t8[q] = (j & 8) ? t16[q + 8] : t16[q];
#pragma unroll
  for (int q = 0; q < 4; ++q) t4[q] = (j & 4) ? t8[q + 4] : t8[q];
#pragma unroll
  for (int q = 0; q < 2; ++q) t2[q] = (j & 2) ? t4[q + 2] : t4[q];
  return (j & 1) ? t2[1] : t2[0];
}

template <int RPT>
__global__ void __launch_bounds__(RPT >= 2 ? kPanelCtaThreads : kMaxThreads, 1)
k_panel(const float* __restrict__ src, int64_t sb_src, int64_t ld_src,
        float* __restrict__ dst, int64_t sb_dst, int64_t ld_dst,
        float* __restrict__ tau_out, int64_t tau_sb, float* __restrict__ T_out,
        int64_t T_sb, int t_ld, float* __restrict__ V_out, float* __restrict__ Vsplit,
        int64_t vs_mat, int64_t vs_plane, int vs_row0, int vs_ld, int vs_zero, int r, int w,
        int cs, int vec_src, int vec_dst) {
  __shared__ float red[2][kMaxThreads / 32][W];  // [parity][warp][slot]
  __shared__ float xch[2][2][W];                 // [parity][0 = CTA slot sums, 1 = row j]
  __shared__ __align__(16) float fbuf[kMaxThreads / 32][W];  // per-warp tau_j * d_k
  __shared__ float Gs[W][W + 1];                 // Gram V^T V, strictly upper part
  __shared__ float taus[W], scales[W], betas[W];

  const int nt = blockDim.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = nt >> 5;
  int rank = 0;
  if (cs > 1) rank = (int)cg::this_cluster().block_rank();
  const int64_t m = blockIdx.x / cs;
  const int row0 = rank * nt * RPT;

  for (int e = tid; e < W * (W + 1); e += nt) (&Gs[0][0])[e] = 0.f;
  if (tid < W) {
    taus[tid] = 0.f;
    scales[tid] = 0.f;
    betas[tid] = 0.f;
  }

  float a[RPT][W];
  int rowi[RPT];
  const float* __restrict__ S = src + m * sb_src;
#pragma unroll
  for (int p = 0; p < RPT; ++p) {
    const int i = row0 + tid + p * nt;
    rowi[p] = i;
    const float* rowp = S + (int64_t)i * ld_src;
    if (i < r && vec_src) {
#pragma unroll
      for (int c4 = 0; c4 < W / 4; ++c4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(rowp) + c4);
        a[p][4 * c4 + 0] = t.x;
        a[p][4 * c4 + 1] = t.y;
        a[p][4 * c4 + 2] = t.z;
        a[p][4 * c4 + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < W; ++c) a[p][c] = (i < r && c < w) ? __ldg(rowp + c) : 0.f;
    }
  }
  __syncthreads();

#pragma unroll 1
  for (int j = 0; j < w; ++j) {  // uniform across the cluster
    const int par = j & 1;

    // Phase A: slot partials over this thread's rows below j.
    float x[RPT];
    float sl[W];
#pragma unroll
    for (int q = 0; q < W; ++q) sl[q] = 0.f;
#pragma unroll
    for (int p = 0; p < RPT; ++p) {
      const float xj = pick32(a[p], j);
      x[p] = xj;
      const float xm = rowi[p] > j ? xj : 0.f;
#pragma unroll
      for (int q = 0; q < W; ++q) sl[q] = fmaf(xm, a[p][q], sl[q]);
      if (rowi[p] == j) {
#pragma unroll
        for (int q = 0; q < W; ++q) xch[par][1][q] = a[p][q];
      }
    }
    reduce_scatter32(sl, lane);
    red[par][warp][lane] = sl[0];
    __syncthreads();

    float tot = 0.f, rowv;
    if (cs > 1) {
      if (warp == 0) {
        for (int w2 = 0; w2 < nwarps; ++w2) tot += red[par][w2][lane];
        xch[par][0][lane] = tot;
      }
      cg::cluster_group cl = cg::this_cluster();
      cl.sync();
      tot = 0.f;
      for (int q = 0; q < cs; ++q) tot += cl.map_shared_rank(&xch[par][0][0], q)[lane];
      rowv = cl.map_shared_rank(&xch[par][1][0], 0)[lane];
    } else {
      for (int w2 = 0; w2 < nwarps; ++w2) tot += red[par][w2][lane];
      rowv = xch[par][1][lane];
    }

    // Every warp forms the reflector from the summed slots (lane = column).
    const float sigma = __shfl_sync(kFull, tot, j);
    const float alpha = __shfl_sync(kFull, rowv, j);
    const Reflector h = make_reflector(alpha, sigma);
    const float d = fmaf(h.scale, tot, rowv);
    fbuf[warp][lane] = lane > j ? h.tau * d : 0.f;
    if (warp == 0) {
      if (lane < j) Gs[lane][j] = scales[lane] * d;
      if (lane == 0) {
        taus[j] = h.tau;
        scales[j] = h.scale;
        betas[j] = h.beta;
      }
    }
    __syncwarp();

    // Phase B: apply H_j to this thread's rows of the trailing columns
    // (f_k = 0 for k <= j leaves the finished columns untouched).
    float vrow[RPT];
#pragma unroll
    for (int p = 0; p < RPT; ++p)
      vrow[p] = rowi[p] > j ? h.scale * x[p] : (rowi[p] == j ? 1.f : 0.f);
#pragma unroll
    for (int k4 = 0; k4 < W / 4; ++k4) {
      const float4 f4 = reinterpret_cast<const float4*>(fbuf[warp])[k4];
#pragma unroll
      for (int p = 0; p < RPT; ++p) {
        a[p][4 * k4 + 0] = fmaf(-f4.x, vrow[p], a[p][4 * k4 + 0]);
        a[p][4 * k4 + 1] = fmaf(-f4.y, vrow[p], a[p][4 * k4 + 1]);
        a[p][4 * k4 + 2] = fmaf(-f4.z, vrow[p], a[p][4 * k4 + 2]);
        a[p][4 * k4 + 3] = fmaf(-f4.w, vrow[p], a[p][4 * k4 + 3]);
      }
    }
    __syncwarp();  // fbuf is rewritten next step
  }
  __syncthreads();  // scales / betas / Gs from warp 0 visible to all

  // Write the factored panel rows back: R above the diagonal, beta on it,
  // v = scale * x below it.
  float* __restrict__ D = dst + m * sb_dst;
#pragma unroll
  for (int p = 0; p < RPT; ++p) {
    const int i = rowi[p];
    if (i >= r) continue;
#pragma unroll
    for (int c = 0; c < W; ++c)
      a[p][c] = i > c ? scales[c] * a[p][c] : (i == c ? betas[c] : a[p][c]);
    const float (&o)[W] = a[p];
    float* rowp = D + (int64_t)i * ld_dst;
    if (vec_dst) {
#pragma unroll
      for (int c4 = 0; c4 < W / 4; ++c4)
        reinterpret_cast<float4*>(rowp)[c4] =
            make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
    } else {
#pragma unroll
      for (int c = 0; c < W; ++c)
        if (c < w) rowp[c] = o[c];
    }
    if (V_out != nullptr) {
      float* vrow = V_out + m * (int64_t)r * w + (int64_t)i * w;
#pragma unroll
      for (int c = 0; c < W; ++c)
        if (c < w) vrow[c] = (i > c) ? o[c] : (i == c ? 1.f : 0.f);
    }
    if (Vsplit != nullptr) {  // the unit-lower reflectors, TF32-split for the tensor cores
      float* vh = Vsplit + m * vs_mat + (int64_t)(vs_row0 + i) * vs_ld;
      float* vl = vh + vs_plane;
#pragma unroll
      for (int c4 = 0; c4 < W / 4; ++c4) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 4 * c4 + e;
          v[e] = (i > c) ? o[c] : (i == c ? 1.f : 0.f);
        }
        float4 hi, lo;
        tc::split4(make_float4(v[0], v[1], v[2], v[3]), hi, lo);
        reinterpret_cast<float4*>(vh)[c4] = hi;
        reinterpret_cast<float4*>(vl)[c4] = lo;
      }
      if (vs_zero && i < W) {  // the next panel's reflectors are zero in these rows
#pragma unroll
        for (int c4 = 0; c4 < W / 4; ++c4) {
          reinterpret_cast<float4*>(vh + W)[c4] = make_float4(0.f, 0.f, 0.f, 0.f);
          reinterpret_cast<float4*>(vl + W)[c4] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  }

  if (rank == 0) {
    if (tid < w) tau_out[m * tau_sb + tid] = taus[tid];
    if (warp == 0 && T_out != nullptr) {
      // Forward LARFT: lane `row` computes row `row` of T.
      const int row = lane;
      float trow[W];
#pragma unroll
      for (int i = 0; i < W; ++i) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < i; ++q) t = fmaf(trow[q], Gs[q][i], t);
        trow[i] = row < i ? -taus[i] * t : (row == i ? taus[i] : 0.f);
      }
      if (row < w) {
        float* Tm = T_out + m * T_sb + (int64_t)row * t_ld;
#pragma unroll
        for (int i = 0; i < W; ++i)
          if (i < t_ld && (t_ld == W || i < w)) Tm[i] = (i < w) ? trow[i] : 0.f;
      } else if (t_ld == W) {
        float* Tm = T_out + m * T_sb + (int64_t)row * t_ld;
#pragma unroll
        for (int i = 0; i < W; ++i) Tm[i] = 0.f;
      }
    }
  }
  if (cs > 1) cg::this_cluster().sync();  // peers may still read our xch
}

template <int RPT>
int launch_panel_rpt(const float* src, int64_t sb_src, int64_t ld_src,
                     float* dst, int64_t sb_dst, int64_t ld_dst, float* tau_out,
                     int64_t tau_sb, float* T_out, int64_t T_sb, int t_ld,
                     float* V_out, float* Vsplit, int64_t vs_mat, int64_t vs_plane,
                     int vs_row0, int vs_ld, int vs_zero, int64_t batch, int r, int w, int cs,
                     int nt, cudaStream_t stream) {
  const bool vec_src = w == W && ld_src % 4 == 0 && sb_src % 4 == 0 &&
                       (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  const bool vec_dst = w == W && ld_dst % 4 == 0 && sb_dst % 4 == 0 &&
                       (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(batch * cs), 1, 1);
  cfg.blockDim = dim3((unsigned)nt, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cs > 1 ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, k_panel<RPT>, src, sb_src, ld_src, dst, sb_dst, ld_dst, tau_out,
      tau_sb, T_out, T_sb, t_ld, V_out, Vsplit, vs_mat, vs_plane, vs_row0, vs_ld, vs_zero, r, w,
      cs, (int)vec_src, (int)vec_dst);
  note_launches(1);
  return e == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace

// Rows per thread: 1 up to 128 rows (one CTA of up to 128 threads), else 4:
// one CTA of up to 256 threads up to 1024 rows, beyond that a cluster of cs
// CTAs of 256 threads (cs a power of two, <= 8 for the launch to be accepted).
// qrb_set_config("panel_rpt") = 1 (CTAs of up to 512 threads) or 2 (up to 256)
// selects that many rows per thread instead (4 where that would need more than
// 8 CTAs).
static void panel_shape(int r, int* rpt, int* cs, int* nt) {
  const int pref = panel_rpt();
  int R = pref > 0 ? pref : (r > 128 ? 4 : 1);
  int c = 1;
  for (;;) {
    const int per_cta_max = (R >= 2 ? kPanelCtaThreads : kMaxThreads) * R;
    const int need = (r + per_cta_max - 1) / per_cta_max;
    c = 1;
    while (c < need) c <<= 1;  // cluster sizes 1, 2, 4, 8
    if (c <= kMaxCluster || R >= 4) break;
    R = 4;
  }
  int threads = (r + R * c - 1) / (R * c);
  threads = ((threads + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  *rpt = R;
  *cs = c;
  *nt = threads;
}

int panel_cluster_size(int r) {
  int rpt, cs, nt;
  panel_shape(r, &rpt, &cs, &nt);
  return cs;
}

int launch_panel(const float* src, int64_t sb_src, int64_t ld_src, float* dst,
                 int64_t sb_dst, int64_t ld_dst, float* tau_out, int64_t tau_sb,
                 float* T_out, int64_t T_sb, int t_ld, float* V_out,
                 int64_t batch, int r, int w, cudaStream_t stream, float* Vsplit,
                 int64_t vs_mat, int64_t vs_plane, int vs_row0, int vs_ld, bool vs_zero) {
  if (r < 1 || w < 1 || w > W) return QRB_ERR_UNSUPPORTED;
  if (Vsplit != nullptr && (w != W || (reinterpret_cast<uintptr_t>(Vsplit) & 15) != 0 ||
                            vs_ld % 4 != 0 || vs_ld < (vs_zero ? 2 * W : W)))
    return QRB_ERR_UNSUPPORTED;
  int rpt, cs, nt;
  panel_shape(r, &rpt, &cs, &nt);
  if (cs > kMaxCluster) return QRB_ERR_UNSUPPORTED;
  if (batch * cs > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  if (rpt == 1)
    return launch_panel_rpt<1>(src, sb_src, ld_src, dst, sb_dst, ld_dst, tau_out,
                               tau_sb, T_out, T_sb, t_ld, V_out, Vsplit, vs_mat, vs_plane, vs_row0, vs_ld, (int)vs_zero, batch, r, w, cs,
                               nt, stream);
  if (rpt == 2)
    return launch_panel_rpt<2>(src, sb_src, ld_src, dst, sb_dst, ld_dst, tau_out,
                               tau_sb, T_out, T_sb, t_ld, V_out, Vsplit, vs_mat, vs_plane, vs_row0, vs_ld, (int)vs_zero, batch, r, w, cs,
                               nt, stream);
  return launch_panel_rpt<4>(src, sb_src, ld_src, dst, sb_dst, ld_dst, tau_out,
                             tau_sb, T_out, T_sb, t_ld, V_out, Vsplit, vs_mat, vs_plane, vs_row0, vs_ld, (int)vs_zero, batch, r, w, cs,
                             nt, stream);
}

}  // namespace qrb

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
// column G[m][j] = v_m(j) + scale * slot[m] (m < j) used by the T recurrence.
// The reduction is a warp reduce-scatter (31 shuffles), a cross-warp sum in
// shared memory, and for clusters a push of each CTA's sums into every rank's
// shared memory (st.async, completing on the receiver's mbarrier; the waits
// are bounded and a timeout sets the device error flag). Every warp forms the
// reflector coefficients itself from the summed slots, so a step costs one
// block barrier (plus one mbarrier wait for clusters); the partial-sum
// buffers alternate by step parity so no second barrier is needed.
//
// The column loop is a runtime loop with a compact body: the register array
// is indexed only by compile-time constants, and the current column is always
// register 0 because every step rotates the columns down by one (the update
// of column j + q + 1 writes register q) and puts the finished column j, in
// its final form (reflector v = x / (alpha - beta) below the diagonal, beta
// on it, R above it), into register 31. After the 32 steps (a panel narrower
// than 32 runs its zero padding columns as tau = 0 steps) every column is
// back in its own register.
//
// Semantics follow the reference panel kernel (src/qrbench/triton_kernels.py
// :839-871 reflectors and packing, :873-884 unit-lower V, :886-909 forward
// LARFT recurrence T[i,i] = tau_i, T[:i,i] = -tau_i T[:i,:i] (V[:,:i]^T v_i)).
#include <cooperative_groups.h>

#include "qrb_common.cuh"
#include "qrb_tc.cuh"
#include "qrb_tma.cuh"

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

// Shared-memory address of the same variable in cluster rank q.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t a, uint32_t q) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(q));
  return r;
}
// Store v into a peer's shared memory; the store completes 4 bytes of
// transactions on the peer's mbarrier at bar.
__device__ __forceinline__ void push_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                   addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
}

template <int RPT>
__global__ void __launch_bounds__(RPT >= 2 ? kPanelCtaThreads : kMaxThreads, 1)
k_panel(const float* __restrict__ src, int64_t sb_src, int64_t ld_src,
        float* __restrict__ dst, int64_t sb_dst, int64_t ld_dst,
        float* __restrict__ tau_out, int64_t tau_sb, float* __restrict__ T_out,
        int64_t T_sb, int t_ld, float* __restrict__ V_out, float* __restrict__ Vsplit,
        int64_t vs_mat, int64_t vs_plane, int vs_row0, int vs_ld, int vs_zero, int r, int w,
        int cs, int vec_src, int vec_dst, int* __restrict__ err, long long wait_limit) {
  __shared__ float red[2][kMaxThreads / 32][W];  // [parity][warp][slot]
  __shared__ float rowj[2][W];                   // [parity] row j of the panel (rotated)
  __shared__ __align__(16) float fbuf[kMaxThreads / 32][W];  // per-warp tau_j * d, shifted
  __shared__ float Gs[W][W + 1];                 // Gram V^T V, strictly upper part
  __shared__ float taus[W];
  __shared__ float Tsm[W][W + 1], Ysm[W][W + 1];  // T and the products of its block steps
  // cluster exchange: [parity][source rank][slot] CTA slot sums, row j from
  // rank 0, one mbarrier per parity
  __shared__ float inbox[2][kMaxCluster][W];
  __shared__ float rowbox[2][W];
  __shared__ __align__(8) uint64_t xbar[2];

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
  if (tid < W) taus[tid] = 0.f;
  if (cs > 1) {
    if (tid == 0) {
      tma::mbar_init(tma::smem_addr(&xbar[0]), 1);
      tma::mbar_init(tma::smem_addr(&xbar[1]), 1);
      tma::mbar_fence_init();
    }
    // the peers may push into this CTA once every rank has arrived here (the
    // wait is after the panel load, which it overlaps)
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
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
  if (cs > 1)
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // peers initialised
  __syncthreads();

  const uint32_t in_mine = tma::smem_addr(&inbox[0][rank][lane]);
  const uint32_t row_mine = tma::smem_addr(&rowbox[0][lane]);
  const uint32_t bar_mine = tma::smem_addr(&xbar[0]);
  constexpr uint32_t kParIn = kMaxCluster * W * 4, kParRow = W * 4, kParBar = 8;
  bool dead = false;  // a bounded wait of this thread ran out

  // Column j is always register 0: each step rotates the columns down by one
  // and puts the finished column, in its final form (reflector below the
  // diagonal, beta on it, R above), into register 31; after 32 steps every
  // column is back in its own register. Padding columns (w < 32) are zero and
  // take tau = 0 steps.
#pragma unroll 1
  for (int j = 0; j < W; ++j) {  // uniform across the cluster
    const int par = j & 1;

    // Phase A: slot partials over this thread's rows below j (slot q =
    // rotated column q: trailing columns j + q for q < 32 - j, finished
    // columns q + j - 32 above).
    float x[RPT];
    float sl[W];
#pragma unroll
    for (int q = 0; q < W; ++q) sl[q] = 0.f;
#pragma unroll
    for (int p = 0; p < RPT; ++p) {
      x[p] = a[p][0];
      const float xm = rowi[p] > j ? x[p] : 0.f;
#pragma unroll
      for (int q = 0; q < W; ++q) sl[q] = fmaf(xm, a[p][q], sl[q]);
      if (rowi[p] == j) {
#pragma unroll
        for (int q = 0; q < W; ++q) rowj[par][q] = a[p][q];
      }
    }
    reduce_scatter32(sl, lane);
    red[par][warp][lane] = sl[0];
    __syncthreads();

    float tot = 0.f, rowv;
    // Sums in a fixed order (warp 0 first, rank 0 first), unrolled to the
    // largest count with a predicate so that the loads issue together.
    auto warp_sum = [&]() {
      float t = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kMaxThreads / 32; ++w2)
        if (w2 < nwarps) t += red[par][w2][lane];
      return t;
    };
    if (cs > 1) {
      // this CTA's sums (and rank 0's row j) go to every rank, the pushes
      // spread over the warps (warp w serves ranks w, w + nwarps, ...); every
      // rank waits for all of them on its own mbarrier
      const uint32_t bar = bar_mine + par * kParBar;
      if (warp < cs) {
        const float ct = warp_sum();
        const float rv = rowj[par][lane];
        for (int q = warp; q < cs; q += nwarps) {
          const uint32_t rb = mapa_rank(bar, (uint32_t)q);
          push_f32(mapa_rank(in_mine + par * kParIn, (uint32_t)q), ct, rb);
          if (rank == 0) push_f32(mapa_rank(row_mine + par * kParRow, (uint32_t)q), rv, rb);
        }
      }
      if (tid == 0) tma::mbar_expect_tx(bar, (uint32_t)((cs + 1) * W * 4));
      if (!dead && !tma::mbar_wait_bounded(bar, (uint32_t)((j >> 1) & 1), wait_limit)) {
        dead = true;
        atomicExch(err, 1);
      }
#pragma unroll
      for (int q = 0; q < kMaxCluster; ++q)
        if (q < cs) tot += inbox[par][q][lane];
      rowv = rowbox[par][lane];
    } else {
      tot = warp_sum();
      rowv = rowj[par][lane];
    }

    // Every warp forms the reflector from the summed slots (lane = rotated
    // column): lane 0 is column j.
    const float sigma = __shfl_sync(kFull, tot, 0);
    const float alpha = __shfl_sync(kFull, rowv, 0);
    const Reflector h = make_reflector(alpha, sigma);
    const float d = fmaf(h.scale, tot, rowv);  // v_j^T (rotated column lane)
    const int live = W - j;                    // lanes 1 .. live - 1: trailing columns
    fbuf[warp][(lane + W - 1) & (W - 1)] = (lane >= 1 && lane < live) ? h.tau * d : 0.f;
    if (warp == 0) {
      if (lane >= live) Gs[lane - live][j] = d;  // finished column lane - live: v^T v_j
      if (lane == 0) taus[j] = h.tau;
    }
    __syncwarp();

    // Phase B: apply H_j to this thread's rows of the trailing columns while
    // rotating: register q takes rotated column q + 1 (f = 0 for finished
    // columns), register 31 the finished column j.
    float vrow[RPT], fin[RPT];
#pragma unroll
    for (int p = 0; p < RPT; ++p) {
      const bool below = rowi[p] > j;
      vrow[p] = below ? h.scale * x[p] : (rowi[p] == j ? 1.f : 0.f);
      fin[p] = below ? vrow[p] : (rowi[p] == j ? h.beta : x[p]);
    }
#pragma unroll
    for (int k4 = 0; k4 < W / 4; ++k4) {
      const float4 f4 = reinterpret_cast<const float4*>(fbuf[warp])[k4];
      const float fk[4] = {f4.x, f4.y, f4.z, f4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = 4 * k4 + e;
        if (q < W - 1) {
#pragma unroll
          for (int p = 0; p < RPT; ++p) a[p][q] = fmaf(-fk[e], vrow[p], a[p][q + 1]);
        }
      }
    }
#pragma unroll
    for (int p = 0; p < RPT; ++p) a[p][W - 1] = fin[p];
    __syncwarp();  // fbuf is rewritten next step
  }
  __syncthreads();  // taus / Gs from warp 0 visible to all

  // Write the factored panel rows back (R above the diagonal, beta on it, v
  // below it: the registers hold the final values).
  float* __restrict__ D = dst + m * sb_dst;
#pragma unroll
  for (int p = 0; p < RPT; ++p) {
    const int i = rowi[p];
    if (i >= r) continue;
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
    if (T_out != nullptr) {
      // T by blocks: T of the first 2b columns from the two T of b columns,
      //   T12 = -T11 (V1^T V2) T22   (V1^T V2 from the Gram, strictly upper),
      // for b = 1, 2, 4, 8, 16, every entry of a level in parallel. The same
      // matrix as the forward column recurrence (src/qrbench/triton_kernels.py
      // :886-909), summed in another order.
      for (int e = tid; e < W * W; e += nt) {
        const int i = e / W, k = e % W;
        Tsm[i][k] = i == k ? taus[i] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int lb = 0; lb < 5; ++lb) {  // block size b = 2^lb (a constant once unrolled)
        const int b = 1 << lb, cnt = (W / 2) * b;  // (W / 2b) pairs x b^2 entries
        for (int e = tid; e < cnt; e += nt) {  // Y = G12 T22
          const int a0 = (e >> (2 * lb)) * 2 * b, b0 = a0 + b;
          const int i = (e >> lb) & (b - 1), k = e & (b - 1);
          float y = 0.f;
#pragma unroll
          for (int q = 0; q < b; ++q)
            if (q <= k) y = fmaf(Gs[a0 + i][b0 + q], Tsm[b0 + q][b0 + k], y);
          Ysm[a0 + i][b0 + k] = y;
        }
        __syncthreads();
        for (int e = tid; e < cnt; e += nt) {  // T12 = -T11 Y
          const int a0 = (e >> (2 * lb)) * 2 * b, b0 = a0 + b;
          const int i = (e >> lb) & (b - 1), k = e & (b - 1);
          float t = 0.f;
#pragma unroll
          for (int q = 0; q < b; ++q)
            if (q >= i) t = fmaf(Tsm[a0 + i][a0 + q], Ysm[a0 + q][b0 + k], t);
          Tsm[a0 + i][b0 + k] = -t;
        }
        __syncthreads();
      }
      for (int e = tid; e < W * W; e += nt) {
        const int row = e / W, i = e % W;
        if (i >= t_ld) continue;
        float* Tm = T_out + m * T_sb + (int64_t)row * t_ld;
        if (row < w) {
          if (t_ld == W || i < w) Tm[i] = (i < w) ? Tsm[row][i] : 0.f;
        } else if (t_ld == W) {
          Tm[i] = 0.f;
        }
      }
    }
  }
  if (cs > 1) cg::this_cluster().sync();  // every push into this CTA has landed
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
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (cs > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)cs;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  na += stream_priority_attr(stream, &attr[na]);
  cfg.attrs = attr;
  cfg.numAttrs = (unsigned)na;
  static int* err_ptr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  if (err_ptr[dev] == nullptr && device_error_ptr(&err_ptr[dev]) != QRB_OK) return QRB_ERR_DEVICE;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, k_panel<RPT>, src, sb_src, ld_src, dst, sb_dst, ld_dst, tau_out,
      tau_sb, T_out, T_sb, t_ld, V_out, Vsplit, vs_mat, vs_plane, vs_row0, vs_ld, vs_zero, r, w,
      cs, (int)vec_src, (int)vec_dst, err_ptr[dev], device_wait_limit());
  note_launches(1);
  return e == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace

// Rows per thread: 1 up to 128 rows (one CTA of up to 512 threads); above,
// 2 when the batch's panels then still fit on the SMs at once (clusters of
// 256-thread CTAs, 512 rows each: the column steps' latency chain is then
// shorter), else 4 (256-thread CTAs of 1024 rows: fewer CTAs when there are
// more than the SMs hold). Beyond 1 CTA, a cluster of cs CTAs (cs a power of
// two, <= 8 for the launch to be accepted). Measured on B200: 16.0 vs
// 16.7 ms with 2 rows per thread at 8 x 4096^2, 4.56 vs 4.41 ms at
// 640 x 512^2 (320 matrices per panel launch). qrb_set_config("panel_rpt") = 1
// (CTAs of up to 512 threads), 2 or 4 forces that many rows per thread (4
// where that would need more than 8 CTAs).
static void panel_shape(int r, int64_t batch, int* rpt, int* cs, int* nt) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      sms = v;
    else
      sms = 148;
  }
  const int pref = panel_rpt();
  int R = pref;
  if (R == 0) {
    if (r <= 128) {
      R = 1;
    } else {
      const int per2 = kPanelCtaThreads * 2;
      int c2 = 1;
      while (c2 * per2 < r) c2 <<= 1;
      R = (c2 <= kMaxCluster && batch * c2 <= sms) ? 2 : 4;
    }
  }
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

int panel_cluster_size(int r, int64_t batch) {
  int rpt, cs, nt;
  panel_shape(r, batch, &rpt, &cs, &nt);
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
  panel_shape(r, batch, &rpt, &cs, &nt);
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

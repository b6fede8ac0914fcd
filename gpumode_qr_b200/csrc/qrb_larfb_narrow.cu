// Narrow trailing update: C <- C - V T^T (V^T C) for the (at most) 64 columns
// next to a panel, in place, FP32 FFMA, with the rows of each matrix split
// across a thread-block cluster (one cluster per matrix and 32-column block).
//
// This is the update the look-ahead puts on the critical path: the next panel
// waits for its own 32 columns, which are a tall r x 32 block (r up to 8192).
// One CTA per matrix would walk all r rows alone; here a cluster of cs CTAs
// (cs <= 8) takes rs rows each:
//   load     the CTA's rows of V (unit lower: the diagonal block is masked in
//            shared memory) and of C, 16-byte cp.async, all requests in flight
//            at once (chunks of at most 512 rows);
//   W_q      lane c of warp w accumulates column c of V_q^T C_q over rows
//            w, w + 8, ...; the 8 warp partials are summed in a fixed order;
//   W        every CTA sums the cs partials W_q over distributed shared
//            memory, rank 0 first, so all CTAs hold the same bits;
//   W'       = T^T W (32 x 32 x 32, shared memory), stored negated;
//   C        lane c of warp w updates column c of rows w, w + 8, ... from the
//            staged V and C and writes them back (128-byte rows per warp).
// Reference semantics: the trailing update of src/qrbench/variants.py:800-804
// (W1 = V^T C, W2 = T^T W1, C -= V W2) on the columns j + w .. j + w + 31.
#include "qrb_common.cuh"

namespace qrb {

namespace {

constexpr int K = kPanelW;       // reflectors and (padded) columns
constexpr int NT = 256;          // threads per CTA
constexpr int NWARP = NT / 32;
constexpr int kMaxChunk = 512;   // rows of V and C staged per chunk
constexpr int kRowsPerCta = 256; // target rows per cluster rank

// Shared memory: V and C chunks (rch x 32 each, row-major as in global
// memory), the per-warp partials, this CTA's W_q (read by the peers), the full
// W, and T.
struct NarrowLayout {
  int rch;
  __host__ __device__ size_t off_v() const { return 0; }
  __host__ __device__ size_t off_c() const { return (size_t)rch * K * 4; }
  __host__ __device__ size_t off_wp() const { return off_c() + (size_t)rch * K * 4; }
  __host__ __device__ size_t off_wq() const { return off_wp() + (size_t)NWARP * K * K * 4; }
  __host__ __device__ size_t off_wf() const { return off_wq() + (size_t)K * K * 4; }
  __host__ __device__ size_t off_t() const { return off_wf() + (size_t)K * K * 4; }
  __host__ __device__ size_t bytes() const { return off_t() + (size_t)K * (K + 1) * 4; }
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The float at shared-memory address p of cluster rank q.
__device__ __forceinline__ float ld_peer(const float* p, uint32_t q) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  float v;
  asm volatile(
      "{\n\t.reg .u32 pa;\n\t"
      "mapa.shared::cluster.u32 pa, %1, %2;\n\t"
      "ld.shared::cluster.f32 %0, [pa];\n\t}"
      : "=f"(v)
      : "r"(a), "r"(q)
      : "memory");
  return v;
}

// Stage rows [row0, row0 + nr) (relative to the panel's diagonal row) of V
// and C into shared memory; the C columns at or beyond cw read as zero.
__device__ __forceinline__ void stage(float* Vs, float* Cs, const float* V, int64_t ldv,
                                      const float* C, int64_t ldc, int row0, int nr, int cw) {
  const int tid = threadIdx.x;
  for (int e = tid; e < nr * (K / 4); e += NT) {
    const int rr = e >> 3, q = e & 7;
    const int64_t g = row0 + rr;
    cp_async16(Vs + rr * K + 4 * q, V + g * ldv + 4 * q);
    if (4 * q < cw)
      cp_async16(Cs + rr * K + 4 * q, C + g * ldc + 4 * q);
    else
      *reinterpret_cast<float4*>(Cs + rr * K + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  cp_async_wait_all();
  __syncthreads();
  if (row0 < K) {  // the diagonal block: unit diagonal, zero above it
    for (int e = tid; e < K * K; e += NT) {
      const int rr = e >> 5, i = e & 31;
      if (rr < nr && row0 + rr < K) {
        const int g = row0 + rr;
        if (i >= g) Vs[rr * K + i] = (i == g) ? 1.f : 0.f;
      }
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NT, 1)
k_larfb_narrow(const float* __restrict__ V, int64_t sVb, int64_t ldv, const float* __restrict__ T,
               int64_t sTb, int t_ld, float* __restrict__ C, int64_t sCb, int64_t ldc, int r,
               int cw, int cs, int rs, int rch) {
  extern __shared__ __align__(16) unsigned char smem[];
  const NarrowLayout L{rch};
  float* Vs = reinterpret_cast<float*>(smem + L.off_v());
  float* Cs = reinterpret_cast<float*>(smem + L.off_c());
  float* Wp = reinterpret_cast<float*>(smem + L.off_wp());
  float* Wq = reinterpret_cast<float*>(smem + L.off_wq());
  float* Wf = reinterpret_cast<float*>(smem + L.off_wf());
  float* Ts = reinterpret_cast<float*>(smem + L.off_t());

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cs > 1 ? cluster_rank() : 0;
  const int64_t m = blockIdx.x / cs;
  const float* Vm = V + m * sVb;
  float* Cm = C + m * sCb + K * blockIdx.y;  // this CTA's block of 32 columns
  cw = min(K, cw - K * (int)blockIdx.y);
  const float* Tm = T + m * sTb;
  for (int e = tid; e < K * K; e += NT) Ts[(e >> 5) * (K + 1) + (e & 31)] = Tm[(e >> 5) * t_ld + (e & 31)];

  const int rbeg = (int)rank * rs;
  const int rend = min(r, rbeg + rs);
  const int nrows = rend > rbeg ? rend - rbeg : 0;
  const int nch = (nrows + rch - 1) / rch;

  // W_q: lane c of warp w accumulates column c over rows w, w + 8, ...
  float acc[K];
#pragma unroll
  for (int i = 0; i < K; ++i) acc[i] = 0.f;
  for (int ch = 0; ch < nch; ++ch) {
    const int row0 = rbeg + ch * rch;
    const int nr = min(rch, rend - row0);
    if (ch > 0) __syncthreads();  // the previous chunk is consumed
    stage(Vs, Cs, Vm, ldv, Cm, ldc, row0, nr, cw);
#pragma unroll 4
    for (int rr = warp; rr < nr; rr += NWARP) {
      const float cv = Cs[rr * K + lane];
      const float4* vr = reinterpret_cast<const float4*>(Vs + rr * K);
#pragma unroll
      for (int q = 0; q < K / 4; ++q) {
        const float4 v = vr[q];
        acc[4 * q + 0] = fmaf(v.x, cv, acc[4 * q + 0]);
        acc[4 * q + 1] = fmaf(v.y, cv, acc[4 * q + 1]);
        acc[4 * q + 2] = fmaf(v.z, cv, acc[4 * q + 2]);
        acc[4 * q + 3] = fmaf(v.w, cv, acc[4 * q + 3]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < K; ++i) Wp[(warp * K + i) * K + lane] = acc[i];
  __syncthreads();
  for (int e = tid; e < K * K; e += NT) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) s += Wp[w * K * K + e];
    Wq[e] = s;
  }
  // W = sum over the cluster ranks in rank order (the same bits everywhere)
  if (cs > 1) {
    cluster_arrive();
    cluster_wait();
    for (int e = tid; e < K * K; e += NT) {
      float s = 0.f;
      for (int q = 0; q < cs; ++q) s += ld_peer(Wq + e, (uint32_t)q);
      Wf[e] = s;
    }
    cluster_arrive();  // done reading the peers' W_q; waited for before exit
  } else {
    for (int e = tid; e < K * K; e += NT) Wf[e] = Wq[e];
  }
  __syncthreads();
  // -W' = -(T^T W), into the (now free) first warp partial
  for (int e = tid; e < K * K; e += NT) {
    const int i = e >> 5, c = e & 31;
    float s = 0.f;
#pragma unroll 8
    for (int j = 0; j < K; ++j) s = fmaf(Ts[j * (K + 1) + i], Wf[j * K + c], s);
    Wp[e] = -s;
  }
  __syncthreads();
  float w2[K];
#pragma unroll
  for (int i = 0; i < K; ++i) w2[i] = Wp[i * K + lane];

  // C -= V W': the staged chunk when the CTA's rows fit one, else restaged
  for (int ch = 0; ch < nch; ++ch) {
    const int row0 = rbeg + ch * rch;
    const int nr = min(rch, rend - row0);
    if (nch > 1) {
      __syncthreads();
      stage(Vs, Cs, Vm, ldv, Cm, ldc, row0, nr, cw);
    }
#pragma unroll 4
    for (int rr = warp; rr < nr; rr += NWARP) {
      float cv = Cs[rr * K + lane];
      const float4* vr = reinterpret_cast<const float4*>(Vs + rr * K);
#pragma unroll
      for (int q = 0; q < K / 4; ++q) {
        const float4 v = vr[q];
        cv = fmaf(v.x, w2[4 * q + 0], cv);
        cv = fmaf(v.y, w2[4 * q + 1], cv);
        cv = fmaf(v.z, w2[4 * q + 2], cv);
        cv = fmaf(v.w, w2[4 * q + 3], cv);
      }
      if (lane < cw) Cm[(int64_t)(row0 + rr) * ldc + lane] = cv;
    }
  }
  if (cs > 1) cluster_wait();  // the peers have read this CTA's W_q
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

void larfb_narrow_shape(int r, int* cs, int* rs, int* rch) {
  int c = (r + kRowsPerCta - 1) / kRowsPerCta;
  if (c < 1) c = 1;
  if (c > kMaxCluster) c = kMaxCluster;
  int s = (r + c - 1) / c;
  s = (s + 31) / 32 * 32;
  *cs = c;
  *rs = s;
  *rch = s < kMaxChunk ? s : kMaxChunk;
}

bool larfb_narrow_supported(const float* V, int64_t sVb, int64_t ldv, const float* C, int64_t sCb,
                            int64_t ldc, int k, int cw) {
  return k == K && cw >= 1 && cw <= 2 * K && cw % 4 == 0 && ldv % 4 == 0 && sVb % 4 == 0 &&
         ldc % 4 == 0 && sCb % 4 == 0 && aligned16(V) && aligned16(C);
}

int launch_larfb_narrow(const float* V, int64_t sVb, int64_t ldv, const float* T, int64_t sTb,
                        int t_ld, float* C, int64_t sCb, int64_t ldc, int64_t batch, int r,
                        int cw, cudaStream_t stream) {
  if (r < 1 || batch < 1 || !larfb_narrow_supported(V, sVb, ldv, C, sCb, ldc, K, cw))
    return QRB_ERR_UNSUPPORTED;
  int cs, rs, rch;
  larfb_narrow_shape(r, &cs, &rs, &rch);
  if (batch * cs > 0x7fffffffLL) return QRB_ERR_UNSUPPORTED;
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QRB_ERR_DEVICE;
  const NarrowLayout L{rch};
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k_larfb_narrow, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)NarrowLayout{kMaxChunk}.bytes()) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(batch * cs), (unsigned)((cw + K - 1) / K), 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = L.bytes();
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_larfb_narrow, V, sVb, ldv, T, sTb, t_ld, C,
                                           sCb, ldc, r, cw, cs, rs, rch);
  note_launches(1);
  return e == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
}

}  // namespace qrb

// Shared device helpers and internal launcher declarations of libqrb200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qrb200.h"

namespace qrb {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kPanelW = 32;        // panel / block-reflector width
constexpr int kFusedMaxN = 32;     // largest n of the warp-per-matrix kernel
constexpr int kFusedMidMaxN = 128; // largest n of the CTA-per-matrix fused kernel
constexpr int64_t kFusedMidMaxBatch = 592;  // 64 < n <= 96: two waves of 2 CTAs per SM
constexpr int kLookaheadMinN = 4096;  // automatic panel look-ahead from this n (measured on B200:
                                      // 29.7 vs 30.5 ms at 8 x 4096, slower at n = 512 and 1024)
constexpr int kMaxN = 8192;        // 4096 rows per CTA-cluster of 8 x 512 x 2
constexpr int kMaxCluster = 8;
constexpr int64_t kHostDirectBlocks = 148;  // direct host-memory kernel: blocks of 4 warps

// Householder coefficients for one column, LAPACK slarfg convention as the
// reference kernels state it (src/qrbench/triton_kernels.py:691-700):
//   sigma = ||x(j+1:)||^2, norm = sqrt(alpha^2 + sigma),
//   beta = -sign(alpha) * norm (alpha >= 0 -> -norm), tau = (beta-alpha)/beta,
//   v = x / (alpha - beta); sigma <= 0 -> tau = 0, beta = alpha (identity).
// Evaluated without divisions by the identities (u = |alpha| + norm > 0)
//   alpha - beta = sign(alpha) * u,   tau = u / norm = 1 + |alpha| / norm,
// with 1/norm from the hardware reciprocal square root and 1/u from the
// hardware reciprocal, each refined by one Newton-Raphson step
// (r <- r (3 - n2 r^2) / 2 and r <- r + r (1 - u r)). Both forms are exact in
// real arithmetic; in FP32 they agree to a few ulp. Outside
// 1e-30 < alpha^2 + sigma < 1e30 the plain IEEE formulas are used.
struct Reflector {
  float beta, tau, scale;
};

// 1/x for normal x of moderate size (1e-16 < |x| < 1e16 here): hardware
// approximation plus one Newton-Raphson step.
__device__ __forceinline__ float recip_nr(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return fmaf(r, fmaf(-x, r, 1.0f), r);
}

__device__ __forceinline__ Reflector make_reflector(float alpha, float sigma) {
  Reflector h;
  if (sigma > 0.f) {
    const float n2 = fmaf(alpha, alpha, sigma);
    const float aa = fabsf(alpha);
    const bool neg = alpha < 0.f;
    if (n2 > 1e-30f && n2 < 1e30f) {
      float r = rsqrtf(n2);
      r = r * fmaf(-0.5f * n2 * r, r, 1.5f);  // one Newton step on 1/sqrt(n2)
      const float norm = n2 * r;
      const float ru = recip_nr(aa + norm);
      h.beta = neg ? norm : -norm;
      h.tau = fmaf(aa, r, 1.0f);
      h.scale = neg ? -ru : ru;
    } else {  // tiny or huge: plain IEEE square root and divisions
      const float norm = sqrtf(n2);
      const float beta = neg ? norm : -norm;
      h.beta = beta;
      h.tau = (beta - alpha) / beta;
      h.scale = 1.0f / (alpha - beta);
    }
  } else {
    h.beta = alpha;
    h.tau = 0.f;
    h.scale = 0.f;
  }
  return h;
}

// Internal launchers (one per kernel family); all return qrb status codes and
// only enqueue work on `stream`.
// Which operands of the fused kernel are page-locked host memory mapped into
// the device's address space (accessed with streaming loads and stores).
enum class HostMem { kNone, kTau, kOutputs /* H and tau */, kAll /* A, H and tau */ };

// max_blocks > 0 caps the grid when A or H is host memory (each warp then
// loops over matrix pairs).
int launch_fused_small(const float* A, int64_t sAb, int64_t sAr, float* H,
                       float* tau, int64_t batch, int n, cudaStream_t stream,
                       HostMem where = HostMem::kNone, int64_t max_blocks = 0);

// CTA-per-matrix fused QR for kFusedMaxN < n <= kFusedMidMaxN (one launch).
int launch_fused_mid(const float* A, int64_t sAb, int64_t sAr, float* H, float* tau,
                     int64_t batch, int n, cudaStream_t stream);
// qrb_set_config("mid_fused"): 1 (default) = 32 < n <= 64 and 96 < n <= 128,
// and 64 < n <= 96 up to kFusedMidMaxBatch matrices, run the CTA-per-matrix
// fused kernel; 2 = every 32 < n <= 128; 0 = always the blocked panel route.
bool mid_fused_enabled();
bool mid_fused_always();

// Factor the r x w panel starting at (row 0, col 0) of src (row stride ld_src,
// matrix stride sb_src) into dst; tau to tau_out[m*tau_sb + c]; T to
// T_out[m*T_sb + row*t_ld + col] (t_ld == 32: a zero-padded 32 x 32 block;
// t_ld == w: a dense w x w block). V_out, when non-null, receives the explicit
// unit-lower reflectors (r x w, contiguous per matrix).
// Vsplit, when non-null (w == 32 only), receives the unit-lower reflectors
// split into a TF32 high part (row vs_row0 + i of matrix m at
// Vsplit + m * vs_mat + (vs_row0 + i) * vs_ld, 32 floats) and the
// TF32-rounded remainder (vs_plane floats further on): the operands of the
// tensor-core update. vs_zero also writes zeros into the 32 floats after each
// of the first 32 rows (where a second panel's reflectors vanish).
int launch_panel(const float* src, int64_t sb_src, int64_t ld_src, float* dst,
                 int64_t sb_dst, int64_t ld_dst, float* tau_out, int64_t tau_sb,
                 float* T_out, int64_t T_sb, int t_ld, float* V_out,
                 int64_t batch, int r, int w, cudaStream_t stream, float* Vsplit = nullptr,
                 int64_t vs_mat = 0, int64_t vs_plane = 0, int vs_row0 = 0, int vs_ld = 32,
                 bool vs_zero = false);

// C_dst <- C_src - V T^T V^T C_src for r x c blocks, k <= 32 reflectors whose
// strictly-lower part is read from V (unit diagonal implied). T is 32 x 32 per
// matrix (leading k x k used) when t_ld == 32, else k x k (t_ld = k).
// tc_pass2: the second product (C -= V W') on the tensor cores (tcgen05,
// 3xTF32) where the operands allow 16-byte vector access and k == 32.
int launch_larfb(const float* V, int64_t sVb, int64_t ldv, const float* T,
                 int64_t sTb, int t_ld, const float* Csrc, int64_t sCsb,
                 int64_t ldcs, float* Cdst, int64_t sCdb, int64_t ldcd,
                 int64_t batch, int r, int k, int c, bool tc_pass2,
                 cudaStream_t stream);

int panel_cluster_size(int r, int64_t batch);
// qrb_set_config("panel_rpt"): rows per thread of the panel kernel, 1, 2 or 4
// (0 = automatic: 1 up to 128 rows, else 2 where the batch's panels still fit
// on the SMs at once, else 4).
int panel_rpt();
// qrb_set_config("gram_tile"): S tile of the Gram kernel, 64 or 128 (0 =
// automatic: 128 above n = 64).
int gram_tile();

// Tensor-core (tcgen05, 3xTF32) trailing update for k = 32 reflectors and
// 16-byte aligned row-major operands; same contract as launch_larfb.
bool larfb_tc_supported(const float* V, int64_t sVb, int64_t ldv, const float* Csrc,
                        int64_t sCsb, int64_t ldcs, const float* Cdst, int64_t sCdb,
                        int64_t ldcd, int k, int c);
int launch_larfb_tc(const float* V, int64_t sVb, int64_t ldv, const float* T,
                    int64_t sTb, int t_ld, const float* Csrc, int64_t sCsb,
                    int64_t ldcs, float* Cdst, int64_t sCdb, int64_t ldcd,
                    int64_t batch, int r, int c, cudaStream_t stream);

// Narrow in-place update C <- C - V T^T V^T C of the cw <= 64 columns next to
// a panel (the next panels' columns): r rows, 32 reflectors read from V's
// strictly lower part (unit diagonal implied), T 32 x 32 with row stride t_ld;
// one cluster per matrix and 32-column block, splitting the rows. Needs
// 16-byte aligned rows and matrices and cw % 4 == 0 (larfb_narrow_supported).
bool larfb_narrow_supported(const float* V, int64_t sVb, int64_t ldv, const float* C, int64_t sCb,
                            int64_t ldc, int k, int cw);
int launch_larfb_narrow(const float* V, int64_t sVb, int64_t ldv, const float* T, int64_t sTb,
                        int t_ld, float* C, int64_t sCb, int64_t ldc, int64_t batch, int r,
                        int cw, cudaStream_t stream);
// Cluster size, rows per cluster rank and rows per staged chunk for r rows.
void larfb_narrow_shape(int r, int* cs, int* rs, int* rch);

// Two-level blocking (64 reflectors = two panels). larfb64: C_dst <- C_src -
// V T^T V^T C_src for r x c blocks (r >= 64) with 64 reflectors read from V's
// strictly lower part and T 64 x 64 per matrix (row stride 64); operands must
// pass larfb64_supported (16-byte aligned rows and matrices, c % 4 == 0).
// t64: fill the cross block of such a T in place from V (r > 64 rows), the
// diagonal blocks T1 and T2 having been written by the two panels.
bool larfb64_supported(const float* V, int64_t sVb, int64_t ldv, const float* Csrc,
                       int64_t sCsb, int64_t ldcs, const float* Cdst, int64_t sCdb,
                       int64_t ldcd, int c);
int launch_larfb64(const float* V, int64_t sVb, int64_t ldv, const float* T, int64_t sTb,
                   const float* Csrc, int64_t sCsb, int64_t ldcs, float* Cdst, int64_t sCdb,
                   int64_t ldcd, int64_t batch, int r, int c, cudaStream_t stream);
int launch_t64(const float* V, int64_t sVb, int64_t ldv, float* T64, int64_t sT64b,
               int64_t batch, int r, cudaStream_t stream);

// Clock-cycle limit of the bounded device-side waits (qrb_set_config
// "wait_limit"; default about one second).
long long device_wait_limit();
// qrb_set_config("test_skip_mma"): the TMA-fed update issues no pass-1 MMAs,
// so its bounded waits run out (tests of the timeout path only).
bool test_skip_mma();
// qrb_set_config("tma_ctas"): most CTAs of one TMA-fed update launch (0 = one
// per SM).
int tma_cta_cap();
// qrb_set_config("tma_split_rows"): the TMA-fed update sums V^T C in two row
// halves when the trailing block has at least this many rows (0 = never).
int tma_split_rows();
// qrb_set_config("tma_pair"): with two halves, 0 = a 2-CTA cluster per tile
// when 2 x tiles <= SMs, 1 = one CTA per tile, 2 = always a pair.
int tma_pair_mode();
// qrb_set_config("tma_dual"): 32-reflector updates without row halves, 0 = two
// CTAs per SM when the launch has more tiles than SMs, 1 = one CTA per SM,
// 2 = always two (the same bits either way).
int tma_dual_mode();
// One probe kernel that waits on an mbarrier nobody arrives at for `limit`
// cycles and then sets the device error flag.
int launch_wait_probe(long long limit, cudaStream_t stream);

// Device-side error flag set by kernels whose bounded waits timed out
// (synchronous read; optionally reset to 0), and its device address.
int device_error_flag(int* value, bool reset);
int device_error_ptr(int** p);

// The blocked route's factor scratch, carved from the caller's workspace of
// `bytes` for `batch` matrices: T one 32 x 32 factor per matrix (required),
// T2 a second one for the panel look-ahead, T64 one 64 x 64 factor per matrix
// for two-level blocking (overlapping T and T2), T64b a second 64 x 64 one
// for two-level blocking with the look-ahead (each nullptr when the workspace
// is too small). Vs: the split reflectors of the tensor-core update, when the
// workspace holds them: for 32-reflector blocks [4][batch][n][32] (planes
// 2 * buf + 0 / 1 = hi / lo of V-buffer buf), for 64-reflector blocks the
// same memory as [4][batch][n][64].
struct FactorScratch {
  float* T = nullptr;
  float* T2 = nullptr;
  float* T64 = nullptr;
  float* T64b = nullptr;
  float* Vs = nullptr;
};
FactorScratch factor_scratch(void* workspace, size_t bytes, int64_t batch, int n);
// Bytes of the split-reflector buffers for (batch, n), 0 where the
// tensor-core update cannot run.
size_t vsplit_bytes(int64_t batch, int n);
// The smallest workspace the blocked route accepts: one T factor per matrix.
size_t min_workspace_bytes(int64_t batch);

// The route of one qrb_geqrf_f32 call (see qrb_route in the public header).
constexpr int kRouteNone = 0, kRouteFusedWarp = 1, kRouteFusedCta = 2, kRouteBlocked = 3;
constexpr int kLarfbFfma = 0, kLarfbTcStaged = 1, kLarfbTcPass2 = 2, kLarfbTma = 3;
// Smallest n the blocked route gives the TMA-fed tensor-core update.
constexpr int kTmaMinN = 129;
struct Plan {
  int route = kRouteNone;
  int larfb = 0;       // trailing update: kLarfb* (0 FFMA, 1 / 2 tcgen05 staged by the
                       // CUDA cores, 3 tcgen05 fed by TMA)
  int groups = 1;      // batch groups on internal streams
  bool lookahead = false;
  bool two_level = false;
  bool deep = false;   // two-level look-ahead of depth two (the wide update off the chain)
};
Plan make_plan(int64_t batch, int n, const FactorScratch& ws);

// The launch attribute that carries the stream's priority into the kernel
// node when a launch is captured into a CUDA graph (an eager launch gets the
// same priority from its stream). Writes *a and returns 1 for a stream of
// non-default priority, else returns 0.
inline int stream_priority_attr(cudaStream_t s, cudaLaunchAttribute* a) {
  int p = 0;
  if (cudaStreamGetPriority(s, &p) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  if (p == 0) return 0;
  a->id = cudaLaunchAttributePriority;
  a->val.priority = p;
  return 1;
}
int route_code(const Plan& p);

// Whole factorization of already validated arguments, enqueued on `stream`
// (no fault injection, no sync check), the blocked route's factors in ws.
// Per-group hooks of the blocked route: before(b0, b1, gs) is called before
// the first kernel of batch group [b0, b1) is enqueued on its stream gs,
// after(b0, b1, gs) after its last (the whole batch is one group on the
// caller's stream when the route has no groups). The host-memory entry point
// uses them to stream each group's copies against the other groups' work.
struct GroupHooks {
  int min_groups = 0;  // at least this many groups (capped at the batch and the stream sets)
  virtual int before(int64_t b0, int64_t b1, cudaStream_t gs) = 0;
  virtual int after(int64_t b0, int64_t b1, cudaStream_t gs) = 0;
 protected:
  ~GroupHooks() = default;
};
// hooks (blocked route only) require A == H: the factorization reads nothing
// a group's hook has not made ready.
int geqrf_enqueue(const float* A, int64_t sAb, int64_t sAr, float* H, float* tau,
                  const FactorScratch& ws, int64_t batch, int n, cudaStream_t stream,
                  GroupHooks* hooks = nullptr);

// CUDA graph replay of repeated blocked calls (qrb_graph.cu): on the second
// call with the same arguments the call is captured, then replayed; sets
// *handled when the call was enqueued that way (else the caller enqueues it).
int geqrf_graph(const float* A, int64_t sAb, int64_t sAr, float* H, float* tau,
                const FactorScratch& fs, const void* ws, size_t ws_bytes, int64_t batch, int n,
                cudaStream_t s, bool* handled);
void graph_cache_clear();
int graph_cache_entries();
// While one lives, this thread's calls enqueue eagerly: graph instantiation
// may allocate device memory (the no-alloc entry point).
struct NoGraphScope {
  NoGraphScope();
  ~NoGraphScope();
  NoGraphScope(const NoGraphScope&) = delete;
  NoGraphScope& operator=(const NoGraphScope&) = delete;
};
// qrb_set_config("graph_cache") and not "sync_check".
bool graph_cache_enabled();
// Bumped by every qrb_set_config call that can change what a call enqueues.
uint64_t config_generation();
// The launch counter (qrb_get_config("launches")).
int64_t launch_count();

// The public entry points' shared epilogue pieces: consume one injected
// failure (fail_next), and apply the sync_check mode to a call's status.
bool take_injected_failure_any();
int finish_call(int rc, cudaStream_t stream);

// qrb_set_config("host_direct") for qrb_geqrf_f32_host with n <= 32 and
// mapped page-locked host buffers: 0 = copies in and out; 1 = the kernel
// reads A and writes H and tau in host memory itself; 2 = copies in, the
// kernel writes H and tau to host memory; 3 = copies in and out for the
// matrices, the kernel writes tau to host memory.
int host_direct_mode();
// qrb_set_config("host_ramp"): 1 = chunk sizes rise and fall (1, 2, .., 2, 1)
// so that the pipeline fills and drains on small pieces; 0 = equal chunks.
bool host_ramp();
// qrb_set_config("host_groups"): qrb_geqrf_f32_host on the blocked route runs
// at least this many batch groups (1..8; 0 = the route's own; default 8).
int host_groups();
// qrb_set_config("direct_blocks"): grid of the direct kernel (0 = automatic).
int64_t host_direct_blocks();

// qrb_set_config("fused_cpl"): columns per lane of the n <= 32 kernel, 2 (two
// matrices per warp), 4 (four matrices per warp) or 0 (by batch size).
int fused_cpl();

// Path taken by the last qrb_geqrf_f32_host call (the host_direct mode that
// ran: 0..3, or 4 for the blocked route's groups as pieces), -1 none yet
// (qrb_get_config("host_path")).
int64_t host_last_path();

// Count of kernel launches enqueued by this library (all devices, all calls);
// read through qrb_get_config("launches").
void note_launches(int64_t count);

}  // namespace qrb

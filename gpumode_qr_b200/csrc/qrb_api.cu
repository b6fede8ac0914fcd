// C ABI of libqrb200: argument validation, configuration hooks and the
// blocked-QR driver (the panel loop of the reference's
// _hh_panel_blocked_qr, src/qrbench/variants.py:761-805, run here on the host
// side of the library as one stream-ordered kernel sequence per call).
#include <atomic>
#include <cstring>
#include <mutex>

#include "qrb_common.cuh"
#include "qrb_tma.cuh"

namespace {

std::atomic<int64_t> g_fail_next{0};
std::atomic<int64_t> g_sync_check{0};
std::atomic<int64_t> g_larfb_kind{-1};  // -1 automatic, else a kLarfb* kind
std::atomic<int64_t> g_launches{0};
std::atomic<int64_t> g_graph{1};           // replay cached CUDA graphs of repeated calls
std::atomic<uint64_t> g_generation{0};     // bumped by routing-relevant qrb_set_config calls
std::atomic<int64_t> g_groups{0};  // 0 = automatic
std::atomic<int64_t> g_host_direct{3};
std::atomic<int64_t> g_direct_blocks{0};
std::atomic<int64_t> g_host_ramp{0};
std::atomic<int64_t> g_host_groups{8};  // pieces of the host pipeline's blocked route
std::atomic<int64_t> g_fused_cpl{0};
std::atomic<int64_t> g_mid_fused{1};
std::atomic<int64_t> g_lookahead{2};  // 0 off, 1 on, 2 from kLookaheadMinN
std::atomic<int64_t> g_two_level{2};  // 0 off, 1 on, 2 automatic
std::atomic<int64_t> g_panel_rpt{0};
std::atomic<int64_t> g_gram_tile{0};
std::atomic<int64_t> g_wait_limit{2000000000LL};  // clock cycles, about 1 s
std::atomic<int64_t> g_skip_mma{0};
std::atomic<int64_t> g_tma_ctas{0};        // 0 = one per SM
std::atomic<int64_t> g_tma_split{1024};    // two row halves from this height (0 = never)
std::atomic<int64_t> g_tma_pair{0};        // halves on: 0 auto, 1 one CTA, 2 a CTA pair per tile
std::atomic<int64_t> g_tma_dual{0};        // 32 reflectors: 0 auto, 1 one CTA per SM, 2 two
std::atomic<int64_t> g_la_depth{0};        // two-level look-ahead depth: 0 auto, 1 or 2 blocks
std::atomic<int64_t> g_narrow{1};          // narrow cluster kernel for the next panel's columns
std::atomic<int64_t> g_panel_priority{1};  // look-ahead stream at the highest priority

// Host-side fault injection: consume one pending injected failure.
bool take_injected_failure() {
  int64_t v = g_fail_next.load();
  while (v > 0) {
    if (g_fail_next.compare_exchange_weak(v, v - 1)) return true;
  }
  return false;
}

int finish(int rc, cudaStream_t stream) {
  if (rc != QRB_OK) return rc;
  if (g_sync_check.load() != 0) {
    if (cudaStreamSynchronize(stream) != cudaSuccess) return QRB_ERR_LAUNCH;
    if (cudaGetLastError() != cudaSuccess) return QRB_ERR_LAUNCH;
    int flag = 0;
    if (qrb::device_error_flag(&flag, false) != QRB_OK) return QRB_ERR_DEVICE;
    if (flag != 0) return QRB_ERR_DEVICE_WAIT;
  }
  return QRB_OK;
}

// Trailing update: the tensor-core kernel where it applies and is selected,
// the FFMA kernel otherwise.
int larfb_any(const float* V, int64_t sVb, int64_t ldv, const float* T, int64_t sTb, int t_ld,
              const float* Csrc, int64_t sCsb, int64_t ldcs, float* Cdst, int64_t sCdb,
              int64_t ldcd, int64_t batch, int r, int k, int c, cudaStream_t s) {
  const int64_t kind = g_larfb_kind.load();
  if (kind == 1 &&
      qrb::larfb_tc_supported(V, sVb, ldv, Csrc, sCsb, ldcs, Cdst, sCdb, ldcd, k, c))
    return qrb::launch_larfb_tc(V, sVb, ldv, T, sTb, t_ld, Csrc, sCsb, ldcs, Cdst, sCdb, ldcd,
                                batch, r, c, s);
  return qrb::launch_larfb(V, sVb, ldv, T, sTb, t_ld, Csrc, sCsb, ldcs, Cdst, sCdb, ldcd, batch,
                           r, k, c, /*tc_pass2=*/kind == 2, s);
}

bool bad_matrix_strides(int64_t sb, int64_t srow, int64_t rows, int64_t cols,
                        int64_t batch) {
  if (srow < cols) return true;                       // rows overlap
  if (batch > 1 && sb < (rows - 1) * srow + cols) return true;  // matrices overlap
  return false;
}

// The blocked factorization of one contiguous group of matrices on `s`:
// per 32-column panel one panel kernel (reflectors, tau, T) and one trailing
// update of the columns to its right. The first step reads A and writes H,
// so no separate copy pass is needed; later steps work in place on H.
// The tensor-core trailing update's operands for one batch group: tensor
// maps over the whole call's batch, the split-reflector planes, and the
// group's first matrix in them.
struct TmaRoute {
  const qrb::LarfbMaps* maps;
  float* Vs;            // plane 0, matrix 0 of the call
  int64_t batch_total;  // matrices the maps and planes cover
  int64_t m0;           // this group's first matrix
  // hi plane of V-buffer `buf` at this group's first matrix
  float* vsplit(int buf, int n) const {
    return Vs + ((int64_t)(2 * buf) * batch_total + m0) * n * qrb::kPanelW;
  }
  int64_t plane(int n) const { return batch_total * n * qrb::kPanelW; }
  // two-level blocks: hi plane [batch][n][64] of V-buffer `buf` at this
  // group's first matrix (the remainder one plane further on)
  float* vsplit64(int buf, int n) const {
    return Vs + ((int64_t)(2 * buf) * batch_total + m0) * n * 2 * qrb::kPanelW;
  }
  int64_t plane64(int n) const { return batch_total * n * 2 * qrb::kPanelW; }
};

// The look-ahead's update on the tensor-core route: columns [col0, n) of rows
// [j0, n) with the 32 reflectors of the panel at (j0, j0) and its factor T
// (row stride t_ld). cols = 32: only the first (at most) 32 columns, which the
// next panel needs first, by the narrow cluster kernel (the TMA-fed kernel
// where the narrow one does not apply or is switched off); cols < 0: the
// columns after them, by the TMA-fed kernel.
int tma_update(const TmaRoute& tr, float* H, const float* T, int64_t sTb, int t_ld,
               int64_t batch, int n, int j0, int col0, int vbuf, int cols, cudaStream_t s) {
  const int W = qrb::kPanelW;
  const int64_t nn = (int64_t)n * n;
  const int c = n - col0, r = n - j0;
  const int ca = c < W ? c : W;
  const float* V = H + (int64_t)j0 * n + j0;
  float* C = H + (int64_t)j0 * n + col0;
  if (cols == W) {
    if (g_narrow.load() != 0 && qrb::larfb_narrow_supported(V, nn, n, C, nn, n, W, ca))
      return qrb::launch_larfb_narrow(V, nn, n, T, sTb, t_ld, C, nn, n, batch, r, ca, s);
    return qrb::launch_larfb_tma(*tr.maps, T, sTb, tr.m0, batch, j0, col0, col0 + ca, n, vbuf, s);
  }
  if (c <= ca) return QRB_OK;
  return qrb::launch_larfb_tma(*tr.maps, T, sTb, tr.m0, batch, j0, col0 + ca, n, n, vbuf, s);
}

// The blocked factorization of one contiguous group of matrices on `s`:
// per 32-column panel one panel kernel (reflectors, tau, T) and one trailing
// update of the columns to its right. On the FFMA route the first step reads
// A and writes H, so no separate copy pass is needed; later steps work in
// place on H. On the tensor-core route (tr non-null) H already holds A, the
// panel also writes its split reflectors and the update is the TMA-fed kernel.
int blocked_qr(const float* A, int64_t strideA_b, int64_t strideA_row, float* H,
               float* tau, float* T, int64_t batch, int n, cudaStream_t s,
               const TmaRoute* tr = nullptr) {
  const int64_t nn = (int64_t)n * n;
  const int W = qrb::kPanelW;
  for (int j0 = 0; j0 < n; j0 += W) {
    const int w = n - j0 < W ? n - j0 : W;
    const int r = n - j0;
    const bool first = j0 == 0 && tr == nullptr;
    const float* src = first ? A : H;
    const int64_t sb = first ? strideA_b : nn;
    const int64_t ld = first ? strideA_row : n;
    float* Hp = H + (int64_t)j0 * n + j0;
    const int c = n - j0 - w;
    float* vs = (tr != nullptr && c > 0) ? tr->vsplit(0, n) : nullptr;
    int rc = qrb::launch_panel(src + (int64_t)j0 * ld + j0, sb, ld, Hp, nn, n, tau + j0, n, T,
                               (int64_t)W * W, W, nullptr, batch, r, w, s, vs,
                               (int64_t)n * W, tr ? tr->plane(n) : 0, j0);
    if (rc != QRB_OK) return rc;
    if (c > 0) {
      rc = tr != nullptr
               ? qrb::launch_larfb_tma(*tr->maps, T, (int64_t)W * W, tr->m0, batch, j0, j0 + w,
                                       n, n, 0, s)
               : larfb_any(Hp, nn, n, T, (int64_t)W * W, W, src + (int64_t)j0 * ld + j0 + w, sb,
                           ld, Hp + w, nn, n, batch, r, w, c, s);
      if (rc != QRB_OK) return rc;
    }
  }
  return QRB_OK;
}

// The blocked factorization with a look-ahead of one panel, on two streams:
// sp runs panel j and the update of panel j + 1's 32 columns (part a), sb the
// update of everything right of them (part b). Panel j + 1 then runs while
// part b of step j does, instead of after it. Part a of step j waits for part
// b of step j - 1 (which last touched those columns), part b of step j for
// panel j. T alternates between T0 and T1 so that panel j + 1 can write its
// factor while part b of step j still reads panel j's. The update is column by
// column, so the split changes no result. Both streams end joined into sb.
int blocked_qr_lookahead(const float* A, int64_t strideA_b, int64_t strideA_row, float* H,
                         float* tau, float* T0, float* T1, int64_t batch, int n,
                         cudaStream_t sb, cudaStream_t sp, cudaEvent_t evP, cudaEvent_t evB,
                         cudaEvent_t joinP, const TmaRoute* tr = nullptr) {
  const int64_t nn = (int64_t)n * n;
  const int W = qrb::kPanelW;
  if (cudaEventRecord(evB, sb) != cudaSuccess || cudaStreamWaitEvent(sp, evB, 0) != cudaSuccess)
    return QRB_ERR_LAUNCH;
  int rc = QRB_OK;
  for (int j0 = 0, step = 0; j0 < n && rc == QRB_OK; j0 += W, ++step) {
    const int buf = step & 1;
    float* T = buf ? T1 : T0;
    const int w = n - j0 < W ? n - j0 : W;
    const int r = n - j0;
    const bool first = j0 == 0 && tr == nullptr;
    const float* src = first ? A : H;
    const int64_t sbt = first ? strideA_b : nn;
    const int64_t ld = first ? strideA_row : n;
    float* Hp = H + (int64_t)j0 * n + j0;
    const int c = n - j0 - w;
    float* vs = (tr != nullptr && c > 0) ? tr->vsplit(buf, n) : nullptr;
    rc = qrb::launch_panel(src + (int64_t)j0 * ld + j0, sbt, ld, Hp, nn, n, tau + j0, n, T,
                           (int64_t)W * W, W, nullptr, batch, r, w, sp, vs, (int64_t)n * W,
                           tr ? tr->plane(n) : 0, j0);
    if (rc != QRB_OK) break;
    if (cudaEventRecord(evP, sp) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
    if (c <= 0) break;
    const int ca = c < W ? c : W, cbw = c - ca;
    const float* ca_src = src + (int64_t)j0 * ld + j0 + w;
    // part a on sp, after part b of the previous step
    if (cudaStreamWaitEvent(sp, evB, 0) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
    rc = tr != nullptr
             ? tma_update(*tr, H, T, (int64_t)W * W, W, batch, n, j0, j0 + w, buf, W, sp)
             : larfb_any(Hp, nn, n, T, (int64_t)W * W, W, ca_src, sbt, ld, Hp + w, nn, n, batch,
                         r, w, ca, sp);
    if (rc != QRB_OK) break;
    // part b on sb, after panel j
    if (cudaStreamWaitEvent(sb, evP, 0) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
    if (cbw > 0) {
      rc = tr != nullptr
               ? tma_update(*tr, H, T, (int64_t)W * W, W, batch, n, j0, j0 + w, buf, -1, sb)
               : larfb_any(Hp, nn, n, T, (int64_t)W * W, W, ca_src + ca, sbt, ld, Hp + w + ca,
                           nn, n, batch, r, w, cbw, sb);
      if (rc != QRB_OK) break;
    }
    if (cudaEventRecord(evB, sb) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
  }
  // join sp into sb (also after an error)
  if (cudaEventRecord(joinP, sp) != cudaSuccess || cudaStreamWaitEvent(sb, joinP, 0) != cudaSuccess)
    if (rc == QRB_OK) rc = QRB_ERR_LAUNCH;
  return rc;
}

// Two-level blocking: per 64 columns two 32-column panels and one trailing
// update with the combined 64-reflector block, so that each trailing column
// is read and written once per 64 reflectors instead of once per 32.
//   panel 1           columns j0 .. j0+31 (T1 on the diagonal of T64)
//   update (k = 32)   panel 1's reflectors on columns j0+32 .. j0+63
//   panel 2           rows and columns from j0+32 (T2 on the diagonal of T64)
//   t64               the cross block of T64 from V1^T V2
//   update (k = 64)   both panels' reflectors on the columns from j0+64.
// Where the 64-wide update's operands are not 16-byte aligned, the two panels
// are applied one after the other instead (the same product).
int blocked_qr2(const float* A, int64_t strideA_b, int64_t strideA_row, float* H, float* tau,
                float* T64, int64_t batch, int n, cudaStream_t s, const TmaRoute* tr = nullptr) {
  const int64_t nn = (int64_t)n * n;
  constexpr int W = qrb::kPanelW;
  constexpr int K2 = 2 * W;
  constexpr int64_t tsb = (int64_t)K2 * K2;
  float* T1 = T64;
  float* T2 = T64 + W * K2 + W;
  for (int j0 = 0; j0 < n; j0 += K2) {
    const int r = n - j0;
    const bool first = j0 == 0 && tr == nullptr;
    const float* src = first ? A : H;
    const int64_t sb = first ? strideA_b : nn;
    const int64_t ld = first ? strideA_row : n;
    float* Hp = H + (int64_t)j0 * n + j0;
    const float* Sp = src + (int64_t)j0 * ld + j0;
    const int w1 = r < W ? r : W;
    // tensor-core route: both panels write their split reflectors into one
    // 64-wide plane when a 64-reflector update follows
    const bool big = tr != nullptr && r > K2;
    float* vs = big ? tr->vsplit64(0, n) : nullptr;
    const int64_t vpl = tr != nullptr ? tr->plane64(n) : 0;
    int rc = qrb::launch_panel(Sp, sb, ld, Hp, nn, n, tau + j0, n, T1, tsb, K2, nullptr, batch,
                               r, w1, s, vs, (int64_t)n * K2, vpl, j0, K2, big);
    if (rc != QRB_OK || r <= W) return rc;
    const int w2 = r - W < W ? r - W : W;
    rc = tr != nullptr && g_narrow.load() != 0 &&
                 qrb::larfb_narrow_supported(Hp, nn, n, Hp + W, nn, n, W, w2)
             ? qrb::launch_larfb_narrow(Hp, nn, n, T1, tsb, K2, Hp + W, nn, n, batch, r, w2, s)
             : larfb_any(Hp, nn, n, T1, tsb, K2, Sp + W, sb, ld, Hp + W, nn, n, batch, r, W, w2,
                         s);
    if (rc != QRB_OK) return rc;
    float* Hq = Hp + (int64_t)W * n + W;
    rc = qrb::launch_panel(Hq, nn, n, Hq, nn, n, tau + j0 + W, n, T2, tsb, K2, nullptr, batch,
                           r - W, w2, s, big ? vs + W : nullptr, (int64_t)n * K2, vpl, j0 + W, K2,
                           false);
    if (rc != QRB_OK) return rc;
    const int c = r - K2;
    if (c <= 0) continue;
    if (big) {
      rc = qrb::launch_t64(Hp, nn, n, T64, tsb, batch, r, s);
      if (rc == QRB_OK)
        rc = qrb::launch_larfb_tma(*tr->maps, T64, tsb, tr->m0, batch, j0, j0 + K2, n, n, 0, s);
    } else if (qrb::larfb64_supported(Hp, nn, n, Sp + K2, sb, ld, Hp + K2, nn, n, c)) {
      rc = qrb::launch_t64(Hp, nn, n, T64, tsb, batch, r, s);
      if (rc != QRB_OK) return rc;
      rc = qrb::launch_larfb64(Hp, nn, n, T64, tsb, Sp + K2, sb, ld, Hp + K2, nn, n, batch, r,
                               c, s);
    } else {
      rc = larfb_any(Hp, nn, n, T1, tsb, K2, Sp + K2, sb, ld, Hp + K2, nn, n, batch, r, W, c, s);
      if (rc == QRB_OK)
        rc = larfb_any(Hq, nn, n, T2, tsb, K2, Hq + W, nn, n, Hq + W, nn, n, batch, r - W, W, c,
                       s);
    }
    if (rc != QRB_OK) return rc;
  }
  return QRB_OK;
}

// Two-level blocking with the look-ahead, tensor-core route only (H holds A,
// tr non-null). Per 64-column block j0 (T64 alternating between two buffers,
// the split reflectors between V-buffers 0 and 1):
//   sp  panel 1                     columns j0 .. j0+31 (T1)
//       narrow update, panel 1      columns j0+32 .. j0+95 (panel 2's and the
//                                   next block's first panel's)
//       panel 2                     rows and columns from j0+32 (T2)
//       narrow update, panel 2      columns j0+64 .. j0+95
//   sb  t64, then the 64-reflector update of the columns from j0+96.
// The sp chain reaches the next block's first panel without waiting for the
// wide update; the next block's first narrow update waits for it (it touches
// the columns from j0+96). Both streams end joined into sb.
int blocked_qr2_lookahead(float* H, float* tau, float* T64a, float* T64b, int64_t batch, int n,
                          cudaStream_t sb, cudaStream_t sp, cudaEvent_t evP, cudaEvent_t evB,
                          cudaEvent_t joinP, const TmaRoute& tr, bool deep) {
  const int64_t nn = (int64_t)n * n;
  constexpr int W = qrb::kPanelW;
  constexpr int K2 = 2 * W;
  constexpr int64_t tsb = (int64_t)K2 * K2;
  const int64_t vpl = tr.plane64(n);
  // the reflectors at Vp (r rows) applied to the cw columns at C: the narrow
  // kernel, or FFMA where its operands do not allow it
  auto narrow = [&](float* Vp, const float* T, int r, float* C, int cw, cudaStream_t st) {
    if (cw <= 0) return (int)QRB_OK;
    if (g_narrow.load() != 0 && qrb::larfb_narrow_supported(Vp, nn, n, C, nn, n, W, cw))
      return qrb::launch_larfb_narrow(Vp, nn, n, T, tsb, K2, C, nn, n, batch, r, cw, st);
    return larfb_any(Vp, nn, n, T, tsb, K2, C, nn, n, C, nn, n, batch, r, W, cw, st);
  };
  if (cudaEventRecord(evB, sb) != cudaSuccess || cudaStreamWaitEvent(sp, evB, 0) != cudaSuccess)
    return QRB_ERR_LAUNCH;
  int rc = QRB_OK;
  for (int j0 = 0, blk = 0; j0 < n && rc == QRB_OK; j0 += K2, ++blk) {
    const int buf = blk & 1;
    float* T64 = buf ? T64b : T64a;
    float* T1 = T64;
    float* T2 = T64 + W * K2 + W;
    const int r = n - j0;
    const int w1 = r < W ? r : W;
    // a 64-reflector update follows (of the columns from j0 + 96, or from
    // j0 + 128 at depth two)
    const bool wide = r > (deep ? 2 * K2 : K2 + W);
    float* Hp = H + (int64_t)j0 * n + j0;
    float* vs = wide ? tr.vsplit64(buf, n) : nullptr;
    rc = qrb::launch_panel(Hp, nn, n, Hp, nn, n, tau + j0, n, T1, tsb, K2, nullptr, batch, r, w1,
                           sp, vs, (int64_t)n * K2, vpl, j0, K2, wide);
    if (rc != QRB_OK || r <= W) break;
    if (deep) {
      // Depth two: the priority stream applies this block's reflectors to the
      // whole next block, so the wide update (columns from j0 + 128) has a
      // block of slack and leaves the critical path. Block k's stream sp:
      // panel 1, its narrow update of panel 2's columns, panel 2, then (once
      // block k-1's wide update, which covered the columns from j0 + 64, is
      // done) both panels' narrow updates of the next 64 columns.
      const int c1 = r - W < W ? r - W : W;
      rc = narrow(Hp, T1, r, Hp + W, c1, sp);
      if (rc != QRB_OK) break;
      float* Hq = Hp + (int64_t)W * n + W;
      rc = qrb::launch_panel(Hq, nn, n, Hq, nn, n, tau + j0 + W, n, T2, tsb, K2, nullptr, batch,
                             r - W, c1, sp, wide ? vs + W : nullptr, (int64_t)n * K2, vpl,
                             j0 + W, K2, false);
      if (rc != QRB_OK) break;
      if (cudaEventRecord(evP, sp) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
      const int c = r - K2;
      if (c <= 0) break;
      if (cudaStreamWaitEvent(sp, evB, 0) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
      const int cb = c < K2 ? c : K2;
      rc = narrow(Hp, T1, r, Hp + K2, cb, sp);
      if (rc == QRB_OK) rc = narrow(Hq, T2, r - W, Hq + W, cb, sp);
      if (rc != QRB_OK) break;
      if (!wide) continue;
      if (cudaStreamWaitEvent(sb, evP, 0) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
      rc = qrb::launch_t64(Hp, nn, n, T64, tsb, batch, r, sb);
      if (rc == QRB_OK)
        rc = qrb::launch_larfb_tma(*tr.maps, T64, tsb, tr.m0, batch, j0, j0 + 2 * K2, n, n, buf,
                                   sb);
      if (rc != QRB_OK) break;
      if (cudaEventRecord(evB, sb) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
      continue;
    }
    // the columns from j0+32 were last written by the previous block's wide update
    if (cudaStreamWaitEvent(sp, evB, 0) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
    const int c1 = r - W < K2 ? r - W : K2;
    rc = narrow(Hp, T1, r, Hp + W, c1, sp);
    if (rc != QRB_OK) break;
    const int w2 = r - W < W ? r - W : W;
    float* Hq = Hp + (int64_t)W * n + W;
    rc = qrb::launch_panel(Hq, nn, n, Hq, nn, n, tau + j0 + W, n, T2, tsb, K2, nullptr, batch,
                           r - W, w2, sp, wide ? vs + W : nullptr, (int64_t)n * K2, vpl, j0 + W,
                           K2, false);
    if (rc != QRB_OK) break;
    if (cudaEventRecord(evP, sp) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
    const int c = r - K2;
    if (c <= 0) break;
    rc = narrow(Hq, T2, r - W, Hq + W, c < W ? c : W, sp);
    if (rc != QRB_OK) break;
    if (!wide) continue;  // the next block is the last, at most 32 columns
    if (cudaStreamWaitEvent(sb, evP, 0) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
    rc = qrb::launch_t64(Hp, nn, n, T64, tsb, batch, r, sb);
    if (rc == QRB_OK)
      rc = qrb::launch_larfb_tma(*tr.maps, T64, tsb, tr.m0, batch, j0, j0 + K2 + W, n, n, buf,
                                 sb);
    if (rc != QRB_OK) break;
    if (cudaEventRecord(evB, sb) != cudaSuccess) { rc = QRB_ERR_LAUNCH; break; }
  }
  if (cudaEventRecord(joinP, sp) != cudaSuccess || cudaStreamWaitEvent(sb, joinP, 0) != cudaSuccess)
    if (rc == QRB_OK) rc = QRB_ERR_LAUNCH;
  return rc;
}

// Internal streams for batch groups, created once per device and kept for the
// life of the process (streams and events, no device memory).
constexpr int kMaxGroups = 8;
struct SideStreams {
  std::mutex mu;
  cudaStream_t s[kMaxGroups] = {};
  cudaEvent_t fork = nullptr;
  cudaEvent_t join[kMaxGroups] = {};
  // look-ahead: per group a panel stream and its events
  cudaStream_t sp[kMaxGroups] = {};
  cudaStream_t spl[kMaxGroups] = {};  // the same at the default priority (test hook)
  cudaEvent_t evP[kMaxGroups] = {}, evB[kMaxGroups] = {}, joinP[kMaxGroups] = {};
  bool ok = false;
};
constexpr int kMaxDevices = 64;
SideStreams g_side[kMaxDevices];
std::once_flag g_side_once[kMaxDevices];

SideStreams* side_streams() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  SideStreams* ss = &g_side[dev];
  std::call_once(g_side_once[dev], [ss] {
    bool ok = cudaEventCreateWithFlags(&ss->fork, cudaEventDisableTiming) == cudaSuccess;
    const unsigned ef = cudaEventDisableTiming;
    // The look-ahead streams (panel and next-panel update: the critical path)
    // get the highest priority, so that their CTAs are placed first whenever
    // trailing-update CTAs leave SMs free.
    int least = 0, greatest = 0;
    ok = ok && cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess;
    for (int g = 0; g < kMaxGroups && ok; ++g) {
      ok = cudaStreamCreateWithFlags(&ss->s[g], cudaStreamNonBlocking) == cudaSuccess &&
           cudaEventCreateWithFlags(&ss->join[g], ef) == cudaSuccess &&
           cudaStreamCreateWithPriority(&ss->sp[g], cudaStreamNonBlocking, greatest) ==
               cudaSuccess &&
           cudaStreamCreateWithFlags(&ss->spl[g], cudaStreamNonBlocking) == cudaSuccess &&
           cudaEventCreateWithFlags(&ss->evP[g], ef) == cudaSuccess &&
           cudaEventCreateWithFlags(&ss->evB[g], ef) == cudaSuccess &&
           cudaEventCreateWithFlags(&ss->joinP[g], ef) == cudaSuccess;
    }
    ss->ok = ok;
  });
  return ss->ok ? ss : nullptr;
}

}  // namespace

namespace qrb {
void note_launches(int64_t count) { g_launches.fetch_add(count); }
int64_t launch_count() { return g_launches.load(); }
bool graph_cache_enabled() { return g_graph.load() != 0 && g_sync_check.load() == 0; }
uint64_t config_generation() { return g_generation.load(); }
}  // namespace qrb

namespace qrb {

bool take_injected_failure_any() { return take_injected_failure(); }
int host_direct_mode() { return (int)g_host_direct.load(); }
bool host_ramp() { return g_host_ramp.load() != 0; }
int host_groups() { return (int)g_host_groups.load(); }
int fused_cpl() { return (int)g_fused_cpl.load(); }
bool mid_fused_enabled() { return g_mid_fused.load() != 0; }
bool mid_fused_always() { return g_mid_fused.load() == 2; }
int panel_rpt() { return (int)g_panel_rpt.load(); }
int gram_tile() { return (int)g_gram_tile.load(); }
int64_t host_direct_blocks() {
  const int64_t b = g_direct_blocks.load();
  return b > 0 ? b : kHostDirectBlocks;
}
int finish_call(int rc, cudaStream_t stream) { return finish(rc, stream); }
long long device_wait_limit() { return (long long)g_wait_limit.load(); }
bool test_skip_mma() { return g_skip_mma.load() != 0; }
int tma_cta_cap() { return (int)g_tma_ctas.load(); }
int tma_split_rows() { return (int)g_tma_split.load(); }
int tma_pair_mode() { return (int)g_tma_pair.load(); }
int tma_dual_mode() { return (int)g_tma_dual.load(); }

size_t vsplit_bytes(int64_t batch, int n) {
  if (batch <= 0 || n < kTmaMinN || n % 4 != 0) return 0;
  return 8 * (size_t)batch * n * kPanelW * sizeof(float);
}

size_t min_workspace_bytes(int64_t batch) {
  return (size_t)batch * kPanelW * kPanelW * sizeof(float);
}

FactorScratch factor_scratch(void* workspace, size_t bytes, int64_t batch, int n) {
  FactorScratch f;
  const size_t unit = (size_t)batch * kPanelW * kPanelW * sizeof(float);
  float* base = static_cast<float*>(workspace);
  if (base == nullptr || batch <= 0 || bytes < unit) return f;
  f.T = base;
  if (bytes >= 2 * unit) f.T2 = base + unit / sizeof(float);
  if (bytes >= 4 * unit) f.T64 = base;
  if (bytes >= 8 * unit) f.T64b = base + 4 * unit / sizeof(float);
  const size_t vb = vsplit_bytes(batch, n);
  if (vb != 0 && bytes >= 8 * unit + vb) f.Vs = base + 8 * unit / sizeof(float);
  return f;
}

// The route of one factorization: which kernels run and how the blocked loop
// is organised. With every test hook at its default this is a pure function
// of (batch, n, the workspace the caller gave), reported by qrb_route().
Plan make_plan(int64_t batch, int n, const FactorScratch& ws) {
  Plan p;
  if (n <= kFusedMaxN) {
    p.route = kRouteFusedWarp;
    return p;
  }
  // The CTA-per-matrix kernel is latency-friendly (one launch) but does more
  // arithmetic than the blocked route and runs in waves of 296 CTAs (2 per SM
  // at 128 threads). Measured on B200 it wins at n <= 64 for every batch, at
  // 96 < n <= 128 for every batch (the blocked route needs four panels there:
  // 1.08 vs 1.75 ms at 4096 x 97, 1.24 vs 1.59 ms at 4096 x 128), and at
  // 64 < n <= 96 up to two waves (145 vs 160 us at 592 x 80; 233 vs 199 us at
  // 740 x 96).
  if (n <= kFusedMidMaxN && mid_fused_enabled() &&
      (n <= 64 || n > 96 || batch <= kFusedMidMaxBatch || mid_fused_always())) {
    p.route = kRouteFusedCta;
    return p;
  }
  if (ws.T == nullptr) return p;  // kRouteNone: the blocked route needs a T factor
  p.route = kRouteBlocked;
  // Trailing update: the TMA-fed tensor-core kernel where the workspace holds
  // the split reflectors and the rows are 16-byte aligned (n % 4 == 0), FFMA
  // elsewhere; the test hook picks a kind explicitly.
  const int64_t kind = g_larfb_kind.load();
  const bool tma_ok = ws.Vs != nullptr && n >= kTmaMinN && larfb_tma_supported(n);
  if (kind < 0)
    p.larfb = tma_ok ? kLarfbTma : kLarfbFfma;
  else
    p.larfb = (kind == kLarfbTma && !tma_ok) ? kLarfbFfma : (int)kind;
  // Automatic blocking for the tensor-core update, from a sweep on B200 over
  // n = 256 .. 4096 and batch 8 .. 640. From n = 1024 two-level blocking
  // (each trailing column read once per 64 reflectors) wins everywhere; with
  // the look-ahead as well while batch * n <= 2^16, where the panels' latency
  // chain sets the time (18.1 vs 20.4 ms one-level with the look-ahead and
  // 23.5 ms two-level alone at 8 x 4096^2; 27.2 vs 29.5 ms at 16 x 4096^2;
  // 10.0 vs 10.8 ms at 32 x 2048^2; 3.45 vs 3.61 ms at 64 x 1024^2), without
  // it above, where the update's traffic does (47.1 vs 48.4 ms at
  // 32 x 4096^2, 6.64 vs 6.93 ms at 160 x 1024^2). Below n = 1024 the plain
  // loop is as fast or faster (4.63 ms two-level, 4.63 plain at 640 x 512^2;
  // 0.40 vs 0.42 ms with the look-ahead at 32 x 256^2). The FFMA update keeps
  // its own rule: the look-ahead from n = 4096, two-level only on request.
  const bool tma_route = p.larfb == kLarfbTma;
  const bool tl_auto = tma_route && n >= 1024;
  const bool la_auto = tma_route ? tl_auto && (double)batch * n <= 65536.0 : n >= kLookaheadMinN;
  const int64_t tl_mode = g_two_level.load();
  const int64_t la_mode = g_lookahead.load();
  p.two_level = ws.T64 != nullptr && (tl_mode == 1 || (tl_mode == 2 && tl_auto));
  const bool la_want = la_mode == 1 || (la_mode == 2 && la_auto);
  // two-level blocking combines with the look-ahead on the tensor-core route
  // (second 64 x 64 factor and double-buffered split reflectors)
  p.lookahead = la_want && (p.two_level ? tma_route && ws.T64b != nullptr : ws.T2 != nullptr);

  // Groups: automatic 4 from n = 1024 (measured on B200: 30.6 vs 32.8 ms for
  // 8 x 4096^2 on the FFMA update; 18.1 vs 18.5 ms and 3.45 vs 3.61 ms at
  // 8 x 4096^2 and 64 x 1024^2 on the tensor-core two-level look-ahead),
  // else 2; at most half the batch.
  int groups = (int)g_groups.load();
  if (groups == 0) groups = n >= 1024 ? 4 : 2;
  if (groups > batch / 2) groups = (int)(batch / 2);
  if (batch < 4) groups = 1;
  p.groups = groups < 1 ? 1 : groups;
  // Look-ahead depth two (the wide update off the critical path) where one
  // group has the GPU to itself at n >= 4096, the panels' chain is the whole
  // time (1 x 4096^2: 8.66 vs 8.98 ms; 2 x 4096^2: 9.01 vs 9.31 ms); with
  // several groups, or below n = 4096, its extra narrow updates cost more
  // (8 x 4096^2: 15.66 vs 15.08 ms; 2 x 2048^2: 3.95 vs 3.70 ms).
  const int64_t depth = g_la_depth.load();
  p.deep = p.lookahead && p.two_level &&
           (depth == 2 || (depth == 0 && p.groups == 1 && n >= 4096));
  return p;
}

int route_code(const Plan& p) {
  if (p.route != kRouteBlocked) return p.route;
  return p.route | (p.larfb << 4) | (p.lookahead ? 1 << 8 : 0) | (p.two_level ? 1 << 9 : 0) |
         (p.deep ? 1 << 10 : 0) | (p.groups << 12);
}

// The whole factorization of validated arguments, enqueued on s, as
// make_plan routes it: the fused warp kernel for n <= 32, the fused CTA kernel
// for 32 < n <= 128 where it wins, the blocked loop otherwise (optionally
// split into batch groups on internal streams, with the panel look-ahead or
// two-level blocking where selected and the workspace holds their factors).
int geqrf_enqueue(const float* A, int64_t strideA_b, int64_t strideA_row, float* H, float* tau,
                  const FactorScratch& ws, int64_t batch, int n, cudaStream_t s,
                  GroupHooks* hooks) {
  const Plan plan = make_plan(batch, n, ws);
  if (plan.route == kRouteFusedWarp)
    return launch_fused_small(A, strideA_b, strideA_row, H, tau, batch, n, s);
  if (plan.route == kRouteFusedCta)
    return launch_fused_mid(A, strideA_b, strideA_row, H, tau, batch, n, s);
  if (plan.route != kRouteBlocked) return QRB_ERR_WORKSPACE;
  if (hooks != nullptr && A != H) return QRB_ERR_INVALID_ARG;
  int groups = plan.groups;
  if (hooks != nullptr && hooks->min_groups > groups) {  // finer pieces (the bits do not change)
    const int64_t g = hooks->min_groups < batch ? hooks->min_groups : batch;
    groups = (int)(g < kMaxGroups ? g : kMaxGroups);
  }
  const bool tl = plan.two_level;
  const bool la = plan.lookahead;
  // Tensor-core route: H must hold A before the first update adds into it in
  // place, and one set of tensor maps covers the whole call.
  LarfbMaps maps;
  const bool tma = plan.larfb == kLarfbTma;
  if (tma) {
    const int64_t nn = (int64_t)n * n;
    if (A != H) {
      cudaError_t e = cudaSuccess;
      if (strideA_b == (int64_t)n * strideA_row) {
        e = cudaMemcpy2DAsync(H, (size_t)n * sizeof(float), A, (size_t)strideA_row * sizeof(float),
                              (size_t)n * sizeof(float), (size_t)(batch * n),
                              cudaMemcpyDeviceToDevice, s);
      } else {
        for (int64_t m = 0; m < batch && e == cudaSuccess; ++m)
          e = cudaMemcpy2DAsync(H + m * nn, (size_t)n * sizeof(float), A + m * strideA_b,
                                (size_t)strideA_row * sizeof(float), (size_t)n * sizeof(float),
                                (size_t)n, cudaMemcpyDeviceToDevice, s);
      }
      if (e != cudaSuccess) return QRB_ERR_LAUNCH;
      A = H;
      strideA_b = nn;
      strideA_row = n;
    }
    const int rc = make_larfb_maps(&maps, H, ws.Vs, batch, n, tl ? 64 : 32);
    if (rc != QRB_OK) return rc;
  }
  auto route_of = [&](int64_t m0) {
    TmaRoute r;
    r.maps = &maps;
    r.Vs = ws.Vs;
    r.batch_total = batch;
    r.m0 = m0;
    return r;
  };
  if (groups <= 1) {
    int rc = hooks != nullptr ? hooks->before(0, batch, s) : QRB_OK;
    if (rc != QRB_OK) return rc;
    const TmaRoute r0 = route_of(0);
    if (!la) {
      rc = tl ? blocked_qr2(A, strideA_b, strideA_row, H, tau, ws.T64, batch, n, s,
                            tma ? &r0 : nullptr)
              : blocked_qr(A, strideA_b, strideA_row, H, tau, ws.T, batch, n, s,
                           tma ? &r0 : nullptr);
    } else {
      SideStreams* ss = side_streams();
      if (ss == nullptr) return QRB_ERR_DEVICE;
      std::lock_guard<std::mutex> lock(ss->mu);
      cudaStream_t sp = g_panel_priority.load() ? ss->sp[0] : ss->spl[0];
      rc = tl  // with la: two-level blocking with the look-ahead
               ? blocked_qr2_lookahead(H, tau, ws.T64, ws.T64b, batch, n, s, sp, ss->evP[0],
                                       ss->evB[0], ss->joinP[0], r0, plan.deep)
               : blocked_qr_lookahead(A, strideA_b, strideA_row, H, tau, ws.T, ws.T2, batch, n,
                                      s, sp, ss->evP[0], ss->evB[0], ss->joinP[0],
                                      tma ? &r0 : nullptr);
    }
    if (rc == QRB_OK && hooks != nullptr) rc = hooks->after(0, batch, s);
    return rc;
  }
  SideStreams* ss = side_streams();
  if (ss == nullptr) return QRB_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(ss->mu);
  // Split the batch into groups that run the same kernel sequence on separate
  // internal streams, forked from and joined back into the caller's stream, so
  // that one group's (latency-bound) panel kernels overlap another group's
  // trailing updates.
  if (cudaEventRecord(ss->fork, s) != cudaSuccess) return QRB_ERR_LAUNCH;
  const int64_t nn = (int64_t)n * n;
  const int64_t tper = (int64_t)kPanelW * kPanelW;
  int rc = QRB_OK;
  for (int g = 0; g < groups && rc == QRB_OK; ++g) {
    const int64_t b0 = batch * g / groups, b1 = batch * (g + 1) / groups;
    if (b1 <= b0) continue;
    cudaStream_t gs = ss->s[g];
    if (cudaStreamWaitEvent(gs, ss->fork, 0) != cudaSuccess) return QRB_ERR_LAUNCH;
    if (hooks != nullptr && (rc = hooks->before(b0, b1, gs)) != QRB_OK) break;
    const TmaRoute rg = route_of(b0);
    if (tl && la)
      rc = blocked_qr2_lookahead(H + b0 * nn, tau + b0 * n, ws.T64 + b0 * 4 * tper,
                                 ws.T64b + b0 * 4 * tper, b1 - b0, n, gs,
                                 g_panel_priority.load() ? ss->sp[g] : ss->spl[g], ss->evP[g],
                                 ss->evB[g], ss->joinP[g], rg, plan.deep);
    else if (tl)
      rc = blocked_qr2(A + b0 * strideA_b, strideA_b, strideA_row, H + b0 * nn, tau + b0 * n,
                       ws.T64 + b0 * 4 * tper, b1 - b0, n, gs, tma ? &rg : nullptr);
    else if (la)
      rc = blocked_qr_lookahead(A + b0 * strideA_b, strideA_b, strideA_row, H + b0 * nn,
                                tau + b0 * n, ws.T + b0 * tper, ws.T2 + b0 * tper, b1 - b0, n,
                                gs, g_panel_priority.load() ? ss->sp[g] : ss->spl[g],
                                ss->evP[g], ss->evB[g], ss->joinP[g],
                                tma ? &rg : nullptr);
    else
      rc = blocked_qr(A + b0 * strideA_b, strideA_b, strideA_row, H + b0 * nn, tau + b0 * n,
                      ws.T + b0 * tper, b1 - b0, n, gs, tma ? &rg : nullptr);
    if (rc == QRB_OK && hooks != nullptr) rc = hooks->after(b0, b1, gs);
    if (cudaEventRecord(ss->join[g], gs) != cudaSuccess && rc == QRB_OK) rc = QRB_ERR_LAUNCH;
    if (cudaStreamWaitEvent(s, ss->join[g], 0) != cudaSuccess && rc == QRB_OK) rc = QRB_ERR_LAUNCH;
  }
  return rc;
}

}  // namespace qrb


extern "C" {

int qrb_version(void) { return 100; }

const char* qrb_status_string(int status) {
  switch (status) {
    case QRB_OK: return "qrb: ok";
    case QRB_ERR_INVALID_ARG: return "qrb: invalid argument";
    case QRB_ERR_UNSUPPORTED: return "qrb: unsupported size";
    case QRB_ERR_WORKSPACE: return "qrb: workspace missing or too small";
    case QRB_ERR_LAUNCH: return "qrb: kernel launch or execution failed";
    case QRB_ERR_DEVICE: return "qrb: no usable CUDA device";
    case QRB_ERR_INJECTED: return "qrb: injected failure (fail_next)";
    case QRB_ERR_DEVICE_WAIT: return "qrb: a device-side wait timed out (device_error set)";
    default: return "qrb: unknown status";
  }
}

int32_t qrb_max_n(void) { return qrb::kMaxN; }
int32_t qrb_fused_max_n(void) { return qrb::kFusedMidMaxN; }

size_t qrb_workspace_bytes(int64_t batch, int32_t n) {
  if (batch <= 0 || n <= qrb::kFusedMaxN) return 0;
  // Eight 32 x 32 units per matrix: one compact-WY factor T is the minimum, a
  // second enables the panel look-ahead, four (one 64 x 64 factor) the
  // two-level blocking, all eight (two 64 x 64 factors) two-level blocking
  // with the look-ahead; then the split reflectors of the tensor-core update
  // (two V buffers x hi / lo, n x 64 each) where that update applies.
  return 8 * (size_t)batch * qrb::kPanelW * qrb::kPanelW * sizeof(float) +
         qrb::vsplit_bytes(batch, n);
}

int qrb_route(int64_t batch, int32_t n, size_t workspace_bytes) {
  if (batch <= 0 || n <= 0 || n > qrb::kMaxN) return 0;
  qrb::FactorScratch fs;
  if (n > qrb::kFusedMaxN) {
    // the same carving as qrb_geqrf_f32 (a stand-in base address: only which
    // factors fit matters here)
    static float dummy[4];
    fs = qrb::factor_scratch(dummy, workspace_bytes, batch, n);
  }
  return qrb::route_code(qrb::make_plan(batch, n, fs));
}

int qrb_fused_qr_f32(const float* A, int64_t strideA_b, int64_t strideA_row,
                     float* H, float* tau, int64_t batch, int32_t n,
                     void* stream) {
  if (batch < 0 || n < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB_OK;
  if (!A || !H || !tau) return QRB_ERR_INVALID_ARG;
  if (n > qrb::kFusedMidMaxN) return QRB_ERR_UNSUPPORTED;
  if (bad_matrix_strides(strideA_b, strideA_row, n, n, batch)) return QRB_ERR_INVALID_ARG;
  if (take_injected_failure()) return QRB_ERR_INJECTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The reference's fused operator covers n <= 128 (src/qrbench/variants.py:698,
  // :741): lanes of a warp per matrix up to n = 32, one CTA per matrix above.
  const int rc = n <= qrb::kFusedMaxN
                     ? qrb::launch_fused_small(A, strideA_b, strideA_row, H, tau, batch, n, s)
                     : qrb::launch_fused_mid(A, strideA_b, strideA_row, H, tau, batch, n, s);
  return finish(rc, s);
}

int qrb_panel_qr_f32(const float* P, int64_t strideP_b, int64_t strideP_row,
                     float* H, float* V, float* tau, float* T, int64_t batch,
                     int32_t r, int32_t w, void* stream) {
  if (batch < 0 || r < 0 || w < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || r == 0 || w == 0) return QRB_OK;
  if (!P || !H || !tau || !T) return QRB_ERR_INVALID_ARG;
  if (w > qrb::kPanelW || r < w) return QRB_ERR_UNSUPPORTED;
  if (qrb::panel_cluster_size(r, batch) > qrb::kMaxCluster) return QRB_ERR_UNSUPPORTED;
  if (bad_matrix_strides(strideP_b, strideP_row, r, w, batch)) return QRB_ERR_INVALID_ARG;
  if (take_injected_failure()) return QRB_ERR_INJECTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = qrb::launch_panel(P, strideP_b, strideP_row, H, (int64_t)r * w, w, tau, w, T,
                                   (int64_t)w * w, w, V, batch, r, w, s);
  return finish(rc, s);
}

int qrb_larfb_f32(const float* V, int64_t strideV_b, int64_t strideV_row,
                  const float* T, float* C, int64_t strideC_b,
                  int64_t strideC_row, int64_t batch, int32_t r, int32_t k,
                  int32_t c, void* stream) {
  if (batch < 0 || r < 0 || k < 0 || c < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || r == 0 || k == 0 || c == 0) return QRB_OK;
  if (!V || !T || !C) return QRB_ERR_INVALID_ARG;
  const bool k64 = k == 2 * qrb::kPanelW;
  if ((k > qrb::kPanelW && !k64) || r < k) return QRB_ERR_UNSUPPORTED;
  if (bad_matrix_strides(strideV_b, strideV_row, r, k, batch)) return QRB_ERR_INVALID_ARG;
  if (bad_matrix_strides(strideC_b, strideC_row, r, c, batch)) return QRB_ERR_INVALID_ARG;
  if (k64 && !qrb::larfb64_supported(V, strideV_b, strideV_row, C, strideC_b, strideC_row, C,
                                     strideC_b, strideC_row, c))
    return QRB_ERR_UNSUPPORTED;
  if (take_injected_failure()) return QRB_ERR_INJECTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k64)
    return finish(qrb::launch_larfb64(V, strideV_b, strideV_row, T, (int64_t)k * k, C, strideC_b,
                                      strideC_row, C, strideC_b, strideC_row, batch, r, c, s),
                  s);
  const int rc = larfb_any(V, strideV_b, strideV_row, T, (int64_t)k * k, k, C, strideC_b,
                           strideC_row, C, strideC_b, strideC_row, batch, r, k, c, s);
  return finish(rc, s);
}

int qrb_geqrf_f32(const float* A, int64_t strideA_b, int64_t strideA_row,
                  float* H, float* tau, int64_t batch, int32_t n,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 0 || n < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB_OK;
  if (!A || !H || !tau) return QRB_ERR_INVALID_ARG;
  if (n > qrb::kMaxN) return QRB_ERR_UNSUPPORTED;
  if (bad_matrix_strides(strideA_b, strideA_row, n, n, batch)) return QRB_ERR_INVALID_ARG;
  if (A == H && (strideA_row != n || strideA_b != (int64_t)n * n)) return QRB_ERR_INVALID_ARG;
  qrb::FactorScratch fs;
  if (n > qrb::kFusedMaxN) {
    const size_t one = qrb::min_workspace_bytes(batch);  // the minimum: one T factor each
    if (workspace == nullptr || workspace_bytes < one) return QRB_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return QRB_ERR_INVALID_ARG;
    fs = qrb::factor_scratch(workspace, workspace_bytes, batch, n);
  }
  if (take_injected_failure()) return QRB_ERR_INJECTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool replayed = false;
  const int rc = qrb::geqrf_graph(A, strideA_b, strideA_row, H, tau, fs, workspace,
                                  workspace_bytes, batch, n, s, &replayed);
  if (rc != QRB_OK || replayed) return finish(rc, s);
  return finish(qrb::geqrf_enqueue(A, strideA_b, strideA_row, H, tau, fs, batch, n, s), s);
}

int qrb_set_config(const char* key, int64_t value) {
  if (!key) return QRB_ERR_INVALID_ARG;
  // every key but the counters and one-shot actions can change what a call
  // enqueues (routes, kernel parameters): cached graphs of older calls no
  // longer match
  if (std::strcmp(key, "launches") != 0 && std::strcmp(key, "device_error") != 0 &&
      std::strcmp(key, "fail_next") != 0 && std::strcmp(key, "wait_probe") != 0)
    g_generation.fetch_add(1);
  if (std::strcmp(key, "graph_cache") == 0) {
    if (value != 0 && value != 1) return QRB_ERR_INVALID_ARG;
    g_graph.store(value);
    if (value == 0) qrb::graph_cache_clear();
    return QRB_OK;
  }
  if (std::strcmp(key, "fail_next") == 0) {
    if (value < 0) return QRB_ERR_INVALID_ARG;
    g_fail_next.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "sync_check") == 0) {
    if (value != 0 && value != 1) return QRB_ERR_INVALID_ARG;
    g_sync_check.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "wait_limit") == 0) {
    if (value < 1000 || value > 100000000000LL) return QRB_ERR_INVALID_ARG;
    g_wait_limit.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "test_skip_mma") == 0) {
    if (value != 0 && value != 1) return QRB_ERR_INVALID_ARG;
    g_skip_mma.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "wait_probe") == 0) {  // run the probe on the legacy stream, synchronously
    if (value < 1000 || value > 100000000000LL) return QRB_ERR_INVALID_ARG;
    const int rc = qrb::launch_wait_probe(value, nullptr);
    if (rc != QRB_OK) return rc;
    return cudaDeviceSynchronize() == cudaSuccess ? QRB_OK : QRB_ERR_LAUNCH;
  }
  if (std::strcmp(key, "tma_ctas") == 0) {
    if (value < 0 || value > 4096) return QRB_ERR_INVALID_ARG;
    g_tma_ctas.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "tma_split_rows") == 0) {
    if (value < 0 || value > (1 << 20)) return QRB_ERR_INVALID_ARG;
    g_tma_split.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "tma_pair") == 0) {
    if (value < 0 || value > 2) return QRB_ERR_INVALID_ARG;
    g_tma_pair.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "tma_dual") == 0) {
    if (value < 0 || value > 2) return QRB_ERR_INVALID_ARG;
    g_tma_dual.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "lookahead_depth") == 0) {
    if (value < 0 || value > 2) return QRB_ERR_INVALID_ARG;
    g_la_depth.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "narrow_update") == 0) {
    if (value != 0 && value != 1) return QRB_ERR_INVALID_ARG;
    g_narrow.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "panel_priority") == 0) {
    if (value != 0 && value != 1) return QRB_ERR_INVALID_ARG;
    g_panel_priority.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "larfb_kind") == 0) {
    if (value < -1 || value > 3) return QRB_ERR_INVALID_ARG;
    g_larfb_kind.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "device_error") == 0) {
    if (value != 0) return QRB_ERR_INVALID_ARG;
    int v = 0;
    return qrb::device_error_flag(&v, true);
  }
  if (std::strcmp(key, "groups") == 0) {
    if (value < 0 || value > kMaxGroups) return QRB_ERR_INVALID_ARG;
    g_groups.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "host_direct") == 0) {
    if (value < 0 || value > 3) return QRB_ERR_INVALID_ARG;
    g_host_direct.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "lookahead") == 0) {
    if (value < 0 || value > 2) return QRB_ERR_INVALID_ARG;
    g_lookahead.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "two_level") == 0) {
    if (value < 0 || value > 2) return QRB_ERR_INVALID_ARG;
    g_two_level.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "panel_rpt") == 0) {
    if (value != 0 && value != 1 && value != 2 && value != 4) return QRB_ERR_INVALID_ARG;
    g_panel_rpt.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "gram_tile") == 0) {
    if (value != 0 && value != 64 && value != 128) return QRB_ERR_INVALID_ARG;
    g_gram_tile.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "mid_fused") == 0) {
    if (value < 0 || value > 2) return QRB_ERR_INVALID_ARG;
    g_mid_fused.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "fused_cpl") == 0) {
    if (value != 0 && value != 2 && value != 4) return QRB_ERR_INVALID_ARG;
    g_fused_cpl.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "host_groups") == 0) {
    if (value < 0 || value > kMaxGroups) return QRB_ERR_INVALID_ARG;
    g_host_groups.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "host_ramp") == 0) {
    if (value != 0 && value != 1) return QRB_ERR_INVALID_ARG;
    g_host_ramp.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "direct_blocks") == 0) {
    if (value < 0 || value > (1 << 20)) return QRB_ERR_INVALID_ARG;
    g_direct_blocks.store(value);
    return QRB_OK;
  }
  if (std::strcmp(key, "launches") == 0) {
    if (value != 0) return QRB_ERR_INVALID_ARG;
    g_launches.store(0);
    return QRB_OK;
  }
  return QRB_ERR_INVALID_ARG;
}

int qrb_get_config(const char* key, int64_t* value) {
  if (!key || !value) return QRB_ERR_INVALID_ARG;
  if (std::strcmp(key, "fail_next") == 0) { *value = g_fail_next.load(); return QRB_OK; }
  if (std::strcmp(key, "sync_check") == 0) { *value = g_sync_check.load(); return QRB_OK; }
  if (std::strcmp(key, "larfb_kind") == 0) { *value = g_larfb_kind.load(); return QRB_OK; }
  if (std::strcmp(key, "wait_limit") == 0) { *value = g_wait_limit.load(); return QRB_OK; }
  if (std::strcmp(key, "test_skip_mma") == 0) { *value = g_skip_mma.load(); return QRB_OK; }
  if (std::strcmp(key, "tma_ctas") == 0) { *value = g_tma_ctas.load(); return QRB_OK; }
  if (std::strcmp(key, "narrow_update") == 0) { *value = g_narrow.load(); return QRB_OK; }
  if (std::strcmp(key, "tma_split_rows") == 0) { *value = g_tma_split.load(); return QRB_OK; }
  if (std::strcmp(key, "tma_pair") == 0) { *value = g_tma_pair.load(); return QRB_OK; }
  if (std::strcmp(key, "tma_dual") == 0) { *value = g_tma_dual.load(); return QRB_OK; }
  if (std::strcmp(key, "graph_cache") == 0) { *value = g_graph.load(); return QRB_OK; }
  if (std::strcmp(key, "graph_cache_entries") == 0) {
    *value = qrb::graph_cache_entries();
    return QRB_OK;
  }
  if (std::strcmp(key, "lookahead_depth") == 0) { *value = g_la_depth.load(); return QRB_OK; }
  if (std::strcmp(key, "panel_priority") == 0) { *value = g_panel_priority.load(); return QRB_OK; }
  if (std::strcmp(key, "device_error") == 0) {
    int v = 0;
    const int rc = qrb::device_error_flag(&v, false);
    *value = v;
    return rc;
  }
  if (std::strcmp(key, "launches") == 0) { *value = g_launches.load(); return QRB_OK; }
  if (std::strcmp(key, "groups") == 0) { *value = g_groups.load(); return QRB_OK; }
  if (std::strcmp(key, "host_direct") == 0) { *value = g_host_direct.load(); return QRB_OK; }
  if (std::strcmp(key, "host_ramp") == 0) { *value = g_host_ramp.load(); return QRB_OK; }
  if (std::strcmp(key, "host_groups") == 0) { *value = g_host_groups.load(); return QRB_OK; }
  if (std::strcmp(key, "fused_cpl") == 0) { *value = g_fused_cpl.load(); return QRB_OK; }
  if (std::strcmp(key, "mid_fused") == 0) { *value = g_mid_fused.load(); return QRB_OK; }
  if (std::strcmp(key, "lookahead") == 0) { *value = g_lookahead.load(); return QRB_OK; }
  if (std::strcmp(key, "two_level") == 0) { *value = g_two_level.load(); return QRB_OK; }
  if (std::strcmp(key, "panel_rpt") == 0) { *value = g_panel_rpt.load(); return QRB_OK; }
  if (std::strcmp(key, "gram_tile") == 0) { *value = g_gram_tile.load(); return QRB_OK; }
  if (std::strcmp(key, "direct_blocks") == 0) { *value = qrb::host_direct_blocks(); return QRB_OK; }
  if (std::strcmp(key, "host_path") == 0) { *value = qrb::host_last_path(); return QRB_OK; }
  return QRB_ERR_INVALID_ARG;
}

}  // extern "C"

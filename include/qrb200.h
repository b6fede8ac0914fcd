/*
 * qrb200.h — C ABI of libqrb200.so, a B200-native (sm_100a) batched FP32
 * compact-Householder QR factorization with torch.geqrf / LAPACK sgeqrf
 * semantics.
 *
 * Layout conventions shared by every entry point:
 *   - Matrices are batched, row-major, FP32: element (i, j) of matrix m lives at
 *     base + m * stride_b + i * stride_row + j (the column stride is 1).
 *   - All pointers are device pointers (qrb_geqrf_f32_host's A_host, H_host and
 *     tau_host excepted); `stream` is a cudaStream_t (NULL = the
 *     legacy default stream). Work is enqueued stream-ordered and the call
 *     returns without synchronising.
 *   - The library allocates no device memory per call. Scratch space, when an
 *     entry point needs it, is passed in by the caller (see
 *     qrb_workspace_bytes).
 *   - Every entry point returns a qrb_status code. Argument errors are detected
 *     on the host before anything is enqueued. There is no CPU fallback.
 *
 * Output convention (identical to torch.geqrf): for A = Q R with
 * Q = H_0 H_1 ... H_{n-1}, H_j = I - tau_j v_j v_j^T, v_j(j) = 1 implicit,
 * the output H holds R on and above the diagonal and the essential part of v_j
 * below the diagonal of column j; tau[j] = tau_j; beta = -sign(alpha)*||x||
 * (alpha >= 0 gives a negative diagonal); a column with nothing below the
 * diagonal to annihilate gets tau = 0.
 */
#ifndef QRB200_H
#define QRB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QRB_API __attribute__((visibility("default")))
#else
#define QRB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
enum {
  QRB_OK = 0,
  QRB_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad stride, ... */
  QRB_ERR_UNSUPPORTED = 2,   /* size outside what the kernels handle */
  QRB_ERR_WORKSPACE = 3,     /* workspace missing or smaller than required */
  QRB_ERR_LAUNCH = 4,        /* a kernel launch failed (cudaGetLastError) */
  QRB_ERR_DEVICE = 5,        /* no usable sm_100 device / device query failed */
  QRB_ERR_INJECTED = 6,      /* failure injected by qrb_set_config("fail_next") */
  QRB_ERR_DEVICE_WAIT = 7    /* a kernel's bounded device-side wait timed out */
};

/* Library version as 10000*major + 100*minor + patch. */
QRB_API int qrb_version(void);

/* Human-readable text for a status code (static storage, never NULL). */
QRB_API const char* qrb_status_string(int status);

/* Largest n that qrb_geqrf_f32 accepts. */
QRB_API int32_t qrb_max_n(void);

/* Bytes of device workspace to give qrb_geqrf_f32 for (batch, n): 0 for
 * n <= 32; otherwise eight 32 x 32 units (32 KiB) per matrix, plus, for
 * n >= 129 with n % 4 == 0, the split reflectors of the tensor-core trailing
 * update (four buffers of n x 32 high parts and n x 32 remainders,
 * 1024 * n bytes per matrix). One 32 x 32 unit per matrix is the minimum
 * accepted; two enable the panel look-ahead ("lookahead" below), four
 * two-level blocking ("two_level"), the whole amount the tensor-core update
 * (and with it two-level blocking with the look-ahead). */
QRB_API size_t qrb_workspace_bytes(int64_t batch, int32_t n);

/*
 * The route qrb_geqrf_f32 takes for (batch, n) given a workspace of
 * workspace_bytes, as a bit field (0 = no route: bad size, or too little
 * workspace for the blocked route):
 *   bits 0-3   1 = fused, lanes of a warp per matrix (n <= 32);
 *              2 = fused, one CTA per matrix (32 < n <= 128);
 *              3 = blocked panel route;
 *   bits 4-7   blocked trailing update: 0 = FP32 FFMA; 1 = tcgen05 3xTF32 with
 *              operands staged by the CUDA cores; 2 = FFMA then tcgen05;
 *              3 = tcgen05 3xTF32 fed by TMA;
 *   bit 8      panel look-ahead on a second stream;
 *   bit 9      two-level (64-reflector) blocking;
 *   bits 12-15 batch groups on internal streams.
 * With every test hook of qrb_set_config at its default, the route is a pure
 * function of (batch, n, workspace_bytes): nothing else that a caller does
 * changes the kernels a call runs. It mirrors the reference's champion
 * dispatch (src/qrbench/variants.py:876-917), which routes by n alone.
 */
QRB_API int qrb_route(int64_t batch, int32_t n, size_t workspace_bytes);

/*
 * Batched square QR: the full hot path, one call per factorization.
 * Replaces the reference's registered impl callable
 *   impl(A: [b, n, n] fp32) -> (H, tau)
 * (src/qrbench/reference.py:15 QRImpl; src/qrbench/variants.py:876-917
 * make_hh_panel_tuned(...).impl, the CHAMPION at variants.py:106), including
 * its dispatch between fused whole-matrix kernels (n <= 32: lanes of a warp
 * per matrix; 32 < n <= 128: one CTA per matrix, see "mid_fused") and the
 * blocked panel route.
 *
 *   A      input, batch x n x n, strides (strideA_b, strideA_row), read only.
 *   H      output, batch x n x n contiguous (stride n*n, row stride n).
 *          H may equal A only when A is itself contiguous (in-place mode).
 *   tau    output, batch x n contiguous.
 */
QRB_API int qrb_geqrf_f32(const float* A, int64_t strideA_b, int64_t strideA_row,
                  float* H, float* tau, int64_t batch, int32_t n,
                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * qrb_geqrf_f32 for callers that cannot allocate device memory (a fixed
 * memory budget reserved up front, a host application that owns the only
 * allocator, a runtime that forbids cudaMalloc after start-up). It has no
 * counterpart in the reference. Same arguments and results as qrb_geqrf_f32
 * minus the workspace: the scratch it needs lives in a 4 MiB array built into
 * the library, which every GPU that loads the library holds until the process
 * exits. It allocates nothing.
 *   - Limit: for n > 32 at most 1024 matrices per call (one 4 KiB T factor
 *     each); a larger batch returns QRB_ERR_UNSUPPORTED before any work is
 *     enqueued. n <= 32 needs no scratch and has no batch limit.
 *   - The first call on a device looks up the array's device address; make it
 *     before any stream capture starts.
 *   - All calls on a device share the array: calls whose GPU work overlaps
 *     (unordered streams) race and give wrong results. Nothing in the array
 *     has to be cleared between calls.
 */
QRB_API int qrb_geqrf_f32_noalloc(const float* A, int64_t strideA_b,
                                  int64_t strideA_row, float* H, float* tau,
                                  int64_t batch, int32_t n, void* stream);

/*
 * Host memory in, host memory out: the batched QR of a host-resident batch,
 * with the host<->device copies pipelined against the factorization. It has
 * no single counterpart in the reference, whose impl takes device tensors; it
 * replaces the round trip a host-side caller of the reference composes,
 *   H, tau = impl(A.to("cuda")); H.cpu(); tau.cpu()
 * (src/qrbench/reference.py:15 QRImpl). Results are bit-identical to
 * qrb_geqrf_f32 on the same data.
 *
 *   A_host    input, batch x n x n contiguous FP32 in host memory.
 *   H_host    output, batch x n x n contiguous (may equal A_host).
 *   tau_host  output, batch x n contiguous.
 *   workspace device memory of qrb_host_workspace_bytes(batch, n) bytes,
 *             256-byte aligned (staging for A/H and tau, plus the T scratch).
 *   chunks    pipeline depth: the batch is cut into this many pieces
 *             (1..64, capped at batch; 0 = automatic: 6 pieces for n <= 64,
 *             4 up to n = 128, and above, where qrb_geqrf_f32 runs its
 *             blocked route, that route's batch groups: one factorization
 *             over the whole batch whose groups each start when their own
 *             matrices have landed and are copied out when done).
 * The pieces run on three internal streams of the current device (copy in,
 * factor, copy out), forked from and joined back into `stream`: synchronise
 * `stream` before reading H_host / tau_host. Page-locked host buffers
 * (cudaHostAlloc / cudaHostRegister) are needed for the copies to overlap;
 * pageable buffers give correct results with serialised copies. Calls on one
 * device share the internal streams and are serialised on them.
 * For n <= 32 the kernel can reach host buffers that lie in page-locked
 * allocations mapped into the current device's address space directly
 * (qrb_set_config("host_direct", mode)): 3 (default) = it writes tau to host
 * memory, the matrices are copied; 1 = it reads A and writes H and tau over
 * PCIe itself in one launch on `stream`, without copies; 2 = A is copied in,
 * it writes H and tau; 0 = copies only. A buffer that fails the mapping check
 * is copied. qrb_get_config("host_path") tells which mode the last call ran.
 */
QRB_API size_t qrb_host_workspace_bytes(int64_t batch, int32_t n);
QRB_API int qrb_geqrf_f32_host(const float* A_host, float* H_host, float* tau_host,
                               int64_t batch, int32_t n, void* workspace,
                               size_t workspace_bytes, int32_t chunks, void* stream);

/*
 * Fused whole-matrix QR for small n (n <= 128), one launch. n <= 32: 16 (or
 * 8) lanes factor one matrix in registers, two (or four) matrices per warp;
 * 32 < n <= 128: one CTA per matrix, one thread per column. Replaces
 * hh_fused_qr / _hh_fused_qr_kernel (src/qrbench/triton_kernels.py:722-755,
 * :641-720) as make_hh_fused_smalln routes it (cap 128,
 * src/qrbench/variants.py:698, :741).
 */
QRB_API int qrb_fused_qr_f32(const float* A, int64_t strideA_b, int64_t strideA_row,
                     float* H, float* tau, int64_t batch, int32_t n,
                     void* stream);

/* Largest n accepted by qrb_fused_qr_f32. */
QRB_API int32_t qrb_fused_max_n(void);

/*
 * Householder factorization of a batch of r x w panels (w <= 32) plus the
 * compact-WY factor T. Replaces hh_panel_qr / _hh_panel_kernel
 * (src/qrbench/triton_kernels.py:912-967, :787-910).
 *
 *   P      input panels, batch x r x w, strides (strideP_b, strideP_row).
 *   H      output, batch x r x w contiguous: R in the top w x w upper triangle,
 *          essential reflectors strictly below the diagonal.
 *   V      optional output (NULL to skip), batch x r x w contiguous: unit lower
 *          reflector matrix (1 on the diagonal, 0 above).
 *   tau    output, batch x w contiguous.
 *   T      output, batch x w x w contiguous, upper triangular, with
 *          Q = I - V T V^T (forward, column-wise LARFT).
 */
QRB_API int qrb_panel_qr_f32(const float* P, int64_t strideP_b, int64_t strideP_row,
                     float* H, float* V, float* tau, float* T,
                     int64_t batch, int32_t r, int32_t w, void* stream);

/*
 * Block-reflector trailing update C <- C - V (T^T (V^T C)), applying Q^T of a
 * factored panel to the trailing columns. Replaces the three batched GEMMs of
 * _hh_panel_blocked_qr (src/qrbench/variants.py:800-804).
 *
 *   V      reflectors, batch x r x k (k <= 32, or k = 64: the two-level
 *          block, which needs 16-byte aligned V and C rows and matrices and
 *          c % 4 == 0, else QRB_ERR_UNSUPPORTED), strides (strideV_b,
 *          strideV_row). Only the strictly lower part is read: the diagonal is
 *          taken as 1 and the upper part as 0, so V may point into a packed H.
 *   T      batch x k x k contiguous (stride k*k), upper triangular.
 *   C      batch x r x c, strides (strideC_b, strideC_row), updated in place.
 */
QRB_API int qrb_larfb_f32(const float* V, int64_t strideV_b, int64_t strideV_row,
                  const float* T, float* C, int64_t strideC_b,
                  int64_t strideC_row, int64_t batch, int32_t r, int32_t k,
                  int32_t c, void* stream);

/*
 * Consumers of a factorization: form Q, or apply Q / Q^T to a matrix. H and
 * tau are as qrb_geqrf_f32 writes them; the first k columns of H hold the
 * reflectors (strictly lower part, unit diagonal implied) and tau is
 * batch x k contiguous (k <= n). Both need qrb_orgqr_workspace_bytes(batch, n)
 * bytes of 16-byte aligned device scratch (one 32 x 32 T factor per matrix).
 *
 * qrb_orgqr_f32: Q (batch x n x n contiguous, must not overlap H) =
 * H_0 H_1 ... H_{k-1}. Replaces torch.linalg.householder_product(H, tau) as
 * the reference's checker calls it (src/qrbench/checker.py:129).
 *
 * qrb_ormqr_f32: C (batch x n x ncols, strides (strideC_b, strideC_row)) is
 * overwritten with Q^T C (transpose != 0) or Q C (transpose == 0). Replaces
 * torch.ormqr(H, tau, C, left=True, transpose=...) (src/qrbench/variants.py:165).
 */
QRB_API size_t qrb_orgqr_workspace_bytes(int64_t batch, int32_t n);
QRB_API int qrb_orgqr_f32(const float* H, int64_t strideH_b, int64_t strideH_row,
                          const float* tau, int32_t k, float* Q, int64_t batch, int32_t n,
                          void* workspace, size_t workspace_bytes, void* stream);
QRB_API int qrb_ormqr_f32(const float* H, int64_t strideH_b, int64_t strideH_row,
                          const float* tau, int32_t k, float* C, int64_t strideC_b,
                          int64_t strideC_row, int64_t batch, int32_t n, int32_t ncols,
                          int32_t transpose, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * The step in front of the factorization in the reference's workload: the
 * statistics S = G G^T of gradients viewed as [basis_dim n, contracted_dim k]
 * (reference AGENTS.md:27, "statistics are formed as G @ G.T, and QR is run on
 * square basis_dim x basis_dim matrices"). No reference function computes it;
 * it replaces the caller's torch G @ G.mT (FP32, no TF32) in front of impl().
 *
 * qrb_gram_f32: G batch x n x k, strides (strideG_b, strideG_row >= k), unit
 * column stride; S batch x n x n contiguous, both triangles written (exactly
 * symmetric). k = 0 gives S = 0. S must not overlap G.
 *
 * qrb_gram_geqrf_f32: (H, tau) = geqrf(G G^T) in one call: the Gram matrix is
 * formed into H and factored in place; the same workspace as qrb_geqrf_f32
 * (qrb_workspace_bytes(batch, n)). H must not overlap G.
 */
QRB_API int qrb_gram_f32(const float* G, int64_t strideG_b, int64_t strideG_row, float* S,
                         int64_t batch, int32_t n, int32_t k, void* stream);
QRB_API int qrb_gram_geqrf_f32(const float* G, int64_t strideG_b, int64_t strideG_row,
                               float* H, float* tau, int64_t batch, int32_t n, int32_t k,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * Test hooks (never needed for correct use). They are process-wide: a value
 * set here changes the route of every later call in the process, on every
 * thread and device, until it is set back, so only tests and benchmarks set
 * them; at their defaults the route depends on (batch, n, workspace) alone
 * (qrb_route). Keys:
 *   "fail_next"   value v > 0: the next v calls of any compute entry point
 *                 return QRB_ERR_INJECTED without enqueuing work (host-side
 *                 fault injection for tests).
 *   "sync_check"  1: every compute call synchronises its stream and reports
 *                 asynchronous kernel faults as QRB_ERR_LAUNCH and device-side
 *                 wait timeouts as QRB_ERR_DEVICE_WAIT (debug mode).
 *   "larfb_kind"  trailing update of the blocked route: -1 (default) =
 *                 automatic (3 where it applies, else 0); 0 = FP32 FFMA;
 *                 1 = tcgen05 3xTF32 for both products with operands staged
 *                 by the CUDA cores; 2 = FFMA for V^T C and tcgen05 3xTF32 for
 *                 C -= V W'; 3 = tcgen05 3xTF32 fed by TMA (n >= 129,
 *                 n % 4 == 0 and the full qrb_workspace_bytes, else FFMA).
 *                 Kinds 1 and 2 apply to 32-reflector blocks with 16-byte
 *                 aligned row-major operands; FFMA elsewhere.
 *   "wait_limit"  clock cycles a kernel's bounded device-side wait lasts
 *                 before it gives up (default 2e9, about one second).
 *   "wait_probe"  value = a cycle limit: runs one probe kernel (synchronously,
 *                 on the legacy stream) whose bounded wait nothing completes,
 *                 so it times out and sets "device_error" (test only).
 *   "test_skip_mma" 1: the TMA-fed update withholds its first MMAs, so its
 *                 bounded waits run out, it abandons the call, sets
 *                 "device_error" and frees its resources (test only; results
 *                 of such calls are wrong).
 *   "tma_ctas"    most CTAs of one TMA-fed update launch, 1..4096 (0, the
 *                 default: one per SM).
 *   "tma_split_rows" 0..2^20: the TMA-fed update sums each tile's V^T C in
 *                 two row halves (each over its own interleaved partial
 *                 accumulators, the two sums added last) when the trailing
 *                 block has at least this many rows (default 1024; 0 =
 *                 never). Results depend on this value, never on the batch,
 *                 its grouping or "tma_pair".
 *   "tma_pair"    with two row halves, 0 (default): a cluster of two CTAs per
 *                 tile (one half each; the partial sums added through
 *                 distributed shared memory) when the launch's tiles fit the
 *                 SMs twice over (2 x tiles <= SMs), else one CTA per tile;
 *                 1: always one CTA; 2: always a pair. The same bits either
 *                 way.
 *   "tma_dual"    32-reflector updates without row halves, 0 (default): two
 *                 CTAs per SM (4 worker warps, 2 pass-1 stages, one pass-2
 *                 accumulator, about 104 KB of shared memory each) when the
 *                 launch has more tiles than SMs, so that one CTA's pass 1
 *                 runs beside the other's pass 2; 1: one CTA per SM; 2: always
 *                 two. The same bits either way.
 *   "graph_cache" 1 (default): a blocked-route call repeated with the same
 *                 arguments (every pointer, stride, size and the workspace)
 *                 and no qrb_set_config change in between is captured into a
 *                 CUDA graph on its second occurrence and replayed from then
 *                 on (forked from and joined back into the caller's stream;
 *                 the same kernels, the same bits; up to 8 graphs cached).
 *                 Calls on a stream being captured, under "sync_check", and
 *                 through qrb_geqrf_f32_noalloc run eagerly. 0: always
 *                 eagerly (drops the cached graphs). Read
 *                 "graph_cache_entries" for the number of graphs held.
 *   "lookahead_depth" 0 (default: 2 where one batch group runs at
 *                 n >= 4096, else 1), 1 or 2: with two-level blocking and the
 *                 look-ahead, depth 2 has the look-ahead stream apply both
 *                 panels' reflectors to all 64 columns of the next block (two
 *                 narrow updates), so the wide update starts at j0 + 128 and
 *                 has a block of slack before the next block needs it.
 *   "narrow_update" 0: the tensor-core route updates the next panel's 32
 *                 columns with the TMA-fed kernel as well, instead of the
 *                 narrow kernel that splits their rows across a cluster
 *                 (1, the default).
 *   "panel_priority" 0: the look-ahead stream (panels and the next panel's
 *                 update) runs at the default stream priority instead of the
 *                 highest (1, the default).
 *   "device_error" read: 1 if a kernel's bounded device-side wait timed out
 *                 since the last reset (synchronous); set to 0 to reset.
 *   "groups"      1..8: batches of 4 or more matrices with n > 32 are split
 *                 into this many groups (at most batch / 2) run on internal
 *                 streams (forked from and joined back into the caller's
 *                 stream) so that panel and trailing-update kernels of
 *                 different groups overlap; 0 (default) = 4 for n >= 1024,
 *                 else 2.
 *   "host_direct" 0..3 (default 3): how qrb_geqrf_f32_host reaches mapped
 *                 page-locked host buffers for n <= 32 (see there).
 *   "direct_blocks" grid of the mode-1 kernel in blocks of 4 warps (0 = 148).
 *   "lookahead"   blocked route: 0 = off, 1 = on, 2 (default) = automatic
 *                 (below); needs the full qrb_workspace_bytes. Panel j + 1
 *                 and the update of its columns run on a second stream (at the
 *                 highest priority) while the rest of step j's update runs.
 *                 With the FFMA update the results are unchanged; with the
 *                 tensor-core update the next panel's 32 columns are updated
 *                 by an FFMA kernel instead, the same results to FP32
 *                 rounding.
 *   "two_level"   blocked route: 0 = off, 1 = on, 2 (default) = automatic;
 *                 needs the full qrb_workspace_bytes. Two 32-column panels
 *                 are combined into one 64-reflector block (T 64 x 64) for the
 *                 trailing update; takes precedence over "lookahead". Same
 *                 results to FP32 rounding.
 *                 Automatic (measured on B200): with the tensor-core update,
 *                 from n = 1024 two-level blocking, with the look-ahead as
 *                 well while batch * n <= 65536 (the panels' latency chain
 *                 sets the time there, the update's traffic above), below
 *                 n = 1024 neither; with the FFMA update, the look-ahead from
 *                 n = 4096 and no two-level blocking. Two-level blocking with
 *                 the look-ahead needs the tensor-core update.
 *   "panel_rpt"   rows per thread of the panel kernel: 0 (default) = 1 up to
 *                 128 rows, else 2 where the batch's panels (clusters of
 *                 256-thread CTAs) all fit on the SMs at once, else 4; 1, 2
 *                 or 4 force that many (CTAs of up to 512 or 256 threads; 4
 *                 where more than 8 CTAs would be needed).
 *   "mid_fused"   1 (default): 32 < n <= 64 and 96 < n <= 128, and
 *                 64 < n <= 96 up to 592 matrices, are factored by one CTA per
 *                 matrix in one launch;
 *                 2: every 32 < n <= 128 that way; 0: always the blocked panel
 *                 route above n = 32.
 *   "fused_cpl"   n <= 32 kernel: 2 or 4 matrices per warp, 0 (default) = 4 up
 *                 to 4736 matrices, else 2. Results are identical either way.
 *   "host_groups" qrb_geqrf_f32_host on the blocked route without the
 *                 look-ahead (automatic depth) runs at least this many batch
 *                 groups, at most one per matrix (1..8; 0 = the route's own
 *                 count; default 8): finer pieces start sooner after their
 *                 copies; the bits do not change.
 *   "host_ramp"   1: qrb_geqrf_f32_host cuts the batch into pieces of relative
 *                 size 1, 2, .., 2, 1 instead of equal pieces (default 0).
 *   "host_path"   read: the path the last qrb_geqrf_f32_host call ran: the
 *                 host_direct mode 0..3, or 4 = the blocked route's batch
 *                 groups as pieces (-1 before the first call).
 *   "launches"    number of kernel launches this library has enqueued since
 *                 load or since the last qrb_set_config("launches", 0).
 * Returns QRB_ERR_INVALID_ARG for an unknown key or value.
 */
QRB_API int qrb_set_config(const char* key, int64_t value);
QRB_API int qrb_get_config(const char* key, int64_t* value);

#ifdef __cplusplus
}
#endif

#endif /* QRB200_H */

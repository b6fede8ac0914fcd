// qrb_geqrf_f32_host: host memory in, host memory out.
//
// For n > 128 on the blocked route with the automatic depth, the pieces are
// the route's batch groups: one factorization call over the whole batch whose
// groups each wait for their own host-to-device copy and hand their H and tau
// to the copy-out stream when done, so the groups' copies and factorizations
// overlap (the blocked factorization of a small piece takes nearly as long as
// that of the whole batch: its panels are a latency chain).
//
// Otherwise the batch is cut into chunks and run as a three-stage pipeline on
// three internal streams of the current device:
//   copy-in   every chunk's host-to-device copy, back to back;
//   compute   each chunk's factorization, in place in the device staging
//             buffer, once that chunk's copy has landed (event);
//   copy-out  each chunk's H and tau device-to-host copies once it is
//             factored (event).
// Host-to-device and device-to-host copies use separate copy engines, so with
// page-locked host buffers the two PCIe directions run at the same time and
// the factorization hides under them. The stages are forked from, and joined
// back into, the caller's stream.
//
// The enqueue loop runs here in C++ so that per-chunk host overhead stays at
// a few microseconds: one cudaMemcpyAsync per copy, two events per chunk.
// Each copy carries a fixed cost of several microseconds on the device side,
// so the default depth is a few large pieces. For n <= 32 with a page-locked
// tau buffer the fused kernel writes tau straight into host memory (one small
// copy fewer per piece, measured about 10 % faster end to end).
//
// Direct path (n <= 32): when A, H and tau are page-locked host memory that
// the current device can address (cudaHostAlloc, or cudaHostRegister with the
// mapped flag), the fused kernel reads A from and writes H and tau to host
// memory itself: one launch, no staging, no copies, the PCIe reads of some
// warps overlapping the PCIe writes of others. Before it is taken, both ends
// of every buffer are checked to lie in one mapped host allocation; anything
// else goes through the copy pipeline.
#include <cuda.h>  // CUpointer_attribute / CUresult types; the entry point is looked up at run time

#include <atomic>
#include <mutex>

#include "qrb_common.cuh"

namespace {

constexpr int kMaxChunks = 64;
constexpr int kAutoChunksSmall = 6;  // n <= 64 (measured best on B200, PCIe 5)
constexpr int kAutoChunksLarge = 4;  // n > 64: fewer pieces, each a full kernel sequence
constexpr size_t kAlign = 256;

std::atomic<int64_t> g_last_path{-1};  // 0 copies, 1 direct, 2 copies in + direct stores,
                                        // 3 copies + tau stores, 4 blocked-route groups

using PointerGetAttributeFn = CUresult (*)(void*, CUpointer_attribute, CUdeviceptr);

PointerGetAttributeFn pointer_get_attribute() {
  static std::once_flag once;
  static PointerGetAttributeFn fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PointerGetAttributeFn>(f);
    else
      (void)cudaGetLastError();
  });
  return fn;
}

// The device address through which the current device reaches the `bytes`
// bytes of host memory at p, or nullptr when that range is not (entirely) in
// one mapped page-locked host allocation.
void* mapped_view(const void* p, size_t bytes) {
  PointerGetAttributeFn get = pointer_get_attribute();
  if (get == nullptr || p == nullptr || bytes == 0) return nullptr;
  const char* ends[2] = {static_cast<const char*>(p), static_cast<const char*>(p) + bytes - 1};
  char* dev[2] = {};
  CUdeviceptr start[2] = {};
  for (int e = 0; e < 2; ++e) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, ends[e]) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    if (at.type != cudaMemoryTypeHost || at.devicePointer == nullptr) return nullptr;
    dev[e] = static_cast<char*>(at.devicePointer);
    if (get(&start[e], CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
            reinterpret_cast<CUdeviceptr>(dev[e])) != CUDA_SUCCESS)
      return nullptr;
  }
  if (start[0] != start[1]) return nullptr;                        // two allocations
  if (dev[1] - dev[0] != static_cast<ptrdiff_t>(bytes - 1)) return nullptr;  // not one linear view
  return dev[0];
}

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// The blocked route's batch groups as the pipeline's pieces: a group's copy in
// (on the copy-in stream) gates that group's first kernel, and its copies out
// (on the copy-out stream) wait for its last, so each group's factorization
// starts as soon as its own matrices have landed and the groups' copies and
// factorizations overlap one another.
struct HostGroupIO final : qrb::GroupHooks {
  cudaStream_t in, out;
  cudaEvent_t* landed;
  cudaEvent_t* factored;
  const float* A_host;
  float* H_host;
  float* tau_host;
  float* M;
  float* tau_d;
  int64_t nn;
  int n;
  int k = 0;  // pieces so far (one event pair each)

  int before(int64_t b0, int64_t b1, cudaStream_t gs) override {
    if (k >= kMaxChunks) return QRB_ERR_UNSUPPORTED;
    const size_t bytes = (size_t)(b1 - b0) * nn * sizeof(float);
    if (cudaMemcpyAsync(M + b0 * nn, A_host + b0 * nn, bytes, cudaMemcpyHostToDevice, in) !=
            cudaSuccess ||
        cudaEventRecord(landed[k], in) != cudaSuccess ||
        cudaStreamWaitEvent(gs, landed[k], 0) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    return QRB_OK;
  }
  int after(int64_t b0, int64_t b1, cudaStream_t gs) override {
    const size_t mbytes = (size_t)(b1 - b0) * nn * sizeof(float);
    const size_t tbytes = (size_t)(b1 - b0) * n * sizeof(float);
    const int e = k++;
    if (cudaEventRecord(factored[e], gs) != cudaSuccess ||
        cudaStreamWaitEvent(out, factored[e], 0) != cudaSuccess ||
        cudaMemcpyAsync(H_host + b0 * nn, M + b0 * nn, mbytes, cudaMemcpyDeviceToHost, out) !=
            cudaSuccess ||
        cudaMemcpyAsync(tau_host + b0 * n, tau_d + b0 * n, tbytes, cudaMemcpyDeviceToHost,
                        out) != cudaSuccess)
      return QRB_ERR_LAUNCH;
    return QRB_OK;
  }
};

struct HostPipe {
  std::mutex mu;
  cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
  cudaEvent_t fork = nullptr, done_in = nullptr, done_comp = nullptr, done_out = nullptr;
  cudaEvent_t landed[kMaxChunks] = {};
  cudaEvent_t factored[kMaxChunks] = {};
  bool ok = false;
};

constexpr int kMaxDevices = 64;
HostPipe g_pipe[kMaxDevices];
std::once_flag g_pipe_once[kMaxDevices];

HostPipe* host_pipe() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  HostPipe* p = &g_pipe[dev];
  std::call_once(g_pipe_once[dev], [p] {
    const unsigned ef = cudaEventDisableTiming;
    bool ok = cudaStreamCreateWithFlags(&p->in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->comp, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&p->fork, ef) == cudaSuccess &&
              cudaEventCreateWithFlags(&p->done_in, ef) == cudaSuccess &&
              cudaEventCreateWithFlags(&p->done_comp, ef) == cudaSuccess &&
              cudaEventCreateWithFlags(&p->done_out, ef) == cudaSuccess;
    for (int c = 0; c < kMaxChunks && ok; ++c)
      ok = cudaEventCreateWithFlags(&p->landed[c], ef) == cudaSuccess &&
           cudaEventCreateWithFlags(&p->factored[c], ef) == cudaSuccess;
    p->ok = ok;
  });
  return p->ok ? p : nullptr;
}

}  // namespace

namespace qrb {
int64_t host_last_path() { return g_last_path.load(); }
}  // namespace qrb

extern "C" {

size_t qrb_host_workspace_bytes(int64_t batch, int32_t n) {
  if (batch <= 0 || n <= 0 || n > qrb::kMaxN) return 0;
  const size_t mats = (size_t)batch * n * n * sizeof(float);
  const size_t taus = (size_t)batch * n * sizeof(float);
  return align_up(mats) + align_up(taus) + qrb_workspace_bytes(batch, n);
}

int qrb_geqrf_f32_host(const float* A_host, float* H_host, float* tau_host, int64_t batch,
                       int32_t n, void* workspace, size_t workspace_bytes, int32_t chunks,
                       void* stream) {
  if (batch < 0 || n < 0 || chunks < 0 || chunks > kMaxChunks) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB_OK;
  if (!A_host || !H_host || !tau_host) return QRB_ERR_INVALID_ARG;
  if (n > qrb::kMaxN) return QRB_ERR_UNSUPPORTED;
  const size_t need = qrb_host_workspace_bytes(batch, n);
  if (workspace == nullptr || workspace_bytes < need) return QRB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0) return QRB_ERR_INVALID_ARG;
  if (qrb::take_injected_failure_any()) return QRB_ERR_INJECTED;

  const int64_t nn = (int64_t)n * n;
  const size_t all_m = (size_t)batch * nn * sizeof(float);
  const size_t all_t = (size_t)batch * n * sizeof(float);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Which operands the fused kernel reaches in host memory (n <= 32 only, and
  // only where the mapping checks pass; anything else is copied).
  const int mode = n <= qrb::kFusedMaxN ? qrb::host_direct_mode() : 0;
  float* dt = mode != 0 ? static_cast<float*>(mapped_view(tau_host, all_t)) : nullptr;
  float* dH = (dt && (mode == 1 || mode == 2)) ? static_cast<float*>(mapped_view(H_host, all_m))
                                               : nullptr;
  const float* dA = (dH && mode == 1) ? static_cast<const float*>(mapped_view(A_host, all_m))
                                      : nullptr;
  if (dA != nullptr) {  // one launch over host memory, no copies
    g_last_path.store(1);
    return qrb::finish_call(qrb::launch_fused_small(dA, nn, n, dH, dt, batch, n, s,
                                                    qrb::HostMem::kAll,
                                                    qrb::host_direct_blocks()),
                            s);
  }
  const qrb::HostMem where = dH ? qrb::HostMem::kOutputs
                                : (dt ? qrb::HostMem::kTau : qrb::HostMem::kNone);
  g_last_path.store(where == qrb::HostMem::kOutputs ? 2 : (where == qrb::HostMem::kTau ? 3 : 0));

  // Chunk plan: nch pieces, equal or with weights 1, 2, .., 2, 1 so that the
  // first copy in and the last copy out (which nothing overlaps) are short.
  int64_t nch = chunks != 0 ? chunks : (n <= 64 ? kAutoChunksSmall : kAutoChunksLarge);
  if (nch < 1) nch = 1;
  if (nch > kMaxChunks) nch = kMaxChunks;
  if (nch > batch) nch = batch;
  int64_t bounds[kMaxChunks + 1];
  {
    int64_t wsum = 0, wacc = 0;
    const bool ramp = qrb::host_ramp();
    for (int64_t c = 0; c < nch; ++c) wsum += ramp ? 1 + (c < nch - 1 - c ? c : nch - 1 - c) : 1;
    bounds[0] = 0;
    for (int64_t c = 0; c < nch; ++c) {
      wacc += ramp ? 1 + (c < nch - 1 - c ? c : nch - 1 - c) : 1;
      bounds[c + 1] = batch * wacc / wsum;
    }
  }

  char* base = static_cast<char*>(workspace);
  float* M = reinterpret_cast<float*>(base);  // A in, H out, in place
  float* tau_d = reinterpret_cast<float*>(base + align_up((size_t)batch * nn * sizeof(float)));
  float* T = reinterpret_cast<float*>(reinterpret_cast<char*>(tau_d) +
                                      align_up((size_t)batch * n * sizeof(float)));

  // one chunk's factors at a time (the chunks run in order on one stream;
  // the group pipeline runs one call over the whole batch)
  const qrb::FactorScratch fs = qrb::factor_scratch(T, qrb_workspace_bytes(batch, n), batch, n);
  HostPipe* p = host_pipe();
  if (p == nullptr) return QRB_ERR_DEVICE;
  int rc = QRB_OK;
  {
    std::lock_guard<std::mutex> lock(p->mu);
    if (cudaEventRecord(p->fork, s) != cudaSuccess) return QRB_ERR_LAUNCH;
    for (cudaStream_t st : {p->in, p->comp, p->out})
      if (cudaStreamWaitEvent(st, p->fork, 0) != cudaSuccess) return QRB_ERR_LAUNCH;
    // Blocked route with the automatic depth: the route's batch groups are
    // the pieces (one factorization call, each group gated by its own copy).
    const qrb::Plan plan = qrb::make_plan(batch, n, fs);
    const bool by_group = chunks == 0 && where == qrb::HostMem::kNone &&
                          plan.route == qrb::kRouteBlocked;
    if (by_group) {
      HostGroupIO io;
      io.in = p->in;
      io.out = p->out;
      io.landed = p->landed;
      io.factored = p->factored;
      io.A_host = A_host;
      io.H_host = H_host;
      io.tau_host = tau_host;
      io.M = M;
      io.tau_d = tau_d;
      io.nn = nn;
      io.n = n;
      // Finer pieces where the route is throughput-bound (no look-ahead):
      // they start sooner after their copies (measured on B200: 39.5k vs
      // 30.1k matrices/s end to end at 640 x 512^2 with 8 groups instead of
      // 2). With the look-ahead each group is a latency chain and more of
      // them only lengthen the tail (224 vs 285 matrices/s at 8 x 4096^2).
      io.min_groups = plan.lookahead ? 0 : qrb::host_groups();
      rc = qrb::geqrf_enqueue(M, nn, n, M, tau_d, fs, batch, n, p->comp, &io);
      g_last_path.store(4);
    }
    for (int64_t c = 0; c < nch && rc == QRB_OK && !by_group; ++c) {
      const int64_t b0 = bounds[c], cnt = bounds[c + 1] - bounds[c];
      if (cnt <= 0) continue;
      float* Mc = M + b0 * nn;
      float* tc = tau_d + b0 * n;
      const size_t mbytes = (size_t)cnt * nn * sizeof(float);
      const size_t tbytes = (size_t)cnt * n * sizeof(float);
      if (cudaMemcpyAsync(Mc, A_host + b0 * nn, mbytes, cudaMemcpyHostToDevice, p->in) !=
              cudaSuccess ||
          cudaEventRecord(p->landed[c], p->in) != cudaSuccess ||
          cudaStreamWaitEvent(p->comp, p->landed[c], 0) != cudaSuccess) {
        rc = QRB_ERR_LAUNCH;
        break;
      }
      if (where == qrb::HostMem::kOutputs) {  // the kernel writes H and tau to host memory
        rc = qrb::launch_fused_small(Mc, nn, n, dH + b0 * nn, dt + b0 * n, cnt, n, p->comp, where);
        continue;
      }
      rc = where == qrb::HostMem::kTau
               ? qrb::launch_fused_small(Mc, nn, n, Mc, dt + b0 * n, cnt, n, p->comp, where)
               : qrb::geqrf_enqueue(Mc, nn, n, Mc, tc, fs, cnt, n, p->comp);
      if (rc != QRB_OK) break;
      if (cudaEventRecord(p->factored[c], p->comp) != cudaSuccess ||
          cudaStreamWaitEvent(p->out, p->factored[c], 0) != cudaSuccess ||
          cudaMemcpyAsync(H_host + b0 * nn, Mc, mbytes, cudaMemcpyDeviceToHost, p->out) !=
              cudaSuccess ||
          (where == qrb::HostMem::kNone &&
           cudaMemcpyAsync(tau_host + b0 * n, tc, tbytes, cudaMemcpyDeviceToHost, p->out) !=
               cudaSuccess)) {
        rc = QRB_ERR_LAUNCH;
        break;
      }
    }
    // Join every stage back into the caller's stream, also after an error, so
    // that nothing the call enqueued outlives the caller's view of it.
    const bool joined = cudaEventRecord(p->done_in, p->in) == cudaSuccess &&
                        cudaEventRecord(p->done_comp, p->comp) == cudaSuccess &&
                        cudaEventRecord(p->done_out, p->out) == cudaSuccess &&
                        cudaStreamWaitEvent(s, p->done_in, 0) == cudaSuccess &&
                        cudaStreamWaitEvent(s, p->done_comp, 0) == cudaSuccess &&
                        cudaStreamWaitEvent(s, p->done_out, 0) == cudaSuccess;
    if (!joined && rc == QRB_OK) rc = QRB_ERR_LAUNCH;
  }
  return qrb::finish_call(rc, s);
}

}  // extern "C"

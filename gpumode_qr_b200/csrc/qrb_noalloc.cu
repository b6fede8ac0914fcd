// qrb_geqrf_f32_noalloc: the batched QR for callers that cannot allocate
// device memory.
//
// Some callers have no way to obtain device scratch: code running inside a
// fixed memory budget where every byte was reserved up front, plugins whose
// host application owns the only allocator, or runtimes that forbid
// cudaMalloc once they have started. qrb_geqrf_f32 needs caller-provided
// workspace for n > 32 (one 32 x 32 T factor per matrix, rewritten every panel
// step); this entry point instead uses a fixed array that is part of the
// library image itself, so it allocates nothing: no cudaMalloc, no cudaFree,
// no allocating library routine.
//
// The array costs every GPU that loads this library kNoAllocScratchBytes of
// device memory until the process exits. Its size caps the batch: for n > 32
// at most kNoAllocMaxBatch matrices per call (n <= 32 needs no scratch at all).
// All calls, on all streams of a device, share the one array, and it keeps
// what the last call left in it. Nothing in it has to start at zero: the panel
// kernel writes every element of a matrix's T block before the trailing
// update reads it. Two calls whose work overlaps on the GPU (different streams
// without ordering between them) race on the array and give wrong results;
// order them, or use qrb_geqrf_f32 with separate workspaces.
//
// The device address of the array is looked up once per device, by the first
// call made on that device (cudaGetSymbolAddress with that device current); a
// lookup that fails is retried by the next call. A
// host-side use of the array's name would only be a host stand-in, never the
// device address, so only the looked-up pointer is ever handed to kernels.
// Make that first call before any stream capture begins.
#include <mutex>

#include "qrb_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int64_t kTBytesPerMatrix = int64_t(qrb::kPanelW) * qrb::kPanelW * sizeof(float);
constexpr int64_t kNoAllocMaxBatch = int64_t(kNoAllocScratchBytes) / kTBytesPerMatrix;  // 1024

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_lookup_mu;
void* g_scratch_ptr[kMaxDevices] = {};  // set only after a successful lookup

// Device address of the scratch array on the current device, looked up by the
// first call on that device that succeeds in doing so; a failed lookup (for
// example one attempted during a stream capture) is not remembered, its CUDA
// error is cleared, and the next call tries again. nullptr with *status set
// on failure.
void* scratch_for_current_device(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = QRB_ERR_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_lookup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      *status = QRB_ERR_DEVICE;
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  *status = QRB_OK;
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int qrb_geqrf_f32_noalloc(const float* A, int64_t strideA_b,
                                     int64_t strideA_row, float* H, float* tau,
                                     int64_t batch, int32_t n, void* stream) {
  if (batch < 0 || n < 0) return QRB_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB_OK;
  qrb::NoGraphScope eager;  // no graph instantiation: it may allocate device memory
  if (n <= qrb::kFusedMaxN)  // the small-n kernel uses no scratch
    return qrb_geqrf_f32(A, strideA_b, strideA_row, H, tau, batch, n, nullptr, 0, stream);
  if (batch > kNoAllocMaxBatch) return QRB_ERR_UNSUPPORTED;
  int status = QRB_OK;
  void* scratch = scratch_for_current_device(&status);
  if (scratch == nullptr) return status;
  return qrb_geqrf_f32(A, strideA_b, strideA_row, H, tau, batch, n, scratch,
                       kNoAllocScratchBytes, stream);
}

// solattn_sol_forward_noalloc: the all-in SOL forward for callers that cannot allocate device
// memory.  Its scratch (pooled K/V/Q means, key moments, thresholds and the status word) lives
// in one fixed, file-scope device array instead of a caller-provided workspace.
//
// Why: some callers of this library have no way to obtain device memory at call time - for
// example a plugin loaded into a host program that owns all device memory through its own
// pool and forbids direct cudaMalloc, or a latency-critical loop where the implicit
// synchronisation of cudaMalloc/cudaFree is not acceptable.  They can still pass their inputs
// and outputs, and this entry point needs nothing else.
//
// Cost and limits:
//   - every GPU that loads libsolattn.so holds kNoAllocScratchBytes (32 MiB) of device memory
//     for this array until the process exits;
//   - problems whose workspace (solattn_workspace_layout) exceeds that size are rejected with
//     SOLATTN_ERR_TOO_LARGE before any GPU work is enqueued;
//   - all calls on a device share the one array, and it keeps the previous call's contents:
//     the status word is cleared at the start of every call and every other byte that a call
//     reads is written by the same call first, but two calls that overlap on the GPU (issued
//     on different streams without ordering, or from different host threads) race on it;
//   - the first call on each device looks the array's device address up with
//     cudaGetSymbolAddress (with that device current) and caches it; make that first call
//     before any stream capture begins.  Later calls on a stream that is not capturing look it
//     up again (cheap, no allocation), so the cache follows a cudaDeviceReset; a call made
//     while its stream is capturing uses the cached address.
//   - device-side errors of a call (a gather index outside its tensor, a bounded wait that ran
//     out) go to the status word at offset 0 of the array: solattn_noalloc_read_status reads
//     and clears it, solattn_noalloc_scratch_address gives its device address for an
//     asynchronous copy (solattn_status_to_host).
#include <mutex>

#include "../../include/solattn.h"
#include "common.cuh"

namespace solattn {
int check_shapes(int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D);  // capi.cu
}  // namespace solattn

namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(32) << 20;
constexpr int kMaxDevices = 128;

}  // namespace

// The scratch array itself.  In host code this name is only a handle for the runtime: the
// device address is obtained below with cudaGetSymbolAddress and passed to the kernels.
static __device__ __align__(256) uint8_t g_solattn_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_solattn_scratch on the current device: looked up on the first call per
// device, and again on every call whose stream is not capturing (`refresh`).
int scratch_address(void** addr, bool refresh) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return SOLATTN_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return SOLATTN_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[dev] || refresh) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_solattn_scratch);
    if (err != cudaSuccess || p == nullptr) return SOLATTN_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  return SOLATTN_OK;
}

}  // namespace

extern "C" {

int64_t solattn_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int solattn_sol_forward_noalloc(const void* q, const void* k, const void* v, int64_t B,
                                int64_t Tq, int64_t Tk, int64_t H, int64_t D, int64_t q_sB,
                                int64_t q_sT, int64_t q_sH, int64_t k_sB, int64_t k_sT,
                                int64_t k_sH, int64_t v_sB, int64_t v_sT, int64_t v_sH,
                                const int64_t* q_idx, const int64_t* kv_idx, int64_t idx_rows,
                                const uint8_t* protect, float scale, float beta, int local,
                                int kv_sink_blocks, int q_sink_blocks, void* out,
                                int32_t* counts, void* stream) {
  // The same code as solattn_sol_forward for a shape it rejects.
  const int shape_rc = solattn::check_shapes(B, Tq, Tk, H, D);
  if (shape_rc != SOLATTN_OK) return shape_rc;
  const int64_t need = solattn_workspace_layout(B, Tq, Tk, H, D, nullptr, nullptr, nullptr,
                                                nullptr, nullptr, nullptr, nullptr, nullptr);
  if (need <= 0) return SOLATTN_ERR_ARG;
  if (need > kNoAllocScratchBytes) return SOLATTN_ERR_TOO_LARGE;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &capture) != cudaSuccess)
    return SOLATTN_ERR_CUDA;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch, capture == cudaStreamCaptureStatusNone);
  if (rc != SOLATTN_OK) return rc;
  return solattn_sol_forward(q, k, v, B, Tq, Tk, H, D, q_sB, q_sT, q_sH, k_sB, k_sT, k_sH, v_sB,
                             v_sT, v_sH, q_idx, kv_idx, idx_rows, protect, scale, beta, local,
                             kv_sink_blocks, q_sink_blocks, scratch, kNoAllocScratchBytes, out,
                             counts, stream);
}

int solattn_noalloc_scratch_address(void** address) {
  if (!address) return SOLATTN_ERR_ARG;
  return scratch_address(address, true);
}

int solattn_noalloc_read_status(int32_t* value, void* stream) {
  if (!value) return SOLATTN_ERR_ARG;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch, true);
  if (rc != SOLATTN_OK) return rc;
  // The status word is the first word of the array (workspace offset 0).
  return solattn_read_status(static_cast<int32_t*>(scratch), value, stream);
}

}  // extern "C"

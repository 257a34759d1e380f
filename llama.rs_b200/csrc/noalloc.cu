// noalloc.cu -- lrs_matvec_noalloc: a matvec that allocates no memory.
//
// lrs_matvec stages the caller's host vectors through device buffers that the
// backend allocates with cudaMalloc on first use (and grows when a larger
// matrix comes along).  Some callers cannot allow that: a host engine that
// hands the library a fixed device-memory budget at start-up and forbids
// allocation afterwards, or one that must not let a call trigger cudaMalloc's
// implicit device-wide synchronization in the middle of its own stream work.
// This entry point serves them: its device staging lives in one file-scope
// __device__ array of fixed size (kScratchBytes below), which every GPU that
// loads the library holds until the process exits.
//
// Properties a caller must know:
// * The first call on a device looks up that device's address of the array
//   (cudaGetSymbolAddress, with the device current) and caches it.  Make that
//   first call before any stream capture is started.  The cached address
//   assumes the device's primary context lives as long as the process (no
//   cudaDeviceReset while the library is loaded).
// * Every call on a device shares the one array, which keeps the previous
//   call's contents; calls whose GPU work overlaps in time race with each
//   other.  The call is synchronous, so calls from one host thread never
//   overlap; calls from several threads (or several backends on one device)
//   must be serialized by the caller.
// * Limits: cols <= kMaxCols (65536) and rows <= kMaxRows (262144); larger
//   matrices are rejected with LRS_ERR_INVALID.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/llamars.h"
#include "common.h"
#include "gemv.cuh"
#include "internal.h"

namespace {

constexpr size_t kMaxCols = 65536;
constexpr size_t kMaxRows = 262144;
constexpr size_t kXOffset = 0;
constexpr size_t kYOffset = kMaxCols * sizeof(float);
constexpr size_t kErrOffset = kYOffset + kMaxRows * sizeof(float);
constexpr size_t kScratchBytes = kErrOffset + 256;  // 1.25 MiB + 256 B

// The scratch: [x: kMaxCols floats][y: kMaxRows floats][error word].
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
int32_t scratch_for(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return lrs::fail(LRS_ERR_INVALID, "device ordinal too large");
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return lrs::fail(LRS_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") +
                                         cudaGetErrorString(e));
    g_scratch_ptr[device] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_ptr[device];
  return LRS_OK;
}

}  // namespace

#define NOALLOC_CUDA(call)                                                               \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return lrs::fail(LRS_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

extern "C" lrs_status lrs_matvec_noalloc(lrs_backend* be, const lrs_tensor* w, const float* in,
                                         size_t n_in, float* out, size_t n_out) try {
  if (!be || !w || !in || !out) return lrs::fail(LRS_ERR_INVALID, "null argument");
  if (n_in != (size_t)w->t.cols)
    return lrs::fail(LRS_ERR_INVALID, "matvec input mismatch: got " + std::to_string(n_in) +
                                          ", expected " + std::to_string(w->t.cols));
  if (n_out != (size_t)w->t.rows)
    return lrs::fail(LRS_ERR_INVALID, "matvec output mismatch: got " + std::to_string(n_out) +
                                          ", expected " + std::to_string(w->t.rows));
  if (n_in > kMaxCols || n_out > kMaxRows)
    return lrs::fail(LRS_ERR_INVALID,
                     "lrs_matvec_noalloc: matrix " + std::to_string(n_out) + " x " +
                         std::to_string(n_in) + " exceeds the fixed scratch (cols <= " +
                         std::to_string(kMaxCols) + ", rows <= " + std::to_string(kMaxRows) + ")");
  NOALLOC_CUDA(cudaSetDevice(be->device));
  unsigned char* base = nullptr;
  int32_t rc = scratch_for(be->device, &base);
  if (rc) return rc;
  float* dx = reinterpret_cast<float*>(base + kXOffset);
  float* dy = reinterpret_cast<float*>(base + kYOffset);
  int* derr = reinterpret_cast<int*>(base + kErrOffset);

  lrs::GemvMat m{};
  m.w = w->t.d;
  m.type = w->t.type;
  m.rows = w->t.rows;
  m.cols = w->t.cols;
  m.out = dy;
  m.out_ld = w->t.rows;
  lrs::GemvParams p;
  if ((rc = lrs::gemv_plan(&p, &m, 1, lrs::EPI_STORE, 1))) return rc;
  p.x = dx;
  p.x_ld = w->t.cols;
  p.error_flag = derr;
  cudaStream_t st = be->stream;
  NOALLOC_CUDA(cudaMemsetAsync(derr, 0, sizeof(int), st));  // the error word must start at zero
  NOALLOC_CUDA(cudaMemcpyAsync(dx, in, n_in * sizeof(float), cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(lrs::gemv_launch(p, st, be->sms, false));
  NOALLOC_CUDA(cudaMemcpyAsync(out, dy, n_out * sizeof(float), cudaMemcpyDeviceToHost, st));
  int herr = 0;
  NOALLOC_CUDA(cudaMemcpyAsync(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
  NOALLOC_CUDA(cudaStreamSynchronize(st));
  if (herr) return lrs::fail(LRS_ERR_DEVICE_TIMEOUT, "a bounded device-side wait gave up");
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

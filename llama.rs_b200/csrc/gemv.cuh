// gemv.cuh -- quantized matrix-vector products (decode GEMV) for sm_100a.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace lrs {

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for `kernel`, once per
// device: the attribute belongs to the current device's context.  `done`
// holds one bit per device ordinal (static per kernel at the call site).
inline cudaError_t set_smem_once(std::atomic<uint64_t>& done, const void* kernel, int smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

enum GemvEpilogue : int {
  EPI_STORE = 0,   // out[b][r] = y (+ bias[r])           LinearLayer::forward, src/model.rs:33-46
  EPI_ADD = 1,     // out[b][r] += y                      residual adds, src/model.rs:236-238, 258-260
  EPI_SWIGLU = 2,  // out[b][r] = silu(y_gate) * y_up     src/model.rs:251-254
  EPI_ARGMAX = 3   // logits (optional) + greedy argmax    src/engine.rs:233-241
};

constexpr int kGemvThreads = 256;
constexpr int kGemvMaxSeg = 3;
constexpr int kGemvMaxStages = 8;

// One output segment: rows of one matrix (or of a gate/up pair for EPI_SWIGLU).
struct GemvSeg {
  const uint8_t* w;   // device block bytes, [rows][rb]
  const uint8_t* w2;  // second matrix of a pair (EPI_SWIGLU), same type and shape
  const float* bias;  // [rows] or null
  float* out;         // out[b * out_ld + r]
  int type, rows, rb, rt, tiles, tile0, out_ld;
  int rr;  // batch-1 kernel: rows per work item (x reuse factor); rt % rr == 0
};

struct GemvParams {
  GemvSeg seg[kGemvMaxSeg];
  int nseg, total_tiles, cols, epi;
  const float* x;    // x[b * x_ld + c]
  int x_ld, batch;
  const float* norm_w;  // fused RMSNorm of x (batch 1 only) or null
  float norm_eps;
  unsigned long long* argmax_keys;  // [batch], EPI_ARGMAX
  int argmax_base;  // added to the row index in the argmax key (batched paths; 0 otherwise)
  int stage_bytes, stages, x_in_smem;
  int fast;  // 1: batch-1 direct-load kernel (int8-split x, dp4a)
  int wpg;   // batch-1 kernel: warps sharing one row group (long rows split across warps)
  int* error_flag;
  // Device scratch for the batched tensor-core paths (gemm_mma.cu, gemm_tc.cu);
  // when null or too small, batches run on the CUDA-core kernel.
  void* scratch;
  size_t scratch_bytes;
};

// Host helpers (gemv.cu).
struct GemvMat {
  const uint8_t* w;
  const uint8_t* w2;
  const float* bias;
  float* out;
  uint32_t type;
  int rows, cols, out_ld;
};
// Fills the tiling of `params` for the given segments; returns 0 or an lrs status.
int gemv_plan(GemvParams* p, const GemvMat* mats, int nmat, int epi, int batch);
// Launches on `stream` (with programmatic dependent launch when pdl != 0).
cudaError_t gemv_launch(const GemvParams& p, cudaStream_t stream, int num_sms, bool pdl);

// Batched (2..64) quantized matmul on the tensor cores with mma.sync (gemm_mma.cu).
bool gemm_supported(const GemvParams& p);
size_t gemm_scratch_bytes(int batch, int max_cols, int sms);
cudaError_t gemm_launch(const GemvParams& p, void* scratch, int sms, cudaStream_t stream);
// Fixed-order sum of K-group partials [segment][pair][kgroups][batch][rows] + epilogue.
cudaError_t gemm_partials_epilogue(const GemvParams& p, const float* const* parts, int kgroups,
                                   cudaStream_t stream);

// Batched Q4_K / Q6_K matmul on tcgen05 (gemm_tc.cu), 4..64 items.
bool gemm_tc_supported(const GemvParams& p);
size_t gemm_tc_scratch_bytes(const GemvParams& p, int sms);
cudaError_t gemm_tc_launch(const GemvParams& p, void* scratch, int sms, cudaStream_t stream);

}  // namespace lrs

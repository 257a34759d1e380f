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

// The last kScratchCounterBytes of a matmul scratch buffer are counters that
// must be zero when the buffer is allocated; kernels that use them leave them
// zero.  Scratch sizes passed in GemvParams include them.
constexpr size_t kScratchCounterBytes = 16384;

// Batched Q4_K / Q6_K matmul on tcgen05 (gemm_tc.cu), 4..64 items.  With
// LRS_TC_FUSED=1 the output step runs in the matmul kernel (gemm_tc_fused_enabled).
bool gemm_tc_supported(const GemvParams& p);
size_t gemm_tc_scratch_bytes(const GemvParams& p, int sms);
cudaError_t gemm_tc_launch(const GemvParams& p, void* scratch, int sms, cudaStream_t stream);
bool gemm_tc_fused_enabled();

// Tensor-parallel row-split projection fused with its all-reduce (the TPX
// variant of gemv_stream_kernel): every CTA stores its rows' partial sums
// into every rank's exchange buffer as its tiles finish, signals the same CTA
// index on the peers, waits for theirs, and adds all ranks' partials of its
// rows onto the output in rank order.
constexpr int kTpSigFused = 64;    // first signal word of the fused path (per rank)
constexpr int kTpMaxGrid = 1024;   // signal words per source rank
struct StreamTp {
  float* const* peer_x;   // [world] every rank's exchange buffer: [world][rows] of this call
  int* local_sig;         // this rank's signal words + kTpSigFused: [world][kTpMaxGrid]
  int* const* peer_sig;   // [world] every rank's signal words (bases)
  unsigned* counters;     // [kTpMaxGrid] this rank's launches per CTA index (zero at creation)
  int rank, world, rows;
  int plan_cols;          // the widest shard of this projection over all ranks (>= cols)
  int* error_flag;
};

// Batch-1 GEMV through a shared-memory ring of bulk copies (gemv_stream.cu),
// for one run of same-type segments planned by gemv_plan (p.fast).  Used
// instead of gemv5_kernel when LRS_GEMV_STREAM=1; with `tp` (one segment, not
// a pair) the fused tensor-parallel variant.  cudaErrorNotSupported: the plan
// does not fit (the caller uses gemv5_kernel).
bool gemv_stream_enabled();
cudaError_t gemv_stream_launch(const GemvParams& p, cudaStream_t stream, int num_sms, bool pdl,
                               const StreamTp* tp = nullptr);

}  // namespace lrs

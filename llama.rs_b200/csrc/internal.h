// internal.h -- handle types shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

struct lrs_backend {
  int device = 0;
  int sms = 148;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  float* d_x = nullptr;
  float* d_y = nullptr;
  size_t x_cap = 0, y_cap = 0;
  void* d_scratch = nullptr;  // batched tensor-core matmul scratch
  size_t scratch_cap = 0;
  uint32_t* d_sample = nullptr;  // sampler: [token, recent window...]
  size_t sample_cap = 0;
};

struct DevTensor {
  uint8_t* d = nullptr;
  size_t nbytes = 0;
  int rows = 0, cols = 0;
  uint32_t type = 0;
};

struct lrs_tensor {
  lrs_backend* be = nullptr;
  DevTensor t;
};

namespace lrs {
// F16 / BF16 (type) values at src to f32 (exact), on stream st (quantize_dev.cu).
cudaError_t launch_widen(const void* src, uint32_t type, size_t n, float* dst, cudaStream_t st);
}  // namespace lrs

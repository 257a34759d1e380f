// quantize_dev.cu -- the load-time GGML encoders on the device, so F32/F16/
// BF16 weights of the 7B/32B models encode in HBM instead of on the host
// (maybe_quantize, src/loader.rs:406-447).  One thread
// encodes one block with the same code as the host (encoders.h); this file is
// compiled with --fmad=false so every f32 operation rounds like the
// reference's, and the bytes equal lrs_quantize_matrix's.
#include <cuda_runtime.h>

#include "../../include/llamars_synth.h"
#include "common.h"
#include "encoders.h"
#include "internal.h"

namespace lrs {
namespace {

__global__ void __launch_bounds__(128)
    quantize_kernel(uint32_t t, const float* v, size_t rows, size_t cols, uint32_t bv, uint32_t bb,
                    uint8_t* out) {
  const size_t per_row = cols / bv;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const size_t r = idx / per_row, b = idx % per_row;
  const float* x = v + r * cols + b * bv;
  uint8_t* o = out + r * (per_row * bb) + b * bb;
  switch (t) {
    case LRS_GGML_F32: memcpy(o, x, 4); break;
    case LRS_GGML_F16: enc::put16(o, enc::f32_to_f16_bits(x[0])); break;
    case LRS_GGML_BF16: enc::put16(o, enc::f32_to_bf16_bits(x[0])); break;
    case LRS_GGML_Q4_0: enc::block_q4_0(x, o); break;
    case LRS_GGML_Q4_1: enc::block_q41_q51(x, o, false); break;
    case LRS_GGML_Q5_0: enc::block_q5_0(x, o); break;
    case LRS_GGML_Q5_1: enc::block_q41_q51(x, o, true); break;
    case LRS_GGML_Q8_0: enc::block_q8_0(x, o); break;
    case LRS_GGML_Q4_K: enc::block_q4k(x, o); break;
    case LRS_GGML_Q5_K: enc::block_q5k(x, o); break;
    case LRS_GGML_Q6_K: enc::block_q6k(x, o); break;
  }
}

// F16 / BF16 values to f32 (exact widening: QuantTensor::to_vec_f32).
__global__ void widen_kernel(const uint16_t* src, uint32_t t, size_t n, float* dst) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint16_t h = src[i];
  dst[i] = t == LRS_GGML_BF16 ? __uint_as_float((uint32_t)h << 16) : enc::f16_bits_to_f32(h);
}

}  // namespace

cudaError_t launch_widen(const void* src, uint32_t type, size_t n, float* dst, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  widen_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint16_t*>(src), type,
                                                              n, dst);
  return cudaGetLastError();
}

}  // namespace lrs

using namespace lrs;

extern "C" lrs_status lrs_quantize_matrix_device(lrs_backend* be, uint32_t t, const float* d_values,
                                                 size_t rows, size_t cols, void* d_out,
                                                 size_t out_cap, uint32_t* out_type,
                                                 size_t* out_len) try {
  if (!be || !d_values || !d_out) return fail(LRS_ERR_INVALID, "null argument");
  uint32_t bv, bb;
  if (!type_geometry(t, &bv, &bb)) return fail(LRS_ERR_UNSUPPORTED, "unsupported GGML type");
  const uint32_t e = enc::effective_type(t, cols);
  const size_t need = lrs_quantized_size(t, rows, cols);
  if (out_cap < need) return fail(LRS_ERR_INVALID, "output buffer too small");
  type_geometry(e, &bv, &bb);
  const size_t blocks = rows * (cols / bv);
  cudaError_t err = cudaSetDevice(be->device);
  if (err == cudaSuccess && blocks) {
    quantize_kernel<<<(unsigned)((blocks + 127) / 128), 128, 0, be->stream>>>(
        e, d_values, rows, cols, bv, bb, static_cast<uint8_t*>(d_out));
    err = cudaGetLastError();
  }
  if (err == cudaSuccess) err = cudaStreamSynchronize(be->stream);
  if (err != cudaSuccess) return fail(LRS_ERR_CUDA, cudaGetErrorString(err));
  if (out_type) *out_type = e;
  if (out_len) *out_len = need;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

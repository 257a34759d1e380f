// gemv.cu -- quantized GEMV for decode (sm_100a).
//
// Replaces CpuBackend::matvec (src/backend.rs:143-162) and the per-row dots
// dot_row_scalar / dot_row_avx2 (src/quant.rs:458-648, src/simd.rs:50-299).
//
// Design (memory-bound; one pass over the weight bytes in HBM):
// * The matrix is split into tiles of `rt` consecutive rows.  A CTA walks its
//   tiles with a grid stride; each tile's block bytes (still in the native GGML
//   layout) are brought into shared memory with one or two cp.async.bulk (TMA)
//   copies completing on an mbarrier, `stages` tiles in flight per CTA.  The
//   weights do not depend on the previous kernel, so the first copies are
//   issued before griddepcontrol.wait (programmatic dependent launch).
// * The input vector (batch 1) is staged once per CTA in shared memory with a
//   4-float pad per 32 columns (conflict-free float4 reads), optionally through
//   a fused RMSNorm (src/model.rs:65-73).  Larger batches read x through L1.
// * Thread t owns row (t % rt) of the tile and pieces t/rt, t/rt + 256/rt, ...
//   of that row; every piece is decoded exactly (value_at) in registers and
//   multiplied into an f32 accumulator; per-row partials are reduced with warp
//   shuffles and one shared-memory pass.
// * Epilogues fuse the bias add, residual add, SwiGLU and greedy argmax.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.h"
#include "device_common.cuh"
#include "gemv.cuh"
#include "gemv_fast.cuh"

namespace lrs {
namespace {

constexpr int kWarps = kGemvThreads / 32;

__host__ __device__ inline int round16(int v) { return (v + 15) & ~15; }
__host__ __device__ inline int red_floats(int nb) { return kWarps * 32 * nb * 2; }
__host__ __device__ inline int stage_offset(int nb) {
  return (64 + red_floats(nb) * 4 + 127) & ~127;
}
__host__ __device__ inline int xs_index(int c) { return c + (c >> 5) * 4; }

// Selects the segment of `tile` with constant indices (a dynamic index into the
// kernel parameters would force a copy to local memory).
__device__ __forceinline__ GemvSeg find_seg(const GemvParams& p, int tile) {
  if (p.nseg > 2 && tile >= p.seg[2].tile0) return p.seg[2];
  if (p.nseg > 1 && tile >= p.seg[1].tile0) return p.seg[1];
  return p.seg[0];
}

// Queues the bulk copies of `tile` into `stage`.
__device__ void issue_tile(const GemvParams& p, int tile, uint8_t* stage, uint64_t* bar,
                           uint64_t policy) {
  const GemvSeg s = find_seg(p, tile);
  int r0 = (tile - s.tile0) * s.rt;
  int nr = min(s.rt, s.rows - r0);
  size_t off = (size_t)r0 * s.rb;
  int mis = (int)(off & 15);
  int size = round16(mis + nr * s.rb);
  bool pair = p.epi == EPI_SWIGLU;
  mbar_expect_tx(bar, (uint32_t)(pair ? 2 * size : size));
  tma_load_1d(stage, s.w + off - mis, (uint32_t)size, bar, policy);
  if (pair) tma_load_1d(stage + size, s.w2 + off - mis, (uint32_t)size, bar, policy);
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int o) {
  uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, o);
  uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), o);
  return ((unsigned long long)hi << 32) | lo;
}

template <int NB>
__device__ __forceinline__ void load_x8(const GemvParams& p, const float* xs, int b0, int col,
                                        float (*xv)[8]) {
  if (NB == 1 && p.x_in_smem) {
    const float4* q = reinterpret_cast<const float4*>(xs + xs_index(col));
    float4 a = q[0], b = q[1];
    xv[0][0] = a.x, xv[0][1] = a.y, xv[0][2] = a.z, xv[0][3] = a.w;
    xv[0][4] = b.x, xv[0][5] = b.y, xv[0][6] = b.z, xv[0][7] = b.w;
  } else {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      if (b0 + b < p.batch) {
        const float4* q = reinterpret_cast<const float4*>(p.x + (size_t)(b0 + b) * p.x_ld + col);
        float4 a = __ldg(q), c = __ldg(q + 1);
        xv[b][0] = a.x, xv[b][1] = a.y, xv[b][2] = a.z, xv[b][3] = a.w;
        xv[b][4] = c.x, xv[b][5] = c.y, xv[b][6] = c.z, xv[b][7] = c.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) xv[b][i] = 0.0f;
      }
    }
  }
}

template <int T, int NB, bool PAIR>
__device__ void process_tile(const GemvParams& p, const GemvSeg& s, int tile, const uint8_t* stage,
                             const float* xs, float* red) {
  using BT = BlockTraits<T>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rt = s.rt;
  const int r0 = (tile - s.tile0) * rt;
  const int nr = min(rt, s.rows - r0);
  const size_t off = (size_t)r0 * s.rb;
  const int mis = (int)(off & 15);
  constexpr bool pair = PAIR;
  const uint8_t* st = stage + mis;
  const uint8_t* st2 = stage + round16(mis + nr * s.rb) + mis;
  const int row = tid % rt;
  const int ppr = p.cols / 32;
  const int pstep = kGemvThreads / rt;

  for (int b0 = 0; b0 < p.batch; b0 += NB) {
    float acc[NB], acc2[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = acc2[b] = 0.0f;
    if (row < nr) {
      const uint8_t* rowp = st + (size_t)row * s.rb;
      const uint8_t* rowp2 = st2 + (size_t)row * s.rb;
      for (int pc = tid / rt; pc < ppr; pc += pstep) {
        const int unit = pc / BT::kPieces, sub = pc % BT::kPieces;
        float w[32];
        decode_piece<T>(rowp + (size_t)unit * BT::kBytes, sub, w);
        float w2[PAIR ? 32 : 1];
        if constexpr (PAIR) decode_piece<T>(rowp2 + (size_t)unit * BT::kBytes, sub, w2);
        const int cbase = unit * BT::kValues;
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const int col = cbase + run_col<T>(sub, r);
          float xv[NB][8];
          load_x8<NB>(p, xs, b0, col, xv);
#pragma unroll
          for (int b = 0; b < NB; b++) {
#pragma unroll
            for (int i = 0; i < 8; i++) acc[b] = fmaf(w[r * 8 + i], xv[b][i], acc[b]);
            if constexpr (PAIR) {
#pragma unroll
              for (int i = 0; i < 8; i++) acc2[b] = fmaf(w2[r * 8 + i], xv[b][i], acc2[b]);
            }
          }
        }
      }
    }
    // Reduce lanes that own the same row (lane == row mod rt).
#pragma unroll
    for (int b = 0; b < NB; b++) {
      for (int o = 16; o >= rt; o >>= 1) {
        acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
        if (pair) acc2[b] += __shfl_xor_sync(0xffffffffu, acc2[b], o);
      }
      if (lane < rt) {
        red[(warp * 32 + lane) * NB + b] = acc[b];
        red[kWarps * 32 * NB + (warp * 32 + lane) * NB + b] = acc2[b];
      }
    }
    __syncthreads();
    if (tid < 32) {
#pragma unroll
      for (int b = 0; b < NB; b++) {
        if (b0 + b >= p.batch) break;
        float y = 0.0f, y2 = 0.0f;
        const int r = r0 + tid;
        if (tid < nr) {
          for (int wv = 0; wv < kWarps; wv++) {
            y += red[(wv * 32 + tid) * NB + b];
            if (pair) y2 += red[kWarps * 32 * NB + (wv * 32 + tid) * NB + b];
          }
          float* out = s.out ? s.out + (size_t)(b0 + b) * s.out_ld + r : nullptr;
          switch (p.epi) {
            case EPI_STORE:
              if (s.bias) y += s.bias[r];
              *out = y;
              break;
            case EPI_ADD:
              *out += y;
              break;
            case EPI_SWIGLU:
              *out = (y / (1.0f + expf(-y))) * y2;
              break;
            default:
              if (out) *out = y;
              break;
          }
        }
        if (p.epi == EPI_ARGMAX) {
          unsigned long long key = tid < nr ? argmax_pack(y, (uint32_t)r) : 0ull;
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) {
            unsigned long long other = shfl_xor_u64(key, o);
            key = other > key ? other : key;
          }
          if (tid == 0) atomicMax(&p.argmax_keys[b0 + b], key);
        }
      }
    }
    __syncthreads();
  }
}

template <int NB, bool PAIR>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + 64);
  uint8_t* stage_base = smem + stage_offset(NB);
  float* xs = reinterpret_cast<float*>(stage_base + (size_t)p.stages * p.stage_bytes);
  const int tid = threadIdx.x;

  if (tid == 0) {
    for (int s = 0; s < p.stages; s++) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t policy = evict_first_policy();
  if (tid == 0) {
    for (int s = 0; s < p.stages; s++) {
      int tile = blockIdx.x + s * gridDim.x;
      if (tile < p.total_tiles) issue_tile(p, tile, stage_base + s * p.stage_bytes, &bars[s], policy);
    }
  }
  pdl_wait();  // x / residual come from the previous kernel
  if (NB == 1 && p.x_in_smem) {
    if (p.norm_w) {
      // RMSNorm::forward, src/model.rs:65-73: x * (inv_rms * w)
      float ss = 0.0f;
      for (int c = tid; c < p.cols; c += kGemvThreads) ss = fmaf(p.x[c], p.x[c], ss);
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((tid & 31) == 0) red[tid >> 5] = ss;
      __syncthreads();
      float tot = 0.0f;
      for (int w = 0; w < kWarps; w++) tot += red[w];
      const float inv = 1.0f / sqrtf(tot / (float)p.cols + p.norm_eps);
      for (int c = tid; c < p.cols; c += kGemvThreads) xs[xs_index(c)] = p.x[c] * (inv * p.norm_w[c]);
    } else {
      for (int c = tid; c < p.cols; c += kGemvThreads) xs[xs_index(c)] = p.x[c];
    }
  }
  __syncthreads();

  int i = 0;
  for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, i++) {
    const int s = i % p.stages;
    const uint32_t parity = (uint32_t)((i / p.stages) & 1);
    if (tile + (int)gridDim.x >= p.total_tiles) pdl_launch_dependents();
    if (!mbar_wait_bounded(&bars[s], parity)) {
      if (tid == 0) {
        atomicExch(p.error_flag, LRS_ERR_DEVICE_TIMEOUT);
        for (int k = 1; k < p.stages; k++) {  // let copies already queued land
          int tk = tile + k * gridDim.x;
          if (tk >= p.total_tiles) break;
          mbar_wait_bounded(&bars[(i + k) % p.stages], (uint32_t)(((i + k) / p.stages) & 1));
        }
      }
      return;
    }
    const GemvSeg sg = find_seg(p, tile);
    const uint8_t* stage = stage_base + s * p.stage_bytes;
    switch (sg.type) {
      case LRS_GGML_F32: process_tile<LRS_GGML_F32, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_F16: process_tile<LRS_GGML_F16, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_BF16: process_tile<LRS_GGML_BF16, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q4_0: process_tile<LRS_GGML_Q4_0, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q4_1: process_tile<LRS_GGML_Q4_1, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q5_0: process_tile<LRS_GGML_Q5_0, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q5_1: process_tile<LRS_GGML_Q5_1, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q8_0: process_tile<LRS_GGML_Q8_0, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q4_K: process_tile<LRS_GGML_Q4_K, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q5_K: process_tile<LRS_GGML_Q5_K, NB, PAIR>(p, sg, tile, stage, xs, red); break;
      case LRS_GGML_Q6_K: process_tile<LRS_GGML_Q6_K, NB, PAIR>(p, sg, tile, stage, xs, red); break;
    }
    // process_tile ends with __syncthreads(): the stage is free again.
    if (tid == 0) {
      int next = tile + p.stages * gridDim.x;
      if (next < p.total_tiles) {
        fence_proxy_async();
        issue_tile(p, next, stage_base + s * p.stage_bytes, &bars[s], policy);
      }
    }
  }
}

// ---- batch-1 kernel with factored per-type dots ---------------------------
// Work item = (block of rr rows, one piece): the piece's x values are read
// from shared memory once and applied to rr rows (and to both matrices of a
// gate/up pair), which keeps shared-memory traffic within the SM's budget.
constexpr int kFastRed = kWarps * 32 * 4 * 2;  // red[warp][lane][k<4] x 2 matrices

__host__ __device__ inline int fast_stage_offset() { return (64 + kFastRed * 4 + 127) & ~127; }

template <int T, bool PAIR>
__device__ void fast_tile(const GemvParams& p, const GemvSeg& s, int tile, const uint8_t* stage,
                          const float* xs, const float* xs8, float* red) {
  using BT = BlockTraits<T>;
  constexpr int PV = fast::Piece<T>::kValues;
  constexpr int PPU = fast::pieces_per_unit<T>();
  constexpr int NRUN = PV / 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rt = s.rt, R = s.rr, nrb = rt / R;
  const int r0 = (tile - s.tile0) * rt;
  const int nr = min(rt, s.rows - r0);
  const size_t off = (size_t)r0 * s.rb;
  const int mis = (int)(off & 15);
  const uint8_t* st = stage + mis;
  const uint8_t* st2 = stage + round16(mis + nr * s.rb) + mis;
  const int rbi = tid % nrb;
  const int ppr = p.cols / PV;
  const int pstep = kGemvThreads / nrb;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int pc = tid / nrb; pc < ppr; pc += pstep) {
    const int unit = pc / PPU, sub = pc % PPU;
    float x[PV], X[NRUN];
#pragma unroll
    for (int r = 0; r < NRUN; r++) {
      const int col = unit * BT::kValues + fast::run_col<T>(sub, r);
      const float4* q = reinterpret_cast<const float4*>(xs + xs_index(col));
      const float4 a = q[0], b = q[1];
      x[8 * r + 0] = a.x, x[8 * r + 1] = a.y, x[8 * r + 2] = a.z, x[8 * r + 3] = a.w;
      x[8 * r + 4] = b.x, x[8 * r + 5] = b.y, x[8 * r + 6] = b.z, x[8 * r + 7] = b.w;
      X[r] = xs8[col >> 3];
    }
    const size_t uoff = (size_t)unit * BT::kBytes;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      if (k < R) {
        const int row = rbi * R + k;
        if (row < nr) {
          acc[k] += fast::piece_dot<T>(st + (size_t)row * s.rb + uoff, sub, x, X);
          if constexpr (PAIR)
            acc2[k] += fast::piece_dot<T>(st2 + (size_t)row * s.rb + uoff, sub, x, X);
        }
      }
    }
  }
  // Lanes with the same row block (lane == rbi mod nrb) reduce together.
#pragma unroll
  for (int k = 0; k < 4; k++) {
    if (k < R) {
      for (int o = 16; o >= nrb; o >>= 1) {
        acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
        if constexpr (PAIR) acc2[k] += __shfl_xor_sync(0xffffffffu, acc2[k], o);
      }
      if (lane < nrb) {
        red[(warp * 32 + lane) * 4 + k] = acc[k];
        if constexpr (PAIR) red[kWarps * 32 * 4 + (warp * 32 + lane) * 4 + k] = acc2[k];
      }
    }
  }
  __syncthreads();
  if (tid < 32) {
    float y = 0.0f, y2 = 0.0f;
    const int r = r0 + tid;
    if (tid < nr) {
      const int b = tid / R, k = tid % R;
      for (int wv = 0; wv < kWarps; wv++) {
        y += red[(wv * 32 + b) * 4 + k];
        if constexpr (PAIR) y2 += red[kWarps * 32 * 4 + (wv * 32 + b) * 4 + k];
      }
      float* out = s.out ? s.out + r : nullptr;
      switch (p.epi) {
        case EPI_STORE:
          if (s.bias) y += s.bias[r];
          *out = y;
          break;
        case EPI_ADD:
          *out += y;
          break;
        case EPI_SWIGLU:
          *out = (y / (1.0f + expf(-y))) * y2;
          break;
        default:
          if (out) *out = y;
          break;
      }
    }
    if (p.epi == EPI_ARGMAX) {
      unsigned long long key = tid < nr ? argmax_pack(y, (uint32_t)r) : 0ull;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        unsigned long long other = shfl_xor_u64(key, o);
        key = other > key ? other : key;
      }
      if (tid == 0) atomicMax(&p.argmax_keys[0], key);
    }
  }
  __syncthreads();
}

template <bool PAIR>
__global__ void __launch_bounds__(kGemvThreads, 1)
    gemv1_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + 64);
  uint8_t* stage_base = smem + fast_stage_offset();
  float* xs = reinterpret_cast<float*>(stage_base + (size_t)p.stages * p.stage_bytes);
  float* xs8 = xs + xs_index(p.cols) + 8;
  const int tid = threadIdx.x;

  if (tid == 0) {
    for (int s = 0; s < p.stages; s++) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t policy = evict_first_policy();
  if (tid == 0) {
    for (int s = 0; s < p.stages; s++) {
      int tile = blockIdx.x + s * gridDim.x;
      if (tile < p.total_tiles) issue_tile(p, tile, stage_base + s * p.stage_bytes, &bars[s], policy);
    }
  }
  pdl_wait();  // x / residual come from the previous kernel
  if (p.norm_w) {
    // RMSNorm::forward, src/model.rs:65-73: x * (inv_rms * w)
    float ss = 0.0f;
    for (int c = tid; c < p.cols; c += kGemvThreads) ss = fmaf(p.x[c], p.x[c], ss);
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < kWarps; w++) tot += red[w];
    const float inv = 1.0f / sqrtf(tot / (float)p.cols + p.norm_eps);
    for (int c = tid; c < p.cols; c += kGemvThreads) xs[xs_index(c)] = p.x[c] * (inv * p.norm_w[c]);
  } else {
    for (int c = tid; c < p.cols; c += kGemvThreads) xs[xs_index(c)] = p.x[c];
  }
  __syncthreads();
  for (int j = tid; j < p.cols / 8; j += kGemvThreads) {
    const float* q = xs + xs_index(j * 8);
    xs8[j] = ((q[0] + q[1]) + (q[2] + q[3])) + ((q[4] + q[5]) + (q[6] + q[7]));
  }
  __syncthreads();

  int i = 0;
  for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, i++) {
    const int s = i % p.stages;
    const uint32_t parity = (uint32_t)((i / p.stages) & 1);
    if (tile + (int)gridDim.x >= p.total_tiles) pdl_launch_dependents();
    if (!mbar_wait_bounded(&bars[s], parity)) {
      if (tid == 0) {
        atomicExch(p.error_flag, LRS_ERR_DEVICE_TIMEOUT);
        for (int k = 1; k < p.stages; k++) {  // let copies already queued land
          int tk = tile + k * gridDim.x;
          if (tk >= p.total_tiles) break;
          mbar_wait_bounded(&bars[(i + k) % p.stages], (uint32_t)(((i + k) / p.stages) & 1));
        }
      }
      return;
    }
    const GemvSeg sg = find_seg(p, tile);
    const uint8_t* stage = stage_base + s * p.stage_bytes;
    switch (sg.type) {
      case LRS_GGML_F32: fast_tile<LRS_GGML_F32, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_F16: fast_tile<LRS_GGML_F16, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_BF16: fast_tile<LRS_GGML_BF16, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q4_0: fast_tile<LRS_GGML_Q4_0, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q4_1: fast_tile<LRS_GGML_Q4_1, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q5_0: fast_tile<LRS_GGML_Q5_0, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q5_1: fast_tile<LRS_GGML_Q5_1, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q8_0: fast_tile<LRS_GGML_Q8_0, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q4_K: fast_tile<LRS_GGML_Q4_K, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q5_K: fast_tile<LRS_GGML_Q5_K, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
      case LRS_GGML_Q6_K: fast_tile<LRS_GGML_Q6_K, PAIR>(p, sg, tile, stage, xs, xs8, red); break;
    }
    if (tid == 0) {
      int next = tile + p.stages * gridDim.x;
      if (next < p.total_tiles) {
        fence_proxy_async();
        issue_tile(p, next, stage_base + s * p.stage_bytes, &bars[s], policy);
      }
    }
  }
}

int fast_piece_values(uint32_t t) {
  return (t == LRS_GGML_Q4_K || t == LRS_GGML_Q5_K) ? 64 : 32;
}

size_t fast_smem_bytes(const GemvParams& p) {
  return fast_stage_offset() + (size_t)p.stages * p.stage_bytes +
         ((size_t)xs_index(p.cols) + 8 + p.cols / 8) * 4 + 16;
}

// Resident CTAs per SM of `kernel` at `smem` bytes (cached per device, kernel, size).
int occupancy(const void* kernel, int smem) {
  struct Entry {
    int dev;
    const void* k;
    int smem, blocks;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  for (auto& c : cache)
    if (c.dev == dev && c.k == kernel && c.smem == smem) return c.blocks;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  int blocks = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kGemvThreads, smem);
  cache.push_back({dev, kernel, smem, blocks});
  return blocks;
}

int gemv_nb(int batch) { return batch == 1 ? 1 : 8; }

size_t smem_bytes(const GemvParams& p, int nb) {
  size_t s = stage_offset(nb) + (size_t)p.stages * p.stage_bytes;
  if (p.x_in_smem) s += (size_t)xs_index(p.cols) * 4 + 16;
  return s;
}

}  // namespace

int gemv_plan(GemvParams* p, const GemvMat* mats, int nmat, int epi, int batch) {
  memset(p, 0, sizeof(*p));
  if (nmat < 1 || nmat > kGemvMaxSeg) return fail(LRS_ERR_INVALID, "gemv: bad segment count");
  if (batch < 1) return fail(LRS_ERR_INVALID, "gemv: batch must be positive");
  const bool pair = epi == EPI_SWIGLU;
  const int cols = mats[0].cols;
  if (cols % 32) return fail(LRS_ERR_UNSUPPORTED, "gemv: the CUDA backend needs cols % 32 == 0");
  int need = 0;
  for (int i = 0; i < nmat; i++) {
    uint32_t bv, bb;
    if (!type_geometry(mats[i].type, &bv, &bb)) return fail(LRS_ERR_UNSUPPORTED, "gemv: bad type");
    if (mats[i].cols != cols) return fail(LRS_ERR_INVALID, "gemv: segments differ in cols");
    if (cols % (int)bv) return fail(LRS_ERR_INVALID, "gemv: cols not divisible by block size");
    int rb = (int)row_bytes(mats[i].type, cols);
    need = std::max(need, (pair ? 2 : 1) * (rb + 32));
  }
  int stage = std::max(16384, (need + 127) & ~127);
  int stages = std::max(2, std::min(kGemvMaxStages, 131072 / stage));
  p->stage_bytes = stage;
  p->stages = stages;
  int tile0 = 0;
  for (int i = 0; i < nmat; i++) {
    GemvSeg& s = p->seg[i];
    s.w = mats[i].w;
    s.w2 = mats[i].w2;
    s.bias = mats[i].bias;
    s.out = mats[i].out;
    s.type = (int)mats[i].type;
    s.rows = mats[i].rows;
    s.out_ld = mats[i].out_ld;
    s.rb = (int)row_bytes(mats[i].type, cols);
    int rt = 32;
    while (rt > 1 && (pair ? 2 : 1) * (rt * s.rb + 32) > stage) rt >>= 1;
    s.rt = rt;
    s.tiles = (s.rows + rt - 1) / rt;
    s.tile0 = tile0;
    tile0 += s.tiles;
  }
  p->nseg = nmat;
  p->total_tiles = tile0;
  p->cols = cols;
  p->epi = epi;
  p->batch = batch;
  p->x_in_smem = 0;
  if (batch == 1) {
    p->x_in_smem = 1;
    if (smem_bytes(*p, 1) > 227 * 1024) p->x_in_smem = 0;
    // Factored batch-1 kernel: per segment pick rows per item (rr, the x
    // reuse factor: 4, or 2 for a gate/up pair) and tile rows rt so that a
    // tile has >= 224 work items and fits a stage of <= 48 KiB.
    const int pf = pair ? 2 : 1;
    GemvParams q = *p;
    int fneed = 0;
    tile0 = 0;
    for (int i = 0; i < nmat; i++) {
      GemvSeg& s = q.seg[i];
      const int ppr = cols / fast_piece_values(s.type);
      int R = pair ? 2 : 4, rt = R;
      for (;;) {
        rt = R;
        while (rt < 32 && (rt / R) * ppr < 224) rt *= 2;
        while (rt > R && pf * (rt * s.rb + 32) > 48 * 1024) rt /= 2;
        if (pf * (rt * s.rb + 32) <= 48 * 1024 || R == 1) break;
        R /= 2;
      }
      s.rr = R;
      s.rt = rt;
      s.tiles = (s.rows + rt - 1) / rt;
      s.tile0 = tile0;
      tile0 += s.tiles;
      fneed = std::max(fneed, pf * (rt * s.rb + 32));
    }
    q.total_tiles = tile0;
    q.stage_bytes = (fneed + 127) & ~127;
    const size_t fixed = fast_stage_offset() + ((size_t)xs_index(cols) + 8 + cols / 8) * 4 + 16;
    q.stages = 4;
    while (q.stages > 2 && fixed + (size_t)q.stages * q.stage_bytes > 227 * 1024) q.stages--;
    if (fixed + (size_t)q.stages * q.stage_bytes <= 227 * 1024) {
      q.fast = 1;
      *p = q;
    }
  }
  return LRS_OK;
}

cudaError_t gemv_launch(const GemvParams& p, cudaStream_t stream, int num_sms, bool pdl) {
  const int nb = gemv_nb(p.batch);
  const bool pair = p.epi == EPI_SWIGLU;
  const void* kernel;
  size_t smem;
  if (p.fast) {
    kernel = pair ? (const void*)gemv1_kernel<true> : (const void*)gemv1_kernel<false>;
    smem = fast_smem_bytes(p);
  } else {
    smem = smem_bytes(p, nb);
    kernel = nb == 1 ? (pair ? (const void*)gemv_kernel<1, true> : (const void*)gemv_kernel<1, false>)
                     : (pair ? (const void*)gemv_kernel<8, true> : (const void*)gemv_kernel<8, false>);
  }
  int occ = occupancy(kernel, (int)smem);
  if (occ < 1) occ = 1;
  int grid = std::min(p.total_tiles, num_sms * occ);
  if (grid < 1) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<GemvParams*>(&p)};
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

}  // namespace lrs

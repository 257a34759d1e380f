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
#include <cstdlib>
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
// Shared-memory x layout of the direct kernel: one 16-byte pad per 2^S columns,
// S chosen per type so that the 8 lanes of each quarter-warp phase read x from
// distinct bank groups (lanes walk consecutive pieces: 64-value pairs for
// Q4_K/Q5_K, (half, octet) pieces for Q6_K, 32-value blocks otherwise).
template <int T>
__host__ __device__ constexpr int xs_shift() {
  return (T == LRS_GGML_Q4_K || T == LRS_GGML_Q5_K) ? 6 : (T == LRS_GGML_Q6_K ? 7 : 5);
}
template <int T>
__host__ __device__ inline int xs_idx(int c) { return c + ((c >> xs_shift<T>()) << 2); }

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

// ---- batch-1 kernel: direct loads, int8-split x, dp4a -------------------------
// x is staged once per CTA in shared memory, per 8-column run r split as
//     x ~= s_r * (xh + xl / 256),  xh, xl int8,  s_r = max|x_run| / 127,
// (about 15 bits of x; the dot's error is ~1e-5 relative) together with the
// exact float sum X_r of the run.  The layout is piece-transposed: 16-byte
// chunk k of piece p sits at (k * npieces + p) * 16, so the lanes of a warp,
// which handle consecutive pieces, read consecutive chunks.
// Each warp then owns groups of R rows (R = 4, or 2 rows of a gate/up pair):
// lane l walks pieces l, l+32, ... of the group, loads the piece bytes of
// all its rows straight from global memory (R loads in flight per lane, no
// staging, no block barrier), multiplies codes by xh and xl with dp4a into
// exact int32 sums per run, and applies the scales (gemv_fast.cuh).  One warp
// reduction per row ends the group.  Dense types (F32/F16/BF16) keep float x
// (XLayout, gemv_fast.cuh).

// Bulk-prefetches the rows of row group g (R rows, both matrices of a pair)
// into L2 so that the lanes' loads of the group hit L2 instead of HBM.
constexpr int kPrefetchPasses = 2;  // row-group passes kept in flight into L2

template <int R, bool PAIR>
__device__ __forceinline__ void prefetch_group(const GemvParams& p, int g) {
  if (g >= p.total_tiles) return;
  const GemvSeg sg = find_seg(p, g);
  const int r0 = (g - sg.tile0) * R;
  const int nr = min(R, sg.rows - r0);
  const size_t lo = (size_t)r0 * sg.rb, hi = lo + (size_t)nr * sg.rb;
  const size_t alo = lo & ~size_t(15);
  const uint32_t bytes = (uint32_t)(((hi - alo) + 15) & ~size_t(15));
  prefetch_l2(sg.w + alo, bytes);
  if (PAIR) prefetch_l2(sg.w2 + alo, bytes);
}

template <int T, bool PAIR>
__global__ void __launch_bounds__(kGemvThreads) gemv5_kernel(const __grid_constant__ GemvParams p) {
  using BT = BlockTraits<T>;
  using P = fast::Piece<T>;
  using XL = XLayout<T>;
  constexpr int NM = PAIR ? 2 : 1;
  constexpr int R = PAIR ? 2 : 4;
  constexpr int PV = XL::PV, NRUN = XL::NRUN, CH = XL::CH, NW = P::kWords;
  constexpr bool kDense = XL::kDense;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem);  // 256 B
  uint8_t* xq = smem + 256;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int npieces = p.cols / PV;
  // piece-transposed arrays
  uint4* xh4 = reinterpret_cast<uint4*>(xq);                      // [CH][npieces]
  uint4* xl4 = xh4 + (size_t)CH * npieces;                        // [CH][npieces]
  float* sxa = reinterpret_cast<float*>(xl4 + (size_t)CH * npieces);  // [NRUN][npieces]
  float* Xa = sxa + (size_t)NRUN * npieces;                       // [NRUN][npieces]
  float* xf = reinterpret_cast<float*>(xq);                       // dense: [npieces][PV]
  // The weights do not depend on the previous kernel: pull this CTA's first
  // two passes of row groups into L2 while it finishes.
  const int gpc0 = kWarps / p.wpg;
  if (tid < kPrefetchPasses * gpc0)
    prefetch_group<R, PAIR>(p, blockIdx.x * gpc0 + (tid / gpc0) * gridDim.x * gpc0 + tid % gpc0);

  pdl_wait();  // x / residual come from the previous kernel
  float inv_rms = 1.0f;
  if (p.norm_w) {
    // RMSNorm::forward, src/model.rs:65-73: x * (inv_rms * w)
    float ss = 0.0f;
    for (int c = tid; c < p.cols; c += kGemvThreads) ss = fmaf(p.x[c], p.x[c], ss);
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < kWarps; w++) tot += red[w];
    inv_rms = 1.0f / sqrtf(tot / (float)p.cols + p.norm_eps);
  }
  // One thread per (piece, run): gather the run's 8 values, normalize, split.
  for (int t = tid; t < npieces * NRUN; t += kGemvThreads) {
    const int pc = t % npieces, r = t / npieces;
    const int unit = pc / P::kPieces, sub = pc % P::kPieces;
    const int col = unit * BT::kValues + P::col(sub, 2 * r);
    float v[8];
    const float4 a = *reinterpret_cast<const float4*>(p.x + col);
    const float4 b = *reinterpret_cast<const float4*>(p.x + col + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    if (p.norm_w) {
      const float4 wa = *reinterpret_cast<const float4*>(p.norm_w + col);
      const float4 wb = *reinterpret_cast<const float4*>(p.norm_w + col + 4);
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int c = 0; c < 8; c++) v[c] = v[c] * (inv_rms * w[c]);
    }
    if constexpr (kDense) {
#pragma unroll
      for (int c = 0; c < 8; c++) xf[(size_t)pc * PV + 8 * r + c] = v[c];
    } else {
      float mx = 0.0f, sum = 0.0f;
#pragma unroll
      for (int c = 0; c < 8; c++) mx = fmaxf(mx, fabsf(v[c]));
      sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
      const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
      const float inv = 1.0f / sc;
      uint32_t hw[2], lw[2];
#pragma unroll
      for (int w = 0; w < 2; w++) {
        hw[w] = lw[w] = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float q = v[4 * w + c] * inv;
          const float h = rintf(q);
          const float l = fminf(fmaxf(rintf((q - h) * 256.0f), -127.0f), 127.0f);
          hw[w] |= ((uint32_t)(int)h & 0xffu) << (8 * c);
          lw[w] |= ((uint32_t)(int)l & 0xffu) << (8 * c);
        }
      }
      // run r = words 2r, 2r+1 of the piece = 8 bytes of chunk r / 2
      uint32_t* hc = reinterpret_cast<uint32_t*>(xh4 + (size_t)(r >> 1) * npieces + pc) + 2 * (r & 1);
      uint32_t* lc = reinterpret_cast<uint32_t*>(xl4 + (size_t)(r >> 1) * npieces + pc) + 2 * (r & 1);
      hc[0] = hw[0], hc[1] = hw[1];
      lc[0] = lw[0], lc[1] = lw[1];
      sxa[(size_t)r * npieces + pc] = sc * (1.0f / 256.0f);
      Xa[(size_t)r * npieces + pc] = sum;
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  // wpg warps share a row group, each taking every wpg-th 32-piece slice;
  // the CTA's 8 warps serve 8 / wpg groups per pass (uniform trip count).
  const int wpg = p.wpg, gpc = kWarps / wpg;
  const int sub_w = warp % wpg;
  for (int gb = blockIdx.x * gpc; gb < p.total_tiles; gb += gridDim.x * gpc) {
    const int g = gb + warp / wpg;
    const bool live = g < p.total_tiles;
    // keep kPrefetchPasses passes ahead in L2
    if (lane == 0 && sub_w == 0) prefetch_group<R, PAIR>(p, g + kPrefetchPasses * gridDim.x * gpc);
    const GemvSeg sg = find_seg(p, live ? g : gb);
    const int r0 = ((live ? g : gb) - sg.tile0) * R;
    const int nr = live ? min(R, sg.rows - r0) : 0;
    const uint8_t* base[NM];
    base[0] = sg.w + (size_t)r0 * sg.rb;
    if constexpr (PAIR) base[1] = sg.w2 + (size_t)r0 * sg.rb;
    float acc[NM][R];
#pragma unroll
    for (int m = 0; m < NM; m++)
#pragma unroll
      for (int r = 0; r < R; r++) acc[m][r] = 0.0f;
    for (int pc = lane + 32 * sub_w; live && pc < npieces; pc += 32 * wpg) {
      const int unit = pc / P::kPieces, sub = pc % P::kPieces;
      const size_t uoff = (size_t)unit * BT::kBytes;
      P pr[NM][R];
#pragma unroll
      for (int m = 0; m < NM; m++)
#pragma unroll
        for (int r = 0; r < R; r++)  // rows past nr re-read row 0 (discarded)
          pr[m][r].template load<false>(base[m] + (size_t)(r < nr ? r : 0) * sg.rb + uoff, sub);
      if constexpr (kDense) {
        const float4* xp = reinterpret_cast<const float4*>(xf + (size_t)pc * PV);
        fast::f2 xa[NW], xb[NW];
#pragma unroll
        for (int i = 0; i < NW; i++) {
          const float4 v = xp[i];
          xa[i] = fast::pk(v.x, v.y);
          xb[i] = fast::pk(v.z, v.w);
        }
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int r = 0; r < R; r++) {
            fast::f2 S0 = 0ull, S1 = 0ull;
#pragma unroll
            for (int i = 0; i < NW; i++) {
              fast::f2 a, b;
              pr[m][r].weights(i, a, b);
              fast::fma2(S0, a, xa[i]);
              fast::fma2(S1, b, xb[i]);
            }
            acc[m][r] += fast::hsum2(S0) + fast::hsum2(S1);
          }
      } else {
        uint32_t xh[PV / 4], xl[PV / 4];
#pragma unroll
        for (int k = 0; k < CH; k++) {
          const uint4 h = xh4[(size_t)k * npieces + pc], l = xl4[(size_t)k * npieces + pc];
          xh[4 * k] = h.x, xh[4 * k + 1] = h.y, xh[4 * k + 2] = h.z, xh[4 * k + 3] = h.w;
          xl[4 * k] = l.x, xl[4 * k + 1] = l.y, xl[4 * k + 2] = l.z, xl[4 * k + 3] = l.w;
        }
        float sx[NRUN], X8[NRUN];
#pragma unroll
        for (int r = 0; r < NRUN; r++) {
          sx[r] = sxa[(size_t)r * npieces + pc];
          X8[r] = Xa[(size_t)r * npieces + pc];
        }
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int r = 0; r < R; r++) {
            float qx[NRUN];
#pragma unroll
            for (int u = 0; u < NRUN; u++) {
              const uint32_t c0 = pr[m][r].icode(2 * u, sub), c1 = pr[m][r].icode(2 * u + 1, sub);
              int hs = __dp4a((int)c0, (int)xh[2 * u], 0);
              hs = __dp4a((int)c1, (int)xh[2 * u + 1], hs);
              int ls = __dp4a((int)c0, (int)xl[2 * u], hs << 8);
              ls = __dp4a((int)c1, (int)xl[2 * u + 1], ls);
              qx[u] = sx[u] * (float)ls;
            }
            acc[m][r] += pr[m][r].finish_i(qx, X8, sub);
          }
      }
    }
#pragma unroll
    for (int m = 0; m < NM; m++)
#pragma unroll
      for (int r = 0; r < R; r++)
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc[m][r] += __shfl_xor_sync(0xffffffffu, acc[m][r], o);
    if (wpg > 1) {  // combine the warps of a group (fixed order: deterministic)
      __syncthreads();
      if (lane == 0)
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int r = 0; r < R; r++) red[(warp * NM + m) * R + r] = acc[m][r];
      __syncthreads();
      if (sub_w == 0 && lane == 0)
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int r = 0; r < R; r++) {
            float t = 0.0f;
            for (int w = 0; w < wpg; w++) t += red[((warp + w) * NM + m) * R + r];
            acc[m][r] = t;
          }
    }
    if (lane == 0 && sub_w == 0 && live) {
      unsigned long long key = 0ull;
#pragma unroll
      for (int r = 0; r < R; r++) {
        if (r >= nr) break;
        const int row = r0 + r;
        float y = acc[0][r];
        float* out = sg.out ? sg.out + row : nullptr;
        switch (p.epi) {
          case EPI_STORE:
            if (sg.bias) y += sg.bias[row];
            *out = y;
            break;
          case EPI_ADD:
            *out += y;
            break;
          case EPI_SWIGLU:
            *out = (y / (1.0f + expf(-y))) * acc[NM - 1][r];
            break;
          default: {
            if (out) *out = y;
            const unsigned long long k2 = argmax_pack(y, (uint32_t)row);
            key = k2 > key ? k2 : key;
          }
        }
      }
      if (p.epi == EPI_ARGMAX) atomicMax(&p.argmax_keys[0], key);
    }
  }
}

size_t fast_x_bytes(uint32_t type, int cols) {
#define LRS_XB(T) \
  case T: return XLayout<T>::bytes(cols / XLayout<T>::PV);
  switch (type) {
    LRS_XB(LRS_GGML_F32)
    LRS_XB(LRS_GGML_F16)
    LRS_XB(LRS_GGML_BF16)
    LRS_XB(LRS_GGML_Q4_0)
    LRS_XB(LRS_GGML_Q4_1)
    LRS_XB(LRS_GGML_Q5_0)
    LRS_XB(LRS_GGML_Q5_1)
    LRS_XB(LRS_GGML_Q8_0)
    LRS_XB(LRS_GGML_Q4_K)
    LRS_XB(LRS_GGML_Q5_K)
    LRS_XB(LRS_GGML_Q6_K)
  }
#undef LRS_XB
  return 0;
}

const void* fast_kernel(int type, bool pair) {
#define LRS_FK(T) \
  case T: return pair ? (const void*)gemv5_kernel<T, true> : (const void*)gemv5_kernel<T, false>;
  switch (type) {
    LRS_FK(LRS_GGML_F32)
    LRS_FK(LRS_GGML_F16)
    LRS_FK(LRS_GGML_BF16)
    LRS_FK(LRS_GGML_Q4_0)
    LRS_FK(LRS_GGML_Q4_1)
    LRS_FK(LRS_GGML_Q5_0)
    LRS_FK(LRS_GGML_Q5_1)
    LRS_FK(LRS_GGML_Q8_0)
    LRS_FK(LRS_GGML_Q4_K)
    LRS_FK(LRS_GGML_Q5_K)
    LRS_FK(LRS_GGML_Q6_K)
  }
#undef LRS_FK
  return nullptr;
}

// Resident CTAs per SM of `kernel` at `smem` bytes (cached per device, kernel, size).
int occupancy(const void* kernel, int smem, int threads = kGemvThreads) {
  struct Entry {
    int dev;
    const void* k;
    int smem, blocks, threads;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  for (auto& c : cache)
    if (c.dev == dev && c.k == kernel && c.smem == smem && c.threads == threads) return c.blocks;
  // the dynamic limit is what the static shared memory leaves of 227 KB
  cudaFuncAttributes fa{};
  const int stat = cudaFuncGetAttributes(&fa, kernel) == cudaSuccess ? (int)fa.sharedSizeBytes : 0;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - stat);
  int blocks = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem);
  cache.push_back({dev, kernel, smem, blocks, threads});
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
    // Direct-load batch-1 kernel: groups of 4 rows (2 for a gate/up pair) per warp.
    GemvParams q = *p;
    const int R = pair ? 2 : 4;
    tile0 = 0;
    bool fits = true;
    for (int i = 0; i < nmat; i++) {
      GemvSeg& s = q.seg[i];
      s.rt = s.rr = R;
      s.tiles = (s.rows + R - 1) / R;
      s.tile0 = tile0;
      tile0 += s.tiles;
      fits = fits && 256 + fast_x_bytes(s.type, cols) <= 200 * 1024;
    }
    q.total_tiles = tile0;
    q.stages = 0;
    q.stage_bytes = 0;
    if (fits) {
      q.fast = 1;
      *p = q;
    }
  }
  return LRS_OK;
}

namespace {

cudaError_t launch_cfg(const void* kernel, size_t smem, int grid, int threads,
                       cudaStream_t stream, bool pdl, const GemvParams& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
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

}  // namespace

cudaError_t gemv_launch(const GemvParams& p, cudaStream_t stream, int num_sms, bool pdl) {
  const bool pair = p.epi == EPI_SWIGLU;
  if (p.scratch && p.batch >= 4) {
    if (gemm_tc_supported(p)) {
      if (p.scratch_bytes >= gemm_tc_scratch_bytes(p, num_sms))
        return gemm_tc_launch(p, p.scratch, num_sms, stream);
    } else if (p.nseg > 1 && !p.fast) {
      // mixed types (q/k/v): each run of same-type segments on its own path
      bool any = false;
      for (int i = 0; i < p.nseg; i++) {
        GemvParams q = p;
        q.nseg = 1;
        q.seg[0] = p.seg[i];
        any = any || gemm_tc_supported(q);
      }
      if (any) {
        int i = 0;
        while (i < p.nseg) {
          int j = i + 1;
          while (j < p.nseg && p.seg[j].type == p.seg[i].type) j++;
          GemvParams q = p;
          q.nseg = j - i;
          const int t0 = p.seg[i].tile0;
          for (int k = 0; k < q.nseg; k++) {
            q.seg[k] = p.seg[i + k];
            q.seg[k].tile0 -= t0;
          }
          q.total_tiles = (j < p.nseg ? p.seg[j].tile0 : p.total_tiles) - t0;
          cudaError_t e = gemv_launch(q, stream, num_sms, pdl);
          if (e != cudaSuccess) return e;
          i = j;
        }
        return cudaSuccess;
      }
    }
  }
  if (p.batch >= 2 && p.scratch && gemm_supported(p) &&
      p.scratch_bytes >= gemm_scratch_bytes(p.batch, p.cols, num_sms))
    return gemm_launch(p, p.scratch, num_sms, stream);
  if (p.fast) {
    // Direct-load batch-1 kernel, one launch per run of same-type segments.
    int i = 0;
    while (i < p.nseg) {
      int j = i + 1;
      while (j < p.nseg && p.seg[j].type == p.seg[i].type) j++;
      GemvParams q = p;
      q.nseg = j - i;
      const int t0 = p.seg[i].tile0;
      for (int k = 0; k < q.nseg; k++) {
        q.seg[k] = p.seg[i + k];
        q.seg[k].tile0 -= t0;
      }
      q.total_tiles = (j < p.nseg ? p.seg[j].tile0 : p.total_tiles) - t0;
      const void* kernel = fast_kernel(q.seg[0].type, pair);
      const size_t smem = 256 + fast_x_bytes(q.seg[0].type, q.cols);
      const int occ = std::max(1, occupancy(kernel, (int)smem, kGemvThreads));
      // Long rows: several warps per row group, ~4 pieces per lane.
      const int pv = (q.seg[0].type == LRS_GGML_Q4_K || q.seg[0].type == LRS_GGML_Q5_K) ? 64 : 32;
      const int ppr = q.cols / pv;
      q.wpg = 1;
      while (q.wpg < kWarps && ppr >= 32 * 4 * 2 * q.wpg) q.wpg *= 2;
      const int gpc = kWarps / q.wpg;
      const int grid = std::min((q.total_tiles + gpc - 1) / gpc, num_sms * occ);
      if (grid > 0) {
        cudaError_t e = launch_cfg(kernel, smem, grid, kGemvThreads, stream, pdl, q);
        if (e != cudaSuccess) return e;
      }
      i = j;
    }
    return cudaSuccess;
  }
  const int nb = gemv_nb(p.batch);
  const size_t smem = smem_bytes(p, nb);
  const void* kernel =
      nb == 1 ? (pair ? (const void*)gemv_kernel<1, true> : (const void*)gemv_kernel<1, false>)
              : (pair ? (const void*)gemv_kernel<8, true> : (const void*)gemv_kernel<8, false>);
  int occ = std::max(1, occupancy(kernel, (int)smem));
  const int grid = std::min(p.total_tiles, num_sms * occ);
  if (grid < 1) return cudaSuccess;
  return launch_cfg(kernel, smem, grid, kGemvThreads, stream, pdl, p);
}

}  // namespace lrs

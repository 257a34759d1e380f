// decode.cu -- embedding, RMSNorm, RoPE + paged KV store, split-K GQA decode
// attention and greedy bookkeeping for the Qwen2 token step (sm_100a).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <cstdlib>

#include "common.h"
#include "decode.cuh"
#include "device_common.cuh"

namespace lrs {
namespace {

// ---- embedding / dequantization (value_at, bit-exact) ---------------------
template <int T>
__global__ void __launch_bounds__(128)
    embed_kernel(const uint8_t* w, int cols, const int* rows, int row0, float* out,
                 unsigned long long* keys) {
  using BT = BlockTraits<T>;
  const int b = blockIdx.x;
  const size_t rb = (size_t)(cols / BT::kValues) * BT::kBytes;
  const int row = rows ? rows[b] : row0 + b;
  const uint8_t* rp = w + (size_t)row * rb;
  float* o = out + (size_t)b * cols;
  if (keys && threadIdx.x == 0) keys[b] = 0ull;
  for (int pc = threadIdx.x; pc < cols / 32; pc += blockDim.x) {
    const int unit = pc / BT::kPieces, sub = pc % BT::kPieces;
    float v[32];
    decode_piece<T>(rp + (size_t)unit * BT::kBytes, sub, v);
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = unit * BT::kValues + run_col<T>(sub, r);
#pragma unroll
      for (int i = 0; i < 8; i++) o[col + i] = v[r * 8 + i];
    }
  }
}

cudaError_t embed_dispatch(const uint8_t* w, uint32_t type, int cols, const int* rows, int row0,
                           int n, float* out, unsigned long long* keys, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  dim3 g(n), b(128);
#define LRS_EMBED(T) \
  case T: embed_kernel<T><<<g, b, 0, st>>>(w, cols, rows, row0, out, keys); break;
  switch (type) {
    LRS_EMBED(LRS_GGML_F32)
    LRS_EMBED(LRS_GGML_F16)
    LRS_EMBED(LRS_GGML_BF16)
    LRS_EMBED(LRS_GGML_Q4_0)
    LRS_EMBED(LRS_GGML_Q4_1)
    LRS_EMBED(LRS_GGML_Q5_0)
    LRS_EMBED(LRS_GGML_Q5_1)
    LRS_EMBED(LRS_GGML_Q8_0)
    LRS_EMBED(LRS_GGML_Q4_K)
    LRS_EMBED(LRS_GGML_Q5_K)
    LRS_EMBED(LRS_GGML_Q6_K)
    default: return cudaErrorInvalidValue;
  }
#undef LRS_EMBED
  return cudaGetLastError();
}

// ---- RMSNorm ---------------------------------------------------------------
__global__ void __launch_bounds__(256)
    rmsnorm_kernel(const float* x, const float* w, float eps, int n, float* out) {
  __shared__ float red[8];
  const float* xb = x + (size_t)blockIdx.x * n;
  float* ob = out + (size_t)blockIdx.x * n;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += 256) ss = fmaf(xb[i], xb[i], ss);
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int k = 0; k < 8; k++) tot += red[k];
  const float inv = 1.0f / sqrtf(tot / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += 256) ob[i] = xb[i] * (inv * w[i]);
}

// ---- RoPE + KV store --------------------------------------------------------
__device__ __forceinline__ size_t kv_offset(const StepIO& io, int b, int p, int nkv, int kvh,
                                            int hd) {
  const int page = io.pages[io.seq[b] * io.max_pages + p / kPageSize];
  return (((size_t)page * nkv + kvh) * kPageSize + (p % kPageSize)) * hd;
}

// One CTA per (item, head): heads [0, nh) rotate q in place; heads
// [nh, nh + nkv) rotate k and store k and v of the item's position.
__global__ void __launch_bounds__(64)
    rope_store_kernel(float* q, const float* k, const float* v, const float* cos_t,
                      const float* sin_t, StepIO io, int nh, int nkv, int hd, void* kpool,
                      void* vpool, int kv_bf16) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int half = hd / 2;
  const int pos = io.pos[b];
  const float* c = cos_t + (size_t)pos * half;
  const float* s = sin_t + (size_t)pos * half;
  // apply_rope_inplace, src/model.rs:86-95 (unfused, as the reference)
  if (h < nh) {
    float* qh = q + ((size_t)b * nh + h) * hd;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float re = qh[i], im = qh[i + half];
      qh[i] = __fsub_rn(__fmul_rn(re, c[i]), __fmul_rn(im, s[i]));
      qh[i + half] = __fadd_rn(__fmul_rn(re, s[i]), __fmul_rn(im, c[i]));
    }
    return;
  }
  const int kvh = h - nh;
  const float* kh = k + ((size_t)b * nkv + kvh) * hd;
  const float* vh = v + ((size_t)b * nkv + kvh) * hd;
  const size_t o = kv_offset(io, b, pos, nkv, kvh, hd);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float re = kh[i], im = kh[i + half];
    const float k0 = __fsub_rn(__fmul_rn(re, c[i]), __fmul_rn(im, s[i]));
    const float k1 = __fadd_rn(__fmul_rn(re, s[i]), __fmul_rn(im, c[i]));
    if (kv_bf16) {
      __nv_bfloat16* kp = reinterpret_cast<__nv_bfloat16*>(kpool) + o;
      __nv_bfloat16* vp = reinterpret_cast<__nv_bfloat16*>(vpool) + o;
      kp[i] = __float2bfloat16_rn(k0);
      kp[i + half] = __float2bfloat16_rn(k1);
      vp[i] = __float2bfloat16_rn(vh[i]);
      vp[i + half] = __float2bfloat16_rn(vh[i + half]);
    } else {
      float* kp = reinterpret_cast<float*>(kpool) + o;
      float* vp = reinterpret_cast<float*>(vpool) + o;
      kp[i] = k0;
      kp[i + half] = k1;
      vp[i] = vh[i];
      vp[i + half] = vh[i + half];
    }
  }
}

// ---- split-K GQA decode attention ------------------------------------------
constexpr int kMaxGroup = 8;  // query heads per KV head handled by one CTA
constexpr int kAttnWarps = 4;
constexpr int kMinSplit = kAttnWarps * 8;  // positions per split (8 per warp at least)

template <int HD, bool BF16>
__device__ __forceinline__ void load_row(const void* pool, size_t off, int d0, float* out) {
  constexpr int DPL = HD / 32;
  if constexpr (BF16) {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(pool) + off + d0;
#pragma unroll
    for (int k = 0; k < DPL; k++) out[k] = __bfloat162float(p[k]);
  } else {
    const float* p = reinterpret_cast<const float*>(pool) + off + d0;
    if constexpr (DPL == 4) {
      float4 t = *reinterpret_cast<const float4*>(p);
      out[0] = t.x, out[1] = t.y, out[2] = t.z, out[3] = t.w;
    } else {
#pragma unroll
      for (int k = 0; k < DPL; k++) out[k] = p[k];
    }
  }
}

// Positions of split `split` of a context of L positions: [s0, s1) with
// chunks a multiple of 32 (blocks of 32 positions never straddle a KV page).
__device__ __forceinline__ int split_chunk(int L, int nsplit) {
  const int c = max((L + nsplit - 1) / nsplit, kMinSplit);
  return (c + 31) & ~31;
}

// Four consecutive K or V values of a row.
template <bool BF16>
__device__ __forceinline__ float4 load4(const void* pool, size_t off) {
  if constexpr (BF16) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(
        reinterpret_cast<const __nv_bfloat16*>(pool) + off));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  } else {
    return __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(pool) + off));
  }
}

// One CTA per (split, kv head, item) serves all G query heads of the GQA
// group, so each K/V row is read once per group.  Warps take blocks of 32
// positions (s0 + 32 * warp, then every 128).  Scores: lane i owns position
// i of the block and dots its K row with the G scaled query rows (shared
// memory broadcasts).  The block's softmax update is one warp max / sum per
// head; the probabilities go through shared memory to the PV product, where
// the lanes cover the head dimension and V rows are read coalesced.
template <int HD, bool BF16>
__global__ void __launch_bounds__(kAttnWarps * 32)
    attn_split_kernel(const float* q, StepIO io, int nh, int nkv, const void* kpool,
                      const void* vpool, int nsplit, float scale, float* part) {
  constexpr int DPL = HD / 32;  // dims per lane in the PV product
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = nh / nkv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int L = io.pos[b] + 1;
  const int chunk = split_chunk(L, nsplit);
  const int s0 = split * chunk, s1 = min(L, s0 + chunk);
  __shared__ float4 qs[kMaxGroup][HD / 4];
  __shared__ float ps[kAttnWarps][kMaxGroup][32];
  __shared__ float wm[kAttnWarps][kMaxGroup], wl[kAttnWarps][kMaxGroup];
  __shared__ float wo[kAttnWarps][kMaxGroup][HD];

  for (int i = threadIdx.x; i < kMaxGroup * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    reinterpret_cast<float*>(qs)[i] = g < G ? q[((size_t)b * nh + kvh * G + g) * HD + d] * scale : 0.0f;
  }
  __syncthreads();
  float m[kMaxGroup], l[kMaxGroup], o[kMaxGroup][DPL];
#pragma unroll
  for (int g = 0; g < kMaxGroup; g++) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int k = 0; k < DPL; k++) o[g][k] = 0.0f;
  }
  for (int blk = s0 + 32 * warp; blk < s1; blk += 32 * kAttnWarps) {
    const size_t base = kv_offset(io, b, blk, nkv, kvh, HD);  // row blk; rows follow at +HD
    const bool valid = blk + lane < s1;
    float sc[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) sc[g] = 0.0f;
    if (valid) {
      const size_t kr = base + (size_t)lane * HD;
#pragma unroll 8
      for (int i = 0; i < HD / 4; i++) {
        const float4 kv = load4<BF16>(kpool, kr + 4 * i);
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
          if (g < G) {
            const float4 qq = qs[g][i];
            sc[g] = fmaf(qq.x, kv.x, fmaf(qq.y, kv.y, fmaf(qq.z, kv.z, fmaf(qq.w, kv.w, sc[g]))));
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) {
      if (g >= G) break;
      const float s = valid ? sc[g] : -INFINITY;
      float bm = s;
      for (int w = 16; w >= 1; w >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, w));
      const float mn = fmaxf(m[g], bm);  // finite: lane 0 is always valid
      const float corr = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
      const float e = valid ? expf(s - mn) : 0.0f;
      float es = e;
      for (int w = 16; w >= 1; w >>= 1) es += __shfl_xor_sync(0xffffffffu, es, w);
      l[g] = l[g] * corr + es;
      m[g] = mn;
      ps[warp][g][lane] = e;
#pragma unroll
      for (int k = 0; k < DPL; k++) o[g][k] *= corr;
    }
    __syncwarp();
    const int nv = min(32, s1 - blk);
#pragma unroll 4
    for (int j = 0; j < nv; j++) {
      const size_t vr = base + (size_t)j * HD + lane * DPL;
      float v[DPL];
      if constexpr (DPL == 4) {
        const float4 t = load4<BF16>(vpool, vr);
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
      } else {
#pragma unroll
        for (int k = 0; k < DPL; k++) {
          if constexpr (BF16)
            v[k] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(vpool)[vr + k]);
          else
            v[k] = __ldg(reinterpret_cast<const float*>(vpool) + vr + k);
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; g++) {
        if (g < G) {
          const float pj = ps[warp][g][j];
#pragma unroll
          for (int k = 0; k < DPL; k++) o[g][k] = fmaf(pj, v[k], o[g][k]);
        }
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int g = 0; g < kMaxGroup; g++) {
    if (g >= G) break;
    if (lane == 0) {
      wm[warp][g] = m[g];
      wl[warp][g] = l[g];
    }
#pragma unroll
    for (int k = 0; k < DPL; k++) wo[warp][g][lane * DPL + k] = o[g][k];
  }
  __syncthreads();
  // Merge the warps; part layout [b][head][split][2 + HD] = (m, l, o[HD]).
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, wm[w][g]);
    float Ls = 0.0f, O = 0.0f;
    for (int w = 0; w < kAttnWarps; w++) {
      const float f = wm[w][g] == -INFINITY ? 0.0f : expf(wm[w][g] - M);
      Ls += wl[w][g] * f;
      O += wo[w][g][d] * f;
    }
    float* pp = part + (((size_t)b * nh + kvh * G + g) * nsplit + split) * (HD + 2);
    if (d == 0) {
      pp[0] = s0 < s1 ? M : -INFINITY;
      pp[1] = s0 < s1 ? Ls : 0.0f;
    }
    pp[2 + d] = s0 < s1 ? O : 0.0f;
  }
}

template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float* part, const int* pos,
                                                          int nh, int nsplit, float* att) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float* pp = part + ((size_t)b * nh + h) * nsplit * (HD + 2);
  const int L = pos[b] + 1;
  const int chunk = split_chunk(L, nsplit);
  const int nact = min(nsplit, (L + chunk - 1) / chunk);  // splits that saw positions
  __shared__ float wsh[64];
  __shared__ float Lsum;
  if (d < 32) {
    // weights exp(m_s - M) of the active splits, and the total softmax denominator
    float m0 = d < nact ? pp[d * (HD + 2)] : -INFINITY;
    float m1 = d + 32 < nact ? pp[(d + 32) * (HD + 2)] : -INFINITY;
    float M = fmaxf(m0, m1);
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float w0 = m0 == -INFINITY ? 0.0f : expf(m0 - M);
    const float w1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
    float l = (d < nact ? pp[d * (HD + 2) + 1] * w0 : 0.0f) +
              (d + 32 < nact ? pp[(d + 32) * (HD + 2) + 1] * w1 : 0.0f);
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    wsh[d] = w0;
    wsh[d + 32] = w1;
    if (d == 0) Lsum = l;
  }
  __syncthreads();
  float O = 0.0f;
  for (int s = 0; s < nact; s++) O += pp[s * (HD + 2) + 2 + d] * wsh[s];
  att[((size_t)b * nh + h) * HD + d] = O / Lsum;
}

__global__ void advance_kernel(const unsigned long long* keys, int* tok, int* pos, int batch,
                               int* step, int n_steps, uint32_t* tokens_out, uint32_t* last) {
  const int s = *step;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    const uint32_t t = (uint32_t)(keys[b] & 0xffffffffull);
    tok[b] = (int)t;
    pos[b] += 1;
    if (last) last[b] = t;
    if (tokens_out && s < n_steps) tokens_out[(size_t)s * batch + b] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = s + 1;
}

}  // namespace

cudaError_t launch_embed(const uint8_t* w, uint32_t type, int cols, const int* rows, int n,
                         float* out, unsigned long long* keys, cudaStream_t st) {
  return embed_dispatch(w, type, cols, rows, 0, n, out, keys, st);
}

cudaError_t launch_dequant_rows(const uint8_t* w, uint32_t type, int cols, int row0, int n,
                                float* out, cudaStream_t st) {
  return embed_dispatch(w, type, cols, nullptr, row0, n, out, nullptr, st);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, int batch, float* out,
                           cudaStream_t st) {
  rmsnorm_kernel<<<batch, 256, 0, st>>>(x, w, eps, n, out);
  return cudaGetLastError();
}

cudaError_t launch_rope_store(float* q, const float* k, const float* v, const float* cos_t,
                              const float* sin_t, StepIO io, int batch, int nh, int nkv, int hd,
                              void* kpool, void* vpool, int kv_bf16, cudaStream_t st) {
  rope_store_kernel<<<dim3(batch, nh + nkv), 64, 0, st>>>(q, k, v, cos_t, sin_t, io, nh, nkv, hd,
                                                          kpool, vpool, kv_bf16);
  return cudaGetLastError();
}

int attention_ctas_per_sm(int hd, int kv_bf16) {
  int n = 1;
  const void* k = hd == 128 ? (kv_bf16 ? (const void*)attn_split_kernel<128, true>
                                       : (const void*)attn_split_kernel<128, false>)
                            : (kv_bf16 ? (const void*)attn_split_kernel<64, true>
                                       : (const void*)attn_split_kernel<64, false>);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kAttnWarps * 32, 0) != cudaSuccess)
    return 1;
  return n < 1 ? 1 : n;
}

cudaError_t launch_attention(const float* q, StepIO io, int batch, int nh, int nkv, int hd,
                             const void* kpool, const void* vpool, int kv_bf16, int nsplit,
                             float* part, float* att, cudaStream_t st) {
  if (nh / nkv > kMaxGroup || nsplit > 64) return cudaErrorInvalidValue;
  const float scale = 1.0f / sqrtf((float)hd);
  dim3 g(nsplit, nkv, batch);
#define LRS_ATTN(HD, BF)                                                                         \
  attn_split_kernel<HD, BF><<<g, kAttnWarps * 32, 0, st>>>(q, io, nh, nkv, kpool, vpool, nsplit, \
                                                            scale, part);                        \
  attn_combine_kernel<HD><<<dim3(nh, batch), HD, 0, st>>>(part, io.pos, nh, nsplit, att);
  if (hd == 128) {
    if (kv_bf16) {
      LRS_ATTN(128, true)
    } else {
      LRS_ATTN(128, false)
    }
  } else if (hd == 64) {
    if (kv_bf16) {
      LRS_ATTN(64, true)
    } else {
      LRS_ATTN(64, false)
    }
  } else {
    return cudaErrorInvalidValue;
  }
#undef LRS_ATTN
  return cudaGetLastError();
}

// dst[b][j] = src[b][j - lo] for lo <= j < lo + n, else 0 (j < width): the
// rank's x of a windowed column shard, zero outside its columns.
__global__ void pad_copy_kernel(const float* src, int n, float* dst, int width, int lo, int batch) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)batch * width) return;
  const int b = (int)(i / width), j = (int)(i % width) - lo;
  dst[i] = j >= 0 && j < n ? src[(size_t)b * n + j] : 0.0f;
}

// g[i] = silu(g[i]) * u[i] (src/model.rs:251-254), for gate and up
// projections of different GGML types that ran as two launches.
__global__ void swiglu_kernel(float* g, const float* u, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float y = g[i];
    g[i] = (y / (1.0f + expf(-y))) * u[i];
  }
}

__global__ void key_offset_kernel(unsigned long long* keys, int n, uint32_t offset) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n && keys[i]) keys[i] += offset;
}

cudaError_t launch_pad_copy(const float* src, int n, float* dst, int width, int lo, int batch,
                            cudaStream_t st) {
  const size_t total = (size_t)batch * width;
  if (total == 0) return cudaSuccess;
  pad_copy_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, n, dst, width, lo, batch);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(float* g, const float* u, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, n);
  return cudaGetLastError();
}

cudaError_t launch_key_offset(unsigned long long* keys, int n, uint32_t offset, cudaStream_t st) {
  key_offset_kernel<<<(n + 63) / 64, 64, 0, st>>>(keys, n, offset);
  return cudaGetLastError();
}

cudaError_t launch_advance(const unsigned long long* keys, int* tok, int* pos, int batch,
                           int* step, int n_steps, uint32_t* tokens_out, uint32_t* last,
                           cudaStream_t st) {
  advance_kernel<<<1, 64, 0, st>>>(keys, tok, pos, batch, step, n_steps, tokens_out, last);
  return cudaGetLastError();
}

}  // namespace lrs

// gemm_i8.cu -- batched quantized matmul (decode batches of 2..64 sequences,
// prefill chunks) on the integer tensor cores of sm_100a
// (mma.sync m16n8k32 / m16n8k16, s8 x s8 -> s32).
//
// Replaces B independent CpuBackend::matvec calls (src/backend.rs:143-162)
// for B >= 2 input vectors: the sequences of a decode batch, or the prompt
// tokens of a prefill chunk (CausalModel::prefill, src/architecture.rs:60-77,
// runs them one by one).
//
// Every quantized GGML type stores integer codes q with a per-group affine
// map  w = ds * q - dm  (value_at, src/quant.rs:349-456):
//   Q4_0: ds = d, dm = 8d        Q4_1: ds = d, dm = -m
//   Q5_0: ds = d, dm = 16d       Q5_1: ds = d, dm = -m
//   Q8_0: ds = d, dm = 0 (signed codes)
//   Q4_K/Q5_K: ds = d*sc, dm = dmin*m per 32 columns
//   Q6_K: ds = d*sc, dm = 32*d*sc per 16 columns
// so that per group  sum_k w_k x_k = ds * sum_k q_k x_k - dm * sum_k x_k.
// The integer part runs on the tensor cores: x of every item is split per
// 32-column group into s * (xh + xl/256) with int8 xh, xl (about 15
// significant bits), and
//     sum_k q_k x_k = s/256 * (256 * (q.xh) + q.xl)
// is formed exactly in int32 by two MMAs (the second one accumulates onto the
// first one's result shifted left by 8).  The A operand is the weight codes,
// decoded straight from the GGML block bytes into the m16n8k32 fragment
// layout; B is the split x staged in shared memory.  Scales and the offset
// term are applied in fp32 per (row, group).  The result matches the
// reference's f32 dot to about 1e-5 relative.
//
// Work split: a CTA of 8 warps owns 128 rows (16 per warp) of one matrix and
// a run of K chunks of 512 columns; per chunk the split x of all items is
// staged in shared memory once and each warp streams its rows' blocks from
// HBM exactly once, holding fp32 accumulators for up to 64 items.  When the
// row CTAs alone fill the GPU the epilogue (bias, residual add, SwiGLU,
// greedy argmax) runs in the kernel; otherwise K is split across CTAs, the
// partial sums go to scratch and gemm_epilogue_kernel adds them in a fixed
// order, so results never depend on scheduling.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "device_common.cuh"
#include "gemv.cuh"

namespace lrs {
namespace {

constexpr int kKC = 512;       // columns per K chunk
constexpr int kWarps = 8;
constexpr int kRowsCTA = 16 * kWarps;
constexpr int kMaxItems = 64;  // items per launch (larger batches loop)
constexpr int kXPad = 16;      // padding bytes per staged x row: conflict-free B fragments
constexpr int kXStride = kKC + kXPad;

__device__ __forceinline__ uint32_t ldg32(const uint8_t* p) {
  uint32_t v;
  asm("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg128(const uint8_t* p) {
  uint4 v;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg16(const uint8_t* p) {
  unsigned short v;
  asm("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
// Four bytes at a 2-byte aligned address (blocks of 18, 22, 34, 210 bytes).
__device__ __forceinline__ uint32_t ldg32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if ((a & 3) == 0) return ldg32(p);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  return __funnelshift_r(ldg32(b), ldg32(b + 4), 16);
}
// Bit j (j = 0..3) of `nib` to bit 0 of byte j.
__device__ __forceinline__ uint32_t spread4(uint32_t nib) {
  return ((nib & 15u) * 0x00204081u) & 0x01010101u;
}
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xffu; }

__device__ __forceinline__ void mma_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1, const int (&c)[4]) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]),
        "r"(c[2]), "r"(c[3]));
}
__device__ __forceinline__ void mma_k16(int (&d)[4], const uint32_t (&a)[2], uint32_t b0,
                                        const int (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%7,%8,%9,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(b0), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// ---- x preparation ---------------------------------------------------------
// xh/xl: [B][cols] int8; sx: [B][cols/32] (scale/256); X16: [B][cols/16] sums
// of x over 16-column halves.  One warp per (item, 32-column group).
__global__ void __launch_bounds__(256)
    xsplit_kernel(const float* x, int x_ld, int cols, int8_t* xh, int8_t* xl, float* sx,
                  float* X16) {
  const int b = blockIdx.y;
  const int g = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (g * 32 >= cols) return;
  const float v = x[(size_t)b * x_ld + g * 32 + lane];
  float mx = fabsf(v);
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s16 = v;
  for (int o = 8; o >= 1; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
  const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
  const float q = v / sc;
  const float h = fminf(fmaxf(rintf(q), -127.0f), 127.0f);
  const float l = fminf(fmaxf(rintf((q - h) * 256.0f), -127.0f), 127.0f);
  xh[(size_t)b * cols + g * 32 + lane] = (int8_t)h;
  xl[(size_t)b * cols + g * 32 + lane] = (int8_t)l;
  if (lane == 0) sx[(size_t)b * (cols / 32) + g] = sc * (1.0f / 256.0f);
  if ((lane & 15) == 0) X16[(size_t)b * (cols / 16) + g * 2 + (lane >> 4)] = s16;
}

// ---- A fragments -------------------------------------------------------------
// For one row (block bytes at rp), 32-column group gc and thread t of the
// quad: the code words of columns 4t..4t+3 (w0) and 16+4t..16+4t+3 (w1) and
// the affine maps of the two 16-column halves (equal except for Q6_K).
template <int T>
struct AFrag {
  uint32_t w0, w1;
  float ds0, dm0, ds1, dm1;

  __device__ __forceinline__ void load(const uint8_t* rp, int gc, int t) {
    if constexpr (T == LRS_GGML_Q4_K || T == LRS_GGML_Q5_K) {
      // d, dmin, scales[12], (qh[32]), qs[128]; value_at, src/quant.rs:404-440
      const uint8_t* u = rp + (size_t)(gc >> 3) * BlockTraits<T>::kBytes;
      const int g = gc & 7;
      constexpr int qs0 = T == LRS_GGML_Q4_K ? 16 : 48;
      const uint8_t* q = u + qs0 + 32 * (g >> 1) + 4 * t;
      const int sh = 4 * (g & 1);
      w0 = (ldg32(q) >> sh) & 0x0F0F0F0Fu;
      w1 = (ldg32(q + 16) >> sh) & 0x0F0F0F0Fu;
      if constexpr (T == LRS_GGML_Q5_K) {
        w0 |= ((ldg32(u + 16 + 4 * t) >> g) & 0x01010101u) << 4;
        w1 |= ((ldg32(u + 32 + 4 * t) >> g) & 0x01010101u) << 4;
      }
      // header as one 16-byte load; scale_min_k4 (src/quant.rs:338-347) on words
      const uint4 hd = ldg128(u);
      uint32_t sc, mn;
      if (g < 4) {
        sc = byte_of(hd.y, g) & 63u;
        mn = byte_of(hd.z, g) & 63u;
      } else {
        const int j = g - 4;
        sc = (byte_of(hd.w, j) & 15u) | ((byte_of(hd.y, j) >> 6) << 4);
        mn = (byte_of(hd.w, j) >> 4) | ((byte_of(hd.z, j) >> 6) << 4);
      }
      ds0 = ds1 = f16_bits((uint16_t)(hd.x & 0xffffu)) * (float)sc;
      dm0 = dm1 = f16_bits((uint16_t)(hd.x >> 16)) * (float)mn;
    } else if constexpr (T == LRS_GGML_Q6_K) {
      // ql[128], qh[64], scales[16] (i8), d; value_at, src/quant.rs:441-456
      const uint8_t* u = rp + (size_t)(gc >> 3) * 210;
      const int gq = gc & 7;
      const int half = gq >> 2, quarter = gq & 3;
      const uint8_t* ql = u + half * 64 + (quarter & 1) * 32 + 4 * t;
      const uint8_t* qh = u + 128 + half * 32 + 4 * t;
      const int nsh = (quarter >> 1) * 4, hsh = 2 * quarter;
      w0 = ((ldg32_a2(ql) >> nsh) & 0x0F0F0F0Fu) | (((ldg32_a2(qh) >> hsh) & 0x03030303u) << 4);
      w1 = ((ldg32_a2(ql + 16) >> nsh) & 0x0F0F0F0Fu) |
           (((ldg32_a2(qh + 16) >> hsh) & 0x03030303u) << 4);
      const float d = f16_bits(ldg16(u + 208));
      const uint16_t sp = ldg16(u + 192 + half * 8 + quarter * 2);
      ds0 = d * (float)(int8_t)(sp & 0xffu);
      ds1 = d * (float)(int8_t)(sp >> 8);
      dm0 = 32.0f * ds0;
      dm1 = 32.0f * ds1;
    } else {
      // 32-value blocks: d, (m), (qh[4]), qs[16] or Q8_0 d, qs[32]
      const uint8_t* u = rp + (size_t)gc * BlockTraits<T>::kBytes;
      const float d = f16_bits(ldg16(u));
      ds0 = ds1 = d;
      if constexpr (T == LRS_GGML_Q8_0) {
        w0 = ldg32_a2(u + 2 + 4 * t);
        w1 = ldg32_a2(u + 18 + 4 * t);
        dm0 = dm1 = 0.0f;
      } else {
        constexpr int qs = T == LRS_GGML_Q4_0 ? 2 : T == LRS_GGML_Q4_1 ? 4 : T == LRS_GGML_Q5_0 ? 6 : 8;
        const uint32_t q = ldg32_a2(u + qs + 4 * t);
        w0 = q & 0x0F0F0F0Fu;
        w1 = (q >> 4) & 0x0F0F0F0Fu;
        if constexpr (T == LRS_GGML_Q5_0 || T == LRS_GGML_Q5_1) {
          const uint32_t qh = ldg32_a2(u + (T == LRS_GGML_Q5_0 ? 2 : 4));
          w0 |= spread4(qh >> (4 * t)) << 4;
          w1 |= spread4(qh >> (16 + 4 * t)) << 4;
        }
        if constexpr (T == LRS_GGML_Q4_1 || T == LRS_GGML_Q5_1) {
          dm0 = dm1 = -f16_bits(ldg16(u + 2));
        } else {
          dm0 = dm1 = (T == LRS_GGML_Q4_0 ? 8.0f : 16.0f) * d;
        }
      }
    }
  }
};

struct GemmArgs {
  GemvSeg seg[kGemvMaxSeg];
  int cta0[kGemvMaxSeg + 1];  // first row-CTA of each segment
  int nseg, cols, batch, epi, kper, kgroups;
  const int8_t* xh;  // [batch][cols]
  const int8_t* xl;
  const float* sx;   // [batch][cols/32]
  const float* X16;  // [batch][cols/16]
  float* part[kGemvMaxSeg];  // [pair][kgroups][batch][rows], kgroups > 1
  unsigned long long* keys;  // [batch], EPI_ARGMAX
};

// Adds one 32-column group of 16 rows x (8 * ntile) items into acc.
template <int T>
__device__ __forceinline__ void group_mma(float (&acc)[8][4], const AFrag<T>& fa,
                                          const AFrag<T>& fb, const int8_t* sxh,
                                          const int8_t* sxl, const float* ssx, const float* sX16,
                                          int g, int ntile, int gid, int t) {
#pragma unroll
  for (int j = 0; j < 8; j++) {
    if (j >= ntile) break;
    const int bn = 8 * j + gid;
    const uint32_t* xh = reinterpret_cast<const uint32_t*>(sxh + bn * kXStride + g * 32 + 4 * t);
    const uint32_t* xl = reinterpret_cast<const uint32_t*>(sxl + bn * kXStride + g * 32 + 4 * t);
    const uint32_t bh0 = xh[0], bh1 = xh[4], bl0 = xl[0], bl1 = xl[4];
    const int i0 = 8 * j + 2 * t;
    const float2 s = *reinterpret_cast<const float2*>(ssx + g * kMaxItems + i0);
    const float2 xa = *reinterpret_cast<const float2*>(sX16 + (2 * g) * kMaxItems + i0);
    const float2 xb = *reinterpret_cast<const float2*>(sX16 + (2 * g + 1) * kMaxItems + i0);
    const int z[4] = {0, 0, 0, 0};
    if constexpr (T != LRS_GGML_Q6_K) {
      const uint32_t A[4] = {fa.w0, fb.w0, fa.w1, fb.w1};
      int d[4], e[4];
      mma_k32(d, A, bh0, bh1, z);
      const int c[4] = {d[0] << 8, d[1] << 8, d[2] << 8, d[3] << 8};
      mma_k32(e, A, bl0, bl1, c);
      const float X0 = xa.x + xb.x, X1 = xa.y + xb.y;
      // e[0], e[1]: row gid, items i0, i0+1; e[2], e[3]: row gid+8
      acc[j][0] = fmaf(fa.ds0, s.x * (float)e[0], fmaf(-fa.dm0, X0, acc[j][0]));
      acc[j][1] = fmaf(fa.ds0, s.y * (float)e[1], fmaf(-fa.dm0, X1, acc[j][1]));
      acc[j][2] = fmaf(fb.ds0, s.x * (float)e[2], fmaf(-fb.dm0, X0, acc[j][2]));
      acc[j][3] = fmaf(fb.ds0, s.y * (float)e[3], fmaf(-fb.dm0, X1, acc[j][3]));
    } else {
      {
        const uint32_t A[2] = {fa.w0, fb.w0};
        int d[4], e[4];
        mma_k16(d, A, bh0, z);
        const int c[4] = {d[0] << 8, d[1] << 8, d[2] << 8, d[3] << 8};
        mma_k16(e, A, bl0, c);
        acc[j][0] = fmaf(fa.ds0, s.x * (float)e[0], fmaf(-fa.dm0, xa.x, acc[j][0]));
        acc[j][1] = fmaf(fa.ds0, s.y * (float)e[1], fmaf(-fa.dm0, xa.y, acc[j][1]));
        acc[j][2] = fmaf(fb.ds0, s.x * (float)e[2], fmaf(-fb.dm0, xa.x, acc[j][2]));
        acc[j][3] = fmaf(fb.ds0, s.y * (float)e[3], fmaf(-fb.dm0, xa.y, acc[j][3]));
      }
      {
        const uint32_t A[2] = {fa.w1, fb.w1};
        int d[4], e[4];
        mma_k16(d, A, bh1, z);
        const int c[4] = {d[0] << 8, d[1] << 8, d[2] << 8, d[3] << 8};
        mma_k16(e, A, bl1, c);
        acc[j][0] = fmaf(fa.ds1, s.x * (float)e[0], fmaf(-fa.dm1, xb.x, acc[j][0]));
        acc[j][1] = fmaf(fa.ds1, s.y * (float)e[1], fmaf(-fa.dm1, xb.y, acc[j][1]));
        acc[j][2] = fmaf(fb.ds1, s.x * (float)e[2], fmaf(-fb.dm1, xb.x, acc[j][2]));
        acc[j][3] = fmaf(fb.ds1, s.y * (float)e[3], fmaf(-fb.dm1, xb.y, acc[j][3]));
      }
    }
  }
}

template <int T, bool PAIR>
__global__ void __launch_bounds__(kWarps * 32) gemm_i8_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ unsigned long long skeys[kMaxItems];
  const int B = a.batch;
  const int ntile = (B + 7) >> 3, Bp = ntile * 8;
  int8_t* sxh = reinterpret_cast<int8_t*>(smem);
  int8_t* sxl = sxh + Bp * kXStride;
  float* ssx = reinterpret_cast<float*>(sxl + Bp * kXStride);  // [kKC/32][kMaxItems]
  float* sX16 = ssx + (kKC / 32) * kMaxItems;                   // [kKC/16][kMaxItems]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, t = lane & 3;

  int s = 0;
  while (s + 1 < a.nseg && (int)blockIdx.x >= a.cta0[s + 1]) s++;
  const uint8_t* W = a.seg[s].w;
  const uint8_t* W2 = a.seg[s].w2;
  const int rows = a.seg[s].rows, rb = a.seg[s].rb;
  const int rbase = ((int)blockIdx.x - a.cta0[s]) * kRowsCTA + warp * 16;
  const int ra = min(rbase + gid, rows - 1), rbr = min(rbase + gid + 8, rows - 1);
  const uint8_t* rpa = W + (size_t)ra * rb;
  const uint8_t* rpb = W + (size_t)rbr * rb;
  const uint8_t* upa = PAIR ? W2 + (size_t)ra * rb : nullptr;
  const uint8_t* upb = PAIR ? W2 + (size_t)rbr * rb : nullptr;
  if (tid < kMaxItems) skeys[tid] = 0ull;

  float acc[8][4], acc2[PAIR ? 8 : 1][4];
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[j][c] = 0.0f;
#pragma unroll
  for (int j = 0; j < (PAIR ? 8 : 1); j++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc2[j][c] = 0.0f;

  const int kch = (a.cols + kKC - 1) / kKC;
  const int k0 = blockIdx.y * a.kper, k1 = min(kch, k0 + a.kper);
  for (int kc = k0; kc < k1; kc++) {
    const int c0 = kc * kKC;
    const int ncol = min(kKC, a.cols - c0);
    const int ng = ncol >> 5;
    __syncthreads();
    for (int i = tid; i < Bp * (ncol >> 4); i += kWarps * 32) {
      const int b = i / (ncol >> 4), c = (i % (ncol >> 4)) * 16;
      uint4 vh = make_uint4(0, 0, 0, 0), vl = vh;
      if (b < B) {
        vh = *reinterpret_cast<const uint4*>(a.xh + (size_t)b * a.cols + c0 + c);
        vl = *reinterpret_cast<const uint4*>(a.xl + (size_t)b * a.cols + c0 + c);
      }
      *reinterpret_cast<uint4*>(sxh + b * kXStride + c) = vh;
      *reinterpret_cast<uint4*>(sxl + b * kXStride + c) = vl;
    }
    for (int i = tid; i < Bp * ng; i += kWarps * 32) {
      const int g = i / Bp, b = i % Bp;
      float v = 0.0f, h0 = 0.0f, h1 = 0.0f;
      if (b < B) {
        v = a.sx[(size_t)b * (a.cols >> 5) + (c0 >> 5) + g];
        h0 = a.X16[(size_t)b * (a.cols >> 4) + (c0 >> 4) + 2 * g];
        h1 = a.X16[(size_t)b * (a.cols >> 4) + (c0 >> 4) + 2 * g + 1];
      }
      ssx[g * kMaxItems + b] = v;
      sX16[(2 * g) * kMaxItems + b] = h0;
      sX16[(2 * g + 1) * kMaxItems + b] = h1;
    }
    __syncthreads();
    if (rbase >= rows) continue;
    const int gc0 = c0 >> 5;
    AFrag<T> fa, fb, ua, ub;
    fa.load(rpa, gc0, t);
    fb.load(rpb, gc0, t);
    if constexpr (PAIR) {
      ua.load(upa, gc0, t);
      ub.load(upb, gc0, t);
    }
    for (int g = 0; g < ng; g++) {
      AFrag<T> na, nb, nua, nub;
      const int gn = g + 1 < ng ? g + 1 : g;  // prefetch the next group's codes
      na.load(rpa, gc0 + gn, t);
      nb.load(rpb, gc0 + gn, t);
      if constexpr (PAIR) {
        nua.load(upa, gc0 + gn, t);
        nub.load(upb, gc0 + gn, t);
      }
      group_mma<T>(acc, fa, fb, sxh, sxl, ssx, sX16, g, ntile, gid, t);
      if constexpr (PAIR) group_mma<T>(acc2, ua, ub, sxh, sxl, ssx, sX16, g, ntile, gid, t);
      fa = na;
      fb = nb;
      if constexpr (PAIR) {
        ua = nua;
        ub = nub;
      }
    }
  }

  // ---- output ----
  if (a.kgroups > 1) {
    if (rbase < rows) {
      float* pp = a.part[s] + (size_t)blockIdx.y * B * rows;
      float* pp2 = pp + (size_t)a.kgroups * B * rows;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (j >= ntile) break;
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int i = 8 * j + 2 * t + (c & 1), r = rbase + gid + (c >> 1) * 8;
          if (i < B && r < rows) {
            pp[(size_t)i * rows + r] = acc[j][c];
            if constexpr (PAIR) pp2[(size_t)i * rows + r] = acc2[PAIR ? j : 0][c];
          }
        }
      }
    }
    return;
  }
  const float* bias = a.seg[s].bias;
  float* out = a.seg[s].out;
  const int out_ld = a.seg[s].out_ld;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    if (j >= ntile) break;
    unsigned long long key[2] = {0ull, 0ull};
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int i = 8 * j + 2 * t + (c & 1), r = rbase + gid + (c >> 1) * 8;
      if (i < B && r < rows) {
        float y = acc[j][c];
        float* o = out ? out + (size_t)i * out_ld + r : nullptr;
        if (a.epi == EPI_STORE) {
          if (bias) y += bias[r];
          *o = y;
        } else if (a.epi == EPI_ADD) {
          *o += y;
        } else if (a.epi == EPI_SWIGLU) {
          if constexpr (PAIR) *o = (y / (1.0f + expf(-y))) * acc2[PAIR ? j : 0][c];
        } else {
          if (o) *o = y;
          const unsigned long long k = argmax_pack(y, (uint32_t)r);
          key[c & 1] = k > key[c & 1] ? k : key[c & 1];
        }
      }
    }
    if (a.epi == EPI_ARGMAX) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        unsigned long long k = key[h];
        for (int o = 4; o <= 16; o <<= 1) {
          const unsigned long long v = __shfl_xor_sync(0xffffffffu, k, o);
          k = v > k ? v : k;
        }
        const int i = 8 * j + 2 * t + h;
        if (gid == 0 && i < B && k) atomicMax(&skeys[i], k);
      }
    }
  }
  if (a.epi == EPI_ARGMAX) {
    __syncthreads();
    if (tid < B && skeys[tid]) atomicMax(&a.keys[tid], skeys[tid]);
  }
}

// Adds the K-group partials in a fixed order and applies the epilogue.
struct EpiArgs {
  GemvSeg seg[kGemvMaxSeg];
  const float* part[kGemvMaxSeg];
  int row0[kGemvMaxSeg + 1];
  int nseg, kgroups, batch, epi;
  unsigned long long* keys;
};

__global__ void __launch_bounds__(256) gemm_epilogue_kernel(const __grid_constant__ EpiArgs e) {
  const int b = blockIdx.y;
  const int row = blockIdx.x * 256 + threadIdx.x;
  unsigned long long key = 0ull;
  if (row < e.row0[e.nseg]) {
    int s = 0;
    while (s + 1 < e.nseg && row >= e.row0[s + 1]) s++;
    const int rows = e.seg[s].rows, r = row - e.row0[s];
    const float* pp = e.part[s] + (size_t)b * rows + r;
    const size_t kstride = (size_t)e.batch * rows;
    float y = 0.0f, y2 = 0.0f;
    for (int k = 0; k < e.kgroups; k++) y += pp[k * kstride];
    if (e.epi == EPI_SWIGLU)
      for (int k = 0; k < e.kgroups; k++) y2 += pp[(e.kgroups + k) * kstride];
    float* out = e.seg[s].out;
    float* o = out ? out + (size_t)b * e.seg[s].out_ld + r : nullptr;
    if (e.epi == EPI_STORE) {
      if (e.seg[s].bias) y += e.seg[s].bias[r];
      *o = y;
    } else if (e.epi == EPI_ADD) {
      *o += y;
    } else if (e.epi == EPI_SWIGLU) {
      *o = (y / (1.0f + expf(-y))) * y2;
    } else {
      if (o) *o = y;
      key = argmax_pack(y, (uint32_t)r);
    }
  }
  if (e.epi == EPI_ARGMAX) {
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long v = __shfl_xor_sync(0xffffffffu, key, o);
      key = v > key ? v : key;
    }
    if ((threadIdx.x & 31) == 0 && key) atomicMax(&e.keys[b], key);
  }
}

size_t gemm_smem(int batch) {
  const int Bp = (batch + 7) & ~7;
  return (size_t)Bp * kXStride * 2 + (size_t)(kKC / 32) * kMaxItems * 4 +
         (size_t)(kKC / 16) * kMaxItems * 4;
}

template <int T, bool PAIR>
cudaError_t launch_t(const GemmArgs& a, dim3 grid, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<T, PAIR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)gemm_smem(kMaxItems));
    if (e != cudaSuccess) return e;
    attr = true;
  }
  gemm_i8_kernel<T, PAIR><<<grid, kWarps * 32, gemm_smem(a.batch), st>>>(a);
  return cudaGetLastError();
}

template <bool PAIR>
cudaError_t launch_type(int type, const GemmArgs& a, dim3 grid, cudaStream_t st) {
  switch (type) {
    case LRS_GGML_Q4_0: return launch_t<LRS_GGML_Q4_0, PAIR>(a, grid, st);
    case LRS_GGML_Q4_1: return launch_t<LRS_GGML_Q4_1, PAIR>(a, grid, st);
    case LRS_GGML_Q5_0: return launch_t<LRS_GGML_Q5_0, PAIR>(a, grid, st);
    case LRS_GGML_Q5_1: return launch_t<LRS_GGML_Q5_1, PAIR>(a, grid, st);
    case LRS_GGML_Q8_0: return launch_t<LRS_GGML_Q8_0, PAIR>(a, grid, st);
    case LRS_GGML_Q4_K: return launch_t<LRS_GGML_Q4_K, PAIR>(a, grid, st);
    case LRS_GGML_Q5_K: return launch_t<LRS_GGML_Q5_K, PAIR>(a, grid, st);
    case LRS_GGML_Q6_K: return launch_t<LRS_GGML_Q6_K, PAIR>(a, grid, st);
  }
  return cudaErrorInvalidValue;
}

bool quantized(int type) {
  switch (type) {
    case LRS_GGML_Q4_0: case LRS_GGML_Q4_1: case LRS_GGML_Q5_0: case LRS_GGML_Q5_1:
    case LRS_GGML_Q8_0: case LRS_GGML_Q4_K: case LRS_GGML_Q5_K: case LRS_GGML_Q6_K:
      return true;
  }
  return false;
}

// K groups for a launch of `row_ctas` row CTAs over `kch` chunks: 1 when the
// rows alone give every SM two CTAs, else enough K groups to get there.
int kgroups_for(int row_ctas, int kch, int sms, int* kper) {
  int kg = 1;
  if (row_ctas < 2 * sms) kg = std::min(kch, (2 * sms + row_ctas - 1) / row_ctas);
  *kper = (kch + kg - 1) / kg;
  return (kch + *kper - 1) / *kper;
}

}  // namespace

bool gemm_supported(const GemvParams& p) {
  if (p.batch < 2 || p.cols % 32 || p.norm_w) return false;
  for (int i = 0; i < p.nseg; i++)
    if (!quantized(p.seg[i].type)) return false;
  return true;
}

size_t gemm_scratch_bytes(int batch, int max_cols, int sms) {
  const size_t B = std::min(batch, kMaxItems);
  const size_t xq = (size_t)batch * max_cols * 2 + (size_t)batch * (max_cols / 32) * 4 +
                    (size_t)batch * (max_cols / 16) * 4 + 1024;
  // kgroups > 1 only when row CTAs < 2*sms, and then kgroups * rows is at
  // most (2*sms + row_ctas) * kRowsCTA per matrix of the pair.
  const size_t parts = (size_t)(4 * sms) * kRowsCTA * B * 4 * 2 + 1024;
  return xq + parts;
}

cudaError_t gemm_launch(const GemvParams& p, void* scratch, int sms, cudaStream_t st) {
  const int Ball = p.batch, cols = p.cols;
  const bool pair = p.epi == EPI_SWIGLU;
  const int kch = (cols + kKC - 1) / kKC;
  auto align = [](void* q) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q) + 255) & ~uintptr_t(255));
  };
  int8_t* xh = reinterpret_cast<int8_t*>(align(scratch));
  int8_t* xl = xh + (size_t)Ball * cols;
  float* sx = reinterpret_cast<float*>(align(xl + (size_t)Ball * cols));
  float* X16 = sx + (size_t)Ball * (cols / 32);
  float* part = reinterpret_cast<float*>(align(X16 + (size_t)Ball * (cols / 16)));
  xsplit_kernel<<<dim3((cols / 32 + 7) / 8, Ball), 256, 0, st>>>(p.x, p.x_ld, cols, xh, xl, sx,
                                                                  X16);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  for (int b0 = 0; b0 < Ball; b0 += kMaxItems) {
    const int B = std::min(kMaxItems, Ball - b0);
    // one launch per run of same-type segments
    int i = 0;
    while (i < p.nseg) {
      int j = i + 1;
      while (j < p.nseg && p.seg[j].type == p.seg[i].type) j++;
      GemmArgs a = {};
      a.nseg = j - i;
      a.cols = cols;
      a.batch = B;
      a.epi = p.epi;
      a.xh = xh + (size_t)b0 * cols;
      a.xl = xl + (size_t)b0 * cols;
      a.sx = sx + (size_t)b0 * (cols / 32);
      a.X16 = X16 + (size_t)b0 * (cols / 16);
      a.keys = p.argmax_keys ? p.argmax_keys + b0 : nullptr;
      int ctas = 0;
      for (int k = 0; k < a.nseg; k++) {
        a.seg[k] = p.seg[i + k];
        if (a.seg[k].out) a.seg[k].out += (size_t)b0 * a.seg[k].out_ld;
        a.cta0[k] = ctas;
        ctas += (a.seg[k].rows + kRowsCTA - 1) / kRowsCTA;
      }
      a.cta0[a.nseg] = ctas;
      a.kgroups = kgroups_for(ctas, kch, sms, &a.kper);
      EpiArgs ea = {};
      if (a.kgroups > 1) {
        float* cur = part;
        int row0 = 0;
        for (int k = 0; k < a.nseg; k++) {
          a.part[k] = cur;
          cur += (size_t)a.kgroups * B * a.seg[k].rows * (pair ? 2 : 1);
          ea.seg[k] = a.seg[k];
          ea.part[k] = a.part[k];
          ea.row0[k] = row0;
          row0 += a.seg[k].rows;
        }
        ea.row0[a.nseg] = row0;
        ea.nseg = a.nseg;
        ea.kgroups = a.kgroups;
        ea.batch = B;
        ea.epi = p.epi;
        ea.keys = a.keys;
      }
      const dim3 grid(ctas, a.kgroups);
      e = pair ? launch_type<true>(a.seg[0].type, a, grid, st)
               : launch_type<false>(a.seg[0].type, a, grid, st);
      if (e != cudaSuccess) return e;
      if (a.kgroups > 1) {
        gemm_epilogue_kernel<<<dim3((ea.row0[ea.nseg] + 255) / 256, B), 256, 0, st>>>(ea);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
      }
      i = j;
    }
  }
  return cudaSuccess;
}

}  // namespace lrs

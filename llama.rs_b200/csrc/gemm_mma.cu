// gemm_mma.cu -- batched quantized matmul (decode batches of 2..64 sequences,
// prefill chunks) on the tensor cores of sm_100a (mma.sync m16n8k16,
// f16 x f16 -> f32).
//
// Replaces B independent CpuBackend::matvec calls (src/backend.rs:143-162)
// for B >= 2 input vectors: the sequences of a decode batch, or the prompt
// tokens of a prefill chunk (CausalModel::prefill, src/architecture.rs:60-77,
// runs them one by one).
//
// Every quantized GGML type stores integer codes q with a per-group affine
// map (value_at, src/quant.rs:349-456).  Written as w = ds * (q - z) - dm:
//   Q4_0: ds = d, z = 8         Q4_1: ds = d, dm = -m
//   Q5_0: ds = d, z = 16        Q5_1: ds = d, dm = -m
//   Q8_0: ds = d (signed codes)
//   Q4_K/Q5_K: ds = d*sc, dm = dmin*m per 32 columns
//   Q6_K: ds = d*sc per 16 columns, z = 32
//   F16 / BF16 rows: ds = 1, the weights themselves are the f16 values
// so per group  sum_k w_k x_k = ds * sum_k (q_k - z) x_k - dm * sum_k x_k.
// The codes minus their zero point are small integers, exact in f16; they are
// decoded from the GGML block bytes straight into the A fragments (a code
// byte or nibble OR 0x6400 is the f16 value 1024 + code, minus 1024 + z).
// x is scaled by a power of two per item s (exact; max |x/s| in [2^13, 2^14),
// so the f16 range is never exceeded) and split into xh = f16(x/s) and
// xl = f16(x/s - xh), together about 22 significant bits.  Per group and 8
// items the tensor cores form sum (q - z) xh + sum (q - z) xl in f32 (every
// product exact), and one FMA per element applies ds (plus one for the dm
// term).  The result matches the reference's f32 dot to about 1e-6 relative.
//
// Column order inside a 32-column group: k-step 0 takes columns 0..15, with
// fragment slots (2t, 2t+1) holding columns (4t, 4t+2) and slots (2t+8, 2t+9)
// holding (4t+1, 4t+3); k-step 1 the same for columns 16..31.  That is the
// order in which lane t finds the codes in the 4-byte word it loads, so each
// A register is one mask and one f16 subtraction.  The split x is stored in
// the same order ("fragment order"): per group g and tile j of 8 items, 32
// lane records of 16 bytes for xh then 32 for xl, lane (gid, t) holding
// {x[4t], x[4t+2]}, {x[4t+1], x[4t+3]}, {x[16+4t], x[16+4t+2]},
// {x[16+4t+1], x[16+4t+3]} of item 8j + gid; then per (g, j, t) a float2
// with sum_k x_k / s of items 8j + 2t and 8j + 2t + 1 (the C fragment's
// columns) for the dm term.
//
// Work split: a CTA of 16 warps (8 for a gate/up pair) owns 16 rows per warp
// of one matrix and a run of K chunks of 256 columns.  The split x of the
// chunk is copied to shared memory with cp.async, double-buffered so the next
// chunk lands while this one is multiplied; each warp streams its rows'
// blocks from HBM exactly once, the next group's codes loaded one group
// ahead.  When the row CTAs alone fill the GPU the epilogue (bias, residual
// add, SwiGLU, greedy argmax) runs in the kernel; otherwise K is split across
// CTAs, the partial sums go to scratch and gemm_epilogue_kernel adds them in a
// fixed order, so results never depend on scheduling.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "device_common.cuh"
#include "gemv.cuh"

namespace lrs {
namespace {

constexpr int kGroupsPerChunk = 8;  // 256 columns
constexpr int kChunkCols = 32 * kGroupsPerChunk;
constexpr int kMaxTiles = 8;        // 64 items per launch (larger batches loop)
constexpr int kMaxItems = 8 * kMaxTiles;
constexpr int kXRec = 1024;         // bytes of x records per (group, tile): 32 x 16 (xh) + 32 x 16 (xl)
constexpr int kSRec = 32;           // bytes of sum records per (group, tile): 4 x float2
constexpr int kAhead = 2;           // K chunks of weight rows prefetched into L2 ahead

template <bool PAIR>
struct Shape {
  static constexpr int kWarps = PAIR ? 8 : 16;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kRows = 16 * kWarps;
};

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
__device__ __forceinline__ uint2 ldg64(const uint8_t* p) {
  uint2 v;
  asm("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg16(const uint8_t* p) {
  unsigned short v;
  asm("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
// Four bytes at a 2-byte aligned address (blocks of 18, 22, 34, 210 bytes).
// Branch-free: two aligned words and a funnel shift.
__device__ __forceinline__ uint32_t ldg32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  return __funnelshift_r(ldg32(b), ldg32(b + 4), (uint32_t)(a & 3) * 8);
}
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xffu; }

// f16 pair (1024 + a, 1024 + b) - (1024 + z, 1024 + z) = (a - z, b - z), exact.
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
constexpr uint32_t kF16Base = 0x64006400u;  // f16 pair (1024, 1024)

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- x preparation ---------------------------------------------------------
// One CTA per item (items >= batch, the tile padding, get zero records).
// xq: [groups][tiles][1024 B]; xs: [groups][tiles][4] float2; xscale: [tiles * 8].
__global__ void __launch_bounds__(256)
    xsplit_kernel(const float* x, int x_ld, int cols, int batch, int tiles, uint8_t* xq,
                  float* xs, float* xscale, const float* norm_w, float norm_eps) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* xr = x + (size_t)b * x_ld;
  __shared__ float red[8];
  // fused RMSNorm (RMSNorm::forward, src/model.rs:65-73): x * (inv * w)
  float inv_rms = 1.0f;
  if (norm_w && b < batch) {
    float ss = 0.0f;
    for (int c = threadIdx.x; c < cols; c += 256) ss = fmaf(xr[c], xr[c], ss);
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < 8; k++) tot += red[k];
    inv_rms = 1.0f / sqrtf(tot / (float)cols + norm_eps);
    __syncthreads();
  }
  auto xval = [&](int c) { return norm_w ? xr[c] * (inv_rms * norm_w[c]) : xr[c]; };
  float mx = 0.0f;
  if (b < batch)
    for (int c = threadIdx.x; c < cols; c += 256) mx = fmaxf(mx, fabsf(xval(c)));
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
  // s = 2^(e - 14) with mx = f * 2^e, f in [0.5, 1): max |x / s| in [2^13, 2^14)
  int e = 14;
  if (mx > 0.0f && isfinite(mx)) frexpf(mx, &e);
  const float inv = ldexpf(1.0f, 14 - e);
  if (threadIdx.x == 0) xscale[b] = ldexpf(1.0f, e - 14);
  const int j = b >> 3, gid = b & 7;
  for (int g = warp; g * 32 < cols; g += 8) {
    const float v = b < batch ? xval(g * 32 + lane) * inv : 0.0f;
    const __half h = __float2half_rn(v);
    const __half l = __float2half_rn(v - __half2float(h));
    float sum = v;
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    uint32_t hp = __half_as_ushort(h), lp = __half_as_ushort(l);
    hp |= __shfl_down_sync(0xffffffffu, hp, 2) << 16;  // pair (c, c + 2)
    lp |= __shfl_down_sync(0xffffffffu, lp, 2) << 16;
    if ((lane & 2) == 0) {
      const int ks = lane >> 4, t = (lane & 15) >> 2, bsel = lane & 1;
      uint8_t* rec = xq + ((size_t)g * tiles + j) * kXRec + (gid * 4 + t) * 16 + ks * 8 + bsel * 4;
      *reinterpret_cast<uint32_t*>(rec) = hp;
      *reinterpret_cast<uint32_t*>(rec + 512) = lp;
    }
    if (lane == 0) xs[((size_t)g * tiles + j) * 8 + gid] = sum;
  }
}

// ---- A fragments -------------------------------------------------------------
// For one row (block bytes at rp), 32-column group gc and thread t of the
// quad: h[0], h[1] = k-step 0 slot pairs (columns (4t, 4t+2), (4t+1, 4t+3)),
// h[2], h[3] = k-step 1 (the same + 16), as f16 (q - z); ds0 / ds1 scale the
// two k-steps (equal except for Q6_K) and ndm = -dm (0 where z holds the offset).
template <int T>
struct AFrag {
  static constexpr bool kAffine = T == LRS_GGML_Q4_1 || T == LRS_GGML_Q5_1 ||
                                  T == LRS_GGML_Q4_K || T == LRS_GGML_Q5_K;
  uint32_t h[4];
  float ds0, ds1, ndm;

  __device__ __forceinline__ void nibbles(uint32_t wa, uint32_t wb) {
    h[0] = wa & 0x000F000Fu;
    h[1] = (wa >> 8) & 0x000F000Fu;
    h[2] = wb & 0x000F000Fu;
    h[3] = (wb >> 8) & 0x000F000Fu;
  }
  __device__ __forceinline__ void finish(uint32_t z) {
    const uint32_t zz = kF16Base + z * 0x00010001u;
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = h2sub(h[i] | kF16Base, zz);
  }

  __device__ __forceinline__ void load(const uint8_t* rp, int gc, int t) {
    if constexpr (T == LRS_GGML_Q4_K || T == LRS_GGML_Q5_K) {
      // d, dmin, scales[12], (qh[32]), qs[128]; value_at, src/quant.rs:404-440
      const uint8_t* u = rp + (size_t)(gc >> 3) * BlockTraits<T>::kBytes;
      const int g = gc & 7;
      constexpr int qs0 = T == LRS_GGML_Q4_K ? 16 : 48;
      const uint8_t* q = u + qs0 + 32 * (g >> 1) + 4 * t;
      const int sh = 4 * (g & 1);
      nibbles(ldg32(q) >> sh, ldg32(q + 16) >> sh);
      if constexpr (T == LRS_GGML_Q5_K) {
        const uint32_t ha = (ldg32(u + 16 + 4 * t) >> g) & 0x01010101u;
        const uint32_t hb = (ldg32(u + 32 + 4 * t) >> g) & 0x01010101u;
        h[0] |= (ha & 0x00010001u) << 4;
        h[1] |= (ha & 0x01000100u) >> 4;
        h[2] |= (hb & 0x00010001u) << 4;
        h[3] |= (hb & 0x01000100u) >> 4;
      }
      finish(0);
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
      ndm = -f16_bits((uint16_t)(hd.x >> 16)) * (float)mn;
    } else if constexpr (T == LRS_GGML_Q6_K) {
      // ql[128], qh[64], scales[16] (i8), d; value_at, src/quant.rs:441-456
      const uint8_t* u = rp + (size_t)(gc >> 3) * 210;
      const int gq = gc & 7;
      const int half = gq >> 2, quarter = gq & 3;
      const uint8_t* ql = u + half * 64 + (quarter & 1) * 32 + 4 * t;
      const uint8_t* qh = u + 128 + half * 32 + 4 * t;
      const int nsh = (quarter >> 1) * 4, hsh = 2 * quarter;
      nibbles(ldg32_a2(ql) >> nsh, ldg32_a2(ql + 16) >> nsh);
      const uint32_t ha = (ldg32_a2(qh) >> hsh) & 0x03030303u;
      const uint32_t hb = (ldg32_a2(qh + 16) >> hsh) & 0x03030303u;
      h[0] |= (ha & 0x00030003u) << 4;
      h[1] |= (ha & 0x03000300u) >> 4;
      h[2] |= (hb & 0x00030003u) << 4;
      h[3] |= (hb & 0x03000300u) >> 4;
      finish(32);
      const float d = f16_bits(ldg16(u + 208));
      const uint16_t sp = ldg16(u + 192 + half * 8 + quarter * 2);
      ds0 = d * (float)(int8_t)(sp & 0xffu);
      ds1 = d * (float)(int8_t)(sp >> 8);
      ndm = 0.0f;
    } else if constexpr (T == LRS_GGML_F16 || T == LRS_GGML_BF16) {
      // dense rows: the f16 weights are the A values (ds = 1); a BF16 weight
      // is rounded to f16, exact for |w| in the f16 normal range
      // [2^-14, 65504] (bf16 keeps 8 significant bits, f16 11), within
      // 2^-25 absolute below it
      const uint8_t* u = rp + (size_t)gc * 64;
      const uint2 a = ldg64(u + 8 * t), b = ldg64(u + 32 + 8 * t);
      uint32_t w[4] = {a.x, a.y, b.x, b.y};
      if constexpr (T == LRS_GGML_BF16) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const __half2 hv = __floats2half2_rn(__uint_as_float(w[i] << 16),
                                               __uint_as_float(w[i] & 0xffff0000u));
          w[i] = *reinterpret_cast<const uint32_t*>(&hv);
        }
      }
      h[0] = __byte_perm(w[0], w[1], 0x5410);  // columns (4t, 4t + 2)
      h[1] = __byte_perm(w[0], w[1], 0x7632);  // columns (4t + 1, 4t + 3)
      h[2] = __byte_perm(w[2], w[3], 0x5410);
      h[3] = __byte_perm(w[2], w[3], 0x7632);
      ds0 = ds1 = 1.0f;
      ndm = 0.0f;
    } else if constexpr (T == LRS_GGML_Q8_0) {
      // d, qs[32] (i8); value_at, src/quant.rs:395-400
      const uint8_t* u = rp + (size_t)gc * 34;
      const uint32_t wa = ldg32_a2(u + 2 + 4 * t) ^ 0x80808080u;  // i8 -> u8 = q + 128
      const uint32_t wb = ldg32_a2(u + 18 + 4 * t) ^ 0x80808080u;
      h[0] = __byte_perm(wa, 0x64646464u, 0x4240);
      h[1] = __byte_perm(wa, 0x64646464u, 0x4341);
      h[2] = __byte_perm(wb, 0x64646464u, 0x4240);
      h[3] = __byte_perm(wb, 0x64646464u, 0x4341);
      const uint32_t zz = kF16Base + 128u * 0x00010001u;
#pragma unroll
      for (int i = 0; i < 4; i++) h[i] = h2sub(h[i], zz);
      ds0 = ds1 = f16_bits(ldg16(u));
      ndm = 0.0f;
    } else {
      // 32-value blocks d, (m), (qh[4]), qs[16]; value_at, src/quant.rs:361-394
      const uint8_t* u = rp + (size_t)gc * BlockTraits<T>::kBytes;
      constexpr int qs = T == LRS_GGML_Q4_0 ? 2 : T == LRS_GGML_Q4_1 ? 4 : T == LRS_GGML_Q5_0 ? 6 : 8;
      const uint32_t w = ldg32_a2(u + qs + 4 * t);
      nibbles(w, w >> 4);  // low nibbles: columns 4t..4t+3; high: 16+4t..16+4t+3
      if constexpr (T == LRS_GGML_Q5_0 || T == LRS_GGML_Q5_1) {
        const uint32_t v = ldg32_a2(u + (T == LRS_GGML_Q5_0 ? 2 : 4)) >> (4 * t);
        h[0] |= ((v & 1u) << 4) | ((v & 4u) << 18);
        h[1] |= ((v & 2u) << 3) | ((v & 8u) << 17);
        h[2] |= ((v >> 12) & 0x10u) | ((v & 0x40000u) << 2);
        h[3] |= ((v >> 13) & 0x10u) | ((v & 0x80000u) << 1);
      }
      finish(T == LRS_GGML_Q4_0 ? 8 : T == LRS_GGML_Q5_0 ? 16 : 0);
      ds0 = ds1 = f16_bits(ldg16(u));
      ndm = kAffine ? f16_bits(ldg16(u + 2)) : 0.0f;
    }
  }
};

struct GemmArgs {
  GemvSeg seg[kGemvMaxSeg];
  int cta0[kGemvMaxSeg + 1];  // first row-CTA of each segment
  int nseg, cols, batch, epi, kgroups, tiles;  // tiles: item tiles of the x layout
  const uint8_t* xq;     // records of tile 0 of this launch's items
  const float* xs;
  const float* xscale;   // [batch] power-of-two item scales
  float* part[kGemvMaxSeg];  // [pair][kgroups][batch][rows], kgroups > 1
  unsigned long long* keys;  // [batch], EPI_ARGMAX
  int argmax_base;
};

// Adds one 32-column group of 16 rows x 8*NT items into acc.  Tiles go in
// pairs so that consecutive MMAs are independent.
template <int T, int NT>
__device__ __forceinline__ void group_mma(float (&acc)[NT][4], const AFrag<T>& fa,
                                          const AFrag<T>& fb, const uint4* xr,
                                          const float2* sr) {
  constexpr int JB = NT < 2 ? NT : 2;
#pragma unroll
  for (int j0 = 0; j0 < NT; j0 += JB) {
    float c[JB][4];
    uint4 xh[JB], xl[JB];
#pragma unroll
    for (int jj = 0; jj < JB; jj++) {
      xh[jj] = xr[(j0 + jj) * 64];
      xl[jj] = xr[(j0 + jj) * 64 + 32];
      c[jj][0] = c[jj][1] = c[jj][2] = c[jj][3] = 0.0f;
    }
#pragma unroll
    for (int jj = 0; jj < JB; jj++)
      mma_f16(c[jj], fa.h[0], fb.h[0], fa.h[1], fb.h[1], xh[jj].x, xh[jj].y);
#pragma unroll
    for (int jj = 0; jj < JB; jj++)
      mma_f16(c[jj], fa.h[0], fb.h[0], fa.h[1], fb.h[1], xl[jj].x, xl[jj].y);
    if constexpr (T == LRS_GGML_Q6_K) {
#pragma unroll
      for (int jj = 0; jj < JB; jj++) {
        float* A = acc[j0 + jj];
        A[0] = fmaf(fa.ds0, c[jj][0], A[0]);
        A[1] = fmaf(fa.ds0, c[jj][1], A[1]);
        A[2] = fmaf(fb.ds0, c[jj][2], A[2]);
        A[3] = fmaf(fb.ds0, c[jj][3], A[3]);
        c[jj][0] = c[jj][1] = c[jj][2] = c[jj][3] = 0.0f;
      }
    }
#pragma unroll
    for (int jj = 0; jj < JB; jj++)
      mma_f16(c[jj], fa.h[2], fb.h[2], fa.h[3], fb.h[3], xh[jj].z, xh[jj].w);
#pragma unroll
    for (int jj = 0; jj < JB; jj++)
      mma_f16(c[jj], fa.h[2], fb.h[2], fa.h[3], fb.h[3], xl[jj].z, xl[jj].w);
    // c[0], c[1]: row gid, items 2t, 2t+1; c[2], c[3]: row gid+8
#pragma unroll
    for (int jj = 0; jj < JB; jj++) {
      float* A = acc[j0 + jj];
      if constexpr (AFrag<T>::kAffine) {
        const float2 X = sr[(j0 + jj) * 4];
        A[0] = fmaf(fa.ds1, c[jj][0], fmaf(fa.ndm, X.x, A[0]));
        A[1] = fmaf(fa.ds1, c[jj][1], fmaf(fa.ndm, X.y, A[1]));
        A[2] = fmaf(fb.ds1, c[jj][2], fmaf(fb.ndm, X.x, A[2]));
        A[3] = fmaf(fb.ds1, c[jj][3], fmaf(fb.ndm, X.y, A[3]));
      } else {
        A[0] = fmaf(fa.ds1, c[jj][0], A[0]);
        A[1] = fmaf(fa.ds1, c[jj][1], A[1]);
        A[2] = fmaf(fb.ds1, c[jj][2], A[2]);
        A[3] = fmaf(fb.ds1, c[jj][3], A[3]);
      }
    }
  }
}

// Copies the x records of chunk kc (all NT tiles) into buffer `buf`.
template <int NT, int THREADS>
__device__ __forceinline__ void stage_chunk(const GemmArgs& a, int kc, uint8_t* buf) {
  const int g0 = kc * kGroupsPerChunk;
  const int ng = min(kGroupsPerChunk, a.cols / 32 - g0);
  uint8_t* sx = buf;
  uint8_t* ss = buf + kGroupsPerChunk * NT * kXRec;
  constexpr int kXU = NT * kXRec / 16, kSU = NT * kSRec / 16;  // 16-byte units per group
  for (int i = threadIdx.x; i < ng * (kXU + kSU); i += THREADS) {
    const int g = i / (kXU + kSU), u = i % (kXU + kSU);
    if (u < kXU) {
      cp_async16(sx + (g * kXU + u) * 16,
                 a.xq + ((size_t)(g0 + g) * a.tiles) * kXRec + u * 16);
    } else {
      cp_async16(ss + (g * kSU + (u - kXU)) * 16,
                 reinterpret_cast<const uint8_t*>(a.xs) + ((size_t)(g0 + g) * a.tiles) * kSRec +
                     (u - kXU) * 16);
    }
  }
}

template <int T, bool PAIR, int NT>
__global__ void __launch_bounds__(Shape<PAIR>::kThreads)
    gemm_mma_kernel(const __grid_constant__ GemmArgs a) {
  using S = Shape<PAIR>;
  constexpr int kBuf = kGroupsPerChunk * NT * (kXRec + kSRec);
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ unsigned long long skeys[kMaxItems];
  const int B = a.batch;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, t = lane & 3;

  int s = 0;
  while (s + 1 < a.nseg && (int)blockIdx.x >= a.cta0[s + 1]) s++;
  const uint8_t* W = a.seg[s].w;
  const uint8_t* W2 = a.seg[s].w2;
  const int rows = a.seg[s].rows, rb = a.seg[s].rb;
  const int rbase = ((int)blockIdx.x - a.cta0[s]) * S::kRows + warp * 16;
  const int ra = min(rbase + gid, rows - 1), rbr = min(rbase + gid + 8, rows - 1);
  const uint8_t* rpa = W + (size_t)ra * rb;
  const uint8_t* rpb = W + (size_t)rbr * rb;
  const uint8_t* upa = PAIR ? W2 + (size_t)ra * rb : nullptr;
  const uint8_t* upb = PAIR ? W2 + (size_t)rbr * rb : nullptr;
  const bool active = rbase < rows;
  if (tid < kMaxItems) skeys[tid] = 0ull;

  float acc[NT][4], acc2[PAIR ? NT : 1][4];
#pragma unroll
  for (int j = 0; j < NT; j++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[j][c] = 0.0f;
#pragma unroll
  for (int j = 0; j < (PAIR ? NT : 1); j++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc2[j][c] = 0.0f;

  const int kch = (a.cols + kChunkCols - 1) / kChunkCols;
  const int k0 = (int)((long long)blockIdx.y * kch / a.kgroups);
  const int k1 = (int)((long long)(blockIdx.y + 1) * kch / a.kgroups);
  const int gend = min(k1 * kGroupsPerChunk, a.cols / 32);
  stage_chunk<NT, S::kThreads>(a, k0, smem);
  cp_async_commit();

  // L2 prefetch of this warp's rows, chunks k0 .. k0 + kAhead - 1 now and
  // chunk kc + kAhead when chunk kc starts: the code loads then hit L2.
  // bytes of one row per 256-column chunk (the last chunk may be shorter)
  constexpr int rbc = BlockTraits<T>::kBytes * (kChunkCols / BlockTraits<T>::kValues);
  auto prefetch_rows = [&](int kc) {
    if (!active || kc >= k1) return;
    const int nbytes = kc + 1 < kch ? rbc : rb - kc * rbc;
    const int lines = (nbytes + 127) / 128 + 1;
    for (int i = lane; i < 16 * lines * (PAIR ? 2 : 1); i += 32) {
      const int r = i % 16, l = (i / 16) % lines, m = i / (16 * lines);
      const int row = min(rbase + r, rows - 1);
      const uint8_t* base = (m ? W2 : W) + (size_t)row * rb + (size_t)kc * rbc;
      const uint8_t* line = base + min(l * 128, nbytes - 1);
      asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
  };
  for (int k = 0; k < kAhead; k++) prefetch_rows(k0 + k);

  AFrag<T> fa, fb, ua, ub;
  int gc = k0 * kGroupsPerChunk;
  if (active) {
    fa.load(rpa, gc, t);
    fb.load(rpb, gc, t);
    if constexpr (PAIR) {
      ua.load(upa, gc, t);
      ub.load(upb, gc, t);
    }
  }
  for (int kc = k0; kc < k1; kc++) {
    uint8_t* buf = smem + ((kc - k0) & 1) * kBuf;
    if (kc + 1 < k1) {
      stage_chunk<NT, S::kThreads>(a, kc + 1, smem + ((kc + 1 - k0) & 1) * kBuf);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    prefetch_rows(kc + kAhead);
    const int ng = min(kGroupsPerChunk, a.cols / 32 - kc * kGroupsPerChunk);
    if (active) {
      const uint4* xr = reinterpret_cast<const uint4*>(buf) + lane;
      const float2* sr = reinterpret_cast<const float2*>(buf + kGroupsPerChunk * NT * kXRec) + t;
#pragma unroll
      for (int g = 0; g < kGroupsPerChunk; g++, gc++) {
        if (g >= ng) break;
        AFrag<T> na, nb, nua, nub;
        const int gn = gc + 1 < gend ? gc + 1 : gc;  // next group's codes, one group ahead
        na.load(rpa, gn, t);
        nb.load(rpb, gn, t);
        if constexpr (PAIR) {
          nua.load(upa, gn, t);
          nub.load(upb, gn, t);
        }
        group_mma<T, NT>(acc, fa, fb, xr + g * NT * 64, sr + g * NT * 4);
        if constexpr (PAIR) group_mma<T, NT>(acc2, ua, ub, xr + g * NT * 64, sr + g * NT * 4);
        fa = na;
        fb = nb;
        if constexpr (PAIR) {
          ua = nua;
          ub = nub;
        }
      }
    }
    __syncthreads();  // buffer kc is refilled by iteration kc + 1's stage of kc + 2
  }

  // undo the item scales (powers of two: exact)
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const float2 sc = *reinterpret_cast<const float2*>(a.xscale + 8 * j + 2 * t);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      acc[j][c] *= (c & 1) ? sc.y : sc.x;
      if constexpr (PAIR) acc2[PAIR ? j : 0][c] *= (c & 1) ? sc.y : sc.x;
    }
  }

  // ---- output ----
  if (a.kgroups > 1) {
    if (active) {
      float* pp = a.part[s] + (size_t)blockIdx.y * B * rows;
      float* pp2 = pp + (size_t)a.kgroups * B * rows;
#pragma unroll
      for (int j = 0; j < NT; j++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int i = 8 * j + 2 * t + (c & 1), r = rbase + gid + (c >> 1) * 8;
          if (i < B && r < rows) {
            pp[(size_t)i * rows + r] = acc[j][c];
            if constexpr (PAIR) pp2[(size_t)i * rows + r] = acc2[PAIR ? j : 0][c];
          }
        }
    }
    return;
  }
  const float* bias = a.seg[s].bias;
  float* out = a.seg[s].out;
  const int out_ld = a.seg[s].out_ld;
#pragma unroll
  for (int j = 0; j < NT; j++) {
    unsigned long long key[2] = {0ull, 0ull};
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int i = 8 * j + 2 * t + (c & 1), r = rbase + gid + (c >> 1) * 8;
      if (active && i < B && r < rows) {
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
          const unsigned long long k = argmax_pack(y, (uint32_t)(r + a.argmax_base));
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
  int nseg, kgroups, batch, epi, argmax_base;
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
      key = argmax_pack(y, (uint32_t)(r + e.argmax_base));
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

template <int NT>
constexpr size_t smem_for() {
  return 2 * (size_t)kGroupsPerChunk * NT * (kXRec + kSRec);
}

template <int T, bool PAIR, int NT>
cudaError_t launch_t(const GemmArgs& a, dim3 grid, cudaStream_t st) {
  static std::atomic<uint64_t> attr{0};
  cudaError_t e = set_smem_once(attr, (const void*)gemm_mma_kernel<T, PAIR, NT>, (int)smem_for<NT>());
  if (e != cudaSuccess) return e;
  gemm_mma_kernel<T, PAIR, NT><<<grid, Shape<PAIR>::kThreads, smem_for<NT>(), st>>>(a);
  return cudaGetLastError();
}

template <int T, bool PAIR>
cudaError_t launch_nt(int nt, const GemmArgs& a, dim3 grid, cudaStream_t st) {
  switch (nt) {
    case 1: return launch_t<T, PAIR, 1>(a, grid, st);
    case 2: return launch_t<T, PAIR, 2>(a, grid, st);
    case 4: return launch_t<T, PAIR, 4>(a, grid, st);
    default: return launch_t<T, PAIR, 8>(a, grid, st);
  }
}

template <bool PAIR>
cudaError_t launch_type(int type, int nt, const GemmArgs& a, dim3 grid, cudaStream_t st) {
  switch (type) {
    case LRS_GGML_Q4_0: return launch_nt<LRS_GGML_Q4_0, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q4_1: return launch_nt<LRS_GGML_Q4_1, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q5_0: return launch_nt<LRS_GGML_Q5_0, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q5_1: return launch_nt<LRS_GGML_Q5_1, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q8_0: return launch_nt<LRS_GGML_Q8_0, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q4_K: return launch_nt<LRS_GGML_Q4_K, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q5_K: return launch_nt<LRS_GGML_Q5_K, PAIR>(nt, a, grid, st);
    case LRS_GGML_Q6_K: return launch_nt<LRS_GGML_Q6_K, PAIR>(nt, a, grid, st);
    case LRS_GGML_F16: return launch_nt<LRS_GGML_F16, PAIR>(nt, a, grid, st);
    case LRS_GGML_BF16: return launch_nt<LRS_GGML_BF16, PAIR>(nt, a, grid, st);
  }
  return cudaErrorInvalidValue;
}

// Types with an A-fragment decoder: every quantized type, and F16 / BF16 rows.
bool mma_type(int type) {
  switch (type) {
    case LRS_GGML_Q4_0: case LRS_GGML_Q4_1: case LRS_GGML_Q5_0: case LRS_GGML_Q5_1:
    case LRS_GGML_Q8_0: case LRS_GGML_Q4_K: case LRS_GGML_Q5_K: case LRS_GGML_Q6_K:
    case LRS_GGML_F16: case LRS_GGML_BF16:
      return true;
  }
  return false;
}

int tiles_for(int items) {  // item tiles of one launch: 1, 2, 4 or 8
  const int need = (items + 7) / 8;
  return need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : 8;
}

// Tiles of the split-x layout for `batch` items: 8 per full 64-item block
// plus the last block's (padded) tile count.
int layout_tiles(int batch) {
  const int full = (batch - 1) / kMaxItems;
  return full * kMaxTiles + tiles_for(batch - full * kMaxItems);
}

}  // namespace

bool gemm_supported(const GemvParams& p) {
  if (p.batch < 2 || p.cols % 32) return false;
  for (int i = 0; i < p.nseg; i++)
    if (!mma_type(p.seg[i].type)) return false;
  return true;
}

size_t gemm_scratch_bytes(int batch, int max_cols, int sms) {
  const size_t tiles = layout_tiles(std::max(batch, 1));
  const size_t xq = (size_t)(max_cols / 32) * tiles * (kXRec + kSRec) + tiles * 32 + 1024;
  // kgroups > 1 only when the row CTAs do not fill the SMs; then kgroups *
  // rows <= 2 * sms * 256 for a launch (a pair has half the rows of a CTA).
  const size_t parts = (size_t)(2 * sms) * 256 * std::min(batch, kMaxItems) * 4 + 1024;
  return xq + parts;
}

cudaError_t gemm_partials_epilogue(const GemvParams& p, const float* const* parts, int kgroups,
                                   cudaStream_t st) {
  EpiArgs ea = {};
  int row0 = 0;
  for (int k = 0; k < p.nseg; k++) {
    ea.seg[k] = p.seg[k];
    ea.part[k] = parts[k];
    ea.row0[k] = row0;
    row0 += p.seg[k].rows;
  }
  ea.row0[p.nseg] = row0;
  ea.nseg = p.nseg;
  ea.kgroups = kgroups;
  ea.batch = p.batch;
  ea.epi = p.epi;
  ea.keys = p.argmax_keys;
  ea.argmax_base = p.argmax_base;
  gemm_epilogue_kernel<<<dim3((row0 + 255) / 256, p.batch), 256, 0, st>>>(ea);
  return cudaGetLastError();
}

cudaError_t gemm_launch(const GemvParams& p, void* scratch, int sms, cudaStream_t st) {
  const int Ball = p.batch, cols = p.cols;
  const bool pair = p.epi == EPI_SWIGLU;
  const int kch = (cols + kChunkCols - 1) / kChunkCols;
  const int tiles = layout_tiles(Ball);
  auto align = [](void* q) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q) + 255) & ~uintptr_t(255));
  };
  uint8_t* xq = align(scratch);
  float* xs = reinterpret_cast<float*>(xq + (size_t)(cols / 32) * tiles * kXRec);
  float* xscale = reinterpret_cast<float*>(
      align(reinterpret_cast<uint8_t*>(xs) + (size_t)(cols / 32) * tiles * kSRec));
  float* part = reinterpret_cast<float*>(align(xscale + tiles * 8));
  xsplit_kernel<<<tiles * 8, 256, 0, st>>>(p.x, p.x_ld, cols, Ball, tiles, xq, xs, xscale,
                                            p.norm_w, p.norm_eps);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int rows_cta = pair ? Shape<true>::kRows : Shape<false>::kRows;
  for (int b0 = 0; b0 < Ball; b0 += kMaxItems) {
    const int B = std::min(kMaxItems, Ball - b0);
    const int nt = tiles_for(B);
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
      a.tiles = tiles;
      a.xq = xq + (size_t)(b0 / 8) * kXRec;
      a.xs = xs + (size_t)(b0 / 8) * (kSRec / 4);
      a.xscale = xscale + b0;
      a.keys = p.argmax_keys ? p.argmax_keys + b0 : nullptr;
      a.argmax_base = p.argmax_base;
      int ctas = 0;
      for (int k = 0; k < a.nseg; k++) {
        a.seg[k] = p.seg[i + k];
        if (a.seg[k].out) a.seg[k].out += (size_t)b0 * a.seg[k].out_ld;
        a.cta0[k] = ctas;
        ctas += (a.seg[k].rows + rows_cta - 1) / rows_cta;
      }
      a.cta0[a.nseg] = ctas;
      // one wave: at most `sms` CTAs (one resident CTA per SM)
      a.kgroups = ctas >= sms ? 1 : std::min(kch, sms / ctas);
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
        ea.argmax_base = p.argmax_base;
      }
      const dim3 grid(ctas, a.kgroups);
      e = pair ? launch_type<true>(a.seg[0].type, nt, a, grid, st)
               : launch_type<false>(a.seg[0].type, nt, a, grid, st);
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

// gemv_fast.cuh -- per-type piece loaders and factored dots for the batch-1 GEMV.
//
// The reference multiplies every dequantized weight by x (dot_row_scalar,
// src/quant.rs:458-648), ~7 GPU instructions per weight: twice what HBM
// bandwidth leaves.  Here the same dot is computed in factored form: per group
// of values sharing a scale,
//     sum_k w_k x_k = scale * sum_k q_k x_k + offset * sum_k x_k,
// with sum_k x_k precomputed per 8-column run.  The default path
// (gemv5_kernel, gemv.cu) takes sum_k q_k x_k in integers: x is split per
// 8-column run as x ~= s_r * (xh + xl / 256) with int8 halves (about 15
// bits), and every 4 codes meet their x bytes in one dp4a (hi and lo sums
// exact in int32, (hi << 8) + lo), then one float multiply per run
// (icode / finish_i below).  Agreement with the reference dot is ~1e-5
// relative (the parity bar is 1e-3).  Dense types multiply float x directly
// with packed fma.rn.f32x2 (weights / finish).  icode and finish_i are built on
// code_word (the 4 codes of a word) and finish (the scales applied to per-group
// sums).
//
// A "piece" is the unit one lane handles: 64 values (a group pair) for
// Q4_K/Q5_K, 32 values otherwise.  load() reads its bytes straight from global
// memory (or shared memory) into registers; icode(i) / code_word(i) yield 4
// codes for x columns col(sub, i)..+3; finish_i() / finish() apply the scales.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "device_common.cuh"

namespace lrs {
namespace fast {

typedef unsigned long long f2;  // two f32 in one 64-bit register

__device__ __forceinline__ f2 pk(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float hsum2(f2 v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return a + b;
}
__device__ __forceinline__ void fma2(f2& acc, f2 a, f2 b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
// The same product-sum as fma2 with two scalar fma.rn.f32.
__device__ __forceinline__ void fma1(f2& acc, f2 a, f2 b) {
  float a0, a1, b0, b1, c0, c1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(b0), "=f"(b1) : "l"(b));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(c0), "=f"(c1) : "l"(acc));
  acc = pk(fmaf(a0, b0, c0), fmaf(a1, b1, c1));
}
__device__ __forceinline__ void add2(f2& acc, f2 a) {
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc) : "l"(a));
}
// Byte k (< 128) of w as the float 0.5 + byte/256.
__device__ __forceinline__ float fq(uint32_t w, int k) {
  return __int_as_float(__byte_perm(w, 0x3F000000u, 0x7044u | ((uint32_t)k << 8)));
}
// Byte k of w as the float 2^23 + byte (exact).
__device__ __forceinline__ float fq23(uint32_t w, int k) {
  return __int_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)k));
}
__device__ __forceinline__ float h2f_lo(uint32_t w) { return f16_bits((uint16_t)(w & 0xffff)); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return f16_bits((uint16_t)(w >> 16)); }
// Spreads the low 4 bits of b to bit 4 of each byte.
__device__ __forceinline__ uint32_t spread4(uint32_t b) {
  return ((b & 15u) * 0x00204081u & 0x01010101u) << 4;
}

// ---- loads (global with SM = false, shared memory with SM = true) --------
template <bool SM>
__device__ __forceinline__ uint32_t ld32(const uint8_t* p) {
  if constexpr (SM) return *reinterpret_cast<const uint32_t*>(p);
  uint32_t v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
template <bool SM>
__device__ __forceinline__ uint4 ld128(const uint8_t* p) {
  if constexpr (SM) return *reinterpret_cast<const uint4*>(p);
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
template <bool SM>
__device__ __forceinline__ uint2 ld64(const uint8_t* p) {
  if constexpr (SM) return *reinterpret_cast<const uint2*>(p);
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
// N little-endian words of the bytes at p (p at least 2-byte aligned).
template <bool SM, int N>
__device__ __forceinline__ void ld_words(const uint8_t* p, uint32_t* w) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 2) * 8;
  uint32_t r[N + 1];
#pragma unroll
  for (int i = 0; i <= N; i++) r[i] = ld32<SM>(b + 4 * i);
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// ---- per-type pieces -------------------------------------------------------
// kValues: values per piece; kWords: 4-value code words; kGroups: scale groups.
template <int T>
struct Piece;

// Q4_0 / Q4_1 / Q5_0 / Q5_1: one 32-value block (src/quant.rs:357-398).
// Word i < 4: low nibbles of qs bytes 4i..4i+3 (columns 4i..); i >= 4: high
// nibbles (columns 16 + 4(i-4)..) -- i.e. column 4i for every i.
template <int T>
struct Piece32Block {
  static constexpr int kValues = 32, kWords = 8, kGroups = 1, kPieces = 1;
  static constexpr bool kFive = T == LRS_GGML_Q5_0 || T == LRS_GGML_Q5_1;
  static constexpr bool kAffine = T == LRS_GGML_Q4_1 || T == LRS_GGML_Q5_1;
  float d, m;
  uint32_t qh, qs[4];
  template <bool SM>
  __device__ __forceinline__ void load(const uint8_t* u, int) {
    if constexpr (T == LRS_GGML_Q4_0) {  // 18 bytes, 2-aligned: d, qs[16]
      uint32_t w[5];
      ld_words<SM, 5>(u, w);
      d = h2f_lo(w[0]);
#pragma unroll
      for (int i = 0; i < 4; i++) qs[i] = __funnelshift_r(w[i], w[i + 1], 16);
    } else if constexpr (T == LRS_GGML_Q4_1) {  // 20 bytes, 4-aligned: d, m, qs[16]
      const uint32_t h = ld32<SM>(u);
      d = h2f_lo(h);
      m = h2f_hi(h);
#pragma unroll
      for (int i = 0; i < 4; i++) qs[i] = ld32<SM>(u + 4 + 4 * i);
    } else if constexpr (T == LRS_GGML_Q5_0) {  // 22 bytes, 2-aligned: d, qh[4], qs[16]
      uint32_t w[6];
      ld_words<SM, 6>(u, w);
      d = h2f_lo(w[0]);
      qh = __funnelshift_r(w[0], w[1], 16);
#pragma unroll
      for (int i = 0; i < 4; i++) qs[i] = __funnelshift_r(w[1 + i], w[2 + i], 16);
    } else {  // Q5_1: 24 bytes, 8-aligned: d, m, qh[4], qs[16]
      const uint2 a = ld64<SM>(u), b = ld64<SM>(u + 8), c = ld64<SM>(u + 16);
      d = h2f_lo(a.x);
      m = h2f_hi(a.x);
      qh = a.y;
      qs[0] = b.x, qs[1] = b.y, qs[2] = c.x, qs[3] = c.y;
    }
  }
  __device__ __forceinline__ static int col(int, int i) { return 4 * i; }
  __device__ __forceinline__ static int group(int) { return 0; }
  __device__ __forceinline__ uint32_t icode(int i, int s) const { return code_word(i, s); }
  // qx[r]: sum over run r (8 columns) of code * x
  __device__ __forceinline__ float finish_i(const float* qx, const float* X8, int) const {
    const float xs = (X8[0] + X8[1]) + (X8[2] + X8[3]);
    const float t = (qx[0] + qx[1]) + (qx[2] + qx[3]);
    if constexpr (kAffine) return d * t + m * xs;
    return d * (t - (kFive ? 16.0f : 8.0f) * xs);
  }
  __device__ __forceinline__ uint32_t code_word(int i, int) const {
    const uint32_t q = i < 4 ? (qs[i] & 0x0F0F0F0Fu) : ((qs[i - 4] >> 4) & 0x0F0F0F0Fu);
    if constexpr (kFive) return q | spread4(qh >> (4 * i));
    return q;
  }
  // xsum: sum of x over the piece's 32 columns
  __device__ __forceinline__ float finish(const float* S, const float* X8, int) const {
    const float xs = (X8[0] + X8[1]) + (X8[2] + X8[3]);
    const float off = kFive ? 16.0f : 8.0f;
    if constexpr (kAffine) return d * (256.0f * S[0] - 128.0f * xs) + m * xs;
    return d * (256.0f * S[0] - (128.0f + off) * xs);
  }
};
template <>
struct Piece<LRS_GGML_Q4_0> : Piece32Block<LRS_GGML_Q4_0> {};
template <>
struct Piece<LRS_GGML_Q4_1> : Piece32Block<LRS_GGML_Q4_1> {};
template <>
struct Piece<LRS_GGML_Q5_0> : Piece32Block<LRS_GGML_Q5_0> {};
template <>
struct Piece<LRS_GGML_Q5_1> : Piece32Block<LRS_GGML_Q5_1> {};

// Q8_0: 34 bytes, 2-aligned: d, qs[32] signed (src/quant.rs:399-402).  Codes
// are signed: handled by the caller through kSigned.
template <>
struct Piece<LRS_GGML_Q8_0> {
  static constexpr int kValues = 32, kWords = 8, kGroups = 1, kPieces = 1;
  float d;
  uint32_t qs[8];
  template <bool SM>
  __device__ __forceinline__ void load(const uint8_t* u, int) {
    uint32_t w[9];
    ld_words<SM, 9>(u, w);
    d = h2f_lo(w[0]);
#pragma unroll
    for (int i = 0; i < 8; i++) qs[i] = __funnelshift_r(w[i], w[i + 1], 16);
  }
  __device__ __forceinline__ static int col(int, int i) { return 4 * i; }
  __device__ __forceinline__ static int group(int) { return 0; }
  __device__ __forceinline__ uint32_t code_word(int i, int) const { return qs[i] ^ 0x80808080u; }
  __device__ __forceinline__ uint32_t icode(int i, int) const { return qs[i]; }  // signed bytes
  __device__ __forceinline__ float finish_i(const float* qx, const float*, int) const {
    return d * ((qx[0] + qx[1]) + (qx[2] + qx[3]));
  }
  __device__ __forceinline__ float finish(const float* S, const float*, int) const { return d * S[0]; }
};

// Q4_K / Q5_K: piece = group pair p (64 values): d*sc*q - dmin*m
// (src/quant.rs:403-436).  Word i < 8: low nibbles of qs[32p + 4i ..]
// (group 2p, columns 4i..); i >= 8: high nibbles (group 2p+1, columns 32 + 4(i-8)..).
template <int T>
struct PieceK4 {
  static constexpr int kValues = 64, kWords = 16, kGroups = 2, kPieces = 4;
  static constexpr bool kFive = T == LRS_GGML_Q5_K;
  uint32_t hd[4];  // d|dmin, scales[0..11]
  uint32_t q[8], h[8];
  template <bool SM>
  __device__ __forceinline__ void load(const uint8_t* u, int p) {
    const uint4 hdr = ld128<SM>(u);
    hd[0] = hdr.x, hd[1] = hdr.y, hd[2] = hdr.z, hd[3] = hdr.w;
    const int qs0 = kFive ? 48 : 16;
    const uint4 a = ld128<SM>(u + qs0 + 32 * p), b = ld128<SM>(u + qs0 + 32 * p + 16);
    q[0] = a.x, q[1] = a.y, q[2] = a.z, q[3] = a.w, q[4] = b.x, q[5] = b.y, q[6] = b.z,
    q[7] = b.w;
    if constexpr (kFive) {
      const uint4 c = ld128<SM>(u + 16), e = ld128<SM>(u + 32);
      h[0] = c.x, h[1] = c.y, h[2] = c.z, h[3] = c.w, h[4] = e.x, h[5] = e.y, h[6] = e.z,
      h[7] = e.w;
    }
  }
  __device__ __forceinline__ static int col(int p, int i) { return p * 64 + 4 * i; }
  __device__ __forceinline__ static int group(int i) { return i >> 3; }
  __device__ __forceinline__ uint32_t icode(int i, int p) const { return code_word(i, p); }
  __device__ __forceinline__ float finish_i(const float* qx, const float* X8, int p) const {
    float S[2];
    S[0] = ((qx[0] + qx[1]) + (qx[2] + qx[3])) * (1.0f / 256.0f) +
           0.5f * ((X8[0] + X8[1]) + (X8[2] + X8[3]));
    S[1] = ((qx[4] + qx[5]) + (qx[6] + qx[7])) * (1.0f / 256.0f) +
           0.5f * ((X8[4] + X8[5]) + (X8[6] + X8[7]));
    return finish(S, X8, p);
  }
  __device__ __forceinline__ uint32_t code_word(int i, int p) const {
    const int k = i & 7;
    uint32_t c = i < 8 ? (q[k] & 0x0F0F0F0Fu) : ((q[k] >> 4) & 0x0F0F0F0Fu);
    if constexpr (kFive) c |= ((h[k] >> (2 * p + (i >> 3))) & 0x01010101u) << 4;
    return c;
  }
  // scale_min_k4 (src/quant.rs:338-347): scales[0..3] = hd[1], [4..7] = hd[2], [8..11] = hd[3].
  // Group pair p: p < 2 -> groups 2p, 2p+1 < 4; p >= 2 -> both >= 4.
  __device__ __forceinline__ float finish(const float* S, const float* X8, int p) const {
    const uint32_t sh = 16 * (p & 1);  // byte offset 2(p&1) within the word
    const uint32_t w0 = hd[1] >> sh, w1 = hd[2] >> sh, w2 = hd[3] >> sh;
    uint32_t sc0, sc1, mn0, mn1;
    if (p < 2) {
      sc0 = w0 & 63, sc1 = (w0 >> 8) & 63, mn0 = w1 & 63, mn1 = (w1 >> 8) & 63;
    } else {
      sc0 = (w2 & 0x0f) | ((w0 >> 2) & 0x30), sc1 = ((w2 >> 8) & 0x0f) | ((w0 >> 10) & 0x30);
      mn0 = ((w2 >> 4) & 0x0f) | ((w1 >> 2) & 0x30), mn1 = ((w2 >> 12) & 0x0f) | ((w1 >> 10) & 0x30);
    }
    const float x0 = (X8[0] + X8[1]) + (X8[2] + X8[3]);
    const float x1 = (X8[4] + X8[5]) + (X8[6] + X8[7]);
    const float qx0 = 256.0f * S[0] - 128.0f * x0, qx1 = 256.0f * S[1] - 128.0f * x1;
    return h2f_lo(hd[0]) * ((float)sc0 * qx0 + (float)sc1 * qx1) -
           h2f_hi(hd[0]) * ((float)mn0 * x0 + (float)mn1 * x1);
  }
};
template <>
struct Piece<LRS_GGML_Q4_K> : PieceK4<LRS_GGML_Q4_K> {};
template <>
struct Piece<LRS_GGML_Q5_K> : PieceK4<LRS_GGML_Q5_K> {};

// Q6_K: piece (half, octet) = 32 values {half*128 + q*32 + oct*8 + i}
// (src/quant.rs:437-454): d * sc_q * (code - 32);  sum (code-32) x =
// 256 S - 160 X per quarter q.  Word i: quarter i/2, lanes oct*8 + 4(i%2)..
template <>
struct Piece<LRS_GGML_Q6_K> {
  static constexpr int kValues = 32, kWords = 8, kGroups = 4, kPieces = 8;
  float d, sc[4];
  uint32_t la[2], lb[2], hb[2];
  template <bool SM>
  __device__ __forceinline__ void load(const uint8_t* u, int sub) {
    const int half = sub >> 2, oct = sub & 3;
    ld_words<SM, 2>(u + half * 64 + oct * 8, la);
    ld_words<SM, 2>(u + half * 64 + 32 + oct * 8, lb);
    ld_words<SM, 2>(u + 128 + half * 32 + oct * 8, hb);
    uint32_t s[2], dw[1];
    ld_words<SM, 2>(u + 192 + half * 8, s);
    ld_words<SM, 1>(u + 208, dw);
    d = h2f_lo(dw[0]);
    const int so = oct >> 1;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int si = 2 * q + so;
      const uint32_t sw = si < 4 ? s[0] : s[1];
      sc[q] = (float)(int8_t)((sw >> (8 * (si & 3))) & 0xff);
    }
  }
  __device__ __forceinline__ static int col(int sub, int i) {
    return (sub >> 2) * 128 + (i >> 1) * 32 + (sub & 3) * 8 + 4 * (i & 1);
  }
  __device__ __forceinline__ static int group(int i) { return i >> 1; }
  __device__ __forceinline__ uint32_t icode(int i, int s) const { return code_word(i, s); }
  __device__ __forceinline__ float finish_i(const float* qx, const float* X8, int) const {
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; q++) acc += sc[q] * (qx[q] - 32.0f * X8[q]);
    return d * acc;
  }
  __device__ __forceinline__ uint32_t code_word(int i, int) const {
    const int r = i >> 1, k = i & 1;
    const uint32_t l = (r & 1) ? lb[k] : la[k];
    return ((l >> ((r >> 1) * 4)) & 0x0F0F0F0Fu) | (((hb[k] >> (2 * r)) & 0x03030303u) << 4);
  }
  __device__ __forceinline__ float finish(const float* S, const float* X8, int) const {
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; q++) acc += sc[q] * (256.0f * S[q] - 160.0f * X8[q]);
    return d * acc;
  }
};

// Dense types: 32 consecutive columns, floats used directly.
template <int T>
struct PieceDense {
  static constexpr int kValues = 32, kWords = 8, kGroups = 1, kPieces = 1;
  uint32_t v[T == LRS_GGML_F32 ? 32 : 16];
  template <bool SM>
  __device__ __forceinline__ void load(const uint8_t* u, int) {
    constexpr int n16 = T == LRS_GGML_F32 ? 8 : 4;
#pragma unroll
    for (int i = 0; i < n16; i++) {
      const uint4 a = ld128<SM>(u + 16 * i);
      v[4 * i] = a.x, v[4 * i + 1] = a.y, v[4 * i + 2] = a.z, v[4 * i + 3] = a.w;
    }
  }
  __device__ __forceinline__ static int col(int, int i) { return 4 * i; }
  __device__ __forceinline__ static int group(int) { return 0; }
  __device__ __forceinline__ uint32_t code_word(int i, int) const { return v[i]; }
  // the 4 weights of word i
  __device__ __forceinline__ void weights(int i, f2& a, f2& b) const {
    if constexpr (T == LRS_GGML_F32) {
      a = pk(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]));
      b = pk(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
    } else if constexpr (T == LRS_GGML_F16) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&v[2 * i]));
      const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&v[2 * i + 1]));
      a = pk(x.x, x.y);
      b = pk(y.x, y.y);
    } else {
      a = pk(__uint_as_float(v[2 * i] << 16), __uint_as_float(v[2 * i] & 0xffff0000u));
      b = pk(__uint_as_float(v[2 * i + 1] << 16), __uint_as_float(v[2 * i + 1] & 0xffff0000u));
    }
  }
  __device__ __forceinline__ float finish(const float* S, const float*, int) const { return S[0]; }
};
template <>
struct Piece<LRS_GGML_F32> : PieceDense<LRS_GGML_F32> {};
template <>
struct Piece<LRS_GGML_F16> : PieceDense<LRS_GGML_F16> {};
template <>
struct Piece<LRS_GGML_BF16> : PieceDense<LRS_GGML_BF16> {};

}  // namespace fast
// ---- x prepared for the factored dots -------------------------------------
// Each 8-column run r of x (after the optional RMSNorm) is split as
//     x ~= s_r * (xh + xl / 256),  xh, xl int8,  s_r = max|x_run| / 127,
// (about 15 bits of x; the dot's error is ~1e-5 relative) together with the
// exact float sum X_r of the run.  The layout is piece-transposed: 16-byte
// chunk k of piece p sits at (k * npieces + p) * 16, so the lanes of a warp,
// which handle consecutive pieces, read consecutive chunks.  Dense types
// (F32/F16/BF16) keep float x, piece-major.
template <int T>
struct XLayout {
  using P = fast::Piece<T>;
  static constexpr bool kDense = T == LRS_GGML_F32 || T == LRS_GGML_F16 || T == LRS_GGML_BF16;
  static constexpr int PV = P::kValues;        // values per piece
  static constexpr int NRUN = PV / 8;          // 8-column runs per piece
  static constexpr int CH = PV / 16;           // 16-byte chunks of xh (and of xl) per piece
  // bytes of the staged x for `npieces` pieces
  __host__ __device__ static size_t bytes(int npieces) {
    if constexpr (kDense) return (size_t)npieces * PV * 4;
    return (size_t)npieces * (2 * CH * 16 + NRUN * 8);
  }
};

// Views of the staged x at xq for `npieces` pieces.
template <int T>
struct XView {
  using XL = XLayout<T>;
  uint4* xh4;  // [CH][npieces]
  uint4* xl4;  // [CH][npieces]
  float* sxa;  // [NRUN][npieces]: s_r / 256
  float* Xa;   // [NRUN][npieces]: X_r
  float* xf;   // dense: [npieces][PV]
  __device__ __forceinline__ XView(uint8_t* xq, int npieces) {
    xh4 = reinterpret_cast<uint4*>(xq);
    xl4 = xh4 + (size_t)XL::CH * npieces;
    sxa = reinterpret_cast<float*>(xl4 + (size_t)XL::CH * npieces);
    Xa = sxa + (size_t)XL::NRUN * npieces;
    xf = reinterpret_cast<float*>(xq);
  }
};

// Stages x (cols values; RMSNorm::forward of src/model.rs:65-73 first when
// norm_w is set) at xq in the XLayout of type T.  NT threads take part (tid in
// [0, NT)); `sync()` is their barrier; red holds NT / 32 floats.  Ends with a
// sync, so xq is ready for all NT threads on return.
template <int T, int NT, class Sync>
__device__ __forceinline__ void prep_x(const float* x, const float* norm_w, float norm_eps, int cols,
                                       uint8_t* xq, float* red, int tid, Sync sync) {
  using BT = BlockTraits<T>;
  using P = fast::Piece<T>;
  using XL = XLayout<T>;
  constexpr int PV = XL::PV, NRUN = XL::NRUN;
  const int lane = tid & 31, warp = tid >> 5;
  const int npieces = cols / PV;
  XView<T> xv(xq, npieces);
  float inv_rms = 1.0f;
  if (norm_w) {
    float ss = 0.0f;
    for (int c = tid; c < cols; c += NT) ss = fmaf(x[c], x[c], ss);
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    sync();
    float tot = 0.0f;
    for (int w = 0; w < NT / 32; w++) tot += red[w];
    inv_rms = 1.0f / sqrtf(tot / (float)cols + norm_eps);
  }
  // One thread per (piece, run): gather the run's 8 values, normalize, split.
  for (int t = tid; t < npieces * NRUN; t += NT) {
    const int pc = t % npieces, r = t / npieces;
    const int unit = pc / P::kPieces, sub = pc % P::kPieces;
    const int col = unit * BT::kValues + P::col(sub, 2 * r);
    float v[8];
    const float4 a = *reinterpret_cast<const float4*>(x + col);
    const float4 b = *reinterpret_cast<const float4*>(x + col + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    if (norm_w) {
      const float4 wa = *reinterpret_cast<const float4*>(norm_w + col);
      const float4 wb = *reinterpret_cast<const float4*>(norm_w + col + 4);
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int c = 0; c < 8; c++) v[c] = v[c] * (inv_rms * w[c]);
    }
    if constexpr (XL::kDense) {
#pragma unroll
      for (int c = 0; c < 8; c++) xv.xf[(size_t)pc * PV + 8 * r + c] = v[c];
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
      uint32_t* hc = reinterpret_cast<uint32_t*>(xv.xh4 + (size_t)(r >> 1) * npieces + pc) + 2 * (r & 1);
      uint32_t* lc = reinterpret_cast<uint32_t*>(xv.xl4 + (size_t)(r >> 1) * npieces + pc) + 2 * (r & 1);
      hc[0] = hw[0], hc[1] = hw[1];
      lc[0] = lw[0], lc[1] = lw[1];
      xv.sxa[(size_t)r * npieces + pc] = sc * (1.0f / 256.0f);
      xv.Xa[(size_t)r * npieces + pc] = sum;
    }
  }
  sync();
}

}  // namespace lrs

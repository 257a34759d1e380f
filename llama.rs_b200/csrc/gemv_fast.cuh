// gemv_fast.cuh -- factored per-type piece dots for the batch-1 GEMV.
//
// The reference multiplies every dequantized weight by x (dot_row_scalar,
// src/quant.rs:458-648).  On the GPU that costs ~7 instructions per weight,
// twice what HBM bandwidth leaves.  These routines compute the same dot in
// factored form: per group of values sharing a scale,
//     sum_k w_k x_k = scale * sum_k q_k x_k + offset * sum_k x_k,
// where sum_k x_k comes precomputed per 8-column run (xs8) and sum_k q_k x_k is
// accumulated from codes turned into floats with one byte-permute each:
// a code q < 128 placed in bits 16..22 of 0x3F000000 is the float
// f = 0.5 + q/256 exactly, so  sum q x = 256 * sum f x - 128 * sum x.
// Products accumulate with packed fma.rn.f32x2.  The result agrees with the
// reference dot to ~1e-6 relative (the parity bar is 1e-3).
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
__device__ __forceinline__ void add2(f2& acc, f2 a) {
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc) : "l"(a));
}
// Byte k (< 128) of w as the float 0.5 + byte/256.
__device__ __forceinline__ float fq(uint32_t w, int k) {
  return __int_as_float(__byte_perm(w, 0x3F000000u, 0x7044u | ((uint32_t)k << 8)));
}
// Byte k of w as the float 2^23 + byte (exact), for signed codes.
__device__ __forceinline__ float fq23(uint32_t w, int k) {
  return __int_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)k));
}
// sum over 4 codes (bytes of w, each < 128) of f(code) * x[0..3]
__device__ __forceinline__ void dot4(f2& acc, uint32_t w, const float* x) {
  fma2(acc, pk(fq(w, 0), fq(w, 1)), pk(x[0], x[1]));
  fma2(acc, pk(fq(w, 2), fq(w, 3)), pk(x[2], x[3]));
}
// Realigned little-endian words of the bytes at p (p 2-byte aligned, shared memory).
template <int N>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t* w) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  uint32_t r[N + 1];
#pragma unroll
  for (int i = 0; i <= N; i++) r[i] = b[i];
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}
__device__ __forceinline__ float h2f_lo(uint32_t w) { return f16_bits((uint16_t)(w & 0xffff)); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return f16_bits((uint16_t)(w >> 16)); }
// Spreads the low 4 bits of b to bit 4 of each byte.
__device__ __forceinline__ uint32_t spread4(uint32_t b) {
  return ((b & 15u) * 0x00204081u & 0x01010101u) << 4;
}

// ---- per-type traits: values per piece, pieces per unit -------------------
template <int T>
struct Piece {
  static constexpr int kValues = 32;
};
template <>
struct Piece<LRS_GGML_Q4_K> {
  static constexpr int kValues = 64;
};
template <>
struct Piece<LRS_GGML_Q5_K> {
  static constexpr int kValues = 64;
};
template <int T>
__host__ __device__ constexpr int pieces_per_unit() {
  return BlockTraits<T>::kValues / Piece<T>::kValues;
}

// Column (within the unit) of the 8-wide run r of piece `sub`; the x
// registers of a piece are run-major, 8 per run.
template <int T>
__device__ __forceinline__ int run_col(int sub, int r) {
  if constexpr (T == LRS_GGML_Q6_K) return (sub >> 2) * 128 + r * 32 + (sub & 3) * 8;
  else return sub * Piece<T>::kValues + r * 8;
}

// Contribution of one piece of one row.  u = the unit (block) in shared
// memory, x = the piece's x values (run-major), X = the piece's 8-run sums.
template <int T>
__device__ __forceinline__ float piece_dot(const uint8_t* u, int sub, const float* x,
                                           const float* X);

// Q4_0: d * (q - 8); sum (q-8) x = 256 S - 136 X   (value_at, src/quant.rs:357-366)
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q4_0>(const uint8_t* u, int, const float* x,
                                                          const float* X) {
  uint32_t w[5];
  load_words<5>(u, w);  // bytes 0..19: d, qs[16]
  const float d = h2f_lo(w[0]);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16);
    dot4(s, q & 0x0F0F0F0Fu, x + 4 * i);
    dot4(s, (q >> 4) & 0x0F0F0F0Fu, x + 16 + 4 * i);
  }
  const float xs = (X[0] + X[1]) + (X[2] + X[3]);
  return d * (256.0f * hsum2(s) - 136.0f * xs);
}

// Q4_1: d * q + m; sum = d (256 S - 128 X) + m X   (src/quant.rs:367-376)
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q4_1>(const uint8_t* u, int, const float* x,
                                                          const float* X) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(u);  // 4-byte aligned (20-byte blocks)
  const uint32_t h = p[0];
  const float d = h2f_lo(h), m = h2f_hi(h);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = p[1 + i];
    dot4(s, q & 0x0F0F0F0Fu, x + 4 * i);
    dot4(s, (q >> 4) & 0x0F0F0F0Fu, x + 16 + 4 * i);
  }
  const float xs = (X[0] + X[1]) + (X[2] + X[3]);
  return d * (256.0f * hsum2(s) - 128.0f * xs) + m * xs;
}

// Q5_0: d * (q - 16); sum = 256 S - 144 X   (src/quant.rs:377-398)
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q5_0>(const uint8_t* u, int, const float* x,
                                                          const float* X) {
  uint32_t w[6];
  load_words<6>(u, w);  // bytes 0..23: d, qh[4], qs[16]
  const float d = h2f_lo(w[0]);
  const uint32_t qh = __funnelshift_r(w[0], w[1], 16);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = __funnelshift_r(w[1 + i], w[2 + i], 16);
    dot4(s, (q & 0x0F0F0F0Fu) | spread4(qh >> (4 * i)), x + 4 * i);
    dot4(s, ((q >> 4) & 0x0F0F0F0Fu) | spread4(qh >> (16 + 4 * i)), x + 16 + 4 * i);
  }
  const float xs = (X[0] + X[1]) + (X[2] + X[3]);
  return d * (256.0f * hsum2(s) - 144.0f * xs);
}

// Q5_1: d * q + m   (src/quant.rs:377-398)
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q5_1>(const uint8_t* u, int, const float* x,
                                                          const float* X) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(u);  // 8-byte aligned (24-byte blocks)
  const float d = h2f_lo(p[0]), m = h2f_hi(p[0]);
  const uint32_t qh = p[1];
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = p[2 + i];
    dot4(s, (q & 0x0F0F0F0Fu) | spread4(qh >> (4 * i)), x + 4 * i);
    dot4(s, ((q >> 4) & 0x0F0F0F0Fu) | spread4(qh >> (16 + 4 * i)), x + 16 + 4 * i);
  }
  const float xs = (X[0] + X[1]) + (X[2] + X[3]);
  return d * (256.0f * hsum2(s) - 128.0f * xs) + m * xs;
}

// Q8_0: d * q with signed q: byte ^ 0x80 placed under exponent 2^23 gives
// 2^23 + 128 + q exactly; subtracting 2^23 + 128 recovers q.   (src/quant.rs:399-402)
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q8_0>(const uint8_t* u, int, const float* x,
                                                          const float*) {
  uint32_t w[9];
  load_words<9>(u, w);  // bytes 0..35: d, qs[32]
  const float d = h2f_lo(w[0]);
  const f2 bias = pk(-8388736.0f, -8388736.0f);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16) ^ 0x80808080u;
    f2 a = pk(fq23(q, 0), fq23(q, 1)), b = pk(fq23(q, 2), fq23(q, 3));
    add2(a, bias);
    add2(b, bias);
    fma2(s, a, pk(x[4 * i], x[4 * i + 1]));
    fma2(s, b, pk(x[4 * i + 2], x[4 * i + 3]));
  }
  return d * hsum2(s);
}

// Q4_K / Q5_K pair piece p (groups 2p, 2p+1): d*sc*q - dmin*m   (src/quant.rs:403-436)
template <int HIGHBITS>
__device__ __forceinline__ float k4_pair(const uint8_t* u, int p, const float* x, const float* X) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(u);  // d, dmin, scales[12]
  const float d = h2f_lo(hdr.x), dmin = h2f_hi(hdr.x);
  // scale_min_k4 (src/quant.rs:338-347) on scales[0..3] = hdr.y, [4..7] = hdr.z, [8..11] = hdr.w
  float sc[2], mn[2];
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int g = 2 * p + k;
    const int j = g & 3;
    const uint32_t b0 = (hdr.y >> (8 * j)) & 0xff, b1 = (hdr.z >> (8 * j)) & 0xff;
    const uint32_t b2 = (hdr.w >> (8 * j)) & 0xff;
    uint32_t a, b;
    if (g < 4) {
      a = b0 & 63;
      b = b1 & 63;
    } else {
      a = (b2 & 0x0f) | ((b0 >> 6) << 4);
      b = (b2 >> 4) | ((b1 >> 6) << 4);
    }
    sc[k] = (float)a;
    mn[k] = (float)b;
  }
  const int qs0 = HIGHBITS ? 48 : 16;
  const uint4 q0 = *reinterpret_cast<const uint4*>(u + qs0 + 32 * p);
  const uint4 q1 = *reinterpret_cast<const uint4*>(u + qs0 + 32 * p + 16);
  const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  uint32_t h[8];
  if (HIGHBITS) {
    const uint4 h0 = *reinterpret_cast<const uint4*>(u + 16);
    const uint4 h1 = *reinterpret_cast<const uint4*>(u + 32);
    h[0] = h0.x, h[1] = h0.y, h[2] = h0.z, h[3] = h0.w;
    h[4] = h1.x, h[5] = h1.y, h[6] = h1.z, h[7] = h1.w;
  }
  f2 slo = 0, shi = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    uint32_t lo = q[i] & 0x0F0F0F0Fu, hi = (q[i] >> 4) & 0x0F0F0F0Fu;
    if (HIGHBITS) {
      lo |= ((h[i] >> (2 * p)) & 0x01010101u) << 4;
      hi |= ((h[i] >> (2 * p + 1)) & 0x01010101u) << 4;
    }
    dot4(slo, lo, x + 4 * i);
    dot4(shi, hi, x + 32 + 4 * i);
  }
  const float x0 = (X[0] + X[1]) + (X[2] + X[3]);
  const float x1 = (X[4] + X[5]) + (X[6] + X[7]);
  const float qx0 = 256.0f * hsum2(slo) - 128.0f * x0;
  const float qx1 = 256.0f * hsum2(shi) - 128.0f * x1;
  return d * (sc[0] * qx0 + sc[1] * qx1) - dmin * (mn[0] * x0 + mn[1] * x1);
}
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q4_K>(const uint8_t* u, int p, const float* x,
                                                          const float* X) {
  return k4_pair<0>(u, p, x, X);
}
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q5_K>(const uint8_t* u, int p, const float* x,
                                                          const float* X) {
  return k4_pair<1>(u, p, x, X);
}

// Q6_K piece (half, octet): d * sc * (q - 32);  sum (q-32) x = 256 S - 160 X
// per 8-value run (one scale each).   (src/quant.rs:437-454)
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_Q6_K>(const uint8_t* u, int sub,
                                                          const float* x, const float* X) {
  const int half = sub >> 2, oct = sub & 3;
  uint32_t la[2], lb[2], hb[2], dw[1], sca[1], scb[1];
  load_words<2>(u + half * 64 + oct * 8, la);
  load_words<2>(u + half * 64 + 32 + oct * 8, lb);
  load_words<2>(u + 128 + half * 32 + oct * 8, hb);
  load_words<1>(u + 208, dw);
  load_words<1>(u + 192 + half * 8, sca);  // scales of the half, bytes 0..3
  load_words<1>(u + 196 + half * 8, scb);  // bytes 4..7
  const float d = h2f_lo(dw[0]);
  const int so = oct >> 1;
  float acc = 0.0f;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const uint32_t* l = (r & 1) ? lb : la;
    const int nsh = (r >> 1) * 4;
    f2 s = 0;
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const uint32_t q = ((l[k] >> nsh) & 0x0F0F0F0Fu) | (((hb[k] >> (2 * r)) & 0x03030303u) << 4);
      dot4(s, q, x + r * 8 + 4 * k);
    }
    const int si = r * 2 + so;  // scale index within the half
    const uint32_t sb = si < 4 ? (sca[0] >> (8 * si)) : (scb[0] >> (8 * (si - 4)));
    const float scv = (float)(int8_t)(sb & 0xff);
    acc += scv * (256.0f * hsum2(s) - 160.0f * X[r]);
  }
  return d * acc;
}

// Dense types: piece = 32 consecutive columns.
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_F32>(const uint8_t* u, int sub, const float* x,
                                                         const float*) {
  const float4* p = reinterpret_cast<const float4*>(u + sub * 128);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float4 v = p[i];
    fma2(s, pk(v.x, v.y), pk(x[4 * i], x[4 * i + 1]));
    fma2(s, pk(v.z, v.w), pk(x[4 * i + 2], x[4 * i + 3]));
  }
  return hsum2(s);
}
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_F16>(const uint8_t* u, int sub, const float* x,
                                                         const float*) {
  const uint4* p = reinterpret_cast<const uint4*>(u + sub * 64);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint4 v = p[i];
    const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&a[k]));
      fma2(s, pk(f.x, f.y), pk(x[8 * i + 2 * k], x[8 * i + 2 * k + 1]));
    }
  }
  return hsum2(s);
}
template <>
__device__ __forceinline__ float piece_dot<LRS_GGML_BF16>(const uint8_t* u, int sub,
                                                          const float* x, const float*) {
  const uint4* p = reinterpret_cast<const uint4*>(u + sub * 64);
  f2 s = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint4 v = p[i];
    const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; k++)
      fma2(s, pk(__uint_as_float(a[k] << 16), __uint_as_float(a[k] & 0xffff0000u)),
           pk(x[8 * i + 2 * k], x[8 * i + 2 * k + 1]));
  }
  return hsum2(s);
}

}  // namespace fast
}  // namespace lrs

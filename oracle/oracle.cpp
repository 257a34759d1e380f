// oracle.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// CPU restatement of llama.rs's scalar token loop.  Every function cites the
// reference file:line it follows.  Compiled with -O2 -ffp-contract=off and no
// fast-math so that f32 arithmetic is unfused and evaluated in the written
// order, as Rust evaluates it.
#include "oracle.h"

#include <immintrin.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <memory>
#include <vector>

#include "pool.h"

namespace {

thread_local std::string g_err;

// --- f16 / bf16 -> f32 (exact), half::f16::to_f32 / bf16::to_f32 ----------
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while ((man & 0x400) == 0);
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
float bf16_to_f32(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
// read_f16 / read_bf16, src/quant.rs:326-332
inline float read_f16(const uint8_t* b, size_t off) { return f16_to_f32(rd16(b + off)); }
inline float read_bf16(const uint8_t* b, size_t off) { return bf16_to_f32(rd16(b + off)); }

bool geometry(uint32_t t, uint32_t* bv, uint32_t* bb) {
  // QuantType::block_size / type_size, src/quant.rs:46-67
  switch (t) {
    case LRS_GGML_F32: *bv = 1; *bb = 4; return true;
    case LRS_GGML_F16: case LRS_GGML_BF16: *bv = 1; *bb = 2; return true;
    case LRS_GGML_Q4_0: *bv = 32; *bb = 18; return true;
    case LRS_GGML_Q4_1: *bv = 32; *bb = 20; return true;
    case LRS_GGML_Q5_0: *bv = 32; *bb = 22; return true;
    case LRS_GGML_Q5_1: *bv = 32; *bb = 24; return true;
    case LRS_GGML_Q8_0: *bv = 32; *bb = 34; return true;
    case LRS_GGML_Q4_K: *bv = 256; *bb = 144; return true;
    case LRS_GGML_Q5_K: *bv = 256; *bb = 176; return true;
    case LRS_GGML_Q6_K: *bv = 256; *bb = 210; return true;
  }
  return false;
}
size_t row_bytes(uint32_t t, size_t cols) {
  uint32_t bv, bb;
  geometry(t, &bv, &bb);
  return cols / bv * bb;
}

// scale_min_k4, src/quant.rs:338-347
inline void scale_min_k4(int i, const uint8_t* s, uint8_t* sc, uint8_t* mn) {
  if (i < 4) {
    *sc = s[i] & 63;
    *mn = s[i + 4] & 63;
  } else {
    *sc = (uint8_t)((s[i + 4] & 0x0f) | ((s[i - 4] >> 6) << 4));
    *mn = (uint8_t)((s[i + 4] >> 4) | ((s[i] >> 6) << 4));
  }
}

// value_at, src/quant.rs:349-456
float value_at(const uint8_t* row, uint32_t ty, size_t col) {
  switch (ty) {
    case LRS_GGML_F32: {
      float f;
      memcpy(&f, row + col * 4, 4);
      return f;
    }
    case LRS_GGML_F16: return read_f16(row, col * 2);
    case LRS_GGML_BF16: return read_bf16(row, col * 2);
    case LRS_GGML_Q4_0: {
      const uint8_t* b = row + col / 32 * 18;
      size_t j = col % 32;
      uint8_t q = j < 16 ? (b[2 + j] & 0x0f) : (b[2 + j - 16] >> 4);
      return read_f16(b, 0) * ((float)q - 8.0f);
    }
    case LRS_GGML_Q4_1: {
      const uint8_t* b = row + col / 32 * 20;
      size_t j = col % 32;
      uint8_t q = j < 16 ? (b[4 + j] & 0x0f) : (b[4 + j - 16] >> 4);
      return read_f16(b, 0) * (float)q + read_f16(b, 2);
    }
    case LRS_GGML_Q5_0:
    case LRS_GGML_Q5_1: {
      size_t bs = ty == LRS_GGML_Q5_0 ? 22 : 24;
      const uint8_t* b = row + col / 32 * bs;
      size_t j = col % 32;
      size_t qh_off = ty == LRS_GGML_Q5_0 ? 2 : 4, qs_off = ty == LRS_GGML_Q5_0 ? 6 : 8;
      uint8_t low = j < 16 ? (b[qs_off + j] & 0x0f) : (b[qs_off + j - 16] >> 4);
      uint8_t high = (b[qh_off + j / 8] >> (j % 8)) & 1;
      uint8_t q = low | (uint8_t)(high << 4);
      if (ty == LRS_GGML_Q5_0) return read_f16(b, 0) * ((float)q - 16.0f);
      return read_f16(b, 0) * (float)q + read_f16(b, 2);
    }
    case LRS_GGML_Q8_0: {
      const uint8_t* b = row + col / 32 * 34;
      return read_f16(b, 0) * (float)(int8_t)b[2 + col % 32];
    }
    case LRS_GGML_Q4_K: {
      const uint8_t* b = row + col / 256 * 144;
      size_t j = col % 256;
      int group = (int)(j / 32);
      uint8_t sc, mn;
      scale_min_k4(group, b + 4, &sc, &mn);
      uint8_t packed = b[16 + (group / 2) * 32 + j % 32];
      uint8_t q = (group % 2 == 0) ? (packed & 0x0f) : (packed >> 4);
      return read_f16(b, 0) * (float)sc * (float)q - read_f16(b, 2) * (float)mn;
    }
    case LRS_GGML_Q5_K: {
      const uint8_t* b = row + col / 256 * 176;
      size_t j = col % 256;
      int group = (int)(j / 32);
      uint8_t sc, mn;
      scale_min_k4(group, b + 4, &sc, &mn);
      uint8_t packed = b[48 + group / 2 * 32 + j % 32];
      uint8_t low = (group % 2 == 0) ? (packed & 0x0f) : (packed >> 4);
      uint8_t mask = (uint8_t)(1u << group);
      uint8_t high = (b[16 + j % 32] & mask) ? 16 : 0;
      return read_f16(b, 0) * (float)sc * (float)(low + high) - read_f16(b, 2) * (float)mn;
    }
    case LRS_GGML_Q6_K: {
      const uint8_t* b = row + col / 256 * 210;
      size_t j = col % 256;
      size_t half = j / 128, within = j % 128, lane = within % 32, quarter = within / 32;
      uint8_t ql;
      switch (quarter) {
        case 0: ql = b[half * 64 + lane] & 0x0f; break;
        case 1: ql = b[half * 64 + 32 + lane] & 0x0f; break;
        case 2: ql = b[half * 64 + lane] >> 4; break;
        default: ql = b[half * 64 + 32 + lane] >> 4; break;
      }
      uint8_t qh = (b[128 + half * 32 + lane] >> (quarter * 2)) & 3;
      float q = (float)((int16_t)(ql | (qh << 4)) - 32);
      float scale = (float)(int8_t)b[192 + half * 8 + quarter * 2 + lane / 16];
      return read_f16(b, 208) * scale * q;
    }
  }
  return 0.0f;
}

// dot_q4k, src/quant.rs:569-593
float dot_q4k(const uint8_t* row, size_t nb, const float* input) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 144;
    float d = read_f16(b, 0), dmin = read_f16(b, 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    const float* x = input + bi * 256;
    for (int g = 0; g < 8; g++) {
      uint8_t sc, mn;
      scale_min_k4(g, scales, &sc, &mn);
      float ds = d * (float)sc, dm = dmin * (float)mn;
      for (int j = 0; j < 32; j++) {
        uint8_t packed = qs[g / 2 * 32 + j];
        uint8_t q = (g % 2 == 0) ? (packed & 0x0f) : (packed >> 4);
        sum += (ds * (float)q - dm) * x[g * 32 + j];
      }
    }
  }
  return sum;
}

// dot_q5k, src/quant.rs:595-622
float dot_q5k(const uint8_t* row, size_t nb, const float* input) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 176;
    float d = read_f16(b, 0), dmin = read_f16(b, 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    const float* x = input + bi * 256;
    for (int g = 0; g < 8; g++) {
      uint8_t sc, mn;
      scale_min_k4(g, scales, &sc, &mn);
      float ds = d * (float)sc, dm = dmin * (float)mn;
      uint8_t mask = (uint8_t)(1u << g);
      for (int j = 0; j < 32; j++) {
        uint8_t packed = qs[g / 2 * 32 + j];
        uint8_t low = (g % 2 == 0) ? (packed & 0x0f) : (packed >> 4);
        uint8_t q = low + ((qh[j] & mask) ? 16 : 0);
        sum += (ds * (float)q - dm) * x[g * 32 + j];
      }
    }
  }
  return sum;
}

// dot_q6k, src/quant.rs:624-648
float dot_q6k(const uint8_t* row, size_t nb, const float* input) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 210;
    float d = read_f16(b, 208);
    const float* x = input + bi * 256;
    for (int half = 0; half < 2; half++) {
      const uint8_t* ql = b + half * 64;
      const uint8_t* qh = b + 128 + half * 32;
      const uint8_t* sc = b + 192 + half * 8;
      int base = half * 128;
      for (int lane = 0; lane < 32; lane++) {
        int si = lane / 16;
        int16_t q1 = (int16_t)((ql[lane] & 0x0f) | ((qh[lane] & 3) << 4)) - 32;
        int16_t q2 = (int16_t)((ql[32 + lane] & 0x0f) | (((qh[lane] >> 2) & 3) << 4)) - 32;
        int16_t q3 = (int16_t)((ql[lane] >> 4) | (((qh[lane] >> 4) & 3) << 4)) - 32;
        int16_t q4 = (int16_t)((ql[32 + lane] >> 4) | (((qh[lane] >> 6) & 3) << 4)) - 32;
        sum += d * (float)(int8_t)sc[si] * (float)q1 * x[base + lane];
        sum += d * (float)(int8_t)sc[si + 2] * (float)q2 * x[base + 32 + lane];
        sum += d * (float)(int8_t)sc[si + 4] * (float)q3 * x[base + 64 + lane];
        sum += d * (float)(int8_t)sc[si + 6] * (float)q4 * x[base + 96 + lane];
      }
    }
  }
  return sum;
}

// dot_row_scalar, src/quant.rs:458-554
float dot_row_scalar(const uint8_t* row, uint32_t ty, const float* input, size_t cols) {
  switch (ty) {
    case LRS_GGML_F32: {
      float sum = 0.0f;
      for (size_t i = 0; i < cols; i++) {
        float w;
        memcpy(&w, row + i * 4, 4);
        sum += w * input[i];
      }
      return sum;
    }
    case LRS_GGML_F16: {
      float sum = 0.0f;
      for (size_t i = 0; i < cols; i++) sum += read_f16(row, i * 2) * input[i];
      return sum;
    }
    case LRS_GGML_BF16: {
      float sum = 0.0f;
      for (size_t i = 0; i < cols; i++) sum += read_bf16(row, i * 2) * input[i];
      return sum;
    }
    case LRS_GGML_Q4_0: {
      float sum = 0.0f;
      for (size_t bi = 0; bi < cols / 32; bi++) {
        const uint8_t* b = row + bi * 18;
        float d = read_f16(b, 0);
        const float* x = input + bi * 32;
        for (int j = 0; j < 16; j++) {
          uint8_t q = b[2 + j];
          sum += d * ((float)(q & 0x0f) - 8.0f) * x[j];
          sum += d * ((float)(q >> 4) - 8.0f) * x[j + 16];
        }
      }
      return sum;
    }
    case LRS_GGML_Q4_1: {
      float sum = 0.0f;
      for (size_t bi = 0; bi < cols / 32; bi++) {
        const uint8_t* b = row + bi * 20;
        float d = read_f16(b, 0), m = read_f16(b, 2);
        const float* x = input + bi * 32;
        for (int j = 0; j < 16; j++) {
          uint8_t q = b[4 + j];
          sum += (d * (float)(q & 0x0f) + m) * x[j];
          sum += (d * (float)(q >> 4) + m) * x[j + 16];
        }
      }
      return sum;
    }
    case LRS_GGML_Q5_0:
    case LRS_GGML_Q5_1: {
      float sum = 0.0f;
      bool q50 = ty == LRS_GGML_Q5_0;
      size_t size = q50 ? 22 : 24;
      for (size_t bi = 0; bi < cols / 32; bi++) {
        const uint8_t* b = row + bi * size;
        float d = read_f16(b, 0);
        float m = q50 ? 0.0f : read_f16(b, 2);
        size_t qh_off = q50 ? 2 : 4, qs_off = q50 ? 6 : 8;
        uint32_t qh = (uint32_t)b[qh_off] | ((uint32_t)b[qh_off + 1] << 8) |
                      ((uint32_t)b[qh_off + 2] << 16) | ((uint32_t)b[qh_off + 3] << 24);
        const float* x = input + bi * 32;
        for (int j = 0; j < 16; j++) {
          uint8_t packed = b[qs_off + j];
          uint32_t q0 = (uint32_t)(packed & 0x0f) | (((qh >> j) & 1) << 4);
          uint32_t q1 = (uint32_t)(packed >> 4) | (((qh >> (j + 16)) & 1) << 4);
          if (q50) {
            sum += d * ((float)q0 - 16.0f) * x[j];
            sum += d * ((float)q1 - 16.0f) * x[j + 16];
          } else {
            sum += (d * (float)q0 + m) * x[j];
            sum += (d * (float)q1 + m) * x[j + 16];
          }
        }
      }
      return sum;
    }
    case LRS_GGML_Q8_0: {
      float sum = 0.0f;
      for (size_t bi = 0; bi < cols / 32; bi++) {
        const uint8_t* b = row + bi * 34;
        float d = read_f16(b, 0);
        const float* x = input + bi * 32;
        for (int j = 0; j < 32; j++) sum += d * (float)(int8_t)b[2 + j] * x[j];
      }
      return sum;
    }
    case LRS_GGML_Q4_K: return dot_q4k(row, cols / 256, input);
    case LRS_GGML_Q5_K: return dot_q5k(row, cols / 256, input);
    case LRS_GGML_Q6_K: return dot_q6k(row, cols / 256, input);
  }
  return 0.0f;
}

// ---- AVX2 restatement of src/simd.rs (the timed CPU baseline) -------------
// hsum, src/simd.rs:11-19
__attribute__((target("avx2,fma"))) inline float hsum(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 s = _mm_add_ps(lo, hi);
  s = _mm_hadd_ps(s, s);
  s = _mm_hadd_ps(s, s);
  return _mm_cvtss_f32(s);
}
__attribute__((target("avx2,fma"))) inline __m256i bytes8_to_i32(const uint8_t* p) {
  return _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i*)p));
}
__attribute__((target("avx2,fma"))) inline __m256i i8x8_to_i32(const uint8_t* p) {
  return _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)p));
}
// dot_f32, src/simd.rs:50-72
__attribute__((target("avx2,fma"))) float avx_dot_f32(const uint8_t* row, const float* in,
                                                      size_t n) {
  __m256 acc = _mm256_setzero_ps();
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    acc = _mm256_fmadd_ps(_mm256_loadu_ps((const float*)(row + i * 4)), _mm256_loadu_ps(in + i),
                          acc);
  float sum = hsum(acc);
  for (; i < n; i++) {
    float w;
    memcpy(&w, row + i * 4, 4);
    sum += w * in[i];
  }
  return sum;
}
// dot_q4, src/simd.rs:74-101
__attribute__((target("avx2,fma"))) float avx_dot_q4(const uint8_t* row, const float* in,
                                                     size_t nb, bool affine) {
  size_t bs = affine ? 20 : 18, qo = affine ? 4 : 2;
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * bs;
    float d = read_f16(b, 0);
    float mn = affine ? read_f16(b, 2) : -8.0f * d;
    const float* x = in + bi * 32;
    __m256 qdot = _mm256_setzero_ps(), xsum = _mm256_setzero_ps();
    for (int half = 0; half < 2; half++)
      for (int ch = 0; ch < 2; ch++) {
        __m256i packed = bytes8_to_i32(b + qo + ch * 8);
        __m256i codes = half == 0 ? _mm256_and_si256(packed, _mm256_set1_epi32(15))
                                  : _mm256_srli_epi32(packed, 4);
        __m256 v = _mm256_loadu_ps(x + half * 16 + ch * 8);
        qdot = _mm256_fmadd_ps(_mm256_cvtepi32_ps(codes), v, qdot);
        xsum = _mm256_add_ps(xsum, v);
      }
    sum += d * hsum(qdot) + mn * hsum(xsum);
  }
  return sum;
}
// dot_q5, src/simd.rs:103-151
__attribute__((target("avx2,fma"))) float avx_dot_q5(const uint8_t* row, const float* in,
                                                     size_t nb, bool affine) {
  size_t bs = affine ? 24 : 22, qho = affine ? 4 : 2, qso = affine ? 8 : 6;
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * bs;
    float d = read_f16(b, 0);
    float mn = affine ? read_f16(b, 2) : -16.0f * d;
    uint32_t qh = (uint32_t)b[qho] | ((uint32_t)b[qho + 1] << 8) | ((uint32_t)b[qho + 2] << 16) |
                  ((uint32_t)b[qho + 3] << 24);
    const float* x = in + bi * 32;
    __m256 qdot = _mm256_setzero_ps(), xsum = _mm256_setzero_ps();
    for (int half = 0; half < 2; half++)
      for (int ch = 0; ch < 2; ch++) {
        int base = ch * 8;
        __m256i packed = bytes8_to_i32(b + qso + base);
        __m256i low = half == 0 ? _mm256_and_si256(packed, _mm256_set1_epi32(15))
                                : _mm256_srli_epi32(packed, 4);
        int bit = half * 16 + base;
        alignas(32) int32_t hv[8];
        for (int k = 0; k < 8; k++) hv[k] = (int32_t)(((qh >> (bit + k)) & 1) << 4);
        __m256i high = _mm256_loadu_si256((const __m256i*)hv);
        __m256i codes = _mm256_add_epi32(low, high);
        __m256 v = _mm256_loadu_ps(x + half * 16 + base);
        qdot = _mm256_fmadd_ps(_mm256_cvtepi32_ps(codes), v, qdot);
        xsum = _mm256_add_ps(xsum, v);
      }
    sum += d * hsum(qdot) + mn * hsum(xsum);
  }
  return sum;
}
// dot_q8, src/simd.rs:153-167
__attribute__((target("avx2,fma"))) float avx_dot_q8(const uint8_t* row, const float* in,
                                                     size_t nb) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 34;
    float d = read_f16(b, 0);
    __m256 acc = _mm256_setzero_ps();
    for (int ch = 0; ch < 4; ch++) {
      __m256i codes = i8x8_to_i32(b + 2 + ch * 8);
      acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(codes), _mm256_loadu_ps(in + bi * 32 + ch * 8), acc);
    }
    sum += d * hsum(acc);
  }
  return sum;
}
// dot_q4k, src/simd.rs:169-197
__attribute__((target("avx2,fma"))) float avx_dot_q4k(const uint8_t* row, const float* in,
                                                      size_t nb) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 144;
    float d = read_f16(b, 0), dmin = read_f16(b, 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    const float* x = in + bi * 256;
    for (int g = 0; g < 8; g++) {
      uint8_t sc, mn;
      scale_min_k4(g, scales, &sc, &mn);
      __m256 qdot = _mm256_setzero_ps(), xsum = _mm256_setzero_ps();
      for (int ch = 0; ch < 4; ch++) {
        __m256i packed = bytes8_to_i32(qs + g / 2 * 32 + ch * 8);
        __m256i codes = g % 2 == 0 ? _mm256_and_si256(packed, _mm256_set1_epi32(15))
                                   : _mm256_srli_epi32(packed, 4);
        __m256 v = _mm256_loadu_ps(x + g * 32 + ch * 8);
        qdot = _mm256_fmadd_ps(_mm256_cvtepi32_ps(codes), v, qdot);
        xsum = _mm256_add_ps(xsum, v);
      }
      sum += d * (float)sc * hsum(qdot) - dmin * (float)mn * hsum(xsum);
    }
  }
  return sum;
}
// dot_q5k, src/simd.rs:199-236
__attribute__((target("avx2,fma"))) float avx_dot_q5k(const uint8_t* row, const float* in,
                                                      size_t nb) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 176;
    float d = read_f16(b, 0), dmin = read_f16(b, 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    const float* x = in + bi * 256;
    for (int g = 0; g < 8; g++) {
      uint8_t sc, mn;
      scale_min_k4(g, scales, &sc, &mn);
      __m256i mask = _mm256_set1_epi32(1 << g);
      __m256 qdot = _mm256_setzero_ps(), xsum = _mm256_setzero_ps();
      for (int ch = 0; ch < 4; ch++) {
        __m256i packed = bytes8_to_i32(qs + g / 2 * 32 + ch * 8);
        __m256i low = g % 2 == 0 ? _mm256_and_si256(packed, _mm256_set1_epi32(15))
                                 : _mm256_srli_epi32(packed, 4);
        __m256i hb = bytes8_to_i32(qh + ch * 8);
        __m256i present = _mm256_cmpgt_epi32(_mm256_and_si256(hb, mask), _mm256_setzero_si256());
        __m256i high = _mm256_and_si256(present, _mm256_set1_epi32(16));
        __m256i codes = _mm256_add_epi32(low, high);
        __m256 v = _mm256_loadu_ps(x + g * 32 + ch * 8);
        qdot = _mm256_fmadd_ps(_mm256_cvtepi32_ps(codes), v, qdot);
        xsum = _mm256_add_ps(xsum, v);
      }
      sum += d * (float)sc * hsum(qdot) - dmin * (float)mn * hsum(xsum);
    }
  }
  return sum;
}
// dot_q6k, src/simd.rs:238-281
__attribute__((target("avx2,fma"))) float avx_dot_q6k(const uint8_t* row, const float* in,
                                                      size_t nb) {
  float sum = 0.0f;
  for (size_t bi = 0; bi < nb; bi++) {
    const uint8_t* b = row + bi * 210;
    float d = read_f16(b, 208);
    const float* x = in + bi * 256;
    __m256 acc = _mm256_setzero_ps();
    for (int half = 0; half < 2; half++) {
      const uint8_t* ql = b + half * 64;
      const uint8_t* qh = b + 128 + half * 32;
      const uint8_t* scales = b + 192 + half * 8;
      for (int quarter = 0; quarter < 4; quarter++) {
        int ql_base = quarter % 2 == 0 ? 0 : 32;
        for (int ch = 0; ch < 4; ch++) {
          __m256i pl = bytes8_to_i32(ql + ql_base + ch * 8);
          __m256i low = quarter < 2 ? _mm256_and_si256(pl, _mm256_set1_epi32(15))
                                    : _mm256_srli_epi32(pl, 4);
          __m256i ph = bytes8_to_i32(qh + ch * 8);
          __m256i sh;
          switch (quarter) {
            case 0: sh = ph; break;
            case 1: sh = _mm256_srli_epi32(ph, 2); break;
            case 2: sh = _mm256_srli_epi32(ph, 4); break;
            default: sh = _mm256_srli_epi32(ph, 6); break;
          }
          __m256i high = _mm256_and_si256(sh, _mm256_set1_epi32(3));
          __m256i codes = _mm256_sub_epi32(_mm256_or_si256(low, _mm256_slli_epi32(high, 4)),
                                           _mm256_set1_epi32(32));
          float scale = (float)(int8_t)scales[quarter * 2 + (ch * 8) / 16] * d;
          __m256 v = _mm256_loadu_ps(x + half * 128 + quarter * 32 + ch * 8);
          __m256 w = _mm256_mul_ps(_mm256_cvtepi32_ps(codes), _mm256_set1_ps(scale));
          acc = _mm256_fmadd_ps(w, v, acc);
        }
      }
    }
    sum += hsum(acc);
  }
  return sum;
}
bool have_avx2() { return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"); }

// dot_row_avx2 -> x86::dot, src/simd.rs:283-311
float dot_row_avx2(const uint8_t* row, uint32_t ty, const float* in, size_t cols) {
  if (!have_avx2()) return dot_row_scalar(row, ty, in, cols);
  switch (ty) {
    case LRS_GGML_F32: return avx_dot_f32(row, in, cols);
    case LRS_GGML_Q4_0: return avx_dot_q4(row, in, cols / 32, false);
    case LRS_GGML_Q4_1: return avx_dot_q4(row, in, cols / 32, true);
    case LRS_GGML_Q5_0: return avx_dot_q5(row, in, cols / 32, false);
    case LRS_GGML_Q5_1: return avx_dot_q5(row, in, cols / 32, true);
    case LRS_GGML_Q8_0: return avx_dot_q8(row, in, cols / 32);
    case LRS_GGML_Q4_K: return avx_dot_q4k(row, in, cols / 256);
    case LRS_GGML_Q5_K: return avx_dot_q5k(row, in, cols / 256);
    case LRS_GGML_Q6_K: return avx_dot_q6k(row, in, cols / 256);
    default: return dot_row_scalar(row, ty, in, cols);  // F16/BF16, src/simd.rs:296
  }
}

inline float dot_kind(int kind, const uint8_t* row, uint32_t ty, const float* in, size_t cols) {
  return kind == ORC_AVX2 ? dot_row_avx2(row, ty, in, cols) : dot_row_scalar(row, ty, in, cols);
}

int resolve_threads(int threads) {
  return threads > 0 ? threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
}

// One persistent pool per thread count, like CpuBackend's owned rayon pool.
ForkJoinPool* pool_for(int threads) {
  static std::mutex mu;
  static std::vector<std::unique_ptr<ForkJoinPool>> pools;
  std::lock_guard<std::mutex> g(mu);
  for (auto& p : pools)
    if (p->size() == threads) return p.get();
  pools.emplace_back(new ForkJoinPool(threads));
  return pools.back().get();
}

// CpuBackend::matvec, src/backend.rs:143-162 (threshold 128Ki MACs, :62)
void matvec(int kind, int threads, const uint8_t* w, uint32_t ty, size_t rows, size_t cols,
            const float* x, float* y) {
  size_t rb = row_bytes(ty, cols);
  size_t work = rows * cols;
  if (threads > 1 && rows >= (size_t)threads * 2 && work >= 128 * 1024) {
    pool_for(threads)->parallel_for((long)rows, [&](long b, long e) {
      for (long r = b; r < e; r++) y[r] = dot_kind(kind, w + r * rb, ty, x, cols);
    });
  } else {
    for (size_t r = 0; r < rows; r++) y[r] = dot_kind(kind, w + r * rb, ty, x, cols);
  }
}

// softmax_inplace, src/model.rs:298-313
void softmax_inplace(float* v, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, v[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    v[i] = expf(v[i] - mx);
    sum += v[i];
  }
  if (std::isfinite(sum) && sum > 0.0f) {
    for (size_t i = 0; i < n; i++) v[i] /= sum;
  } else {
    float u = 1.0f / (float)n;
    for (size_t i = 0; i < n; i++) v[i] = u;
  }
}

// RMSNorm::forward, src/model.rs:65-73
void rmsnorm(float* h, const float* w, size_t n, float eps) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += h[i] * h[i];
  float mean_sq = ss / (float)n;
  float inv = 1.0f / sqrtf(mean_sq + eps);
  for (size_t i = 0; i < n; i++) h[i] *= inv * w[i];
}

// apply_rope_inplace, src/model.rs:86-95
void apply_rope(float* x, size_t len, const float* c, const float* s) {
  size_t half = len / 2;
  for (size_t i = 0; i < half; i++) {
    float re = x[i], im = x[i + half];
    x[i] = re * c[i] - im * s[i];
    x[i + half] = re * s[i] + im * c[i];
  }
}

// Ordering key of f32::total_cmp (sign-magnitude -> two's complement).
inline int32_t total_key(float f) {
  int32_t b;
  memcpy(&b, &f, 4);
  b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
  return b;
}

}  // namespace

struct orc_model {
  lrs_model_desc d;
  std::vector<lrs_layer_desc> layers;
  int kind, threads;
  size_t max_seq_len;
  // KVCache (src/cache.rs:4-10): dense f32 [layer][pos * kv_width + kvh * hd + d]
  std::vector<std::vector<float>> kc, vc;
  // InferenceBuffers (src/cache.rs:60-101)
  std::vector<float> hidden, residual, q, k, v, att, proj, gate, up, down, scores, rc, rs, logits;
  std::vector<float> zeros_h, zeros_kv;
};

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }

int orc_type_geometry(uint32_t t, uint32_t* bv, uint32_t* bb) { return geometry(t, bv, bb) ? 0 : 2; }

float orc_value_at(const uint8_t* row, uint32_t t, size_t col) { return value_at(row, t, col); }

void orc_dequantize_row(const uint8_t* row, uint32_t t, size_t cols, float* out) {
  for (size_t c = 0; c < cols; c++) out[c] = value_at(row, t, c);
}

float orc_dot_row(int kind, const uint8_t* row, uint32_t t, const float* x, size_t cols) {
  return dot_kind(kind, row, t, x, cols);
}

int orc_avx2_available(void) { return have_avx2() ? 1 : 0; }

int orc_matvec(int kind, int threads, const uint8_t* w, uint32_t t, size_t rows, size_t cols,
               const float* x, float* y) {
  uint32_t bv, bb;
  if (!geometry(t, &bv, &bb)) return 2;
  if (cols % bv) return 1;
  matvec(kind, resolve_threads(threads), w, t, rows, cols, x, y);
  return 0;
}

uint32_t orc_sample(const float* logits, size_t n, const uint32_t* recent, size_t n_recent,
                    float temperature, float top_p, size_t top_k, float repetition_penalty,
                    float u, float* margin_out) {
  // sample_current_logits, src/engine.rs:253-325, step by step.
  float margin = INFINITY;
  if (margin_out) *margin_out = margin;
  if (n == 0) return 0;
  std::vector<char> seen(n, 0);
  for (size_t i = 0; i < n_recent; i++)
    if (recent[i] < n) seen[recent[i]] = 1;
  std::vector<std::pair<uint32_t, float>> cand;
  cand.reserve(n);
  for (size_t t = 0; t < n; t++) {
    float value = logits[t];
    if (repetition_penalty != 1.0f && seen[t])
      value = value > 0.0f ? value / repetition_penalty : value * repetition_penalty;
    if (temperature > 0.0f) value /= temperature;
    if (!std::isfinite(value)) value = -INFINITY;
    cand.emplace_back((uint32_t)t, value);
  }
  // sort_unstable_by(|a, b| b.1.total_cmp(&a.1)); equal values: larger index first
  std::sort(cand.begin(), cand.end(), [](const std::pair<uint32_t, float>& a,
                                         const std::pair<uint32_t, float>& b) {
    const int32_t ka = total_key(a.second), kb = total_key(b.second);
    return ka != kb ? ka > kb : a.first > b.first;
  });
  if (temperature <= 0.0f) return cand[0].first;
  if (top_k > 0 && top_k < cand.size()) cand.resize(top_k);
  const float mx = cand[0].second;
  float sum = 0.0f;
  for (auto& c : cand) {
    c.second = std::exp(c.second - mx);
    sum += c.second;
  }
  if (!std::isfinite(sum) || sum <= 0.0f) return cand[0].first;
  for (auto& c : cand) c.second /= sum;
  float cumulative = 0.0f;
  size_t cutoff = cand.size();
  for (size_t i = 0; i < cand.size(); i++) {
    const float before = cumulative;
    cumulative += cand[i].second;
    if (cumulative >= top_p) {
      cutoff = i + 1;
      margin = std::min(margin, std::min(cumulative - top_p, top_p - before));
      break;
    }
  }
  float kept_sum = 0.0f;
  for (size_t i = 0; i < cutoff; i++) kept_sum += cand[i].second;
  float random = u * kept_sum;
  for (size_t i = 0; i < cutoff; i++) {
    const float before = random;
    random -= cand[i].second;
    if (random <= 0.0f) {
      if (margin_out) *margin_out = std::min(margin, std::min(before, -random));
      return cand[i].first;
    }
  }
  if (margin_out) *margin_out = std::min(margin, std::fabs(random));
  return cand[cutoff - 1].first;
}

uint32_t orc_argmax(const float* logits, size_t n) {
  // argmax_current_logits, src/engine.rs:233-241: Iterator::max_by keeps the
  // LAST of equal maxima under f32::total_cmp.
  if (n == 0) return 0;
  size_t best = 0;
  int32_t bk = total_key(logits[0]);
  for (size_t i = 1; i < n; i++) {
    int32_t k = total_key(logits[i]);
    if (k >= bk) {
      bk = k;
      best = i;
    }
  }
  return (uint32_t)best;
}

orc_model* orc_model_create(const lrs_model_desc* desc, size_t max_seq_len, int kind, int threads) {
  const lrs_config& c = desc->config;
  if (max_seq_len == 0 || max_seq_len > c.max_position_embeddings) {
    g_err = "max_seq_len must be in 1..=max_position_embeddings";
    return nullptr;
  }
  orc_model* m = new orc_model();
  m->d = *desc;
  m->layers.assign(desc->layers, desc->layers + c.num_hidden_layers);
  m->d.layers = m->layers.data();
  m->kind = kind;
  m->threads = resolve_threads(threads);
  m->max_seq_len = max_seq_len;
  size_t kvw = (size_t)c.num_key_value_heads * c.head_dim;
  m->kc.assign(c.num_hidden_layers, std::vector<float>(max_seq_len * kvw, 0.0f));
  m->vc.assign(c.num_hidden_layers, std::vector<float>(max_seq_len * kvw, 0.0f));
  size_t h = c.hidden_size, I = c.intermediate_size;
  m->hidden.assign(h, 0);
  m->residual.assign(h, 0);
  m->q.assign(h, 0);
  m->k.assign(kvw, 0);
  m->v.assign(kvw, 0);
  m->att.assign(h, 0);
  m->proj.assign(h, 0);
  m->gate.assign(I, 0);
  m->up.assign(I, 0);
  m->down.assign(h, 0);
  m->scores.assign(max_seq_len, 0);
  m->rc.assign(c.head_dim / 2, 0);
  m->rs.assign(c.head_dim / 2, 0);
  m->logits.assign(c.vocab_size, 0);
  return m;
}

void orc_model_destroy(orc_model* m) { delete m; }

static void linear(orc_model* m, const lrs_tensor_desc& t, const float* bias, const float* in,
                   float* out) {
  // LinearLayer::forward, src/model.rs:33-46
  matvec(m->kind, m->threads, (const uint8_t*)t.data, t.ggml_type, t.rows, t.cols, in, out);
  if (bias)
    for (size_t i = 0; i < t.rows; i++) out[i] += bias[i];
}

int orc_model_forward_token(orc_model* m, uint32_t token, size_t pos, int compute_logits,
                            float* logits_out) {
  // Qwen2Model::forward_impl, src/model.rs:135-270
  const lrs_config& c = m->d.config;
  if (token >= c.vocab_size) {
    g_err = "token id is outside vocabulary";
    return 1;
  }
  if (pos >= m->max_seq_len) {
    g_err = "position exceeds configured context";
    return 1;
  }
  size_t hidden = c.hidden_size, hd = c.head_dim, nh = c.num_attention_heads,
         nkv = c.num_key_value_heads, kvw = nkv * hd, groups = nh / nkv;
  float scale = 1.0f / sqrtf((float)hd);
  // prepare_rope, src/model.rs:76-84
  for (size_t i = 0; i < hd / 2; i++) {
    float inv_freq = 1.0f / powf(c.rope_theta, 2.0f * (float)i / (float)hd);
    float angle = (float)pos * inv_freq;
    m->rs[i] = sinf(angle);
    m->rc[i] = cosf(angle);
  }
  // embed_tokens.row_into, src/model.rs:170-171
  const lrs_tensor_desc& E = m->d.embed_tokens;
  const uint8_t* erow = (const uint8_t*)E.data + (size_t)token * row_bytes(E.ggml_type, E.cols);
  for (size_t i = 0; i < hidden; i++) m->residual[i] = value_at(erow, E.ggml_type, i);

  for (uint32_t li = 0; li < c.num_hidden_layers; li++) {
    const lrs_layer_desc& L = m->d.layers[li];
    m->hidden = m->residual;
    rmsnorm(m->hidden.data(), L.input_layernorm, hidden, c.rms_norm_eps);
    linear(m, L.q_proj, L.q_bias, m->hidden.data(), m->q.data());
    linear(m, L.k_proj, L.k_bias, m->hidden.data(), m->k.data());
    linear(m, L.v_proj, L.v_bias, m->hidden.data(), m->v.data());
    for (size_t h = 0; h < nh; h++) apply_rope(&m->q[h * hd], hd, m->rc.data(), m->rs.data());
    for (size_t h = 0; h < nkv; h++) apply_rope(&m->k[h * hd], hd, m->rc.data(), m->rs.data());
    // KVCache::update, src/cache.rs:38-53
    memcpy(&m->kc[li][pos * kvw], m->k.data(), kvw * 4);
    memcpy(&m->vc[li][pos * kvw], m->v.data(), kvw * 4);
    std::fill(m->att.begin(), m->att.end(), 0.0f);
    for (size_t h = 0; h < nh; h++) {
      size_t kvh = h / groups;
      const float* qh = &m->q[h * hd];
      float* sc = m->scores.data();
      for (size_t p = 0; p <= pos; p++) {
        const float* key = &m->kc[li][p * kvw + kvh * hd];
        float s = 0.0f;
        for (size_t d = 0; d < hd; d++) s += qh[d] * key[d];
        sc[p] = s * scale;
      }
      softmax_inplace(sc, pos + 1);
      float* out = &m->att[h * hd];
      for (size_t p = 0; p <= pos; p++) {
        const float* val = &m->vc[li][p * kvw + kvh * hd];
        float w = sc[p];
        for (size_t d = 0; d < hd; d++) out[d] += w * val[d];
      }
    }
    linear(m, L.o_proj, nullptr, m->att.data(), m->proj.data());
    for (size_t i = 0; i < hidden; i++) m->residual[i] += m->proj[i];
    m->hidden = m->residual;
    rmsnorm(m->hidden.data(), L.post_attention_layernorm, hidden, c.rms_norm_eps);
    linear(m, L.gate_proj, nullptr, m->hidden.data(), m->gate.data());
    linear(m, L.up_proj, nullptr, m->hidden.data(), m->up.data());
    for (size_t i = 0; i < c.intermediate_size; i++) {
      float g = m->gate[i];
      m->gate[i] = (g / (1.0f + expf(-g))) * m->up[i];
    }
    linear(m, L.down_proj, nullptr, m->gate.data(), m->down.data());
    for (size_t i = 0; i < hidden; i++) m->residual[i] += m->down[i];
  }
  if (compute_logits) {
    m->hidden = m->residual;
    rmsnorm(m->hidden.data(), m->d.final_norm, hidden, c.rms_norm_eps);
    linear(m, m->d.lm_head, nullptr, m->hidden.data(), m->logits.data());
    if (logits_out) memcpy(logits_out, m->logits.data(), c.vocab_size * 4);
  }
  return 0;
}

int orc_model_prefill(orc_model* m, const uint32_t* tokens, size_t n, size_t start_pos,
                      float* logits_out) {
  // CausalModel::prefill default, src/architecture.rs:60-77
  if (n == 0) {
    g_err = "prefill requires at least one token";
    return 1;
  }
  for (size_t i = 0; i < n; i++) {
    int rc = orc_model_forward_token(m, tokens[i], start_pos + i, i + 1 == n,
                                     i + 1 == n ? logits_out : nullptr);
    if (rc) return rc;
  }
  return 0;
}

static float top2_margin(const float* l, size_t n) {
  float a = -INFINITY, b = -INFINITY;
  for (size_t i = 0; i < n; i++) {
    if (l[i] > a) {
      b = a;
      a = l[i];
    } else if (l[i] > b) {
      b = l[i];
    }
  }
  return a - b;
}

int orc_benchmark_tokens(orc_model* m, const uint32_t* prompt, size_t n, size_t decode,
                         uint32_t* tokens_out, float* step_logits, float* margins,
                         double* prefill_s, double* decode_s) {
  // InferenceEngine::benchmark_tokens, src/engine.rs:189-223
  const size_t V = m->d.config.vocab_size;
  if (n == 0 || n + decode > m->max_seq_len) {
    g_err = "benchmark token counts exceed context";
    return 1;
  }
  auto t0 = std::chrono::steady_clock::now();
  int rc = orc_model_prefill(m, prompt, n, 0, nullptr);
  if (rc) return rc;
  auto t1 = std::chrono::steady_clock::now();
  if (step_logits) memcpy(step_logits, m->logits.data(), V * 4);
  if (margins) margins[0] = top2_margin(m->logits.data(), V);
  for (size_t s = 0; s < decode; s++) {
    uint32_t tok = orc_argmax(m->logits.data(), V);
    if (tokens_out) tokens_out[s] = tok;
    rc = orc_model_forward_token(m, tok, n + s, 1, nullptr);
    if (rc) return rc;
    if (step_logits) memcpy(step_logits + (s + 1) * V, m->logits.data(), V * 4);
    if (margins) margins[s + 1] = top2_margin(m->logits.data(), V);
  }
  auto t2 = std::chrono::steady_clock::now();
  if (prefill_s) *prefill_s = std::chrono::duration<double>(t1 - t0).count();
  if (decode_s) *decode_s = std::chrono::duration<double>(t2 - t1).count();
  return 0;
}

}  // extern "C"

// encoders.h -- the load-time GGML encoders and the q4k / q4km fallbacks,
// shared by the host (quantize.cpp) and the device (quantize_dev.cu).
//
// The reference quantizes F32/F16/BF16 weights once at load time
// (maybe_quantize, src/loader.rs:406-447) with the encoders in
// src/quant.rs:187-259 and 650-967; they are restated here so the synthetic
// models get the bytes the reference would build.  Every operation is a
// single IEEE f32 operation in the reference's order: the host build uses
// -ffp-contract=off and the device build --fmad=false (Rust never fuses
// a*b+c), and f32 -> f16 rounds to nearest even on both sides, so host and
// device encoders produce identical bytes.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/llamars.h"
#if defined(__CUDACC__)
#define LRS_ENC __host__ __device__ inline
#else
#define LRS_ENC inline
#endif

namespace lrs {
namespace enc {

// f32::max / f32::min with one rule for a tie of signed zeros on host and
// device: a NaN operand yields the other one, an equal pair yields `b` (the
// x86 maxss/minss result the host build gets; CUDA's max.f32 would give +0).
LRS_ENC float fmax_(float a, float b) {
  if (a != a) return b;
  if (b != b) return a;
  return a > b ? a : b;
}
LRS_ENC float fmin_(float a, float b) {
  if (a != a) return b;
  if (b != b) return a;
  return a < b ? a : b;
}

// --- Rust `as` casts from f32 saturate and send NaN to 0 ------------------
LRS_ENC uint8_t as_u8(float v) {
  if (!(v == v) || v <= 0.0f) return 0;
  if (v >= 255.0f) return 255;
  return (uint8_t)v;
}
LRS_ENC int8_t as_i8(float v) {
  if (!(v == v)) return 0;
  if (v <= -128.0f) return -128;
  if (v >= 127.0f) return 127;
  return (int8_t)v;
}
LRS_ENC int32_t as_i32(float v) {
  if (!(v == v)) return 0;
  if (v <= -2147483648.0f) return INT32_MIN;
  if (v >= 2147483647.0f) return INT32_MAX;
  return (int32_t)v;
}
// f32::clamp (NaN passes through).
LRS_ENC float clampf(float v, float lo, float hi) {
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}
// f32::round rounds half away from zero == roundf.
LRS_ENC float rround(float v) { return roundf(v); }

// half::f16::from_f32 / bf16::from_f32: round to nearest even.
// f32 <-> f16 bits in integer arithmetic, round to nearest even (what
// half::f16::from_f32 does), so host and device share one definition.
LRS_ENC uint32_t f32_bits(float v) {
  uint32_t x;
  memcpy(&x, &v, 4);
  return x;
}
LRS_ENC uint16_t f32_to_f16_bits(float v) {
  const uint32_t x = f32_bits(v), sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));  // NaN
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // >= 65520 rounds to inf
  const uint32_t e = ax >> 23;
  uint32_t r, rem, half;
  if (e < 113) {  // below 2^-14: subnormal result, unit 2^-24
    const uint32_t s = 126 - e;
    if (s > 24) return (uint16_t)sign;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    r = m >> s;
    rem = m & ((1u << s) - 1u);
    half = 1u << (s - 1);
  } else {
    r = ((e - 112) << 10) | ((ax & 0x7fffffu) >> 13);
    rem = ax & 0x1fffu;
    half = 0x1000u;
  }
  if (rem > half || (rem == half && (r & 1u))) r++;
  return (uint16_t)(sign | r);
}
LRS_ENC float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    float f = (float)m * 5.9604644775390625e-8f;  // m * 2^-24, exact
    return sign ? -f : f;
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}
LRS_ENC uint16_t f32_to_bf16_bits(float v) {
  uint32_t x;
  memcpy(&x, &v, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40);  // quiet NaN
  uint32_t bias = 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)((x + bias) >> 16);
}
LRS_ENC void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}
// write_f16, src/quant.rs:334-336
LRS_ENC void write_f16(uint8_t* p, float v) { put16(p, f32_to_f16_bits(v)); }
LRS_ENC float f16_round(float v) { return f16_bits_to_f32(f32_to_f16_bits(v)); }

// quantize_block_q8_0, src/quant.rs:650-662
LRS_ENC void block_q8_0(const float* v, uint8_t* out) {
  float abs_max = 0.0f;
  for (int i = 0; i < 32; i++) abs_max = fmax_(abs_max, fabsf(v[i]));
  float d = abs_max / 127.0f;
  float inv = d == 0.0f ? 0.0f : 1.0f / d;
  write_f16(out, d);
  for (int i = 0; i < 32; i++) out[2 + i] = (uint8_t)as_i8(clampf(rround(v[i] * inv), -127.0f, 127.0f));
}

// make_qx_quants_16, src/quant.rs:726-777
LRS_ENC float make_qx_quants_16(const float* values, uint8_t* codes) {
  float max = 0.0f, abs_max = 0.0f;
  for (int i = 0; i < 16; i++) {
    if (fabsf(values[i]) > abs_max) {
      abs_max = fabsf(values[i]);
      max = values[i];
    }
  }
  if (abs_max < 1e-15f) {
    memset(codes, 0, 16);
    return 0.0f;
  }
  float inv_scale = -32.0f / max;
  float sum_lx = 0.0f, sum_l2 = 0.0f;
  for (int i = 0; i < 16; i++) {
    int32_t level = as_i32(clampf(rround(inv_scale * values[i]), -32.0f, 31.0f));
    codes[i] = (uint8_t)(level + 32);
    float weight = values[i] * values[i];
    sum_lx += weight * values[i] * (float)level;
    sum_l2 += weight * (float)(level * level);
  }
  float scale = sum_l2 > 0.0f ? sum_lx / sum_l2 : 0.0f;
  float best = scale * sum_lx;
  for (int step = -9; step <= 9; step++) {
    if (step == 0) continue;
    inv_scale = -(32.0f + 0.1f * (float)step) / max;
    sum_lx = 0.0f;
    sum_l2 = 0.0f;
    for (int i = 0; i < 16; i++) {
      float value = values[i];
      int32_t level = as_i32(clampf(rround(inv_scale * value), -32.0f, 31.0f));
      float weight = value * value;
      sum_lx += weight * value * (float)level;
      sum_l2 += weight * (float)(level * level);
    }
    if (sum_l2 > 0.0f && sum_lx * sum_lx > best * sum_l2) {
      for (int i = 0; i < 16; i++) {
        int32_t level = as_i32(clampf(rround(inv_scale * values[i]), -32.0f, 31.0f));
        codes[i] = (uint8_t)(level + 32);
      }
      scale = sum_lx / sum_l2;
      best = scale * sum_lx;
    }
  }
  return scale;
}

// quantize_block_q6k, src/quant.rs:664-724
LRS_ENC void block_q6k(const float* values, uint8_t* out) {
  uint8_t codes[256];
  float scales[16];
  float max_scale = 0.0f, max_abs_scale = 0.0f;
  for (int g = 0; g < 16; g++) {
    float s = make_qx_quants_16(values + g * 16, codes + g * 16);
    scales[g] = s;
    if (fabsf(s) > max_abs_scale) {
      max_abs_scale = fabsf(s);
      max_scale = s;
    }
  }
  if (max_abs_scale < 1e-15f) {
    memset(out, 0, 210);
    return;
  }
  float inv_scale = -128.0f / max_scale;
  float d = 1.0f / inv_scale;
  float d_f16 = f16_round(d);
  int8_t scale_codes[16];
  for (int g = 0; g < 16; g++) {
    scale_codes[g] = as_i8(fmin_(rround(inv_scale * scales[g]), 127.0f));
    float group_d = d_f16 * (float)scale_codes[g];
    if (group_d == 0.0f) continue;
    for (int i = 0; i < 16; i++) {
      int32_t level = as_i32(clampf(rround(values[g * 16 + i] / group_d), -32.0f, 31.0f));
      codes[g * 16 + i] = (uint8_t)(level + 32);
    }
  }
  uint8_t* low = out;
  uint8_t* high = out + 128;
  for (int half = 0; half < 2; half++) {
    int base = half * 128;
    for (int lane = 0; lane < 32; lane++) {
      uint8_t q1 = codes[base + lane], q2 = codes[base + 32 + lane], q3 = codes[base + 64 + lane],
              q4 = codes[base + 96 + lane];
      low[half * 64 + lane] = (uint8_t)((q1 & 0x0f) | ((q3 & 0x0f) << 4));
      low[half * 64 + 32 + lane] = (uint8_t)((q2 & 0x0f) | ((q4 & 0x0f) << 4));
      high[half * 32 + lane] =
          (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  for (int g = 0; g < 16; g++) out[192 + g] = (uint8_t)scale_codes[g];
  write_f16(out + 208, d);
}

// quantize_block_q5_0, src/quant.rs:779-807
LRS_ENC void block_q5_0(const float* v, uint8_t* out) {
  float max_value = 0.0f, abs_max = 0.0f;
  for (int i = 0; i < 32; i++) {
    if (fabsf(v[i]) > abs_max) {
      abs_max = fabsf(v[i]);
      max_value = v[i];
    }
  }
  float d = abs_max == 0.0f ? 0.0f : max_value / -16.0f;
  float inv = d == 0.0f ? 0.0f : 1.0f / d;
  write_f16(out, d);
  uint32_t high = 0;
  for (int j = 0; j < 16; j++) {
    uint8_t q0 = as_u8(clampf(floorf(v[j] * inv + 16.5f), 0.0f, 31.0f));
    uint8_t q1 = as_u8(clampf(floorf(v[j + 16] * inv + 16.5f), 0.0f, 31.0f));
    out[6 + j] = (uint8_t)((q0 & 0x0f) | ((q1 & 0x0f) << 4));
    high |= (((uint32_t)q0 >> 4) & 1u) << j;
    high |= (((uint32_t)q1 >> 4) & 1u) << (j + 16);
  }
  for (int k = 0; k < 4; k++) out[2 + k] = (uint8_t)(high >> (8 * k));
}

// make_qkx2_quants, src/quant.rs:892-967
LRS_ENC float make_qkx2_quants(const float* values, const float* weights, uint8_t* codes, float* out_min) {
  uint8_t aux[32];
  float mn = values[0], mx = values[0];
  float sum_weight = weights[0];
  float sum_value = weights[0] * values[0];
  for (int i = 1; i < 32; i++) {
    mn = fmin_(mn, values[i]);
    mx = fmax_(mx, values[i]);
    sum_weight += weights[i];
    sum_value += weights[i] * values[i];
  }
  mn = fmin_(mn, 0.0f);
  if (mx == mn) {
    memset(codes, 0, 32);
    *out_min = -mn;
    return 0.0f;
  }
  float range = mx - mn;
  float inv_scale = 15.0f / range;
  float scale = 1.0f / inv_scale;
  float best_error = 0.0f;
  for (int i = 0; i < 32; i++) {
    uint8_t code = as_u8(clampf(rround(inv_scale * (values[i] - mn)), 0.0f, 15.0f));
    codes[i] = code;
    float diff = scale * (float)code + mn - values[i];
    best_error += weights[i] * diff * diff;
  }
  for (int step = 0; step <= 20; step++) {
    inv_scale = (-1.0f + 0.1f * (float)step + 15.0f) / range;
    float sum_l = 0.0f, sum_l2 = 0.0f, sum_xl = 0.0f;
    for (int i = 0; i < 32; i++) {
      uint8_t code = as_u8(clampf(rround(inv_scale * (values[i] - mn)), 0.0f, 15.0f));
      aux[i] = code;
      float wc = weights[i] * (float)code;
      sum_l += wc;
      sum_l2 += wc * (float)code;
      sum_xl += wc * values[i];
    }
    float det = sum_weight * sum_l2 - sum_l * sum_l;
    if (det > 0.0f) {
      float cs = (sum_weight * sum_xl - sum_value * sum_l) / det;
      float cm = (sum_l2 * sum_value - sum_l * sum_xl) / det;
      if (cm > 0.0f) {
        cm = 0.0f;
        cs = sum_xl / sum_l2;
      }
      float error = 0.0f;
      for (int i = 0; i < 32; i++) {
        float diff = cs * (float)aux[i] + cm - values[i];
        error += weights[i] * diff * diff;
      }
      if (error < best_error) {
        memcpy(codes, aux, 32);
        best_error = error;
        scale = cs;
        mn = cm;
      }
    }
  }
  *out_min = -mn;
  return scale;
}

// Packs 8 six-bit scale codes and 8 six-bit min codes the Q4_K/Q5_K way
// (src/quant.rs:851-862; decoded by scale_min_k4, :338-347).
LRS_ENC void pack_scales_k(const uint8_t* sc, const uint8_t* mc, uint8_t* scales) {
  memset(scales, 0, 12);
  for (int g = 0; g < 8; g++) {
    if (g < 4) {
      scales[g] = sc[g];
      scales[g + 4] = mc[g];
    } else {
      scales[g + 4] = (uint8_t)((sc[g] & 0x0f) | ((mc[g] & 0x0f) << 4));
      scales[g - 4] |= (uint8_t)((sc[g] >> 4) << 6);
      scales[g] |= (uint8_t)((mc[g] >> 4) << 6);
    }
  }
}

// quantize_block_q4k, src/quant.rs:809-890
LRS_ENC void block_q4k(const float* values, uint8_t* out) {
  float local_scales[8], local_mins[8];
  float max_scale = 0.0f, max_min = 0.0f;
  uint8_t codes[256];
  for (int g = 0; g < 8; g++) {
    const float* gv = values + g * 32;
    float sum_sq = 0.0f;
    for (int i = 0; i < 32; i++) sum_sq += gv[i] * gv[i];
    float average = sqrtf(sum_sq / 32.0f);
    float weights[32];
    for (int i = 0; i < 32; i++) weights[i] = average + fabsf(gv[i]);
    float mn = 0.0f;
    float s = make_qkx2_quants(gv, weights, codes + g * 32, &mn);
    local_scales[g] = s;
    local_mins[g] = mn;
    max_scale = fmax_(max_scale, s);
    max_min = fmax_(max_min, mn);
  }
  float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
  float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
  uint8_t sc_codes[8], min_codes[8];
  for (int g = 0; g < 8; g++) {
    sc_codes[g] = as_u8(clampf(rround(inv_scale * local_scales[g]), 0.0f, 63.0f));
    min_codes[g] = as_u8(clampf(rround(inv_min * local_mins[g]), 0.0f, 63.0f));
  }
  float d = max_scale / 63.0f;
  float dmin = max_min / 63.0f;
  write_f16(out, d);
  write_f16(out + 2, dmin);
  pack_scales_k(sc_codes, min_codes, out + 4);
  d = f16_round(d);
  dmin = f16_round(dmin);
  for (int g = 0; g < 8; g++) {
    float scale = d * (float)sc_codes[g];
    if (scale == 0.0f) continue;
    float mnv = dmin * (float)min_codes[g];
    for (int i = 0; i < 32; i++)
      codes[g * 32 + i] = as_u8(clampf(rround((values[g * 32 + i] + mnv) / scale), 0.0f, 15.0f));
  }
  for (int pair = 0; pair < 4; pair++)
    for (int i = 0; i < 32; i++)
      out[16 + pair * 32 + i] = (uint8_t)(codes[pair * 64 + i] | (codes[pair * 64 + 32 + i] << 4));
}

// ---- Encoders with no counterpart in the reference ------------------------
// The reference can read Q4_0, Q4_1, Q5_1 and Q5_K tensors from GGUF files but
// cannot produce them.  The GEMV sweep needs such matrices, so these plain
// min/max encoders emit valid blocks of the layouts value_at decodes
// (src/quant.rs:357-436).  Their quality is irrelevant to parity: the CUDA
// kernels are checked against value_at / dot_row_scalar on whatever bytes
// these produce.

// Q4_0: d = (value of largest magnitude) / -8, q = floor(v/d + 8.5) in [0,15].
LRS_ENC void block_q4_0(const float* v, uint8_t* out) {
  float amax = 0.0f, max = 0.0f;
  for (int i = 0; i < 32; i++)
    if (fabsf(v[i]) > amax) {
      amax = fabsf(v[i]);
      max = v[i];
    }
  float d = max / -8.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  write_f16(out, d);
  for (int j = 0; j < 16; j++) {
    uint8_t q0 = as_u8(clampf(floorf(v[j] * id + 8.5f), 0.0f, 15.0f));
    uint8_t q1 = as_u8(clampf(floorf(v[j + 16] * id + 8.5f), 0.0f, 15.0f));
    out[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}
// Q4_1 / Q5_1: m = min, d = (max - min) / levels, q = round((v - m) / d).
LRS_ENC void block_q41_q51(const float* v, uint8_t* out, bool five) {
  float mn = v[0], mx = v[0];
  for (int i = 1; i < 32; i++) {
    mn = fmin_(mn, v[i]);
    mx = fmax_(mx, v[i]);
  }
  float levels = five ? 31.0f : 15.0f;
  float d = (mx - mn) / levels;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  write_f16(out, d);
  write_f16(out + 2, mn);
  uint32_t qh = 0;
  uint8_t* qs = out + (five ? 8 : 4);
  for (int j = 0; j < 16; j++) {
    uint8_t q0 = as_u8(clampf(floorf((v[j] - mn) * id + 0.5f), 0.0f, levels));
    uint8_t q1 = as_u8(clampf(floorf((v[j + 16] - mn) * id + 0.5f), 0.0f, levels));
    qs[j] = (uint8_t)((q0 & 0x0f) | ((q1 & 0x0f) << 4));
    qh |= (uint32_t)((q0 >> 4) & 1) << j;
    qh |= (uint32_t)((q1 >> 4) & 1) << (j + 16);
  }
  if (five)
    for (int k = 0; k < 4; k++) out[4 + k] = (uint8_t)(qh >> (8 * k));
}
// Q5_K: per 32-value group, scale = (max - min') / 31 with min' = min(min, 0);
// six-bit scale/min codes packed like Q4_K; codes recomputed from the rounded
// scales.
LRS_ENC void block_q5k(const float* values, uint8_t* out) {
  float ls[8], lm[8], max_scale = 0.0f, max_min = 0.0f;
  for (int g = 0; g < 8; g++) {
    const float* gv = values + g * 32;
    float mn = gv[0], mx = gv[0];
    for (int i = 1; i < 32; i++) {
      mn = fmin_(mn, gv[i]);
      mx = fmax_(mx, gv[i]);
    }
    mn = fmin_(mn, 0.0f);
    ls[g] = (mx - mn) / 31.0f;
    lm[g] = -mn;
    max_scale = fmax_(max_scale, ls[g]);
    max_min = fmax_(max_min, lm[g]);
  }
  float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
  float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
  uint8_t sc[8], mc[8];
  for (int g = 0; g < 8; g++) {
    sc[g] = as_u8(clampf(rround(inv_scale * ls[g]), 0.0f, 63.0f));
    mc[g] = as_u8(clampf(rround(inv_min * lm[g]), 0.0f, 63.0f));
  }
  float d = max_scale / 63.0f, dmin = max_min / 63.0f;
  write_f16(out, d);
  write_f16(out + 2, dmin);
  pack_scales_k(sc, mc, out + 4);
  d = f16_round(d);
  dmin = f16_round(dmin);
  uint8_t* qh = out + 16;
  uint8_t* qs = out + 48;
  memset(qh, 0, 32);
  uint8_t codes[256];
  for (int g = 0; g < 8; g++) {
    float scale = d * (float)sc[g];
    float mnv = dmin * (float)mc[g];
    for (int i = 0; i < 32; i++)
      codes[g * 32 + i] =
          scale == 0.0f ? 0 : as_u8(clampf(rround((values[g * 32 + i] + mnv) / scale), 0.0f, 31.0f));
  }
  for (int g = 0; g < 8; g++)
    for (int i = 0; i < 32; i++)
      if (codes[g * 32 + i] & 16) qh[i] |= (uint8_t)(1u << g);
  for (int pair = 0; pair < 4; pair++)
    for (int i = 0; i < 32; i++)
      qs[pair * 32 + i] =
          (uint8_t)((codes[pair * 64 + i] & 15) | ((codes[pair * 64 + 32 + i] & 15) << 4));
}


// Resolves the reference encoders' fallbacks (src/quant.rs:190-259).
LRS_ENC uint32_t effective_type(uint32_t t, size_t cols) {
  switch (t) {
    case LRS_GGML_Q4_K:
      if (cols % 256 == 0) return t;
      return cols % 32 == 0 ? LRS_GGML_Q5_0 : LRS_GGML_F32;
    case LRS_GGML_Q6_K:
      if (cols % 256 == 0) return t;
      return cols % 32 == 0 ? LRS_GGML_Q8_0 : LRS_GGML_F32;
    case LRS_GGML_Q5_K:
      return cols % 256 == 0 ? t : (uint32_t)LRS_GGML_F32;
    case LRS_GGML_Q4_0:
    case LRS_GGML_Q4_1:
    case LRS_GGML_Q5_0:
    case LRS_GGML_Q5_1:
    case LRS_GGML_Q8_0:
      return cols % 32 == 0 ? t : (uint32_t)LRS_GGML_F32;
    default:
      return t;
  }
}

// Encodes one row of `cols` values as `t` (already an effective type).
LRS_ENC void quantize_row(uint32_t t, const float* v, size_t cols, uint8_t* out) {
  switch (t) {
    case LRS_GGML_F32: memcpy(out, v, cols * 4); break;
    case LRS_GGML_F16:
      for (size_t i = 0; i < cols; i++) put16(out + 2 * i, f32_to_f16_bits(v[i]));
      break;
    case LRS_GGML_BF16:
      for (size_t i = 0; i < cols; i++) put16(out + 2 * i, f32_to_bf16_bits(v[i]));
      break;
    case LRS_GGML_Q4_0:
      for (size_t b = 0; b < cols / 32; b++) block_q4_0(v + b * 32, out + b * 18);
      break;
    case LRS_GGML_Q4_1:
      for (size_t b = 0; b < cols / 32; b++) block_q41_q51(v + b * 32, out + b * 20, false);
      break;
    case LRS_GGML_Q5_0:
      for (size_t b = 0; b < cols / 32; b++) block_q5_0(v + b * 32, out + b * 22);
      break;
    case LRS_GGML_Q5_1:
      for (size_t b = 0; b < cols / 32; b++) block_q41_q51(v + b * 32, out + b * 24, true);
      break;
    case LRS_GGML_Q8_0:
      for (size_t b = 0; b < cols / 32; b++) block_q8_0(v + b * 32, out + b * 34);
      break;
    case LRS_GGML_Q4_K:
      for (size_t b = 0; b < cols / 256; b++) block_q4k(v + b * 256, out + b * 144);
      break;
    case LRS_GGML_Q5_K:
      for (size_t b = 0; b < cols / 256; b++) block_q5k(v + b * 256, out + b * 176);
      break;
    case LRS_GGML_Q6_K:
      for (size_t b = 0; b < cols / 256; b++) block_q6k(v + b * 256, out + b * 210);
      break;
  }
}


}  // namespace enc
}  // namespace lrs

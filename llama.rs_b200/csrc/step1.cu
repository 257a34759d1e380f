// step1.cu -- the batch-1 decode step as one persistent kernel (sm_100a).
//
// Replaces, for one sequence, the per-token forward of Qwen2Model::forward_impl
// (src/model.rs:135-270) with the greedy argmax of benchmark_tokens
// (src/engine.rs:189-241), and CpuBackend::matvec (src/backend.rs:143-162) at
// batch 1.
//
// Roles.  One CTA per SM (cooperative launch), 11 consumer warps and one
// producer warp.
// * The producer walks the weight chunks of the whole step in order (every
//   layer's q/k/v, o, gate/up, down, then the LM head): CTA b of G owns rows
//   [rows*b/G, rows*(b+1)/G) of every matrix, a contiguous byte range, and
//   copies it chunk by chunk with cp.async.bulk into a ring of 32 KB slots.
//   The weights do not depend on the activations, so the producer never waits
//   for a phase boundary, only for free slots: the ring (4-6 slots per SM)
//   stays full across the grid barriers.
// * The consumers run the phases.  Before a projection they stage its input
//   vector in shared memory (RMSNorm fused where the reference applies one),
//   split per 32-column group into three int8 parts with one f32 scale:
//   x ~= s * (hi + mid / 2^8 + lo / 2^16), 23 bits per value.  Each lane
//   takes block "pieces" of R rows (the x piece is read once for R rows): the
//   codes meet the int8 parts in dp4a (exact int32 sums), and one float step
//   per group applies the block scales -- the per-row dot of dot_row_scalar
//   (src/quant.rs:458-648) to about f32 rounding.
// * A chunk's row sums are reduced in a fixed order (deterministic) by the
//   last consumer warp to finish it, which applies the epilogue: bias,
//   residual add, silu(gate) * up, or the argmax key.
// * Attention (src/model.rs:188-231): the (KV head, context split) pairs are
//   spread over the CTAs; each rotates q (RoPE, src/model.rs:86-95), computes
//   its split's scores, softmax partials and PV product; the CTA whose split
//   holds the new position rotates k and stores k and v in the paged cache
//   (KVCache::update, src/cache.rs:38-53).  The CTA that finishes last for a
//   KV head merges the splits.
// * Grid barriers: one counter, zeroed before the launch, and acquire spins.
// Every wait is bounded in time (LRS_ERR_DEVICE_TIMEOUT on the host); after a
// timeout every CTA skips its remaining waits, lets its copies land and exits.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <string>

#include "common.h"
#include "decode.cuh"
#include "device_common.cuh"
#include "gemv.cuh"
#include "step1.cuh"

namespace lrs {
namespace {

constexpr int kW = kS1Warps;
constexpr int kCT = 32 * kW;            // consumer threads
constexpr int kRedPerSlot = 128;        // partial sums per slot (<= 88 used)
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: bound of every wait

// ---------------------------------------------------------------- helpers --
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) {
  return *reinterpret_cast<const volatile int*>(p);
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}
// N little-endian words at a 2-byte aligned shared-memory address.
template <int N>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t* w) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 2) * 8;
  uint32_t r[N + 1];
#pragma unroll
  for (int i = 0; i <= N; i++) r[i] = b[i];
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}
__device__ __forceinline__ float h2f(uint32_t bits16) { return f16_bits((uint16_t)(bits16 & 0xffffu)); }
// Bit k (k < 4) of b to bit 4 of byte k.
__device__ __forceinline__ uint32_t spread4(uint32_t b) {
  return ((b & 15u) * 0x00204081u & 0x01010101u) << 4;
}
// sum_k c_k (2^16 hi_k + 2^8 mid_k + lo_k) over 8 words (32 values) as f32;
// codes < 128 or signed bytes.  Both int32 parts are exact: |sum c hi| <
// 32 * 128 * 127 and |sum c (256 mid + lo)| < 32 * 128 * 32639 < 2^31.
__device__ __forceinline__ float idot8(const uint32_t* c, const uint32_t* hi, const uint32_t* mid,
                                       const uint32_t* lo) {
  int a = 0, b = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) a = __dp4a((int)c[i], (int)hi[i], a);
#pragma unroll
  for (int i = 0; i < 8; i++) b = __dp4a((int)c[i], (int)mid[i], b);
  b <<= 8;
#pragma unroll
  for (int i = 0; i < 8; i++) b = __dp4a((int)c[i], (int)lo[i], b);
  return fmaf((float)a, 65536.0f, (float)b);
}

// ------------------------------------------------------------ staged x -----
// Class A (32-column groups, every block type but Q6_K and the dense ones):
//   hi, mid, lo [2][G] uint4 each, s [G] (scale / 2^16), X [G] (sum of x).
// Class B (Q6_K pieces: columns u*256 + h*128 + q*32 + o*8 + i of piece
//   p = u*8 + h*4 + o, run-major): hi, mid, lo [2][P], HI [P] int4 (per run
//   sum of hi), XI [P] int4 (per run sum of 256 mid + lo), s [P].
// Class D (dense types): x as f32.
struct XStage {
  const uint4 *ah, *am, *al;
  const float *as, *aX;
  int ag;
  const uint4 *bh, *bm, *bl;
  const int4 *bH, *bI;
  const float* bs;
  int bp;
  const float* d;
};

__host__ __device__ constexpr int xa_bytes(int cols) { return (cols / 32) * 104; }
__host__ __device__ constexpr int xb_bytes(int cols) { return (cols / 32) * 132; }

__device__ __forceinline__ XStage xstage_at(uint8_t* smem, const S1Smem& L, int cols) {
  XStage x;
  const int G = cols / 32, P = cols / 32;
  uint8_t* a = smem + L.xa;
  x.ah = reinterpret_cast<const uint4*>(a);
  x.am = x.ah + 2 * G;
  x.al = x.am + 2 * G;
  x.as = reinterpret_cast<const float*>(a + 96 * G);
  x.aX = x.as + G;
  x.ag = G;
  uint8_t* b = smem + L.xb;
  x.bh = reinterpret_cast<const uint4*>(b);
  x.bm = x.bh + 2 * P;
  x.bl = x.bm + 2 * P;
  x.bH = reinterpret_cast<const int4*>(b + 96 * P);
  x.bI = x.bH + P;
  x.bs = reinterpret_cast<const float*>(b + 128 * P);
  x.bp = P;
  x.d = reinterpret_cast<const float*>(smem + L.xd);
  return x;
}

// Source of a staged vector: v_i = src_i * (inv_rms * norm_i) (RMSNorm::forward,
// src/model.rs:65-73), or silu(src_i) * src2_i (SwiGLU, src/model.rs:251-254),
// or src_i.  src may live in shared memory (the embedding row).
struct XSrc {
  const float* src;
  const float* src2;
  const float* norm;
  float eps;
  int cols;
  bool smem;
};

__device__ __forceinline__ float ld_act(const float* p, bool smem) { return smem ? *p : __ldcg(p); }

// Splits 32 values into hi / mid / lo int8 words, x ~= s (hi + mid/2^8 +
// lo/2^16); returns s / 2^16.  hs / xi (may be null): per-word sums of hi and
// of 256 mid + lo.
__device__ __forceinline__ float split32(const float* v, uint32_t* hw, uint32_t* mw, uint32_t* lw,
                                         int* hs, int* xi) {
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; i++) mx = fmaxf(mx, fabsf(v[i]));
  const float s = mx > 0.0f && isfinite(mx) ? mx / 127.0f : 1.0f;
  const float inv = 1.0f / s;
#pragma unroll
  for (int w = 0; w < 8; w++) {
    uint32_t h = 0, m = 0, l = 0;
    int sh = 0, sx = 0;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const float q = v[4 * w + c] * inv;
      const float hq = fminf(fmaxf(rintf(q), -127.0f), 127.0f);
      const float r1 = (q - hq) * 256.0f;
      const float mq = fminf(fmaxf(rintf(r1), -127.0f), 127.0f);
      const float lq = fminf(fmaxf(rintf((r1 - mq) * 256.0f), -127.0f), 127.0f);
      h |= ((uint32_t)(int)hq & 0xffu) << (8 * c);
      m |= ((uint32_t)(int)mq & 0xffu) << (8 * c);
      l |= ((uint32_t)(int)lq & 0xffu) << (8 * c);
      sh += (int)hq;
      sx += 256 * (int)mq + (int)lq;
    }
    hw[w] = h;
    mw[w] = m;
    lw[w] = l;
    if (hs) hs[w] = sh, xi[w] = sx;
  }
  return s * (1.0f / 65536.0f);
}

// Stages `x` for the classes in `mask` (bit 0: A, 1: B, 2: D).  Run by the
// consumer threads; ends with their barrier.  red: >= kW floats.
__device__ __noinline__ void stage_x(const XSrc x, int mask, uint8_t* smem, const S1Smem L,
                                     float* red, int ctid) {
  float inv_rms = 1.0f;
  if (x.norm) {
    float ss = 0.0f;
    for (int c = ctid; c < x.cols; c += kCT) {
      const float v = ld_act(x.src + c, x.smem);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((ctid & 31) == 0) red[ctid >> 5] = ss;
    consumer_sync();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kW; w++) tot += red[w];
    inv_rms = 1.0f / sqrtf(tot / (float)x.cols + x.eps);
    consumer_sync();  // red is reused below
  }
  auto val = [&](int c) -> float {
    const float a = ld_act(x.src + c, x.smem);
    if (x.norm) return a * (inv_rms * __ldg(x.norm + c));
    if (x.src2) return (a / (1.0f + expf(-a))) * __ldcg(x.src2 + c);
    return a;
  };
  const int G = x.cols / 32;
  if (mask & 1) {
    uint8_t* a = smem + L.xa;
    uint4* ah = reinterpret_cast<uint4*>(a);
    uint4* am = ah + 2 * G;
    uint4* al = am + 2 * G;
    float* as = reinterpret_cast<float*>(a + 96 * G);
    float* aX = as + G;
    for (int g = ctid; g < G; g += kCT) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i++) v[i] = val(32 * g + i);
      uint32_t hw[8], mw[8], lw[8];
      const float s = split32(v, hw, mw, lw, nullptr, nullptr);
      float X = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; i++) X += v[i];
      ah[g] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      ah[G + g] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
      am[g] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
      am[G + g] = make_uint4(mw[4], mw[5], mw[6], mw[7]);
      al[g] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      al[G + g] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
      as[g] = s;
      aX[g] = X;
    }
  }
  if (mask & 2) {
    uint8_t* b = smem + L.xb;
    uint4* bh = reinterpret_cast<uint4*>(b);
    uint4* bm = bh + 2 * G;
    uint4* bl = bm + 2 * G;
    int4* bH = reinterpret_cast<int4*>(b + 96 * G);
    int4* bI = bH + G;
    float* bs = reinterpret_cast<float*>(b + 128 * G);
    for (int p = ctid; p < G; p += kCT) {
      const int u = p >> 3, hh = (p >> 2) & 1, o = p & 3;
      const int c0 = u * 256 + hh * 128 + o * 8;
      float v[32];
#pragma unroll
      for (int q = 0; q < 4; q++)
#pragma unroll
        for (int i = 0; i < 8; i++) v[q * 8 + i] = val(c0 + q * 32 + i);
      uint32_t hw[8], mw[8], lw[8];
      int hs[8], xi[8];
      const float s = split32(v, hw, mw, lw, hs, xi);
      bh[p] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      bh[G + p] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
      bm[p] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
      bm[G + p] = make_uint4(mw[4], mw[5], mw[6], mw[7]);
      bl[p] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      bl[G + p] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
      bH[p] = make_int4(hs[0] + hs[1], hs[2] + hs[3], hs[4] + hs[5], hs[6] + hs[7]);
      bI[p] = make_int4(xi[0] + xi[1], xi[2] + xi[3], xi[4] + xi[5], xi[6] + xi[7]);
      bs[p] = s;
    }
  }
  if (mask & 4) {
    float* d = reinterpret_cast<float*>(smem + L.xd);
    for (int c = ctid; c < x.cols; c += kCT) d[c] = val(c);
  }
  consumer_sync();
}

// ------------------------------------------------------- per-type pieces ---
// A piece is the unit one lane handles per row: one 32-value block (Q4_0 ..
// Q8_0), a pair of 32-column groups (Q4_K, Q5_K), a (half, octet) set of 32
// values (Q6_K), or 32 consecutive values (dense types).
template <int T>
struct PT;
#define LRS_PT(T, PPU, UB, CLS) \
  template <>                   \
  struct PT<T> {                \
    static constexpr int kPPU = PPU, kUB = UB, kClass = CLS; \
  };
LRS_PT(LRS_GGML_F32, 1, 128, 2)
LRS_PT(LRS_GGML_F16, 1, 64, 2)
LRS_PT(LRS_GGML_BF16, 1, 64, 2)
LRS_PT(LRS_GGML_Q4_0, 1, 18, 0)
LRS_PT(LRS_GGML_Q4_1, 1, 20, 0)
LRS_PT(LRS_GGML_Q5_0, 1, 22, 0)
LRS_PT(LRS_GGML_Q5_1, 1, 24, 0)
LRS_PT(LRS_GGML_Q8_0, 1, 34, 0)
LRS_PT(LRS_GGML_Q4_K, 4, 144, 0)
LRS_PT(LRS_GGML_Q5_K, 4, 176, 0)
LRS_PT(LRS_GGML_Q6_K, 8, 210, 1)
#undef LRS_PT

__device__ __forceinline__ void ld8(const uint4* p, int stride, uint32_t* w) {
  const uint4 a = p[0], b = p[stride];
  w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
}

// x registers of one piece.
template <int T, int CLS = PT<T>::kClass, int NGRP = PT<T>::kPPU == 4 ? 2 : 1>
struct XP;
template <int T, int NGRP>
struct XP<T, 0, NGRP> {  // class A: NGRP consecutive 32-column groups
  uint32_t h[8 * NGRP], m[8 * NGRP], l[8 * NGRP];
  float s[NGRP], X[NGRP];
  __device__ __forceinline__ void load(const XStage& x, int piece) {
#pragma unroll
    for (int k = 0; k < NGRP; k++) {
      const int g = piece * NGRP + k;
      ld8(x.ah + g, x.ag, h + 8 * k);
      ld8(x.am + g, x.ag, m + 8 * k);
      ld8(x.al + g, x.ag, l + 8 * k);
      s[k] = x.as[g];
      X[k] = x.aX[g];
    }
  }
};
template <int T, int NGRP>
struct XP<T, 1, NGRP> {  // class B: one Q6_K piece
  uint32_t h[8], m[8], l[8];
  int H[4], I[4];
  float s;
  __device__ __forceinline__ void load(const XStage& x, int piece) {
    ld8(x.bh + piece, x.bp, h);
    ld8(x.bm + piece, x.bp, m);
    ld8(x.bl + piece, x.bp, l);
    const int4 h4 = x.bH[piece], i4 = x.bI[piece];
    H[0] = h4.x, H[1] = h4.y, H[2] = h4.z, H[3] = h4.w;
    I[0] = i4.x, I[1] = i4.y, I[2] = i4.z, I[3] = i4.w;
    s = x.bs[piece];
  }
};
template <int T, int NGRP>
struct XP<T, 2, NGRP> {  // dense: 32 f32 values
  float v[32];
  __device__ __forceinline__ void load(const XStage& x, int piece) {
    const float4* p = reinterpret_cast<const float4*>(x.d + 32 * piece);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 t = p[i];
      v[4 * i] = t.x, v[4 * i + 1] = t.y, v[4 * i + 2] = t.z, v[4 * i + 3] = t.w;
    }
  }
};

// Row contribution of piece `sub` of the unit at `u` (shared memory).
template <int T>
__device__ __forceinline__ float pdot(const uint8_t* u, int sub, const XP<T>& x);

template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q4_0>(const uint8_t* u, int, const XP<LRS_GGML_Q4_0>& x) {
  uint32_t w[5];
  lds_words<5>(u, w);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16);
    c[i] = q & 0x0F0F0F0Fu;
    c[4 + i] = (q >> 4) & 0x0F0F0F0Fu;
  }
  const float L = idot8(c, x.h, x.m, x.l);
  return h2f(w[0]) * fmaf(x.s[0], L, -8.0f * x.X[0]);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q4_1>(const uint8_t* u, int, const XP<LRS_GGML_Q4_1>& x) {
  const uint32_t hd = lds32(u);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = lds32(u + 4 + 4 * i);
    c[i] = q & 0x0F0F0F0Fu;
    c[4 + i] = (q >> 4) & 0x0F0F0F0Fu;
  }
  const float L = idot8(c, x.h, x.m, x.l);
  return fmaf(h2f(hd) * x.s[0], L, h2f(hd >> 16) * x.X[0]);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q5_0>(const uint8_t* u, int, const XP<LRS_GGML_Q5_0>& x) {
  uint32_t w[6];
  lds_words<6>(u, w);
  const uint32_t qh = __funnelshift_r(w[0], w[1], 16);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = __funnelshift_r(w[1 + i], w[2 + i], 16);
    c[i] = (q & 0x0F0F0F0Fu) | spread4(qh >> (4 * i));
    c[4 + i] = ((q >> 4) & 0x0F0F0F0Fu) | spread4(qh >> (16 + 4 * i));
  }
  const float L = idot8(c, x.h, x.m, x.l);
  return h2f(w[0]) * fmaf(x.s[0], L, -16.0f * x.X[0]);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q5_1>(const uint8_t* u, int, const XP<LRS_GGML_Q5_1>& x) {
  const uint32_t hd = lds32(u), qh = lds32(u + 4);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t q = lds32(u + 8 + 4 * i);
    c[i] = (q & 0x0F0F0F0Fu) | spread4(qh >> (4 * i));
    c[4 + i] = ((q >> 4) & 0x0F0F0F0Fu) | spread4(qh >> (16 + 4 * i));
  }
  const float L = idot8(c, x.h, x.m, x.l);
  return fmaf(h2f(hd) * x.s[0], L, h2f(hd >> 16) * x.X[0]);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q8_0>(const uint8_t* u, int, const XP<LRS_GGML_Q8_0>& x) {
  uint32_t w[9];
  lds_words<9>(u, w);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 8; i++) c[i] = __funnelshift_r(w[i], w[i + 1], 16);
  const float L = idot8(c, x.h, x.m, x.l);
  return h2f(w[0]) * x.s[0] * L;
}
// Q4_K / Q5_K piece p: groups 2p and 2p+1 (src/quant.rs:403-436).
template <int T>
__device__ __forceinline__ float pdot_k45(const uint8_t* u, int p, const XP<T>& x) {
  constexpr bool k5 = T == LRS_GGML_Q5_K;
  const uint4 hd = lds128(u);
  const uint8_t* qs = u + (k5 ? 48 : 16) + 32 * p;
  const uint4 a = lds128(qs), b = lds128(qs + 16);
  const uint32_t q[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t c0[8], c1[8];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    c0[i] = q[i] & 0x0F0F0F0Fu;
    c1[i] = (q[i] >> 4) & 0x0F0F0F0Fu;
  }
  if constexpr (k5) {
    const uint4 e = lds128(u + 16), f = lds128(u + 32);
    const uint32_t qh[8] = {e.x, e.y, e.z, e.w, f.x, f.y, f.z, f.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      c0[i] |= ((qh[i] >> (2 * p)) & 0x01010101u) << 4;
      c1[i] |= ((qh[i] >> (2 * p + 1)) & 0x01010101u) << 4;
    }
  }
  const float L0 = idot8(c0, x.h, x.m, x.l), L1 = idot8(c1, x.h + 8, x.m + 8, x.l + 8);
  // scale_min_k4 (src/quant.rs:338-347) of groups 2p, 2p+1: bytes 2(p&1), +1
  // of the 32-bit words holding scales[0..3], [4..7], [8..11]
  const uint32_t sh = 16u * (uint32_t)(p & 1);
  const uint32_t w0 = hd.y >> sh, w1 = hd.z >> sh, w2 = hd.w >> sh;
  uint32_t sc0, sc1, mn0, mn1;
  if (p < 2) {
    sc0 = w0 & 63u, sc1 = (w0 >> 8) & 63u, mn0 = w1 & 63u, mn1 = (w1 >> 8) & 63u;
  } else {
    sc0 = (w2 & 0x0fu) | ((w0 >> 2) & 0x30u), sc1 = ((w2 >> 8) & 0x0fu) | ((w0 >> 10) & 0x30u);
    mn0 = ((w2 >> 4) & 0x0fu) | ((w1 >> 2) & 0x30u), mn1 = ((w2 >> 12) & 0x0fu) | ((w1 >> 10) & 0x30u);
  }
  const float t = fmaf((float)sc0 * x.s[0], L0, (float)sc1 * x.s[1] * L1);
  const float m = fmaf((float)mn0, x.X[0], (float)mn1 * x.X[1]);
  return fmaf(h2f(hd.x), t, -h2f(hd.x >> 16) * m);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q4_K>(const uint8_t* u, int p, const XP<LRS_GGML_Q4_K>& x) {
  return pdot_k45<LRS_GGML_Q4_K>(u, p, x);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q5_K>(const uint8_t* u, int p, const XP<LRS_GGML_Q5_K>& x) {
  return pdot_k45<LRS_GGML_Q5_K>(u, p, x);
}
// Q6_K piece (h, o) = sub: d * sum_q sc[q] * sum_i (code - 32) x (src/quant.rs:437-454).
template <>
__device__ __forceinline__ float pdot<LRS_GGML_Q6_K>(const uint8_t* u, int sub, const XP<LRS_GGML_Q6_K>& x) {
  const int hh = sub >> 2, o = sub & 3;
  uint32_t la[2], lb[2], qh[2], sw[2], dw[1];
  lds_words<2>(u + hh * 64 + o * 8, la);
  lds_words<2>(u + hh * 64 + 32 + o * 8, lb);
  lds_words<2>(u + 128 + hh * 32 + o * 8, qh);
  lds_words<2>(u + 192 + hh * 8, sw);
  lds_words<1>(u + 208, dw);
  float L[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t c[2];
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const uint32_t l = (q & 1) ? lb[k] : la[k];
      const uint32_t lo = (q & 2) ? ((l >> 4) & 0x0F0F0F0Fu) : (l & 0x0F0F0F0Fu);
      const uint32_t hb = q == 0 ? (qh[k] << 4) : q == 1 ? (qh[k] << 2) : q == 2 ? qh[k] : (qh[k] >> 2);
      c[k] = lo | (hb & 0x30303030u);
    }
    // sum (code - 32) x over the run, in the two exact int32 parts
    int a = __dp4a((int)c[0], (int)x.h[2 * q], 0);
    a = __dp4a((int)c[1], (int)x.h[2 * q + 1], a);
    int b = __dp4a((int)c[0], (int)x.m[2 * q], 0);
    b = __dp4a((int)c[1], (int)x.m[2 * q + 1], b);
    b <<= 8;
    b = __dp4a((int)c[0], (int)x.l[2 * q], b);
    b = __dp4a((int)c[1], (int)x.l[2 * q + 1], b);
    L[q] = fmaf((float)(a - 32 * x.H[q]), 65536.0f, (float)(b - 32 * x.I[q]));
  }
  // scales sc[2q + o/2] (int8): bytes (o>>1), 2+(o>>1) of sw[0] and of sw[1]
  const int so = o >> 1;
  const int s0 = (int)(int8_t)(sw[0] >> (8 * so)), s1 = (int)(int8_t)(sw[0] >> (8 * (2 + so)));
  const int s2 = (int)(int8_t)(sw[1] >> (8 * so)), s3 = (int)(int8_t)(sw[1] >> (8 * (2 + so)));
  const float acc = fmaf((float)s0, L[0], fmaf((float)s1, L[1], fmaf((float)s2, L[2], (float)s3 * L[3])));
  return h2f(dw[0]) * x.s * acc;
}
template <int T>
__device__ __forceinline__ float pdot_dense(const uint8_t* u, const XP<T>& x) {
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  if constexpr (T == LRS_GGML_F32) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 w = *reinterpret_cast<const float4*>(u + 16 * i);
      a0 = fmaf(w.x, x.v[4 * i], a0);
      a1 = fmaf(w.y, x.v[4 * i + 1], a1);
      a2 = fmaf(w.z, x.v[4 * i + 2], a2);
      a3 = fmaf(w.w, x.v[4 * i + 3], a3);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint4 w = lds128(u + 16 * i);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        float lo, hi;
        if constexpr (T == LRS_GGML_F16) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[k]));
          lo = f.x, hi = f.y;
        } else {
          lo = __uint_as_float(ww[k] << 16), hi = __uint_as_float(ww[k] & 0xffff0000u);
        }
        const int c = 8 * i + 2 * k;
        if (k & 1) {
          a2 = fmaf(lo, x.v[c], a2);
          a3 = fmaf(hi, x.v[c + 1], a3);
        } else {
          a0 = fmaf(lo, x.v[c], a0);
          a1 = fmaf(hi, x.v[c + 1], a1);
        }
      }
    }
  }
  return (a0 + a1) + (a2 + a3);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_F32>(const uint8_t* u, int, const XP<LRS_GGML_F32>& x) {
  return pdot_dense<LRS_GGML_F32>(u, x);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_F16>(const uint8_t* u, int, const XP<LRS_GGML_F16>& x) {
  return pdot_dense<LRS_GGML_F16>(u, x);
}
template <>
__device__ __forceinline__ float pdot<LRS_GGML_BF16>(const uint8_t* u, int, const XP<LRS_GGML_BF16>& x) {
  return pdot_dense<LRS_GGML_BF16>(u, x);
}

// -------------------------------------------------------------- the ring ---
struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int ns;
};

struct Shared {  // per-CTA control words (shared memory)
  int abort;
  int last;        // this CTA combines a KV head
  unsigned long long key;  // CTA argmax key
  int cnt[8];      // per-slot consumer-warp counters
};

// Bounded wait on an mbarrier phase; false on timeout or abort.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          const int* gerr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtime();
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255) {
      if (*abort || (gerr && ld_volatile_i32(gerr))) return false;
      if (gtime() - t0 > kWaitNs) return false;
    }
  }
}

__device__ __forceinline__ void cta_rows(int rows, int b, int G, int& r0, int& r1) {
  r0 = (int)((long long)rows * b / G);
  r1 = (int)((long long)rows * (b + 1) / G);
}

// ----------------------------------------------------------- the producer --
struct Producer {
  Ring ring;
  uint64_t policy;
  int seq;
  volatile int* abort;
  const int* gerr;
  bool ok;
};

// Issues the bulk copies of every chunk of this CTA's rows of ms[0..n).
__device__ __noinline__ void produce(Producer& pr, const S1Mat* ms, int n, int b, int G) {
  const Ring ring = pr.ring;
  const uint64_t policy = pr.policy;
  int seq = pr.seq;
  bool ok = pr.ok;
  for (int mi = 0; mi < n && ok; mi++) {
    const S1Mat m = ms[mi];
    int r0, r1;
    cta_rows(m.rows, b, G, r0, r1);
    const int nkc = (m.units + m.ku - 1) / m.ku;
    const int nm = m.w2 ? 2 : 1;
    for (int row = r0; row < r1 && ok; row += m.kr) {
      const int kr = min(m.kr, r1 - row);
      for (int kc = 0; kc < nkc && ok; kc++) {
        const int u0 = kc * m.ku, nu = min(m.ku, m.units - u0);
        const int s = seq % ring.ns, k = seq / ring.ns;
        if (k >= 1) {
          ok = ring_wait(&ring.empty[s], (uint32_t)((k - 1) & 1), pr.abort, pr.gerr);
          if (!ok) break;
          fence_proxy_async();
        }
        const size_t len = (size_t)(kr - 1) * m.rb + (size_t)nu * m.ub;
        uint32_t total = 0;
        uintptr_t lo[2];
        uint32_t sz[2];
#pragma unroll
        for (int mm = 0; mm < 2; mm++) {
          if (mm >= nm) break;
          const uintptr_t a =
              reinterpret_cast<uintptr_t>((mm ? m.w2 : m.w) + (size_t)row * m.rb + (size_t)u0 * m.ub);
          lo[mm] = a & ~uintptr_t(15);
          sz[mm] = (uint32_t)(((a + len + 15) & ~uintptr_t(15)) - lo[mm]);
          total += sz[mm];
        }
        mbar_expect_tx(&ring.full[s], total);
#pragma unroll
        for (int mm = 0; mm < 2; mm++) {
          if (mm >= nm) break;
          tma_load_1d(ring.base + (size_t)s * kS1Slot + (size_t)mm * m.part,
                      reinterpret_cast<const void*>(lo[mm]), sz[mm], &ring.full[s], policy);
        }
        seq++;
      }
    }
  }
  pr.seq = seq;
  pr.ok = ok;
}

// ----------------------------------------------------------- the consumer --
struct Consumer {
  Ring ring;
  int seq;
  float* red;        // [ns][kRedPerSlot]
  Shared* sh;
  const int* gerr;
  int* error_flag;
  int warp, lane;
  bool ok;
};

template <int T, int R, int NM>
__device__ __forceinline__ void group_pieces(const uint8_t* const* base, int rb, int nvalid, int u0,
                                             int nu, int li, int nl, const XStage& xs,
                                             float (&acc)[NM][R]) {
  constexpr int PPU = PT<T>::kPPU, UB = PT<T>::kUB;
  const int np = nu * PPU;
  for (int pl = li; pl < np; pl += nl) {
    const int unit = pl / PPU, sub = pl - unit * PPU;
    XP<T> x;
    x.load(xs, (u0 + unit) * PPU + sub);
#pragma unroll
    for (int mm = 0; mm < NM; mm++)
#pragma unroll
      for (int r = 0; r < R; r++)
        if (r < nvalid) acc[mm][r] += pdot<T>(base[mm] + (size_t)r * rb + (size_t)unit * UB, sub, x);
  }
}

// Fixed-order sum of a chunk's partials and the output step (lane = row).
template <int NM>
__device__ __forceinline__ void chunk_epilogue(const S1Mat& m, const float* red, Shared* sh,
                                               int row0, int kr, int R, int wpg, int lane) {
  const int i = lane;
  unsigned long long key = 0ull;
  if (i < kr) {
    const int g = i / R, r = i - g * R;
    float y[NM];
#pragma unroll
    for (int mm = 0; mm < NM; mm++) {
      float a = 0.0f;
      for (int w = 0; w < wpg; w++) a += red[((g * wpg + w) * NM + mm) * R + r];
      y[mm] = a;
    }
    const int row = row0 + i;
    switch (m.epi) {
      case EPI_STORE:
        m.out[row] = m.bias ? y[0] + __ldg(m.bias + row) : y[0];
        break;
      case EPI_ADD:
        m.out[row] = __ldcg(m.out + row) + y[0];
        break;
      case EPI_SWIGLU:
        m.out[row] = (y[0] / (1.0f + expf(-y[0]))) * y[NM - 1];
        break;
      default:
        if (m.out) m.out[row] = y[0];
        key = argmax_pack(y[0], (uint32_t)row);
    }
  }
  if (m.epi == EPI_ARGMAX) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
      key = k2 > key ? k2 : key;
    }
    if (lane == 0 && key) atomicMax(&sh->key, key);
  }
}

// One matrix of a phase: every chunk of this CTA's rows.  The matrix, the
// staged-x views and the consumer state are copied into registers first.
template <int T, int R, int NM>
__device__ __forceinline__ void run_mat(Consumer& c, const S1Mat& mg, int b, int G,
                                        const XStage& xsg) {
  const S1Mat m = mg;
  const XStage xs = xsg;
  const Ring ring = c.ring;
  float* const red = c.red;
  Shared* const sh = c.sh;
  const int* const gerr = c.gerr;
  int* const error_flag = c.error_flag;
  const int warp = c.warp, lane = c.lane;
  int seq = c.seq;
  bool ok = c.ok;
  int r0, r1;
  cta_rows(m.rows, b, G, r0, r1);
  const int nkc = (m.units + m.ku - 1) / m.ku;
  float acc[NM][R];
  for (int row = r0; row < r1 && ok; row += m.kr) {
    const int kr = min(m.kr, r1 - row);
    const int NG = (kr + R - 1) / R;
    const int wpg = NG >= kW ? 1 : kW / NG;
#pragma unroll
    for (int mm = 0; mm < NM; mm++)
#pragma unroll
      for (int r = 0; r < R; r++) acc[mm][r] = 0.0f;
    for (int kc = 0; kc < nkc && ok; kc++) {
      const int u0 = kc * m.ku, nu = min(m.ku, m.units - u0);
      const int s = seq % ring.ns, k = seq / ring.ns;
      // every lane waits: the completed phase orders the bulk copy's writes
      // before its own reads of the slot
      const bool got =
          __all_sync(0xffffffffu, ring_wait(&ring.full[s], (uint32_t)(k & 1), &sh->abort, gerr));
      if (!got) {
        if (lane == 0) {
          sh->abort = 1;
          if (error_flag) atomicExch(error_flag, LRS_ERR_DEVICE_TIMEOUT);
        }
        ok = false;
        break;
      }
      const uint8_t* slot = ring.base + (size_t)s * kS1Slot;
      const size_t off = (size_t)row * m.rb + (size_t)u0 * m.ub;
      const bool last_kc = kc == nkc - 1;
      const int g_first = NG >= kW ? warp : warp / wpg;
      const int ws = NG >= kW ? 0 : warp % wpg;
      float* red_s = red + s * kRedPerSlot;
      if (NG >= kW || warp < NG * wpg) {
        for (int g = g_first; g < NG; g += kW) {
          const uint8_t* base[NM];
#pragma unroll
          for (int mm = 0; mm < NM; mm++) {
            const uintptr_t a = reinterpret_cast<uintptr_t>((mm ? m.w2 : m.w) + off);
            base[mm] = slot + (size_t)mm * m.part + (a & 15) + (size_t)(g * R) * m.rb;
          }
          if (NG >= kW) {
#pragma unroll
            for (int mm = 0; mm < NM; mm++)
#pragma unroll
              for (int r = 0; r < R; r++) acc[mm][r] = 0.0f;
          }
          group_pieces<T, R, NM>(base, m.rb, kr - g * R, u0, nu, ws * 32 + lane, 32 * wpg, xs, acc);
          if (last_kc) {
#pragma unroll
            for (int mm = 0; mm < NM; mm++)
#pragma unroll
              for (int r = 0; r < R; r++) {
                float v = acc[mm][r];
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) red_s[((g * wpg + ws) * NM + mm) * R + r] = v;
              }
          }
          if (NG < kW) break;
        }
      }
      __syncwarp();
      bool last_warp = false;
      if (last_kc) {
        if (lane == 0) {
          __threadfence_block();
          last_warp = atomicAdd(&sh->cnt[s], 1) == kW - 1;
        }
        last_warp = __shfl_sync(0xffffffffu, last_warp, 0);
      }
      if (last_warp) {
        __threadfence_block();
        chunk_epilogue<NM>(m, red_s, sh, row, kr, R, wpg, lane);
        if (lane == 0) sh->cnt[s] = 0;
        __syncwarp();
      }
      if (lane == 0) mbar_arrive1(&ring.empty[s]);
      seq++;
    }
  }
  c.seq = seq;
  c.ok = ok;
}

template <int T>
__device__ __forceinline__ void run_mat_t(Consumer& c, const S1Mat& m, int b, int G, const XStage& xs) {
  if (m.w2) {
    if (m.R == 2) run_mat<T, 2, 2>(c, m, b, G, xs);
    else run_mat<T, 1, 2>(c, m, b, G, xs);
  } else {
    if (m.R == 4) run_mat<T, 4, 1>(c, m, b, G, xs);
    else if (m.R == 2) run_mat<T, 2, 1>(c, m, b, G, xs);
    else run_mat<T, 1, 1>(c, m, b, G, xs);
  }
}

__device__ __noinline__ void consume(Consumer& c, const S1Mat& m, int b, int G, const XStage& xs) {
  switch (m.type) {
    case LRS_GGML_F32: run_mat_t<LRS_GGML_F32>(c, m, b, G, xs); break;
    case LRS_GGML_F16: run_mat_t<LRS_GGML_F16>(c, m, b, G, xs); break;
    case LRS_GGML_BF16: run_mat_t<LRS_GGML_BF16>(c, m, b, G, xs); break;
    case LRS_GGML_Q4_0: run_mat_t<LRS_GGML_Q4_0>(c, m, b, G, xs); break;
    case LRS_GGML_Q4_1: run_mat_t<LRS_GGML_Q4_1>(c, m, b, G, xs); break;
    case LRS_GGML_Q5_0: run_mat_t<LRS_GGML_Q5_0>(c, m, b, G, xs); break;
    case LRS_GGML_Q5_1: run_mat_t<LRS_GGML_Q5_1>(c, m, b, G, xs); break;
    case LRS_GGML_Q8_0: run_mat_t<LRS_GGML_Q8_0>(c, m, b, G, xs); break;
    case LRS_GGML_Q4_K: run_mat_t<LRS_GGML_Q4_K>(c, m, b, G, xs); break;
    case LRS_GGML_Q5_K: run_mat_t<LRS_GGML_Q5_K>(c, m, b, G, xs); break;
    case LRS_GGML_Q6_K: run_mat_t<LRS_GGML_Q6_K>(c, m, b, G, xs); break;
  }
}

__device__ __forceinline__ int class_mask(const S1Mat* ms, int n) {
  int mask = 0;
  for (int i = 0; i < n; i++) {
    const int t = ms[i].type;
    mask |= t == LRS_GGML_Q6_K ? 2 : (t == LRS_GGML_F32 || t == LRS_GGML_F16 || t == LRS_GGML_BF16) ? 4 : 1;
  }
  return mask;
}

// Shared-memory carve-up common to both kernels.
struct Carve {
  Ring ring;
  float* red;
  float* work;
  Shared* sh;
};
__device__ __forceinline__ Carve carve(uint8_t* smem, const S1Smem& L) {
  Carve c;
  c.ring.base = smem;
  c.ring.ns = L.nslots;
  c.ring.full = reinterpret_cast<uint64_t*>(smem + L.bars);
  c.ring.empty = c.ring.full + L.nslots;
  c.red = reinterpret_cast<float*>(smem + L.red);
  c.work = reinterpret_cast<float*>(smem + L.work);
  c.sh = reinterpret_cast<Shared*>(smem + L.misc);
  return c;
}

__device__ void init_shared(const Carve& c, int tid) {
  if (tid == 0) {
    for (int s = 0; s < c.ring.ns; s++) {
      mbar_init(&c.ring.full[s], 1);
      mbar_init(&c.ring.empty[s], kW);
    }
    fence_barrier_init();
    c.sh->abort = 0;
    c.sh->last = 0;
    c.sh->key = 0ull;
    for (int s = 0; s < 8; s++) c.sh->cnt[s] = 0;
  }
  __syncthreads();
}

// After an abort: the copies the producer issued must land before the CTA exits.
__device__ void drain(const Producer& p) {
  const int n = min(p.seq, p.ring.ns);
  const uint64_t t0 = gtime();
  for (int i = p.seq - n; i < p.seq; i++) {
    const int s = i % p.ring.ns;
    const uint32_t par = (uint32_t)((i / p.ring.ns) & 1);
    while (!mbar_try_wait(&p.ring.full[s], par))
      if (gtime() - t0 > kWaitNs) return;
  }
}

// ---------------------------------------------------------- one GEMV kernel --
__global__ void __launch_bounds__(kS1Threads, 1)
    s1_gemv_kernel(const __grid_constant__ S1Mat m, const float* x, int* error_flag,
                   const __grid_constant__ S1Smem L) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Carve c = carve(smem, L);
  init_shared(c, tid);
  const int b = blockIdx.x, G = gridDim.x;
  if (warp == kW) {
    if (lane == 0) {
      Producer p{c.ring, evict_first_policy(), 0, &c.sh->abort, error_flag, true};
      produce(p, &m, 1, b, G);
      if (!p.ok) drain(p);
    }
    return;
  }
  const int mask = class_mask(&m, 1);
  stage_x(XSrc{x, nullptr, nullptr, 0.0f, m.cols, false}, mask, smem, L, c.red, tid);
  const XStage xs = xstage_at(smem, L, m.cols);
  Consumer cons{c.ring, 0, c.red, c.sh, error_flag, error_flag, warp, lane, true};
  consume(cons, m, b, G, xs);
}

// ------------------------------------------------------ the decode step ----
// Grid barrier of the consumers (all CTAs): false when aborted.
struct GridSync {
  unsigned* ctr;
  unsigned n;  // barriers passed (thread 0 of the CTA)
  __device__ bool sync(Shared* sh, int ctid, int* error_flag) {
    consumer_sync();
    if (ctid == 0) {
      n++;
      const unsigned target = n * gridDim.x;
      __threadfence();
      atomicAdd(ctr, 1u);
      if (!sh->abort) {
        const uint64_t t0 = gtime();
        for (uint32_t i = 0;; i++) {
          if (ld_acquire_u32(ctr) >= target) break;
          if ((i & 63) == 63) {
            if (error_flag && ld_volatile_i32(error_flag)) {
              sh->abort = 1;
              break;
            }
            if (gtime() - t0 > kWaitNs) {
              sh->abort = 1;
              if (error_flag) atomicExch(error_flag, LRS_ERR_DEVICE_TIMEOUT);
              break;
            }
          }
        }
      }
    }
    consumer_sync();
    return !*reinterpret_cast<volatile int*>(&sh->abort);
  }
};

// N consecutive K or V values of a cached row (written by earlier launches).
template <bool BF16, int N>
__device__ __forceinline__ void ld_kv(const void* pool, size_t off, float* o) {
  if constexpr (BF16) {
    const uint16_t* p = reinterpret_cast<const uint16_t*>(pool) + off;
    if constexpr (N == 4) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
      o[0] = __uint_as_float(u.x << 16), o[1] = __uint_as_float(u.x & 0xffff0000u);
      o[2] = __uint_as_float(u.y << 16), o[3] = __uint_as_float(u.y & 0xffff0000u);
    } else {
      const uint32_t u = __ldg(reinterpret_cast<const uint32_t*>(p));
      o[0] = __uint_as_float(u << 16), o[1] = __uint_as_float(u & 0xffff0000u);
    }
  } else {
    const float* p = reinterpret_cast<const float*>(pool) + off;
    if constexpr (N == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p));
      o[0] = t.x, o[1] = t.y, o[2] = t.z, o[3] = t.w;
    } else {
      const float2 t = __ldg(reinterpret_cast<const float2*>(p));
      o[0] = t.x, o[1] = t.y;
    }
  }
}

__device__ __forceinline__ size_t kv_off(const S1Model& M, int seq, int p, int kvh) {
  const int page = __ldcg(M.pages + seq * M.max_pages + p / kPageSize);
  return (((size_t)page * M.nkv + kvh) * kPageSize + (p % kPageSize)) * M.hd;
}

// Attention of one (KV head, split) pair (src/model.rs:188-231).
template <bool BF16, int HD>
__device__ __noinline__ void attention(const S1Model& M, const S1Layer& Ly, float* work, Shared* sh,
                                       int b, int ctid) {
  const int warp = ctid >> 5, lane = ctid & 31;
  constexpr int hd = HD, half = HD / 2, dpl = HD / 32;
  const int nkv = M.nkv, G = M.nh / nkv;
  const int pos = __ldcg(M.pos), seq = __ldcg(M.seq), L = pos + 1;
  int nsplit = min(M.max_split, max(1, (L + 63) / 64));
  const int chunk = (L + nsplit - 1) / nsplit;
  nsplit = (L + chunk - 1) / chunk;  // splits that hold positions
  const int kvh = b % nkv, split = b / nkv;
  if (split >= nsplit || chunk > M.split_cap) return;
  const int s0 = split * chunk, s1 = min(L, s0 + chunk), n = s1 - s0;
  const int cap = M.split_cap;
  float* qs = work;                   // [G][hd]
  float* sc = qs + kS1MaxGroup * hd;  // [G][split_cap]
  float* kn = sc + kS1MaxGroup * cap;  // [hd] rotated k of the new position
  float* vn = kn + hd;                 // [hd]
  float* ml = vn + hd;                 // [G][2]: m, l
  const float* cs = M.rope_cos + (size_t)pos * half;
  const float* sn = M.rope_sin + (size_t)pos * half;
  // q rotated and scaled: split-half RoPE, unfused like apply_rope_inplace
  for (int i = ctid; i < G * half; i += kCT) {
    const int g = i / half, j = i - g * half;
    const float* qh = M.q + (size_t)(kvh * G + g) * hd;
    const float re = __ldcg(qh + j), im = __ldcg(qh + j + half);
    const float c = __ldg(cs + j), s = __ldg(sn + j);
    qs[g * hd + j] = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s)) * M.attn_scale;
    qs[g * hd + j + half] = __fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c)) * M.attn_scale;
  }
  if (s1 == L) {  // this split holds the new position: rotate k, store k and v
    const size_t o = kv_off(M, seq, pos, kvh);
    const float* kh = M.k + (size_t)kvh * hd;
    const float* vh = M.v + (size_t)kvh * hd;
    for (int j = ctid; j < half; j += kCT) {
      const float re = __ldcg(kh + j), im = __ldcg(kh + j + half);
      const float c = __ldg(cs + j), s = __ldg(sn + j);
      float k0 = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s));
      float k1 = __fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c));
      float v0 = __ldcg(vh + j), v1 = __ldcg(vh + j + half);
      if constexpr (BF16) {
        __nv_bfloat16* kp = reinterpret_cast<__nv_bfloat16*>(Ly.kpool) + o;
        __nv_bfloat16* vp = reinterpret_cast<__nv_bfloat16*>(Ly.vpool) + o;
        const __nv_bfloat16 a = __float2bfloat16_rn(k0), bb = __float2bfloat16_rn(k1);
        const __nv_bfloat16 c2 = __float2bfloat16_rn(v0), d2 = __float2bfloat16_rn(v1);
        kp[j] = a, kp[j + half] = bb, vp[j] = c2, vp[j + half] = d2;
        // what a later step reads back
        k0 = __bfloat162float(a), k1 = __bfloat162float(bb);
        v0 = __bfloat162float(c2), v1 = __bfloat162float(d2);
      } else {
        float* kp = reinterpret_cast<float*>(Ly.kpool) + o;
        float* vp = reinterpret_cast<float*>(Ly.vpool) + o;
        kp[j] = k0, kp[j + half] = k1, vp[j] = v0, vp[j + half] = v1;
      }
      kn[j] = k0, kn[j + half] = k1, vn[j] = v0, vn[j + half] = v1;
    }
  }
  consumer_sync();
  // scores: warps over positions, lanes over the head dimension
  float qr[kS1MaxGroup][dpl];
#pragma unroll
  for (int g = 0; g < kS1MaxGroup; g++)
#pragma unroll
    for (int i = 0; i < dpl; i++) qr[g][i] = g < G ? qs[g * hd + lane * dpl + i] : 0.0f;
  for (int j = warp; j < n; j += kW) {
    const int p = s0 + j;
    float kv[dpl];
    if (p == pos) {
#pragma unroll
      for (int i = 0; i < dpl; i++) kv[i] = kn[lane * dpl + i];
    } else {
      ld_kv<BF16, dpl>(Ly.kpool, kv_off(M, seq, p, kvh) + lane * dpl, kv);
    }
#pragma unroll
    for (int g = 0; g < kS1MaxGroup; g++) {
      if (g >= G) break;
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < dpl; i++) d = fmaf(qr[g][i], kv[i], d);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (lane == 0) sc[g * cap + j] = d;
    }
  }
  consumer_sync();
  // softmax partials (softmax_inplace, src/model.rs:298-313): warp g, head g
  if (warp < G) {
    float* row = sc + warp * cap;
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.0f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(row[j] - mx);
      row[j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) ml[2 * warp] = mx, ml[2 * warp + 1] = l;
  }
  consumer_sync();
  // PV: warp g accumulates head g over the split, lanes over the dimension
  if (warp < G) {
    const float* e = sc + warp * cap;
    float o[dpl];
#pragma unroll
    for (int i = 0; i < dpl; i++) o[i] = 0.0f;
    for (int j = 0; j < n; j++) {
      const int p = s0 + j;
      float vv[dpl];
      if (p == pos) {
#pragma unroll
        for (int i = 0; i < dpl; i++) vv[i] = vn[lane * dpl + i];
      } else {
        ld_kv<BF16, dpl>(Ly.vpool, kv_off(M, seq, p, kvh) + lane * dpl, vv);
      }
      const float ej = e[j];
#pragma unroll
      for (int i = 0; i < dpl; i++) o[i] = fmaf(ej, vv[i], o[i]);
    }
    float* pp = M.part + ((size_t)(kvh * M.max_split + split) * G + warp) * (2 + hd);
    if (lane == 0) pp[0] = ml[2 * warp], pp[1] = ml[2 * warp + 1];
#pragma unroll
    for (int i = 0; i < dpl; i++) pp[2 + lane * dpl + i] = o[i];
  }
  // the last split to finish for this KV head merges them
  consumer_sync();
  if (ctid == 0) {
    __threadfence();
    sh->last = atomicAdd(&M.attn_cnt[kvh], 1u) == (unsigned)(nsplit - 1);
  }
  consumer_sync();
  if (!sh->last) return;
  __threadfence();
  for (int i = ctid; i < G * hd; i += kCT) {
    const int g = i / hd, d = i - g * hd;
    float mx = -INFINITY;
    for (int s = 0; s < nsplit; s++)
      mx = fmaxf(mx, __ldcg(M.part + ((size_t)(kvh * M.max_split + s) * G + g) * (2 + hd)));
    float l = 0.0f, acc = 0.0f;
    for (int s = 0; s < nsplit; s++) {
      const float* pp = M.part + ((size_t)(kvh * M.max_split + s) * G + g) * (2 + hd);
      const float w = expf(__ldcg(pp) - mx);
      l = fmaf(__ldcg(pp + 1), w, l);
      acc = fmaf(__ldcg(pp + 2 + d), w, acc);
    }
    M.att[(size_t)(kvh * G + g) * hd + d] = acc / l;
  }
  consumer_sync();
  if (ctid == 0) {
    M.attn_cnt[kvh] = 0u;
    sh->last = 0;
  }
}

// The embedding row (row_into with value_at, bit-exact) into `e`.
__device__ __noinline__ void embed_row(const S1Model& M, float* e, int ctid) {
  const int tok = __ldcg(M.tok);
  const int h = M.h;
  switch (M.embed_type) {
#define LRS_EMB(T)                                                                         \
  case T: {                                                                                \
    using BT = BlockTraits<T>;                                                             \
    const uint8_t* rp = M.embed + (size_t)tok * (h / BT::kValues) * BT::kBytes;            \
    for (int pc = ctid; pc < h / 32; pc += kCT) {                                          \
      const int unit = pc / BT::kPieces, sub = pc % BT::kPieces;                           \
      float v[32];                                                                         \
      decode_piece<T>(rp + (size_t)unit * BT::kBytes, sub, v);                             \
      for (int r = 0; r < 4; r++)                                                          \
        for (int i = 0; i < 8; i++) e[unit * BT::kValues + run_col<T>(sub, r) + i] = v[r * 8 + i]; \
    }                                                                                      \
  } break;
    LRS_EMB(LRS_GGML_F32)
    LRS_EMB(LRS_GGML_F16)
    LRS_EMB(LRS_GGML_BF16)
    LRS_EMB(LRS_GGML_Q4_0)
    LRS_EMB(LRS_GGML_Q4_1)
    LRS_EMB(LRS_GGML_Q5_0)
    LRS_EMB(LRS_GGML_Q5_1)
    LRS_EMB(LRS_GGML_Q8_0)
    LRS_EMB(LRS_GGML_Q4_K)
    LRS_EMB(LRS_GGML_Q5_K)
    LRS_EMB(LRS_GGML_Q6_K)
#undef LRS_EMB
  }
}

__global__ void __launch_bounds__(kS1Threads, 1)
    s1_step_kernel(const S1Model* __restrict__ Mp, int advance) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const S1Model& M = *Mp;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const S1Smem Ls = M.sm;
  const Carve c = carve(smem, Ls);
  init_shared(c, tid);
  const int b = blockIdx.x, G = gridDim.x;
  if (warp == kW) {
    // ---- producer: every weight chunk of the step, in consumption order ----
    if (lane == 0) {
      Producer p{c.ring, evict_first_policy(), 0, &c.sh->abort, M.error_flag, true};
      for (int l = 0; l < M.L && p.ok; l++) {
        const S1Layer* Ly = M.layers + l;
        produce(p, Ly->qkv, 3, b, G);
        produce(p, &Ly->o, 1, b, G);
        produce(p, Ly->gu, Ly->ngu, b, G);
        produce(p, &Ly->down, 1, b, G);
      }
      produce(p, &M.lm, 1, b, G);
      if (!p.ok) drain(p);
    }
    return;
  }
  // ---- consumers ----
  GridSync gs{M.bar_ctr, 0u};
  Consumer cons{c.ring, 0, c.red, c.sh, M.error_flag, M.error_flag, warp, lane, true};
  const int ctid = tid;
  if (b == 0 && ctid == 0) *M.keys = 0ull;
  embed_row(M, c.work, ctid);
  consumer_sync();
  if (b == 0)
    for (int i = ctid; i < M.h; i += kCT) M.residual[i] = c.work[i];
  bool ok = true;
  for (int l = 0; l < M.L && ok; l++) {
    const S1Layer& Ly = M.layers[l];
    // input_layernorm + q/k/v with bias (src/model.rs:175-186)
    {
      stage_x(XSrc{l == 0 ? c.work : M.residual, nullptr, Ly.in_norm, M.eps, M.h, l == 0},
              class_mask(Ly.qkv, 3), smem, Ls, c.red, ctid);
      const XStage xs = xstage_at(smem, Ls, M.h);
      for (int i = 0; i < 3 && cons.ok; i++) consume(cons, Ly.qkv[i], b, G, xs);
    }
    if (!(ok = gs.sync(c.sh, ctid, M.error_flag) && cons.ok)) break;
    // RoPE, KV store, attention (src/model.rs:188-231)
    if (M.hd == 128) {
      if (M.kv_bf16) attention<true, 128>(M, Ly, c.work, c.sh, b, ctid);
      else attention<false, 128>(M, Ly, c.work, c.sh, b, ctid);
    } else {
      if (M.kv_bf16) attention<true, 64>(M, Ly, c.work, c.sh, b, ctid);
      else attention<false, 64>(M, Ly, c.work, c.sh, b, ctid);
    }
    if (!(ok = gs.sync(c.sh, ctid, M.error_flag))) break;
    // o_proj + residual (src/model.rs:233-238)
    {
      stage_x(XSrc{M.att, nullptr, nullptr, 0.0f, M.nh * M.hd, false}, class_mask(&Ly.o, 1), smem,
              Ls, c.red, ctid);
      consume(cons, Ly.o, b, G, xstage_at(smem, Ls, M.nh * M.hd));
    }
    if (!(ok = gs.sync(c.sh, ctid, M.error_flag) && cons.ok)) break;
    // post_attention_layernorm + gate/up + SwiGLU (src/model.rs:241-254)
    {
      stage_x(XSrc{M.residual, nullptr, Ly.post_norm, M.eps, M.h, false}, class_mask(Ly.gu, Ly.ngu),
              smem, Ls, c.red, ctid);
      const XStage xs = xstage_at(smem, Ls, M.h);
      for (int i = 0; i < Ly.ngu && cons.ok; i++) consume(cons, Ly.gu[i], b, G, xs);
    }
    if (!(ok = gs.sync(c.sh, ctid, M.error_flag) && cons.ok)) break;
    // down_proj + residual (src/model.rs:255-260)
    {
      stage_x(XSrc{M.act, Ly.ngu == 2 ? M.act2 : nullptr, nullptr, 0.0f, M.inter, false},
              class_mask(&Ly.down, 1), smem, Ls, c.red, ctid);
      consume(cons, Ly.down, b, G, xstage_at(smem, Ls, M.inter));
    }
    if (!(ok = gs.sync(c.sh, ctid, M.error_flag) && cons.ok)) break;
  }
  if (ok) {
    // final norm + lm_head + greedy argmax (src/model.rs:263-268, src/engine.rs:233-241)
    stage_x(XSrc{M.residual, nullptr, M.final_norm, M.eps, M.h, false}, class_mask(&M.lm, 1), smem,
            Ls, c.red, ctid);
    consume(cons, M.lm, b, G, xstage_at(smem, Ls, M.h));
    consumer_sync();
    if (ctid == 0 && c.sh->key) atomicMax(M.keys, c.sh->key);
    ok = gs.sync(c.sh, ctid, M.error_flag) && cons.ok;
  }
  if (ok && advance && b == 0 && ctid == 0) {
    // advance_kernel: the token fed to the next step, position, output row
    const int s = *M.step;
    const uint32_t t = (uint32_t)(__ldcg(M.keys) & 0xffffffffull);
    *M.tok = (int)t;
    *M.pos += 1;
    if (M.last) *M.last = t;
    if (M.tokens_out && s < M.n_steps_cap) M.tokens_out[s] = t;
    *M.step = s + 1;
  }
}

std::atomic<uint64_t> g_attr_gemv{0}, g_attr_step{0};

}  // namespace

int s1_xclass(int type) {
  if (type == LRS_GGML_Q6_K) return 1;
  if (type == LRS_GGML_F32 || type == LRS_GGML_F16 || type == LRS_GGML_BF16) return 2;
  return 0;
}

bool s1_plan_mat(S1Mat* m, int nm, int grid) {
  uint32_t bv, bb;
  if (!type_geometry((uint32_t)m->type, &bv, &bb)) return false;
  const bool dense = bv == 1;
  m->ub = dense ? (int)bb * 32 : (int)bb;
  m->units = m->cols / (dense ? 32 : (int)bv);
  m->rb = (int)row_bytes((uint32_t)m->type, (size_t)m->cols);
  m->part = nm == 2 ? (kS1Slot / 2) & ~15 : kS1Slot;
  const int avail = m->part - 32;  // alignment slop and the word past a 2-byte aligned piece
  if (m->rb <= avail) {
    m->kr = std::min(kS1MaxRows, avail / m->rb);
    m->ku = m->units;
  } else {
    m->kr = 1;
    m->ku = std::max(1, avail / m->ub);
  }
  // a CTA's rows: no more than its share
  const int share = std::max(1, (m->rows + grid - 1) / grid);
  if (m->ku == m->units) m->kr = std::min(m->kr, share);
  // rows sharing an x piece: the largest that keeps the lanes busy
  const int ppu = m->type == LRS_GGML_Q6_K ? 8 : (m->type == LRS_GGML_Q4_K || m->type == LRS_GGML_Q5_K) ? 4 : 1;
  const int P = m->ku * ppu;
  double best = 1e30;
  int bestR = 1;
  const int cands[3] = {4, 2, 1};
  for (int R : cands) {
    if (nm == 2 && R == 4) continue;
    if (dense && R > 1) continue;
    const int kr = m->kr;
    const int NG = (kr + R - 1) / R;
    const int wpg = NG >= kS1Warps ? 1 : kS1Warps / NG;
    const int passes = ((P + 32 * wpg - 1) / (32 * wpg)) * ((NG + kS1Warps - 1) / kS1Warps);
    const double cost = passes * (R * nm + 1.0);
    if (cost < best * 0.999) best = cost, bestR = R;
  }
  m->R = bestR;
  return true;
}

bool s1_plan_smem(S1Smem* s, int cols_a, int cols_b, int cols_d, int work_floats) {
  int off = 0;
  auto take = [&](int bytes) {
    const int o = off;
    off += (bytes + 127) & ~127;
    return o;
  };
  const int xa = xa_bytes(cols_a), xb = xb_bytes(cols_b), xd = cols_d * 4;
  const int fixed = ((xa + 127) & ~127) + ((xb + 127) & ~127) + ((xd + 127) & ~127) +
                    ((work_floats * 4 + 127) & ~127) + 8 * kRedPerSlot * 4 + 256 + 128;
  const int budget = 227 * 1024;
  const int ns = std::min(8, (budget - fixed) / kS1Slot);
  if (ns < 2) return false;
  s->nslots = ns;
  take(ns * kS1Slot);
  s->xa = take(xa);
  s->xb = take(xb);
  s->xd = take(xd);
  s->work = take(work_floats * 4);
  s->red = take(ns * kRedPerSlot * 4);
  s->bars = take(2 * ns * 8);
  s->misc = take((int)sizeof(Shared));
  s->total = off;
  return off <= budget;
}

int s1_occupancy(int smem) {
  if (set_smem_once(g_attr_step, (const void*)s1_step_kernel, 227 * 1024) != cudaSuccess) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, s1_step_kernel, kS1Threads, smem) != cudaSuccess)
    return 0;
  return n;
}

cudaError_t s1_launch_step(const S1Model& hm, const S1Model* d_model, int num_sms, cudaStream_t st) {
  cudaError_t e = set_smem_once(g_attr_step, (const void*)s1_step_kernel, 227 * 1024);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(hm.bar_ctr, 0, sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kS1Threads);
  cfg.dynamicSmemBytes = hm.sm.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int advance = 1;
  void* args[] = {const_cast<S1Model**>(&d_model), &advance};
  return cudaLaunchKernelExC(&cfg, (const void*)s1_step_kernel, args);
}

cudaError_t s1_launch_gemv(const S1Mat& m0, const float* x, int* error_flag, int num_sms,
                           cudaStream_t st) {
  S1Mat m = m0;
  const int grid = std::max(1, std::min(num_sms, m.rows));
  if (!s1_plan_mat(&m, m.w2 ? 2 : 1, grid)) return cudaErrorInvalidValue;
  const int cls = s1_xclass(m.type);
  S1Smem L{};
  if (!s1_plan_smem(&L, cls == 0 ? m.cols : 0, cls == 1 ? m.cols : 0, cls == 2 ? m.cols : 0, 0))
    return cudaErrorNotSupported;
  cudaError_t e = set_smem_once(g_attr_gemv, (const void*)s1_gemv_kernel, 227 * 1024);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kS1Threads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  void* args[] = {&m, const_cast<float**>(&x), &error_flag, &L};
  return cudaLaunchKernelExC(&cfg, (const void*)s1_gemv_kernel, args);
}

}  // namespace lrs

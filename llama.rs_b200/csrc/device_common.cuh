// device_common.cuh -- device helpers shared by the llama.rs sm_100a kernels.
//
// * Exact dequantization of every GGML block type (value_at, src/quant.rs:349-456).
//   Products and differences use __fmul_rn / __fsub_rn / __fadd_rn so nvcc can
//   never contract them into an FMA: the results are bit-identical to the
//   reference's unfused f32 arithmetic.
// * "Pieces": every block type is consumed as pieces of 32 values laid out as
//   four runs of 8 consecutive columns.  A piece is one 32-value block
//   (Q4_0..Q8_0), one 32-value group of a K-quant super-block (Q4_K, Q5_K), or
//   for Q6_K the 32 values {half*128 + q*32 + octet*8 + i}; F32/F16/BF16 use 32
//   consecutive columns.
// * TMA bulk copies (cp.async.bulk) completing on an mbarrier, with waits that
//   give up after a bounded number of polls.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/llamars.h"

namespace lrs {

// Bounded polls of an mbarrier before a kernel reports LRS_ERR_DEVICE_TIMEOUT.
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ float f16_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ float bf16_bits(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t ld16(const uint8_t* p) {
  return (uint16_t)(p[0] | ((uint16_t)p[1] << 8));
}

// scale_min_k4, src/quant.rs:338-347
__device__ __forceinline__ void scale_min_k4(int i, const uint8_t* s, float* sc, float* mn) {
  uint32_t a, b;
  if (i < 4) {
    a = s[i] & 63;
    b = s[i + 4] & 63;
  } else {
    a = (s[i + 4] & 0x0f) | ((s[i - 4] >> 6) << 4);
    b = (s[i + 4] >> 4) | ((s[i] >> 6) << 4);
  }
  *sc = (float)a;
  *mn = (float)b;
}

template <int T>
struct BlockTraits;
#define LRS_TRAITS(T, BV, BB, PPB) \
  template <>                      \
  struct BlockTraits<T> {          \
    static constexpr int kValues = BV, kBytes = BB, kPieces = PPB; \
  };
// kValues/kBytes: QuantType::block_size/type_size (src/quant.rs:46-67);
// kPieces: 32-value pieces per "unit" of kBytes.  Dense types use a unit of 32
// values (128 or 64 bytes).
LRS_TRAITS(LRS_GGML_F32, 32, 128, 1)
LRS_TRAITS(LRS_GGML_F16, 32, 64, 1)
LRS_TRAITS(LRS_GGML_BF16, 32, 64, 1)
LRS_TRAITS(LRS_GGML_Q4_0, 32, 18, 1)
LRS_TRAITS(LRS_GGML_Q4_1, 32, 20, 1)
LRS_TRAITS(LRS_GGML_Q5_0, 32, 22, 1)
LRS_TRAITS(LRS_GGML_Q5_1, 32, 24, 1)
LRS_TRAITS(LRS_GGML_Q8_0, 32, 34, 1)
LRS_TRAITS(LRS_GGML_Q4_K, 256, 144, 8)
LRS_TRAITS(LRS_GGML_Q5_K, 256, 176, 8)
LRS_TRAITS(LRS_GGML_Q6_K, 256, 210, 8)
#undef LRS_TRAITS

// Column (within the unit) of run r (0..3) of piece `sub`; each run is 8 columns.
template <int T>
__device__ __forceinline__ int run_col(int sub, int r) {
  if constexpr (T == LRS_GGML_Q6_K) {
    return (sub >> 2) * 128 + r * 32 + (sub & 3) * 8;
  } else {
    return sub * 32 + r * 8;
  }
}

// Decodes piece `sub` of the unit at `u` into w[32] (run-major: w[r*8+i] is
// column run_col(sub, r) + i).  Every value equals value_at bit for bit.
template <int T>
__device__ __forceinline__ void decode_piece(const uint8_t* u, int sub, float* w) {
  if constexpr (T == LRS_GGML_F32) {
#pragma unroll
    for (int k = 0; k < 32; k++) w[k] = reinterpret_cast<const float*>(u)[k];
  } else if constexpr (T == LRS_GGML_F16) {
#pragma unroll
    for (int k = 0; k < 32; k++) w[k] = f16_bits(ld16(u + 2 * k));
  } else if constexpr (T == LRS_GGML_BF16) {
#pragma unroll
    for (int k = 0; k < 32; k++) w[k] = bf16_bits(ld16(u + 2 * k));
  } else if constexpr (T == LRS_GGML_Q4_0 || T == LRS_GGML_Q4_1) {
    const int qo = T == LRS_GGML_Q4_0 ? 2 : 4;
    float d = f16_bits(ld16(u));
    float m = T == LRS_GGML_Q4_1 ? f16_bits(ld16(u + 2)) : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      uint32_t q = u[qo + j];
      float q0 = (float)(q & 15), q1 = (float)(q >> 4);
      if constexpr (T == LRS_GGML_Q4_0) {
        w[j] = __fmul_rn(d, __fsub_rn(q0, 8.0f));
        w[j + 16] = __fmul_rn(d, __fsub_rn(q1, 8.0f));
      } else {
        w[j] = __fadd_rn(__fmul_rn(d, q0), m);
        w[j + 16] = __fadd_rn(__fmul_rn(d, q1), m);
      }
    }
  } else if constexpr (T == LRS_GGML_Q5_0 || T == LRS_GGML_Q5_1) {
    const int qho = T == LRS_GGML_Q5_0 ? 2 : 4, qso = T == LRS_GGML_Q5_0 ? 6 : 8;
    float d = f16_bits(ld16(u));
    float m = T == LRS_GGML_Q5_1 ? f16_bits(ld16(u + 2)) : 0.0f;
    uint32_t qh = (uint32_t)u[qho] | ((uint32_t)u[qho + 1] << 8) | ((uint32_t)u[qho + 2] << 16) |
                  ((uint32_t)u[qho + 3] << 24);
#pragma unroll
    for (int j = 0; j < 16; j++) {
      uint32_t q = u[qso + j];
      float q0 = (float)((q & 15) | (((qh >> j) & 1) << 4));
      float q1 = (float)((q >> 4) | (((qh >> (j + 16)) & 1) << 4));
      if constexpr (T == LRS_GGML_Q5_0) {
        w[j] = __fmul_rn(d, __fsub_rn(q0, 16.0f));
        w[j + 16] = __fmul_rn(d, __fsub_rn(q1, 16.0f));
      } else {
        w[j] = __fadd_rn(__fmul_rn(d, q0), m);
        w[j + 16] = __fadd_rn(__fmul_rn(d, q1), m);
      }
    }
  } else if constexpr (T == LRS_GGML_Q8_0) {
    float d = f16_bits(ld16(u));
#pragma unroll
    for (int j = 0; j < 32; j++) w[j] = __fmul_rn(d, (float)(int8_t)u[2 + j]);
  } else if constexpr (T == LRS_GGML_Q4_K || T == LRS_GGML_Q5_K) {
    float d = f16_bits(ld16(u)), dmin = f16_bits(ld16(u + 2));
    float sc, mn;
    scale_min_k4(sub, u + 4, &sc, &mn);
    float ds = __fmul_rn(d, sc), dm = __fmul_rn(dmin, mn);
    const int qs0 = T == LRS_GGML_Q4_K ? 16 : 48;
    const uint8_t* qs = u + qs0 + (sub >> 1) * 32;
    const int sh = (sub & 1) * 4;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      uint32_t q = (qs[j] >> sh) & 15;
      if constexpr (T == LRS_GGML_Q5_K) q += ((u[16 + j] >> sub) & 1) << 4;
      w[j] = __fsub_rn(__fmul_rn(ds, (float)q), dm);
    }
  } else if constexpr (T == LRS_GGML_Q6_K) {
    const int half = sub >> 2, oct = sub & 3;
    float d = f16_bits(ld16(u + 208));
    const uint8_t* ql = u + half * 64 + oct * 8;
    const uint8_t* qh = u + 128 + half * 32 + oct * 8;
    const uint8_t* scl = u + 192 + half * 8 + (oct >> 1);
#pragma unroll
    for (int r = 0; r < 4; r++) {
      float ds = __fmul_rn(d, (float)(int8_t)scl[r * 2]);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        uint32_t lo = (r & 1) ? ql[32 + i] : ql[i];
        lo = (r & 2) ? (lo >> 4) : (lo & 15);
        uint32_t hi = (qh[i] >> (2 * r)) & 3;
        float q = (float)((int)(lo | (hi << 4)) - 32);
        w[r * 8 + i] = __fmul_rn(ds, q);
      }
    }
  }
}

// value_at for one column of a row (src/quant.rs:349-456), via the piece decoder.
template <int T>
__device__ __forceinline__ float value_at_dev(const uint8_t* row, int col) {
  using BT = BlockTraits<T>;
  const uint8_t* u = row + (size_t)(col / BT::kValues) * BT::kBytes;
  int c = col % BT::kValues;
  int sub, r, i;
  if constexpr (T == LRS_GGML_Q6_K) {
    int half = c / 128, within = c % 128, q = within / 32, lane = within % 32;
    sub = half * 4 + lane / 8;
    r = q;
    i = lane % 8;
  } else {
    sub = c / 32;
    r = (c % 32) / 8;
    i = c % 8;
  }
  float w[32];
  decode_piece<T>(u, sub, w);
  return w[r * 8 + i];
}

// ---- TMA bulk copy + mbarrier --------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// 1-D bulk copy global -> shared; dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Returns false if the phase did not complete within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bulk prefetch of [src, src + bytes) into L2 (src 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the upstream grid's memory, and
// allow the downstream grid to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Ordering key of f32::total_cmp, widened so that an unsigned 64-bit max over
// (key << 32 | index) picks the largest value and, among equal values, the
// largest index -- the element Iterator::max_by returns (src/engine.rs:233-241).
__device__ __forceinline__ unsigned long long argmax_pack(float v, uint32_t idx) {
  int32_t b = __float_as_int(v);
  b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
  uint32_t key = (uint32_t)b ^ 0x80000000u;  // signed order -> unsigned order
  return ((unsigned long long)key << 32) | idx;
}

}  // namespace lrs

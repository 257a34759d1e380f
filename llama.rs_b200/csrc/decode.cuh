// decode.cuh -- non-GEMV kernels of the Qwen2 token step (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace lrs {

// Paged KV cache: per layer, K and V pools of [page][kv_head][kPageSize][head_dim]
// elements; pages[seq * max_pages + i] is the physical page of positions
// [i * kPageSize, (i + 1) * kPageSize) of sequence slot `seq`.
constexpr int kPageSize = 64;

struct StepIO {
  const int* tok;  // [B] input token per item
  const int* pos;  // [B] position per item
  const int* seq;  // [B] sequence slot per item
  const int* pages;
  int max_pages;
};

// Dequantizes rows tok[b] of the embedding into out[b][cols] (value_at,
// bit-exact) and clears keys[b] (argmax accumulators) when keys != null.
cudaError_t launch_embed(const uint8_t* w, uint32_t type, int cols, const int* rows, int n,
                         float* out, unsigned long long* keys, cudaStream_t st);
// Dequantizes rows [row0, row0 + n) into out[n][cols] (lrs_dequantize_rows).
cudaError_t launch_dequant_rows(const uint8_t* w, uint32_t type, int cols, int row0, int n,
                                float* out, cudaStream_t st);
// out[b][i] = x[b][i] * (inv_rms_b * w[i])  (RMSNorm::forward, src/model.rs:65-73)
cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, int batch, float* out,
                           cudaStream_t st);
// RoPE on q and k (src/model.rs:86-95, table rows indexed by position) and
// KVCache::update (src/cache.rs:38-53) into the paged pools.
cudaError_t launch_rope_store(float* q, const float* k, const float* v, const float* cos_t,
                              const float* sin_t, StepIO io, int batch, int nh, int nkv, int hd,
                              void* kpool, void* vpool, int kv_bf16, cudaStream_t st);
// Split-K GQA decode attention over the paged cache (src/model.rs:206-231 with
// softmax_inplace :298-313) into att[b][nh*hd].  Unfused: q already rotated
// and the position's K/V already stored (launch_rope_store), a combine kernel
// merges the splits.  Fused (every item a different sequence): the kernel
// rotates q and k, stores the position's K/V and merges the splits itself
// (cnt: [B][nkv] zeroed counters, left zeroed).  `err` is set to 1 if a tile
// copy never completes (bounded wait).
struct AttnLaunch {
  const float *q, *k, *v, *cos_t, *sin_t;
  StepIO io;
  int batch, nh, nkv, hd, kv_bf16, nsplit;
  void *kpool, *vpool;
  float *part, *att;
  unsigned* cnt;
  int* err;
  bool fused;
};
// Resident attention CTAs per SM (occupancy of the split kernel).
int attention_ctas_per_sm(int hd, int kv_bf16);
cudaError_t launch_attention(const AttnLaunch& l, cudaStream_t st);
// Greedy bookkeeping after the LM head: tok[b] = argmax, pos[b] += 1,
// tokens_out[step * B + b] = argmax while step < n_steps; step += 1.
// x of a windowed tensor-parallel column shard: dst[b][0..width) holds
// src[b][0..n) at offset lo and zeros elsewhere.
cudaError_t launch_pad_copy(const float* src, int n, float* dst, int width, int lo, int batch,
                            cudaStream_t st);
// g[i] = silu(g[i]) * u[i] over n floats (SwiGLU of separately computed gate / up).
cudaError_t launch_swiglu(float* g, const float* u, size_t n, cudaStream_t st);
// keys[i] += offset (the packed argmax keys of a vocabulary shard; 0 stays 0).
cudaError_t launch_key_offset(unsigned long long* keys, int n, uint32_t offset, cudaStream_t st);
cudaError_t launch_advance(const unsigned long long* keys, int* tok, int* pos, int batch,
                           int* step, int n_steps, uint32_t* tokens_out, uint32_t* last,
                           cudaStream_t st);

}  // namespace lrs

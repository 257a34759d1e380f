/*
 * llamars_synth.h -- host-side model construction for the CUDA backend.
 *
 * The reference builds its quantized weights at load time: ModelLoader reads
 * F32/F16/BF16 tensors and `maybe_quantize` (src/loader.rs:406-447) encodes
 * them with the GGML encoders of src/quant.rs:187-259, 650-967.  This header
 * exposes the same encoders and recipes, and a builder for the seeded
 * synthetic Qwen2 models the benchmarks use (weights and biases N(0, std),
 * norm weights 1.0), producing an lrs_model_desc that lrs_model_create takes.
 */
#ifndef LLAMARS_SYNTH_H
#define LLAMARS_SYNTH_H
#include "llamars.h"

#ifdef __cplusplus
extern "C" {
#endif

/* LoadQuantization (src/loader.rs:16-25). */
enum { LRS_RECIPE_NONE = 0, LRS_RECIPE_Q4K = 1, LRS_RECIPE_Q4KM = 2 };

/* GGML type that maybe_quantize (src/loader.rs:406-447) picks for a 2-D F32
 * tensor called `name` of shape [rows, cols], including the encoders'
 * fallbacks (Q4_K -> Q5_0 -> F32, src/quant.rs:190-208; Q6_K -> Q8_0,
 * src/quant.rs:244-251; Q8_0/Q5_0 -> F32 when cols % 32 != 0). */
uint32_t lrs_recipe_type(uint32_t recipe, const char* name, size_t rows, size_t cols);

/* Encodes a row-major F32 matrix as `ggml_type`.  Q4_K, Q5_0, Q8_0 and Q6_K
 * follow the reference encoders byte for byte (QuantTensor::quantize_*,
 * src/quant.rs:190-259), including their fallbacks; *out_type reports the
 * type actually produced.  F16/BF16 round to nearest even.  Q4_0, Q4_1, Q5_1
 * and Q5_K have no encoder in the reference: they use plain min/max encoders
 * that emit valid GGML blocks (documented in quantize.cpp).
 * `out` must hold lrs_quantized_size(type, rows, cols) bytes. */
lrs_status lrs_quantize_matrix(uint32_t ggml_type, const float* values, size_t rows, size_t cols,
                               void* out, size_t out_cap, uint32_t* out_type, size_t* out_len);
size_t lrs_quantized_size(uint32_t ggml_type, size_t rows, size_t cols);

/* The same encoders on the GPU (no counterpart in the reference, which
 * encodes on the host): `d_values` and `d_out` are device pointers, one
 * thread per block on the backend's stream; returns when the bytes are
 * written.  The bytes equal lrs_quantize_matrix's for the same input. */
lrs_status lrs_quantize_matrix_device(lrs_backend* backend, uint32_t ggml_type,
                                      const float* d_values, size_t rows, size_t cols, void* d_out,
                                      size_t out_cap, uint32_t* out_type, size_t* out_len);

/* Deterministic N(0, std) values of the synthetic models: element i of the
 * tensor called `name` under `seed` (counter-based, so any slice can be
 * generated independently).  Writes out[0..n) = value(offset + k). */
void lrs_synth_fill(uint64_t seed, const char* name, float stddev, uint64_t offset, size_t n,
                    float* out);

typedef struct lrs_synth_spec {
  lrs_config config;
  uint64_t seed;
  uint32_t recipe;              /* LRS_RECIPE_* applied to every 2-D weight */
  uint32_t tie_word_embeddings; /* 1: no lm_head.weight; the head reuses the embedding */
  float init_std;               /* 0.02 in every benchmark config */
  uint32_t threads;             /* host threads for generation, 0 = all */
} lrs_synth_spec;

typedef struct lrs_synth_model lrs_synth_model;
lrs_status lrs_synth_model_create(const lrs_synth_spec* spec, lrs_synth_model** out);
const lrs_model_desc* lrs_synth_model_desc(const lrs_synth_model* model);
void lrs_synth_model_destroy(lrs_synth_model* model);

#ifdef __cplusplus
}
#endif
#endif

/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of llama.rs's scalar token loop, used as the checker for
 * the CUDA backend and as the timed CPU baseline.  Nothing in the product
 * (the CUDA library, its Python host module) links, loads or calls this code;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * Parity status: the reference (Rust) cannot be built in this image (no cargo
 * or rustc), and its own tests hold no golden vectors -- only self-consistency
 * properties (src/quant.rs:973-1063), which tests/test_oracle.py re-checks
 * against this restatement, plus hand-derived known-answer blocks.  The
 * restatement is therefore pinned to those properties, not to outputs of the
 * reference binary.
 */
#ifndef LLAMARS_ORACLE_H
#define LLAMARS_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#include "../include/llamars.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Kernel kinds of the reference CpuBackend (src/backend.rs:31-36). */
enum { ORC_SCALAR = 0, ORC_AVX2 = 1 };

int orc_type_geometry(uint32_t ggml_type, uint32_t* block_values, uint32_t* block_bytes);
float orc_value_at(const uint8_t* row, uint32_t ggml_type, size_t col);
void orc_dequantize_row(const uint8_t* row, uint32_t ggml_type, size_t cols, float* out);
float orc_dot_row(int kind, const uint8_t* row, uint32_t ggml_type, const float* x, size_t cols);
/* CpuBackend::matvec with its row-parallel threshold; threads = 0 -> all cores. */
int orc_matvec(int kind, int threads, const uint8_t* w, uint32_t ggml_type, size_t rows,
               size_t cols, const float* x, float* y);
int orc_avx2_available(void);

typedef struct orc_model orc_model;
orc_model* orc_model_create(const lrs_model_desc* desc, size_t max_seq_len, int kind, int threads);
void orc_model_destroy(orc_model* m);
int orc_model_forward_token(orc_model* m, uint32_t token, size_t pos, int compute_logits,
                            float* logits_out);
int orc_model_prefill(orc_model* m, const uint32_t* tokens, size_t n, size_t start_pos,
                      float* logits_out);
/* InferenceEngine::benchmark_tokens: prefill + `decode` greedy steps.
 * tokens_out[decode] receives the token fed to each decode step; step_logits
 * (may be NULL) receives [decode + 1][vocab] logits (after prefill, then after
 * every step); top2_margin (may be NULL) receives decode+1 margins. */
int orc_benchmark_tokens(orc_model* m, const uint32_t* prompt, size_t n, size_t decode,
                         uint32_t* tokens_out, float* step_logits, float* top2_margin,
                         double* prefill_s, double* decode_s);
/* Greedy argmax of the reference (last maximal index under f32::total_cmp). */
uint32_t orc_argmax(const float* logits, size_t n);
/* InferenceEngine::sample_current_logits (src/engine.rs:253-325) over `n`
 * logits with the recent-token window `recent` (the seen flags), and the
 * uniform draw `u` in [0, 1) that the reference takes from
 * rand::thread_rng().gen::<f32>().  Equal values, whose order
 * sort_unstable_by leaves unspecified, are ordered larger index first.
 * *margin_out (may be NULL) receives the smallest distance, in probability
 * units, between a decision and its boundary (the top-p cutoff and the draw);
 * +inf when no such decision was made.  No reference test covers this
 * function: it is pinned to the source only (tests/test_sampler.py restates
 * it again in Python). */
uint32_t orc_sample(const float* logits, size_t n, const uint32_t* recent, size_t n_recent,
                    float temperature, float top_p, size_t top_k, float repetition_penalty,
                    float u, float* margin_out);
const char* orc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif

/*
 * llamars_sample.h -- the stochastic sampler on the device.
 *
 * Replaces InferenceEngine::sample_current_logits (src/engine.rs:253-325) so
 * that the non-greedy chat path (InferenceEngine::forward_step, :96-106, and
 * generate_with_metrics, :115-165) keeps the logits on the GPU: one launch
 * turns the vocabulary logits into the next token and 4 bytes come back
 * instead of the 4 * vocab bytes of logits.
 *
 * The reference draws u = rand::thread_rng().gen::<f32>() in [0, 1); here the
 * caller passes u (the Rust shim draws it the same way), so for a given u the
 * token is a deterministic function of the logits:
 *   repetition penalty on the distinct recent tokens, temperature,
 *   non-finite -> -inf, descending order under f32::total_cmp (equal values:
 *   larger index first -- sort_unstable_by leaves them unordered), top-k,
 *   softmax, top-p cutoff, draw -- each step in the reference's f32 order.
 * Device limit: 1 <= top_k <= LRS_SAMPLE_MAX_TOP_K (or top_k >= vocab when the
 * vocabulary itself is that small); top_k = 0 (off) and larger values return
 * LRS_ERR_UNSUPPORTED, and the shim keeps the reference's host sampler for
 * them, as for vocabularies above about 1.39 million tokens (the device's
 * seen-token bitmap must fit in shared memory).  temperature <= 0 is the
 * greedy argmax whatever top_k is.
 */
#ifndef LLAMARS_SAMPLE_H
#define LLAMARS_SAMPLE_H
#include "llamars.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LRS_SAMPLE_MAX_TOP_K 4096

/* EngineOptions' sampling fields (src/engine.rs:11-33; defaults 0.7, 0.9, 40, 1.1). */
typedef struct lrs_sampler {
  float temperature;
  float top_p;
  uint32_t top_k;
  float repetition_penalty;
} lrs_sampler;

/* validate_sampling (src/engine.rs:327-339), with its messages; plus the
 * device limits on top_k and the vocabulary (LRS_ERR_UNSUPPORTED).  No CUDA call. */
lrs_status lrs_sampler_check(const lrs_sampler* params, size_t vocab);

/* Samples from `vocab` logits in device memory (d_logits) on the backend
 * stream; recent[n_recent] (host) is the recent-token window
 * (InferenceEngine::remember, :243-251); u in [0, 1).  Synchronous: the token
 * is in *token_out on return. */
lrs_status lrs_sample_logits(lrs_backend* backend, const float* d_logits, size_t vocab,
                             const lrs_sampler* params, const uint32_t* recent, size_t n_recent,
                             float u, uint32_t* token_out);

/* InferenceEngine::forward_step (src/engine.rs:96-106) without the logits
 * copy: forward_token(token, pos, LogitsMode::Compute) for sequence slot `seq`,
 * then the device sampler.  Under tensor parallelism every rank calls it with
 * the same arguments and gets the same token. */
lrs_status lrs_model_forward_sample(lrs_model* model, uint32_t seq, uint32_t token_id,
                                    uint32_t pos, const lrs_sampler* params,
                                    const uint32_t* recent, size_t n_recent, float u,
                                    uint32_t* next_out);

#ifdef __cplusplus
}
#endif
#endif /* LLAMARS_SAMPLE_H */

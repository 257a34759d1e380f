// sample.cuh -- the device sampler's entry points inside the library (sample.cu).
#pragma once
#include <cuda_runtime.h>

#include "../../include/llamars_sample.h"
#include "internal.h"

namespace lrs {

// Queues sample_current_logits (src/engine.rs:253-325) for `vocab` logits at
// d_logits with the window d_recent[n_recent]; the token lands in *d_out.
// The parameters must have passed lrs_sampler_check.
cudaError_t launch_sample(const float* d_logits, int vocab, const uint32_t* d_recent, int n_recent,
                          const lrs_sampler& p, float u, uint32_t* d_out, cudaStream_t st);

// Backend-owned device buffers: the window copied from recent[n] (queued on
// the backend stream) and one slot for the token.
int32_t sample_buffers(lrs_backend* be, const uint32_t* recent, size_t n, uint32_t** d_recent,
                       uint32_t** d_out);

}  // namespace lrs

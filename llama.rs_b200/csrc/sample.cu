// sample.cu -- InferenceEngine::sample_current_logits (src/engine.rs:253-325)
// on the device.
//
// One CTA of 1024 threads per call:
//  1. The seen flags of the recent tokens become a bitmap in shared memory.
//     Every pass recomputes a candidate's value from the logits in the
//     reference's order: repetition penalty (v / p if v > 0, else v * p),
//     temperature (v / t), non-finite -> -inf.
//  2. Candidates are ordered by a 64-bit composite key, total_cmp key << 32 |
//     index, so equal values order larger index first.  temperature <= 0
//     returns the first candidate (a block max of the key).
//  3. top-k (k <= 4096): a most-significant-digit radix select over the key
//     (six passes of up to 11 bits, warp-aggregated counts into 2048 bins,
//     one block scan per pass) finds the k-th key; the k candidates are
//     gathered and bitonic-sorted in shared memory.
//  4. exp(v - max) per candidate in parallel; then one thread runs the sum,
//     the top-p cumulative, the kept sum and the draw sequentially in f32, in
//     sorted order -- the reference's arithmetic.
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "common.h"
#include "sample.cuh"

namespace lrs {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kBins = 2048;
constexpr size_t kSampleMaxSmem = 227 * 1024;  // dynamic shared memory of one CTA

struct SampleArgs {
  const float* logits;
  const uint32_t* recent;
  uint32_t* out;
  int vocab, n_recent, k;
  float temperature, top_p, penalty, u;
};

__device__ __forceinline__ uint32_t order_key(float v) {
  // f32::total_cmp order as an unsigned key
  int32_t b = __float_as_int(v);
  b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
  return (uint32_t)b ^ 0x80000000u;
}

__device__ __forceinline__ float cand_value(const SampleArgs& a, const uint32_t* seen, int i) {
  float v = a.logits[i];
  if (a.penalty != 1.0f && ((seen[i >> 5] >> (i & 31)) & 1u))
    v = v > 0.0f ? v / a.penalty : v * a.penalty;
  if (a.temperature > 0.0f) v = v / a.temperature;
  if (!isfinite(v)) v = -INFINITY;
  return v;
}

__device__ __forceinline__ unsigned long long composite(float v, int i) {
  return ((unsigned long long)order_key(v) << 32) | (uint32_t)i;
}

__device__ __forceinline__ unsigned long long shfl_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long w =
        ((unsigned long long)__shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), o) << 32) |
        __shfl_xor_sync(0xffffffffu, (uint32_t)v, o);
    v = w > v ? w : v;
  }
  return v;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int V = a.vocab;
  const int words = (V + 31) / 32;
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem);        // [4096]
  float* vals = reinterpret_cast<float*>(cand + LRS_SAMPLE_MAX_TOP_K);           // [4096]
  uint32_t* hist = reinterpret_cast<uint32_t*>(vals + LRS_SAMPLE_MAX_TOP_K);     // [2048]
  uint32_t* wsum = hist + kBins;                                                 // [32]
  unsigned long long* wmax = reinterpret_cast<unsigned long long*>(wsum + 32);   // [32]
  uint32_t* misc = reinterpret_cast<uint32_t*>(wmax + 32);                       // [4]
  uint32_t* seen = misc + 4;                                                     // [words]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int iters = (V + kSampleThreads - 1) / kSampleThreads;

  for (int w = tid; w < words; w += kSampleThreads) seen[w] = 0;
  __syncthreads();
  for (int r = tid; r < a.n_recent; r += kSampleThreads) {
    const uint32_t t = a.recent[r];
    if (t < (uint32_t)V) atomicOr(&seen[t >> 5], 1u << (t & 31));
  }
  __syncthreads();

  // the first candidate in the reference's order
  unsigned long long best = 0ull;
  for (int it = 0; it < iters; it++) {
    const int i = tid + it * kSampleThreads;
    if (i < V) {
      const unsigned long long c = composite(cand_value(a, seen, i), i);
      best = c > best ? c : best;
    }
  }
  best = shfl_max_u64(best);
  if (lane == 0) wmax[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = shfl_max_u64(wmax[lane]);
    if (lane == 0) wmax[0] = best;
  }
  __syncthreads();
  const unsigned long long first = wmax[0];
  if (a.temperature <= 0.0f) {
    if (tid == 0) *a.out = (uint32_t)first;
    return;
  }

  // k-th largest key: digits of bits [63,53] [52,42] [41,31] [30,20] [19,9] [8,0]
  const int K = a.k;
  unsigned long long thr = 0ull;
  if (K < V) {
    unsigned long long prefix = 0ull;
    uint32_t rank = (uint32_t)K;  // 1-based, from the top
    for (int pass = 0; pass < 6; pass++) {
      const int hi = 63 - 11 * pass, lo = pass == 5 ? 0 : hi - 10;
      const int nbits = hi - lo + 1;
      for (int b = tid; b < kBins; b += kSampleThreads) hist[b] = 0;
      __syncthreads();
      for (int it = 0; it < iters; it++) {
        const int i = tid + it * kSampleThreads;
        bool valid = false;
        uint32_t d = 0;
        if (i < V) {
          const unsigned long long c = composite(cand_value(a, seen, i), i);
          valid = hi == 63 || (c >> (hi + 1)) == (prefix >> (hi + 1));
          d = (uint32_t)(c >> lo) & ((1u << nbits) - 1u);
        }
        const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
        if (valid) {
          const uint32_t grp = __match_any_sync(vmask, d);
          if (lane == __ffs(grp) - 1) atomicAdd(&hist[d], (uint32_t)__popc(grp));
        }
      }
      __syncthreads();
      // descending digits: thread t owns digits 2047 - 2t and 2046 - 2t
      const uint32_t h0 = hist[kBins - 1 - 2 * tid], h1 = hist[kBins - 2 - 2 * tid];
      uint32_t incl = h0 + h1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (lane == 31) wsum[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        uint32_t t = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t n = __shfl_up_sync(0xffffffffu, t, o);
          if (lane >= o) t += n;
        }
        wsum[lane] = t;  // inclusive warp prefix
      }
      __syncthreads();
      const uint32_t base = (warp ? wsum[warp - 1] : 0u) + incl - (h0 + h1);
      if (base < rank && rank <= base + h0) {
        misc[0] = kBins - 1 - 2 * tid;
        misc[1] = base;
      } else if (base + h0 < rank && rank <= base + h0 + h1) {
        misc[0] = kBins - 2 - 2 * tid;
        misc[1] = base + h0;
      }
      __syncthreads();
      rank -= misc[1];
      prefix |= (unsigned long long)misc[0] << lo;
      __syncthreads();
    }
    thr = prefix;
  }

  // gather the K candidates (keys >= thr), pad to a power of two, sort descending
  if (tid == 0) misc[2] = 0;
  __syncthreads();
  for (int it = 0; it < iters; it++) {
    const int i = tid + it * kSampleThreads;
    if (i < V) {
      const unsigned long long c = composite(cand_value(a, seen, i), i);
      if (c >= thr) {
        const uint32_t slot = atomicAdd(&misc[2], 1u);
        if (slot < LRS_SAMPLE_MAX_TOP_K) cand[slot] = c;
      }
    }
  }
  __syncthreads();
  const int n = min((int)misc[2], LRS_SAMPLE_MAX_TOP_K);
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int s = n + tid; s < n2; s += kSampleThreads) cand[s] = 0ull;
  __syncthreads();
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = tid; t < n2 / 2; t += kSampleThreads) {
        const int i = 2 * t - (t & (stride - 1));  // lower index of the pair
        const int j = i + stride;
        const bool desc = (i & size) == 0;
        const unsigned long long x = cand[i], y = cand[j];
        if ((x < y) == desc) {
          cand[i] = y;
          cand[j] = x;
        }
      }
      __syncthreads();
    }
  }

  // softmax numerators in parallel, then the reference's sequential steps
  const float mx = cand_value(a, seen, (int)(uint32_t)cand[0]);
  for (int r = tid; r < n; r += kSampleThreads)
    vals[r] = expf(cand_value(a, seen, (int)(uint32_t)cand[r]) - mx);
  __syncthreads();
  if (tid != 0) return;
  float sum = 0.0f;
  for (int r = 0; r < n; r++) sum += vals[r];
  if (!isfinite(sum) || sum <= 0.0f) {
    *a.out = (uint32_t)cand[0];
    return;
  }
  float cumulative = 0.0f;
  int cutoff = n;
  for (int r = 0; r < n; r++) {
    vals[r] = vals[r] / sum;
    cumulative += vals[r];
    if (cumulative >= a.top_p) {
      cutoff = r + 1;
      break;
    }
  }
  float kept = 0.0f;
  for (int r = 0; r < cutoff; r++) kept += vals[r];
  float random = a.u * kept;
  for (int r = 0; r < cutoff; r++) {
    random -= vals[r];
    if (random <= 0.0f) {
      *a.out = (uint32_t)cand[r];
      return;
    }
  }
  *a.out = (uint32_t)cand[cutoff - 1];
}

size_t sample_smem(size_t vocab) {
  return (size_t)LRS_SAMPLE_MAX_TOP_K * 12 + kBins * 4 + 32 * 4 + 32 * 8 + 16 +
         (vocab + 31) / 32 * 4;
}

}  // namespace

// Queues the sampler for `vocab` logits at d_logits; the token lands in d_out.
cudaError_t launch_sample(const float* d_logits, int vocab, const uint32_t* d_recent, int n_recent,
                          const lrs_sampler& p, float u, uint32_t* d_out, cudaStream_t st) {
  SampleArgs a;
  a.logits = d_logits;
  a.recent = d_recent;
  a.out = d_out;
  a.vocab = vocab;
  a.n_recent = n_recent;
  a.k = p.top_k == 0 || p.top_k >= (uint32_t)vocab ? vocab : (int)p.top_k;
  a.temperature = p.temperature;
  a.top_p = p.top_p;
  a.penalty = p.repetition_penalty;
  a.u = u;
  const size_t smem = sample_smem((size_t)vocab);
  cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  sample_kernel<<<1, kSampleThreads, smem, st>>>(a);
  return cudaGetLastError();
}

// Copies recent[n] into backend-owned device memory (grown on demand) and
// returns it with a device slot for the token right after it.
int32_t sample_buffers(lrs_backend* be, const uint32_t* recent, size_t n, uint32_t** d_recent,
                       uint32_t** d_out) {
  const size_t need = n + 1;
  if (be->sample_cap < need) {
    cudaFree(be->d_sample);  // synchronizes with work that may still use it
    be->d_sample = nullptr;
    be->sample_cap = 0;
    const size_t cap = need < 256 ? 256 : need;
    if (cudaMalloc(&be->d_sample, cap * 4) != cudaSuccess)
      return fail(LRS_ERR_OOM, "cudaMalloc of sampler buffers failed");
    be->sample_cap = cap;
  }
  if (n) {
    cudaError_t e = cudaMemcpyAsync(be->d_sample + 1, recent, n * 4, cudaMemcpyHostToDevice,
                                    be->stream);
    if (e != cudaSuccess) return fail(LRS_ERR_CUDA, cudaGetErrorString(e));
  }
  *d_out = be->d_sample;
  *d_recent = be->d_sample + 1;
  return LRS_OK;
}

}  // namespace lrs

using namespace lrs;

extern "C" lrs_status lrs_sampler_check(const lrs_sampler* p, size_t vocab) try {
  // validate_sampling, src/engine.rs:327-339
  if (!p) return fail(LRS_ERR_INVALID, "null sampler parameters");
  if (!std::isfinite(p->temperature) || p->temperature < 0.0f)
    return fail(LRS_ERR_INVALID, "temperature must be finite and non-negative");
  if (!std::isfinite(p->top_p) || !(0.0f < p->top_p && p->top_p <= 1.0f))
    return fail(LRS_ERR_INVALID, "top_p must be in (0, 1]");
  if (!std::isfinite(p->repetition_penalty) || p->repetition_penalty <= 0.0f)
    return fail(LRS_ERR_INVALID, "repetition_penalty must be finite and positive");
  if (vocab == 0 || vocab > (1u << 24)) return fail(LRS_ERR_INVALID, "vocabulary size out of range");
  if (sample_smem(vocab) > kSampleMaxSmem)  // the seen bitmap lives in shared memory
    return fail(LRS_ERR_UNSUPPORTED, "device sampler: vocabulary too large (the host sampler applies)");
  const size_t k = p->top_k == 0 || p->top_k >= vocab ? vocab : p->top_k;
  if (p->temperature > 0.0f && k > LRS_SAMPLE_MAX_TOP_K)
    return fail(LRS_ERR_UNSUPPORTED, "device sampler: top_k must be in 1.." +
                                         std::to_string(LRS_SAMPLE_MAX_TOP_K) +
                                         " (top_k = 0 and larger values use the host sampler)");
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

extern "C" lrs_status lrs_sample_logits(lrs_backend* be, const float* d_logits, size_t vocab,
                                        const lrs_sampler* p, const uint32_t* recent,
                                        size_t n_recent, float u, uint32_t* token_out) try {
  if (!be || !d_logits || !token_out || (n_recent && !recent))
    return fail(LRS_ERR_INVALID, "null argument");
  int32_t rc = lrs_sampler_check(p, vocab);
  if (rc) return rc;
  if (!(u >= 0.0f && u < 1.0f)) return fail(LRS_ERR_INVALID, "u must be in [0, 1)");
  cudaError_t e = cudaSetDevice(be->device);
  if (e != cudaSuccess) return fail(LRS_ERR_CUDA, cudaGetErrorString(e));
  uint32_t *d_recent, *d_out;
  if ((rc = sample_buffers(be, recent, n_recent, &d_recent, &d_out))) return rc;
  e = launch_sample(d_logits, (int)vocab, d_recent, (int)n_recent, *p, u, d_out, be->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(token_out, d_out, 4, cudaMemcpyDeviceToHost, be->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
  if (e != cudaSuccess) return fail(LRS_ERR_CUDA, cudaGetErrorString(e));
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

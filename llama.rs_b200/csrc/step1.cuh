// step1.cuh -- the batch-1 decode step as one persistent kernel (step1.cu).
//
// One CTA per SM runs the whole token step of Qwen2Model::forward_impl
// (src/model.rs:135-270) for one sequence: embedding, every layer's
// projections, RoPE + KV store, attention, SwiGLU, residual adds, the final
// norm and the LM head with the greedy argmax (src/engine.rs:189-241).  The
// phases meet at grid-wide barriers; the weights, which do not depend on the
// activations, stream through a shared-memory ring of bulk copies that one
// producer warp keeps filling across the barriers, so HBM never waits for a
// phase boundary.  The same GEMV machinery serves lrs_matvec at batch 1 as a
// one-phase launch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace lrs {

// 12 warps: 3 per SM sub-partition, which leaves 168 registers per thread.
constexpr int kS1Warps = 11;                    // consumer warps per CTA
constexpr int kS1Threads = 32 * kS1Warps + 32;  // + the producer warp
constexpr int kS1Slot = 32 * 1024;              // bytes per ring slot
constexpr int kS1MaxRows = 32;                  // rows per chunk
constexpr int kS1MaxGroup = 8;                  // query heads per KV head

// One matrix of a GEMV phase (or a gate/up pair: w2, same type and shape).
// The CTA of index b among G owns rows [rows*b/G, rows*(b+1)/G); its rows are
// consumed in chunks of kr whole rows, or, when a row does not fit a slot,
// one row in chunks of ku block units.
struct S1Mat {
  const uint8_t* w;
  const uint8_t* w2;
  const float* bias;  // EPI_STORE: added per row (LinearLayer::forward)
  float* out;         // output vector (EPI_ARGMAX: logits, may be null)
  int type, rows, cols, rb;
  int units, ub;      // block units per row, bytes per unit (dense types: 32 values)
  int kr, ku;         // rows per chunk; units per chunk (== units unless kr == 1)
  int R;              // rows sharing one x piece in a consumer lane (1, 2 or 4)
  int part;           // bytes of a slot per matrix of a pair
  int epi;            // EPI_STORE / EPI_ADD / EPI_SWIGLU / EPI_ARGMAX
};

struct S1Layer {
  S1Mat qkv[3];
  S1Mat o;
  S1Mat gu[2];        // one pair (EPI_SWIGLU), or gate and up stored separately
  S1Mat down;
  int ngu;            // 1: pair; 2: separate (down's x is silu(gate) * up)
  const float* in_norm;
  const float* post_norm;
  void* kpool;
  void* vpool;
};

// Shared-memory plan of a launch (host-computed, the same for every CTA).
struct S1Smem {
  int nslots;
  int xa, xb, xd;       // offsets of the staged-x regions (class A / B / dense)
  int work;             // offset of the float work area
  int red, bars, misc;  // partial sums, mbarriers, flags
  int total;
};

// Everything the step kernel reads (device memory, built at model creation).
struct S1Model {
  int L, h, nh, nkv, hd, inter, vocab;
  float eps, attn_scale;
  int kv_bf16;
  const S1Layer* layers;
  const uint8_t* embed;
  int embed_type;
  S1Mat lm;             // out: logits (null: argmax only)
  const float* final_norm;
  const float* rope_cos;  // [max_seq][hd/2]
  const float* rope_sin;
  float *residual, *q, *k, *v, *att, *act, *act2;
  float* part;          // attention partials [nkv][max_split][G][2 + hd]
  int max_split;        // attention splits per KV head
  int split_cap;        // positions per split the work area holds
  unsigned* attn_cnt;   // [nkv] combine counters (zero between launches)
  unsigned* bar_ctr;    // grid barrier counter (zeroed before every launch)
  unsigned long long* keys;  // argmax key of the step
  // greedy bookkeeping (advance_kernel)
  int *tok, *pos, *seq, *pages;
  int max_pages;
  int* step;
  int n_steps_cap;
  uint32_t* tokens_out;
  uint32_t* last;
  int* error_flag;
  S1Smem sm;
};

// Fills the chunk plan of a matrix (kr, ku, R, part, units, ub, rb) for a
// launch of `grid` CTAs; false if the type is unknown.
bool s1_plan_mat(S1Mat* m, int nm, int grid);
// Shared-memory layout for phases whose widest x has `cols_a` columns of a
// 32-group type, `cols_b` of Q6_K, `cols_d` of a dense type; `work` floats.
bool s1_plan_smem(S1Smem* s, int cols_a, int cols_b, int cols_d, int work_floats);
// Class of a type's staged x: 0 (32-column groups), 1 (Q6_K pieces), 2 (dense).
int s1_xclass(int type);
// The whole decode step of one sequence (cooperative launch, one CTA per SM).
// `d_model` is the device copy of `host_model`.
cudaError_t s1_launch_step(const S1Model& host_model, const S1Model* d_model, int num_sms,
                           cudaStream_t st);
// Resident CTAs of the step kernel per SM with `smem` bytes.
int s1_occupancy(int smem);
// y = W x for one matrix at batch 1 (lrs_matvec): x, y device vectors.
cudaError_t s1_launch_gemv(const S1Mat& m, const float* x, int* error_flag, int num_sms,
                           cudaStream_t st);

}  // namespace lrs

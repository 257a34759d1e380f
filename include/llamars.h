/*
 * llamars.h -- C ABI of the B200 (sm_100a) CUDA backend for llama.rs's Qwen2
 * token loop.
 *
 * The reference engine (llama.rs, Rust) reaches its numerical kernels through
 * two traits:
 *   - KernelBackend { name, threads, matvec }        src/backend.rs:69-73
 *   - CausalModel   { forward_token, prefill, ... }   src/architecture.rs:42-78
 * This header is the plain-C surface a Rust `CudaBackend: KernelBackend` and a
 * `CudaQwen2Model: CausalModel` bind through `extern "C"`.  Every entry point
 * returns an lrs_status (0 = success); the message of the last failure on the
 * calling thread is available from lrs_last_error().  Nothing here aborts,
 * throws across the boundary or takes a torch type.
 *
 * Shapes follow the reference: a matrix is row-major [rows, cols] of GGML
 * blocks (src/quant.rs:105-173), blocks never straddle rows, and a row of
 * `cols` values occupies cols / block_size * type_size bytes.
 */
#ifndef LLAMARS_H
#define LLAMARS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status -- */
typedef int32_t lrs_status;
enum {
  LRS_OK = 0,
  LRS_ERR_INVALID = 1,      /* bad argument / shape (reference: ensure! failures) */
  LRS_ERR_UNSUPPORTED = 2,  /* unsupported GGML type id (src/quant.rs:40-42) */
  LRS_ERR_CUDA = 3,         /* CUDA runtime error */
  LRS_ERR_OOM = 4,          /* device or pool allocation failed */
  LRS_ERR_DEVICE_TIMEOUT = 5 /* a bounded device-side wait gave up */
};

/* GGML tensor type ids accepted by QuantType::from_ggml_type (src/quant.rs:27-44). */
enum {
  LRS_GGML_F32 = 0,
  LRS_GGML_F16 = 1,
  LRS_GGML_Q4_0 = 2,
  LRS_GGML_Q4_1 = 3,
  LRS_GGML_Q5_0 = 6,
  LRS_GGML_Q5_1 = 7,
  LRS_GGML_Q8_0 = 8,
  LRS_GGML_Q4_K = 12,
  LRS_GGML_Q5_K = 13,
  LRS_GGML_Q6_K = 14,
  LRS_GGML_BF16 = 30
};

/* LogitsMode (src/architecture.rs:34-38). */
enum { LRS_LOGITS_SKIP = 0, LRS_LOGITS_COMPUTE = 1 };

/* Message of the last failed call on this thread ("" if none). */
const char* lrs_last_error(void);

/* Block geometry of a GGML type: values per block and bytes per block
 * (QuantType::block_size / type_size, src/quant.rs:46-67). */
lrs_status lrs_type_geometry(uint32_t ggml_type, uint32_t* block_values, uint32_t* block_bytes);

/* ------------------------------------------------------------- backend -- */
typedef struct lrs_backend lrs_backend;

/* Creates a backend bound to one CUDA device (replaces CpuBackend::new,
 * src/backend.rs:98-121, and the hard-wired construction at src/loader.rs:99,242). */
lrs_status lrs_backend_create(int device, lrs_backend** out);
void lrs_backend_destroy(lrs_backend* backend);
/* KernelBackend::name (src/backend.rs:70): returns "cuda-sm100a". */
const char* lrs_backend_name(const lrs_backend* backend);
/* KernelBackend::threads (src/backend.rs:71): the device's SM count. */
size_t lrs_backend_threads(const lrs_backend* backend);
/* Blocks until all work queued by this backend has finished. */
lrs_status lrs_backend_synchronize(lrs_backend* backend);

/* --------------------------------------------------------------- tensor -- */
typedef struct lrs_tensor lrs_tensor;

/* Uploads the bytes of a QuantTensor once to HBM in their native block layout
 * (QuantTensor::from_data validation, src/quant.rs:132-157).  `data` is a host
 * pointer of `nbytes` bytes; the Rust shim keys the handle by the tensor's
 * data pointer so later matvec calls find the device copy. */
lrs_status lrs_tensor_upload(lrs_backend* backend, const void* data, size_t nbytes, size_t rows,
                             size_t cols, uint32_t ggml_type, lrs_tensor** out);
void lrs_tensor_free(lrs_tensor* tensor);
/* Device address of the uploaded block bytes (for callers that launch their own work). */
const void* lrs_tensor_device_ptr(const lrs_tensor* tensor);

/* Dequantizes rows [row0, row0 + nrows) to f32 into the HOST buffer `out`
 * (nrows * cols floats).  Bit-exact with value_at (src/quant.rs:349-456) and
 * QuantTensor::row_into (src/quant.rs:261-272). */
lrs_status lrs_dequantize_rows(lrs_backend* backend, const lrs_tensor* tensor, size_t row0,
                               size_t nrows, float* out);

/* KernelBackend::matvec (src/backend.rs:69-73, CpuBackend::matvec :143-162):
 * out[r] = dot(row r, in).  Host buffers; synchronous; validates exactly like
 * QuantTensor::validate_matvec (src/quant.rs:303-318). */
lrs_status lrs_matvec(lrs_backend* backend, const lrs_tensor* weight, const float* in, size_t n_in,
                      float* out, size_t n_out);

/* Batched matvec over `batch` independent input vectors (row-major [batch, cols]
 * in, [batch, rows] out), host buffers.  The reference has no batched form; it
 * equals `batch` calls of KernelBackend::matvec.  1 <= batch <= 64. */
lrs_status lrs_matvec_batched(lrs_backend* backend, const lrs_tensor* weight, const float* in,
                              size_t batch, size_t n_in, float* out, size_t n_out);

/* lrs_matvec for callers that cannot allocate device memory.  This entry point
 * has no counterpart in the reference.  lrs_matvec stages the host vectors
 * through device buffers it cudaMalloc's on first use; callers that run on a
 * device-memory budget fixed at start-up, or that must not let a call trigger
 * cudaMalloc's device-wide synchronization, call this instead: it stages
 * through one fixed-size __device__ array built into the library (1.25 MiB,
 * held by every GPU that loads the library until exit) and allocates nothing.
 * Limits: cols <= 65536, rows <= 262144 (larger matrices: LRS_ERR_INVALID).
 * The first call on a device looks up the array's address there; make it
 * before any stream capture.  That address is cached for the life of the
 * process: it assumes the device's primary context is never reset
 * (cudaDeviceReset) while the library is loaded.  All calls on a device share the array: calls
 * whose GPU work overlaps race, so callers on several threads must serialize
 * them.  Synchronous; same validation and results as lrs_matvec. */
lrs_status lrs_matvec_noalloc(lrs_backend* backend, const lrs_tensor* weight, const float* in,
                              size_t n_in, float* out, size_t n_out);

/* Device-pointer form of lrs_matvec_batched: `d_in` / `d_out` are device
 * addresses, the work is queued on `stream` (a cudaStream_t, NULL = the
 * backend's stream) and the call returns without synchronizing. */
lrs_status lrs_matvec_device(lrs_backend* backend, const lrs_tensor* weight, const float* d_in,
                             size_t batch, float* d_out, void* stream);

/* ---------------------------------------------------------------- model -- */

/* LlamaConfig (src/config.rs:18-39) after validate(); head_dim is explicit. */
typedef struct lrs_config {
  uint32_t hidden_size;
  uint32_t intermediate_size;
  uint32_t num_attention_heads;
  uint32_t num_key_value_heads;
  uint32_t num_hidden_layers;
  uint32_t vocab_size;
  uint32_t head_dim;
  uint32_t max_position_embeddings;
  float rms_norm_eps;
  float rope_theta;
} lrs_config;

/* A QuantTensor view: host bytes in GGML block layout. */
typedef struct lrs_tensor_desc {
  const void* data;
  uint64_t nbytes;
  uint64_t rows;
  uint64_t cols;
  uint32_t ggml_type;
  uint32_t reserved;
} lrs_tensor_desc;

/* TransformerBlock (src/model.rs:97-108).  Biases may be NULL (treated as zeros,
 * src/loader.rs:489-493).  Norm weights are f32 [hidden_size]. */
typedef struct lrs_layer_desc {
  const float* input_layernorm;
  const float* post_attention_layernorm;
  lrs_tensor_desc q_proj, k_proj, v_proj, o_proj;
  lrs_tensor_desc gate_proj, up_proj, down_proj;
  const float* q_bias;
  const float* k_bias;
  const float* v_bias;
} lrs_layer_desc;

/* Qwen2Model (src/model.rs:110-118).  A tied head passes the embedding again. */
typedef struct lrs_model_desc {
  lrs_config config;
  lrs_tensor_desc embed_tokens;
  lrs_tensor_desc lm_head;
  const float* final_norm;
  const lrs_layer_desc* layers; /* num_hidden_layers entries */
} lrs_model_desc;

/* KV-cache element type on the device. */
enum { LRS_KV_F32 = 0, LRS_KV_BF16 = 1 };

typedef struct lrs_model_options {
  uint32_t max_seq_len;   /* context per sequence (KVCache::new max_seq_len, src/cache.rs:12-36) */
  uint32_t max_sequences; /* concurrent sequences (slots) */
  uint32_t kv_dtype;      /* LRS_KV_F32 (default, parity) or LRS_KV_BF16 */
  uint32_t use_graph;     /* capture decode steps in a CUDA graph (1 = yes) */
  uint32_t device_recipe; /* LRS_RECIPE_* (llamars_synth.h): F32/F16/BF16 matrices are encoded
                             on the GPU at creation (maybe_quantize, src/loader.rs:406-447); 0 = as given */
  uint32_t tp_allreduce;  /* tensor-parallel models: LRS_TP_ALLREDUCE_NCCL (default) or
                             LRS_TP_ALLREDUCE_P2P (one kernel over peer memory) */
  uint32_t persistent_decode; /* 1: batch-1 greedy decode steps run as one persistent
                                 kernel per step (step1.cu); 0 (default): one CUDA graph of
                                 per-operation kernels */
} lrs_model_options;

enum { LRS_TP_ALLREDUCE_NCCL = 0, LRS_TP_ALLREDUCE_P2P = 1 };

typedef struct lrs_model lrs_model;

/* Uploads every tensor of the model once and allocates the paged KV cache and
 * activation buffers (InferenceBuffers::new, src/cache.rs:79-101). */
lrs_status lrs_model_create(lrs_backend* backend, const lrs_model_desc* desc,
                            const lrs_model_options* options, lrs_model** out);
/* ---- tensor parallelism (c4) ---------------------------------------------
 * No counterpart in the reference (one CPU process): the model is split over
 * `world` processes, one GPU each.  q/k/v/gate/up and the LM head are split by
 * rows (heads, MLP width, vocabulary), o and down by columns; after o and
 * after down one NCCL sum all-reduce rebuilds the residual on every rank, and
 * the greedy argmax is a MAX all-reduce of the packed (value, index) keys.
 * Every rank passes the FULL model description and makes the same calls in
 * the same order.  world must divide the KV heads, the MLP width and the
 * vocabulary, and the column splits must fall on block boundaries. */
#define LRS_TP_ID_BYTES 128
/* Rank 0 makes the id and shares it with the other ranks out of band. */
lrs_status lrs_tp_unique_id(uint8_t* id_out /* LRS_TP_ID_BYTES */);
lrs_status lrs_model_create_tp(lrs_backend* backend, const lrs_model_desc* desc,
                               const lrs_model_options* options, uint32_t rank, uint32_t world,
                               const uint8_t* id /* LRS_TP_ID_BYTES */, lrs_model** out);
uint32_t lrs_model_tp_world(const lrs_model* model);

void lrs_model_destroy(lrs_model* model);

/* Forgets the contents of a sequence slot (KVCache::reset, src/cache.rs:55-57). */
lrs_status lrs_model_reset(lrs_model* model, uint32_t seq);

/* CausalModel::forward_token (src/architecture.rs:50-57, Qwen2Model::forward_impl
 * src/model.rs:135-270) for sequence slot `seq`.  With LRS_LOGITS_COMPUTE the
 * vocabulary logits are copied into `logits_out` (may be NULL) and the greedy
 * token (last maximal index under total order, src/engine.rs:233-241) into
 * `argmax_out` (may be NULL). */
lrs_status lrs_model_forward_token(lrs_model* model, uint32_t seq, uint32_t token_id, uint32_t pos,
                                   int logits_mode, float* logits_out, uint32_t* argmax_out);

/* CausalModel::prefill (src/architecture.rs:60-77): runs `n_tokens` prompt
 * tokens at positions start_pos.. and computes logits only for the last one. */
lrs_status lrs_model_prefill(lrs_model* model, uint32_t seq, const uint32_t* tokens,
                             size_t n_tokens, uint32_t start_pos, float* logits_out,
                             uint32_t* argmax_out);

/* The decode half of InferenceEngine::benchmark_tokens (src/engine.rs:189-223)
 * with the argmax on the device: for each of `n_seqs` sequences (slots
 * seqs[i], next input token first_tokens[i] at position start_pos[i]) runs
 * n_steps greedy steps; tokens_out is [n_steps][n_seqs]: row s is the token
 * step s produced (the argmax of its logits), which the reference loop feeds
 * to step s + 1. */
lrs_status lrs_model_decode_greedy(lrs_model* model, size_t n_seqs, const uint32_t* seqs,
                                   const uint32_t* first_tokens, const uint32_t* start_pos,
                                   size_t n_steps, uint32_t* tokens_out);

/* Device-resident decode for benchmarking: like lrs_model_decode_greedy but
 * queues the steps on the backend stream and leaves the tokens on the device;
 * lrs_model_read_tokens copies them out afterwards. */
lrs_status lrs_model_decode_enqueue(lrs_model* model, size_t n_seqs, const uint32_t* seqs,
                                    const uint32_t* first_tokens, const uint32_t* start_pos,
                                    size_t n_steps);
lrs_status lrs_model_read_tokens(lrs_model* model, size_t n_seqs, size_t n_steps,
                                 uint32_t* tokens_out);

/* Measurement hook (no counterpart in the reference): runs ONE greedy step for
 * the given items outside any CUDA graph, with every GEMV launch bracketed by
 * CUDA events on the model's stream.  Reports the summed GEMV time, the number
 * of GEMV launches, the whole step's time and the summed time of the per-layer
 * RoPE/KV-store + attention launches (milliseconds; any pointer may be NULL).
 * The step writes the KV cache at `pos` like a normal decode step. */
lrs_status lrs_model_profile_step(lrs_model* model, size_t n_seqs, const uint32_t* seqs,
                                  const uint32_t* tokens, const uint32_t* pos, float* gemv_ms,
                                  uint32_t* gemv_launches, float* step_ms, float* attn_ms);

/* Kernel launches in one decode step of the most recent decode_enqueue
 * (kernel nodes of its CUDA graph); 0 before the first graph-captured step. */
uint32_t lrs_model_step_kernels(const lrs_model* model);

/* Device stream (cudaStream_t) the model and backend queue work on. */
void* lrs_backend_stream(lrs_backend* backend);

/* Bytes of weights the decode step streams per token (algorithmic). */
uint64_t lrs_model_weight_bytes(const lrs_model* model);
/* FNV-1a 64-bit digest of the weight bytes the model holds on the device
 * (embedding, every layer's matrices in q, k, v, o, gate, up, down order, the
 * LM head).  No counterpart in the reference: an integrity check that two
 * models (for example one encoded on the host and one by device_recipe) hold
 * the same bytes.  Synchronous; copies each tensor through host memory. */
lrs_status lrs_model_weights_digest(lrs_model* model, uint64_t* digest_out);

#ifdef __cplusplus
}
#endif
#endif /* LLAMARS_H */

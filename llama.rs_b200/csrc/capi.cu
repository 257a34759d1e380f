// capi.cu -- the extern "C" surface of include/llamars.h.
//
// Host side of the CUDA backend: the KernelBackend::matvec equivalent
// (src/backend.rs:69-73), tensor upload, and a CausalModel equivalent
// (src/architecture.rs:42-78, src/model.rs:135-270) that owns the device
// weights, the paged KV cache and the activation buffers, and replays the
// per-token decode step as one CUDA graph.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/llamars.h"
#include "../../include/llamars_synth.h"
#include "common.h"
#include "decode.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "sample.cuh"
#include "step1.cuh"
#include "tp_p2p.cuh"

namespace lrs {
thread_local std::string g_last_error;
int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
void clear_error() { g_last_error.clear(); }
}  // namespace lrs

using namespace lrs;

#define LRS_CUDA(call)                                                                      \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      return fail(LRS_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));        \
  } while (0)

namespace {

// NCCL, resolved at run time from the process (or libnccl.so.2) the first time
// a tensor-parallel model is made, so the library loads without NCCL.
struct NcclApi {
  bool ok = false;
  std::string err;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.err = std::string("NCCL not found: ") + dlerror();
      return a;
    }
#define LRS_NCCL_SYM(f) a.f = reinterpret_cast<decltype(a.f)>(dlsym(h, "nccl" #f))
    LRS_NCCL_SYM(GetUniqueId);
    LRS_NCCL_SYM(CommInitRank);
    LRS_NCCL_SYM(AllReduce);
    LRS_NCCL_SYM(AllGather);
    LRS_NCCL_SYM(CommDestroy);
    LRS_NCCL_SYM(GetErrorString);
#undef LRS_NCCL_SYM
    a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.AllGather && a.CommDestroy &&
           a.GetErrorString;
    if (!a.ok) a.err = "NCCL is missing required symbols";
    return a;
  }();
  return api;
}

#define LRS_NCCL(call)                                                                      \
  do {                                                                                      \
    ncclResult_t r_ = (call);                                                               \
    if (r_ != ncclSuccess)                                                                  \
      return fail(LRS_ERR_CUDA, std::string("NCCL: ") + nccl().GetErrorString(r_));        \
  } while (0)

int32_t check_device_error(lrs_backend* be) {
  int h = 0;
  LRS_CUDA(cudaMemcpy(&h, be->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) {
    cudaMemset(be->d_err, 0, sizeof(int));
    return fail(LRS_ERR_DEVICE_TIMEOUT, "a bounded device-side wait gave up (TMA copy not completed)");
  }
  return LRS_OK;
}

int32_t validate_tensor(size_t nbytes, size_t rows, size_t cols, uint32_t type) {
  // QuantTensor::from_data, src/quant.rs:132-157
  uint32_t bv, bb;
  if (!type_geometry(type, &bv, &bb))
    return fail(LRS_ERR_UNSUPPORTED,
                "unsupported GGML tensor type " + std::to_string(type) +
                    "; supported: F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K");
  if (rows == 0 || cols == 0) return fail(LRS_ERR_INVALID, "empty tensor");
  if (cols % bv)
    return fail(LRS_ERR_INVALID, "last dimension " + std::to_string(cols) + " is not divisible by " +
                                     std::to_string(bv) + " for " + type_name(type));
  size_t expected = rows * (cols / bv) * bb;
  if (nbytes != expected)
    return fail(LRS_ERR_INVALID, std::string("bad ") + type_name(type) + " tensor byte length: got " +
                                     std::to_string(nbytes) + ", expected " + std::to_string(expected));
  if (cols % 32)
    return fail(LRS_ERR_UNSUPPORTED, "the CUDA backend requires cols % 32 == 0");
  return LRS_OK;
}

int32_t upload(const void* data, size_t nbytes, size_t rows, size_t cols, uint32_t type,
               DevTensor* out) {
  int32_t rc = validate_tensor(nbytes, rows, cols, type);
  if (rc) return rc;
  uint8_t* d = nullptr;
  // +256: tiles are copied in 16-byte granules that may run past the last row.
  if (cudaMalloc(&d, nbytes + 256) != cudaSuccess)
    return fail(LRS_ERR_OOM, "cudaMalloc of " + std::to_string(nbytes) + " bytes failed");
  cudaMemset(d + nbytes, 0, 256);
  // a copy from pageable memory may return before its DMA lands; kernels on
  // other (non-blocking) streams must not start before it has
  if (cudaMemcpy(d, data, nbytes, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaStreamSynchronize(cudaStreamLegacy) != cudaSuccess) {
    cudaFree(d);
    return fail(LRS_ERR_CUDA, "upload copy failed");
  }
  out->d = d;
  out->nbytes = nbytes;
  out->rows = (int)rows;
  out->cols = (int)cols;
  out->type = type;
  return LRS_OK;
}

template <typename T>
int32_t dalloc(T** p, size_t count) {
  if (cudaMalloc((void**)p, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess)
    return fail(LRS_ERR_OOM, "cudaMalloc failed (" + std::to_string(count * sizeof(T)) + " bytes)");
  return LRS_OK;
}

int32_t ensure_cap(float** p, size_t* cap, size_t n) {
  if (*cap >= n) return LRS_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  int32_t rc = dalloc(p, n);
  if (rc) return rc;
  *cap = n;
  return LRS_OK;
}

GemvMat mat_of(const DevTensor& t, float* out, int out_ld, const float* bias = nullptr,
               const DevTensor* t2 = nullptr) {
  GemvMat m{};
  m.w = t.d;
  m.w2 = t2 ? t2->d : nullptr;
  m.bias = bias;
  m.out = out;
  m.type = t.type;
  m.rows = t.rows;
  m.cols = t.cols;
  m.out_ld = out_ld;
  return m;
}

}  // namespace

extern "C" {

const char* lrs_last_error(void) { return g_last_error.c_str(); }

lrs_status lrs_type_geometry(uint32_t t, uint32_t* bv, uint32_t* bb) {
  uint32_t a, b;
  if (!type_geometry(t, &a, &b)) return fail(LRS_ERR_UNSUPPORTED, "unsupported GGML type");
  if (bv) *bv = a;
  if (bb) *bb = b;
  return LRS_OK;
}

lrs_status lrs_backend_create(int device, lrs_backend** out) try {
  if (!out) return fail(LRS_ERR_INVALID, "null out");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
    return fail(LRS_ERR_CUDA, "no CUDA device is available");
  if (device < 0 || device >= n) return fail(LRS_ERR_INVALID, "device ordinal out of range");
  LRS_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  LRS_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(LRS_ERR_UNSUPPORTED, std::string("this build targets sm_100a (B200); device is ") +
                                         prop.name);
  auto* be = new lrs_backend();
  be->device = device;
  be->sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&be->d_err, sizeof(int)) != cudaSuccess) {
    delete be;
    return fail(LRS_ERR_CUDA, "stream / flag allocation failed");
  }
  cudaMemset(be->d_err, 0, sizeof(int));
  *out = be;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

void lrs_backend_destroy(lrs_backend* be) {
  if (!be) return;
  cudaSetDevice(be->device);
  cudaStreamSynchronize(be->stream);
  cudaFree(be->d_err);
  cudaFree(be->d_x);
  cudaFree(be->d_y);
  cudaFree(be->d_scratch);
  cudaFree(be->d_sample);
  cudaStreamDestroy(be->stream);
  delete be;
}

const char* lrs_backend_name(const lrs_backend*) { return "cuda-sm100a"; }
size_t lrs_backend_threads(const lrs_backend* be) { return be ? (size_t)be->sms : 0; }
void* lrs_backend_stream(lrs_backend* be) { return be ? (void*)be->stream : nullptr; }

lrs_status lrs_backend_synchronize(lrs_backend* be) try {
  if (!be) return fail(LRS_ERR_INVALID, "null backend");
  LRS_CUDA(cudaSetDevice(be->device));
  LRS_CUDA(cudaStreamSynchronize(be->stream));
  return check_device_error(be);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_tensor_upload(lrs_backend* be, const void* data, size_t nbytes, size_t rows,
                             size_t cols, uint32_t type, lrs_tensor** out) try {
  if (!be || !data || !out) return fail(LRS_ERR_INVALID, "null argument");
  LRS_CUDA(cudaSetDevice(be->device));
  auto* t = new lrs_tensor();
  t->be = be;
  int32_t rc = upload(data, nbytes, rows, cols, type, &t->t);
  if (rc) {
    delete t;
    return rc;
  }
  *out = t;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

void lrs_tensor_free(lrs_tensor* t) {
  if (!t) return;
  cudaSetDevice(t->be->device);
  cudaFree(t->t.d);
  delete t;
}

const void* lrs_tensor_device_ptr(const lrs_tensor* t) { return t ? t->t.d : nullptr; }

lrs_status lrs_dequantize_rows(lrs_backend* be, const lrs_tensor* t, size_t row0, size_t nrows,
                               float* out) try {
  if (!be || !t || !out) return fail(LRS_ERR_INVALID, "null argument");
  if (row0 + nrows > (size_t)t->t.rows) return fail(LRS_ERR_INVALID, "row range out of bounds");
  if (nrows == 0) return LRS_OK;
  LRS_CUDA(cudaSetDevice(be->device));
  size_t n = nrows * (size_t)t->t.cols;
  int32_t rc = ensure_cap(&be->d_y, &be->y_cap, n);
  if (rc) return rc;
  LRS_CUDA(launch_dequant_rows(t->t.d, t->t.type, t->t.cols, (int)row0, (int)nrows, be->d_y,
                               be->stream));
  LRS_CUDA(cudaMemcpyAsync(out, be->d_y, n * 4, cudaMemcpyDeviceToHost, be->stream));
  LRS_CUDA(cudaStreamSynchronize(be->stream));
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_matvec_device(lrs_backend* be, const lrs_tensor* w, const float* d_in,
                             size_t batch, float* d_out, void* stream) try {
  if (!be || !w || !d_in || !d_out) return fail(LRS_ERR_INVALID, "null argument");
  if (batch < 1 || batch > 64) return fail(LRS_ERR_INVALID, "batch must be in 1..=64");
  GemvMat m = mat_of(w->t, d_out, w->t.rows);
  GemvParams p;
  int32_t rc = gemv_plan(&p, &m, 1, EPI_STORE, (int)batch);
  if (rc) return rc;
  p.x = d_in;
  p.x_ld = w->t.cols;
  p.error_flag = be->d_err;
  if (batch > 1 && gemm_supported(p)) {
    const size_t need = gemm_scratch_bytes((int)batch, w->t.cols, be->sms);
    if (be->scratch_cap < need) {
      cudaFree(be->d_scratch);  // synchronizes with work that may still use it
      be->d_scratch = nullptr;
      be->scratch_cap = 0;
      if (cudaMalloc(&be->d_scratch, need) != cudaSuccess)
        return fail(LRS_ERR_OOM, "cudaMalloc of matmul scratch failed");
      LRS_CUDA(cudaMemset(be->d_scratch, 0, need));  // the tail counters start at zero
      be->scratch_cap = need;
    }
    p.scratch = be->d_scratch;
    p.scratch_bytes = be->scratch_cap;
  }
  cudaStream_t st = stream ? (cudaStream_t)stream : be->stream;
  LRS_CUDA(gemv_launch(p, st, be->sms, false));
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_matvec_batched(lrs_backend* be, const lrs_tensor* w, const float* in, size_t batch,
                              size_t n_in, float* out, size_t n_out) try {
  if (!be || !w || !in || !out) return fail(LRS_ERR_INVALID, "null argument");
  // QuantTensor::validate_matvec, src/quant.rs:303-318
  if (n_in != (size_t)w->t.cols)
    return fail(LRS_ERR_INVALID, "matvec input mismatch: got " + std::to_string(n_in) +
                                     ", expected " + std::to_string(w->t.cols));
  if (n_out != (size_t)w->t.rows)
    return fail(LRS_ERR_INVALID, "matvec output mismatch: got " + std::to_string(n_out) +
                                     ", expected " + std::to_string(w->t.rows));
  if (batch < 1 || batch > 64) return fail(LRS_ERR_INVALID, "batch must be in 1..=64");
  LRS_CUDA(cudaSetDevice(be->device));
  int32_t rc = ensure_cap(&be->d_x, &be->x_cap, batch * n_in);
  if (rc) return rc;
  rc = ensure_cap(&be->d_y, &be->y_cap, batch * n_out);
  if (rc) return rc;
  LRS_CUDA(cudaMemcpyAsync(be->d_x, in, batch * n_in * 4, cudaMemcpyHostToDevice, be->stream));
  rc = lrs_matvec_device(be, w, be->d_x, batch, be->d_y, be->stream);
  if (rc) return rc;
  LRS_CUDA(cudaMemcpyAsync(out, be->d_y, batch * n_out * 4, cudaMemcpyDeviceToHost, be->stream));
  LRS_CUDA(cudaStreamSynchronize(be->stream));
  return check_device_error(be);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_matvec(lrs_backend* be, const lrs_tensor* w, const float* in, size_t n_in,
                      float* out, size_t n_out) try {
  return lrs_matvec_batched(be, w, in, 1, n_in, out, n_out);
} catch (...) {
  return lrs::status_of_current_exception();
}

}  // extern "C"

// =============================================================== model ====

namespace {

struct Layer {
  DevTensor q, k, v, o, gate, up, down;
  // tensor parallelism: column windows of the row-split o / down shards.  A
  // shard holds whole blocks [c0 - lo, c0 - lo + cols); when that is wider
  // than the rank's columns, x is zero-padded to it (launch_pad_copy).
  int o_lo = 0, d_lo = 0;
  float *in_norm = nullptr, *post_norm = nullptr, *qb = nullptr, *kb = nullptr, *vb = nullptr;
  void *kpool = nullptr, *vpool = nullptr;
};

struct GraphKey {
  int batch;
  const void* tokens_out;
  bool operator<(const GraphKey& o) const {
    return batch != o.batch ? batch < o.batch : tokens_out < o.tokens_out;
  }
};

}  // namespace

struct lrs_model {
  lrs_backend* be = nullptr;
  lrs_config c{};
  lrs_model_options opt{};
  std::vector<Layer> layers;
  DevTensor embed, lm;
  bool tied = false;
  float* final_norm = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  std::vector<void*> allocs;  // everything cudaMalloc'd except the tensors above
  // paged KV
  int pages_per_seq = 0, total_pages = 0;
  std::vector<int> free_pages;
  std::vector<std::vector<int>> seq_pages;
  int* d_pages = nullptr;
  size_t kv_elem = 4;
  // activations, for up to max_items items per step
  int max_items = 0, max_split = 64;
  float *residual = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr,
        *att = nullptr, *act = nullptr, *logits = nullptr, *part = nullptr;
  float *att_pad = nullptr, *act_pad = nullptr;  // zero-padded x of windowed o / down shards
  // tensor parallelism over peer memory (LRS_TP_P2P=1): exchange buffers
  // [2][max_items * hidden], signal words [world], a launch counter, and the
  // device arrays of every rank's (IPC-mapped) pointers
  bool tp_p2p = false;
  float* xbuf = nullptr;
  int* tp_sig = nullptr;
  unsigned* tp_tickets = nullptr;
  const float** d_parts = nullptr;  // [2][world]
  int** d_peer_sig = nullptr;       // [world]
  std::vector<void*> ipc_opened;
  float* act2 = nullptr;    // up projection when a layer's gate and up differ in type
  // the batch-1 decode step as one persistent kernel (step1.cu)
  bool s1_ok = false;
  S1Model s1{};
  S1Model* d_s1 = nullptr;
  const void* s1_tokens = nullptr;  // tokens_out the device copy holds
  int s1_cap = -1;
  void* gemm_scratch = nullptr;  // batched tensor-core matmul scratch
  // tensor parallelism: this process holds shard tp_rank of tp_world
  int tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;
  uint32_t vocab_full = 0;  // the model's vocabulary (c.vocab_size is this shard's head rows)
  int vocab0 = 0;           // first LM-head row of this shard
  float* logits_full = nullptr;
  size_t gemm_scratch_bytes = 0;
  unsigned long long* keys = nullptr;
  int *d_tok = nullptr, *d_pos = nullptr, *d_seq = nullptr, *d_step = nullptr;
  unsigned* d_attn_cnt = nullptr;  // [max_items][kv heads] split counters of the fused attention
  // batch-1 steps run the projections of a second GGML type among q/k/v (v
  // in Q8_0 under q4km) on a side stream, beside the first type's launch
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  uint32_t* d_last = nullptr;
  uint32_t* d_tokens_out = nullptr;
  size_t tokens_out_cap = 0;  // in elements
  std::map<GraphKey, cudaGraphExec_t> graphs;
  std::map<GraphKey, uint32_t> graph_kernels;  // kernel nodes per captured step
  uint32_t last_step_kernels = 0;
  uint64_t weight_bytes = 0;
  // When set, every GEMV launch of enqueue_step is bracketed by two events.
  std::vector<cudaEvent_t>* prof = nullptr;
  // When set, each layer's RoPE/KV store + attention launches are bracketed too.
  std::vector<cudaEvent_t>* prof_attn = nullptr;
};

namespace {

int32_t model_alloc(lrs_model* m, void** p, size_t bytes) {
  if (cudaMalloc(p, std::max<size_t>(bytes, 4)) != cudaSuccess)
    return fail(LRS_ERR_OOM, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
  m->allocs.push_back(*p);
  return LRS_OK;
}

// One projection (with per-launch events when profiling).
cudaError_t model_gemv(lrs_model* m, const GemvParams& p0, cudaStream_t st, int sms) {
  GemvParams p = p0;
  p.scratch = m->gemm_scratch;
  p.scratch_bytes = m->gemm_scratch_bytes;
  auto run = [&](bool pdl) { return gemv_launch(p, st, sms, pdl); };
  if (!m->prof) return run(true);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  m->prof->push_back(a);
  m->prof->push_back(b);
  cudaEventRecord(a, st);
  cudaError_t e = run(false);
  cudaEventRecord(b, st);
  return e;
}

int32_t upload_vec(lrs_model* m, const float* h, size_t n, float** out) {
  if (!h) {
    *out = nullptr;
    return LRS_OK;
  }
  int32_t rc = model_alloc(m, (void**)out, n * 4);
  if (rc) return rc;
  LRS_CUDA(cudaMemcpy(*out, h, n * 4, cudaMemcpyHostToDevice));
  return LRS_OK;
}

int32_t upload_mat(const lrs_tensor_desc& d, size_t rows, size_t cols, const char* what,
                   DevTensor* out) {
  if (d.rows != rows || d.cols != cols)
    return fail(LRS_ERR_INVALID, std::string("tensor ") + what + " has shape [" +
                                     std::to_string(d.rows) + ", " + std::to_string(d.cols) +
                                     "], expected [" + std::to_string(rows) + ", " +
                                     std::to_string(cols) + "]");
  return upload(d.data, d.nbytes, rows, cols, d.ggml_type, out);
}

// The peer-memory all-reduce: every rank allocates its exchange buffers and
// signal words, the ranks swap CUDA IPC handles with one NCCL all-gather, and
// each rank maps its peers' allocations (collective: all ranks call it).
int32_t setup_tp_p2p(lrs_model* m, int h) {
  const int world = m->tp_world, rank = m->tp_rank;
  cudaStream_t st = m->be->stream;
  const size_t xcount = 2 * (size_t)m->max_items * h;
  // own cudaMalloc allocations: an IPC handle names the base of an allocation
  LRS_CUDA(cudaMalloc((void**)&m->xbuf, xcount * 4));
  m->allocs.push_back(m->xbuf);
  // signal words [0, world) of tp_allreduce_add_kernel
  const size_t sig_bytes = (size_t)world * 4;
  LRS_CUDA(cudaMalloc((void**)&m->tp_sig, sig_bytes));
  m->allocs.push_back(m->tp_sig);
  LRS_CUDA(cudaMemset(m->tp_sig, 0, sig_bytes));
  int32_t rc;
  if ((rc = model_alloc(m, (void**)&m->tp_tickets, 4))) return rc;
  LRS_CUDA(cudaMemset(m->tp_tickets, 0, 4));
  if ((size_t)world > (size_t)m->max_items)
    return fail(LRS_ERR_UNSUPPORTED, "peer-memory all-reduce: more ranks than item slots");
  cudaIpcMemHandle_t mine[2];
  LRS_CUDA(cudaIpcGetMemHandle(&mine[0], m->xbuf));
  LRS_CUDA(cudaIpcGetMemHandle(&mine[1], m->tp_sig));
  uint8_t* d_hs = nullptr;
  if ((rc = model_alloc(m, (void**)&d_hs, sizeof(mine) * (world + 1)))) return rc;
  LRS_CUDA(cudaMemcpy(d_hs, mine, sizeof(mine), cudaMemcpyHostToDevice));
  LRS_NCCL(nccl().AllGather(d_hs, d_hs + sizeof(mine), sizeof(mine), ncclInt8, m->comm, st));
  std::vector<cudaIpcMemHandle_t> all(2 * (size_t)world);
  LRS_CUDA(cudaMemcpyAsync(all.data(), d_hs + sizeof(mine), sizeof(mine) * world,
                           cudaMemcpyDeviceToHost, st));
  LRS_CUDA(cudaStreamSynchronize(st));
  std::vector<const float*> parts(2 * (size_t)world);
  std::vector<int*> sigs(world);
  for (int p = 0; p < world; p++) {
    float* x = m->xbuf;
    int* g = m->tp_sig;
    if (p != rank) {
      void* px = nullptr;
      void* pg = nullptr;
      LRS_CUDA(cudaIpcOpenMemHandle(&px, all[2 * p], cudaIpcMemLazyEnablePeerAccess));
      m->ipc_opened.push_back(px);
      LRS_CUDA(cudaIpcOpenMemHandle(&pg, all[2 * p + 1], cudaIpcMemLazyEnablePeerAccess));
      m->ipc_opened.push_back(pg);
      x = static_cast<float*>(px);
      g = static_cast<int*>(pg);
    }
    parts[p] = x;
    parts[world + p] = x + (size_t)m->max_items * h;
    sigs[p] = g;
  }
  if ((rc = model_alloc(m, (void**)&m->d_parts, parts.size() * sizeof(float*))) ||
      (rc = model_alloc(m, (void**)&m->d_peer_sig, sigs.size() * sizeof(int*))))
    return rc;
  LRS_CUDA(cudaMemcpy(m->d_parts, parts.data(), parts.size() * sizeof(float*), cudaMemcpyHostToDevice));
  LRS_CUDA(cudaMemcpy(m->d_peer_sig, sigs.data(), sigs.size() * sizeof(int*), cudaMemcpyHostToDevice));
  m->tp_p2p = true;
  return LRS_OK;
}

// Splits of each sequence's context: about eight waves of resident attention
// CTAs (batch * kv heads * splits CTAs), so that CTAs of different lengths
// even out across the SMs and each SM's second CTA streams while the first
// starts or finishes.
int nsplit_for(const lrs_model* m, int batch) {
  const int slots = m->be->sms * attention_ctas_per_sm((int)m->c.head_dim,
                                                       m->opt.kv_dtype == LRS_KV_BF16);
  int want = 8 * slots / (batch * (int)m->c.num_key_value_heads);
  // at least 128 positions per split of a full context: a split's tiles are
  // copied back to back, and the merge reads fewer partials
  int maxs = std::max(1, (int)((m->opt.max_seq_len + 127) / 128));
  return std::max(1, std::min({want, m->max_split, maxs}));
}

int32_t ensure_pages(lrs_model* m, int seq, uint32_t last_pos) {
  size_t need = last_pos / kPageSize + 1;
  auto& pg = m->seq_pages[seq];
  if (pg.size() >= need) return LRS_OK;
  size_t old = pg.size();
  while (pg.size() < need) {
    if (m->free_pages.empty()) return fail(LRS_ERR_OOM, "KV page pool exhausted");
    pg.push_back(m->free_pages.back());
    m->free_pages.pop_back();
  }
  LRS_CUDA(cudaMemcpyAsync(m->d_pages + (size_t)seq * m->pages_per_seq + old, pg.data() + old,
                           (pg.size() - old) * sizeof(int), cudaMemcpyHostToDevice, m->be->stream));
  return LRS_OK;
}

// Queues one forward step for items 0..B-1 (d_tok / d_pos / d_seq already set):
// Qwen2Model::forward_impl, src/model.rs:135-270, for B tokens at once.  When
// `lm_item` >= 0 only that item runs the final norm + LM head (prefill);
// lm_item == -1 runs it for every item; -2 skips it.
int32_t enqueue_step(lrs_model* m, int B, int lm_item, bool want_logits, bool greedy_advance,
                     int n_steps_cap) {
  const lrs_config& c = m->c;
  cudaStream_t st = m->be->stream;
  const int h = c.hidden_size, I = c.intermediate_size, nh = c.num_attention_heads,
            nkv = c.num_key_value_heads, hd = c.head_dim, kvw = nkv * hd, qw = nh * hd;
  const int sms = m->be->sms;
  const bool tp = m->tp_world > 1;
  // Row-split projections (o, down): every rank adds its partial sum of the
  // residual update; rank 0 adds onto the residual, the others overwrite their
  // copy with the partial, and one sum all-reduce rebuilds the residual.
  // With the peer-memory all-reduce every rank stores its partial into the
  // exchange buffer of the call's parity instead, and tp_allreduce_add_kernel
  // adds all ranks' partials onto the residual.
  const int res_epi = tp && (m->tp_p2p || m->tp_rank != 0) ? EPI_STORE : EPI_ADD;
  int ar_calls = 0;  // all-reduces queued by this step (2 per layer: parities alternate)
  auto res_out = [&]() -> float* {
    return m->tp_p2p ? m->xbuf + (size_t)(ar_calls & 1) * m->max_items * h : m->residual;
  };
  auto allreduce_residual = [&]() -> int32_t {
    if (tp && m->tp_p2p) {
      TpArgs a;
      a.residual = m->residual;
      a.n = (size_t)B * h;
      a.parts0 = m->d_parts;
      a.parts1 = m->d_parts + m->tp_world;
      a.parity = ar_calls & 1;
      a.local_sig = m->tp_sig;
      a.peer_sig = m->d_peer_sig;
      a.tickets = m->tp_tickets;
      a.rank = m->tp_rank;
      a.world = m->tp_world;
      a.error_flag = m->be->d_err;
      LRS_CUDA(launch_tp_allreduce_add(a, st));
    } else if (tp) {
      LRS_NCCL(nccl().AllReduce(m->residual, m->residual, (size_t)B * h, ncclFloat32, ncclSum,
                                m->comm, st));
    }
    ar_calls++;
    return LRS_OK;
  };
  StepIO io{m->d_tok, m->d_pos, m->d_seq, m->d_pages, m->pages_per_seq};
  const int kv_bf16 = m->opt.kv_dtype == LRS_KV_BF16;
  const int nsplit = nsplit_for(m, B);
  int32_t rc;
  LRS_CUDA(launch_embed(m->embed.d, m->embed.type, h, m->d_tok, B, m->residual, m->keys, st));
  for (size_t li = 0; li < m->layers.size(); li++) {
    Layer& L = m->layers[li];
    GemvParams p;
    // input_layernorm + q/k/v projections with bias (src/model.rs:175-186)
    GemvMat qkv[3] = {mat_of(L.q, m->q, qw, L.qb), mat_of(L.k, m->k, kvw, L.kb),
                      mat_of(L.v, m->v, kvw, L.vb)};
    // batch 1, two GGML types among q/k/v, not profiling: the second type's
    // segments on the side stream (its launch is a separate one anyway)
    GemvMat first[3], second[3];
    int nf = 0, ns = 0;
    for (int i = 0; i < 3; i++) {
      if (qkv[i].type == qkv[0].type) first[nf++] = qkv[i];
      else second[ns++] = qkv[i];
    }
    bool fork = B == 1 && ns > 0 && !m->prof && m->side;
    for (int i = 1; i < ns; i++) fork = fork && second[i].type == second[0].type;
    auto qkv_input = [&](GemvParams& q) {
      q.error_flag = m->be->d_err;
      q.x = m->residual;  // the norm is fused into the x preparation
      q.norm_w = L.in_norm;
      q.norm_eps = c.rms_norm_eps;
      q.x_ld = h;
    };
    if (fork) {
      GemvParams p2;
      if ((rc = gemv_plan(&p, first, nf, EPI_STORE, B)) ||
          (rc = gemv_plan(&p2, second, ns, EPI_STORE, B)))
        return rc;
      qkv_input(p);
      qkv_input(p2);
      LRS_CUDA(cudaEventRecord(m->ev_fork, st));
      LRS_CUDA(cudaStreamWaitEvent(m->side, m->ev_fork, 0));
      LRS_CUDA(model_gemv(m, p2, m->side, sms));
      LRS_CUDA(cudaEventRecord(m->ev_join, m->side));
      LRS_CUDA(model_gemv(m, p, st, sms));
      LRS_CUDA(cudaStreamWaitEvent(st, m->ev_join, 0));
    } else {
      if ((rc = gemv_plan(&p, qkv, 3, EPI_STORE, B))) return rc;
      p.error_flag = m->be->d_err;
      if (B == 1 || gemm_supported(p)) {  // the norm is fused into the x preparation
        qkv_input(p);
      } else {
        LRS_CUDA(launch_rmsnorm(m->residual, L.in_norm, c.rms_norm_eps, h, B, m->xn, st));
        p.x = m->xn;
        p.x_ld = h;
      }
      LRS_CUDA(model_gemv(m, p, st, sms));
    }
    // RoPE + KV store (src/model.rs:188-205), attention (:206-231)
    cudaEvent_t a0 = nullptr, a1 = nullptr;
    if (m->prof_attn) {
      cudaEventCreate(&a0);
      cudaEventCreate(&a1);
      m->prof_attn->push_back(a0);
      m->prof_attn->push_back(a1);
      cudaEventRecord(a0, st);
    }
    // every item its own sequence (a decode step): RoPE, the KV store and the
    // split merge run inside the attention kernel; prefill chunks (items of
    // one sequence read each other's rows) store every row first
    const bool fused_attn = lm_item == -1 || B == 1;
    if (!fused_attn)
      LRS_CUDA(launch_rope_store(m->q, m->k, m->v, m->rope_cos, m->rope_sin, io, B, nh, nkv, hd,
                                 L.kpool, L.vpool, kv_bf16, st));
    AttnLaunch al{};
    al.q = m->q, al.k = m->k, al.v = m->v, al.cos_t = m->rope_cos, al.sin_t = m->rope_sin;
    al.io = io;
    al.batch = B, al.nh = nh, al.nkv = nkv, al.hd = hd, al.kv_bf16 = kv_bf16, al.nsplit = nsplit;
    al.kpool = L.kpool, al.vpool = L.vpool;
    al.part = m->part, al.att = m->att, al.cnt = m->d_attn_cnt, al.err = m->be->d_err;
    al.fused = fused_attn;
    LRS_CUDA(launch_attention(al, st));
    if (a1) cudaEventRecord(a1, st);
    // o_proj + residual (src/model.rs:233-238)
    GemvMat om = mat_of(L.o, res_out(), h);
    if ((rc = gemv_plan(&p, &om, 1, res_epi, B))) return rc;
    p.error_flag = m->be->d_err;
    p.x = m->att;
    p.x_ld = qw;
    if (L.o.cols != qw) {  // a windowed column shard: x zero-padded to its blocks
      LRS_CUDA(launch_pad_copy(m->att, qw, m->att_pad, L.o.cols, L.o_lo, B, st));
      p.x = m->att_pad;
      p.x_ld = L.o.cols;
    }
    LRS_CUDA(model_gemv(m, p, st, sms));
    if ((rc = allreduce_residual())) return rc;
    // post_attention_layernorm + gate/up + SwiGLU (src/model.rs:241-254)
    bool xn_ready = false;
    auto ffn_input = [&](GemvParams& q) -> int32_t {
      q.error_flag = m->be->d_err;
      if (B == 1 || gemm_supported(q)) {  // the norm is fused into the x preparation
        q.x = m->residual;
        q.norm_w = L.post_norm;
        q.norm_eps = c.rms_norm_eps;
      } else {
        if (!xn_ready)
          LRS_CUDA(launch_rmsnorm(m->residual, L.post_norm, c.rms_norm_eps, h, B, m->xn, st));
        xn_ready = true;
        q.x = m->xn;
      }
      q.x_ld = h;
      return LRS_OK;
    };
    if (L.gate.type == L.up.type) {  // one launch over the row pair, SwiGLU in its epilogue
      GemvMat gu = mat_of(L.gate, m->act, I, nullptr, &L.up);
      if ((rc = gemv_plan(&p, &gu, 1, EPI_SWIGLU, B)) || (rc = ffn_input(p))) return rc;
      LRS_CUDA(model_gemv(m, p, st, sms));
    } else {  // mixed files: gate and up of different types, then SwiGLU
      GemvMat gm = mat_of(L.gate, m->act, I), um = mat_of(L.up, m->act2, I);
      if ((rc = gemv_plan(&p, &gm, 1, EPI_STORE, B)) || (rc = ffn_input(p))) return rc;
      LRS_CUDA(model_gemv(m, p, st, sms));
      if ((rc = gemv_plan(&p, &um, 1, EPI_STORE, B)) || (rc = ffn_input(p))) return rc;
      LRS_CUDA(model_gemv(m, p, st, sms));
      LRS_CUDA(launch_swiglu(m->act, m->act2, (size_t)B * I, st));
    }
    // down_proj + residual (src/model.rs:255-260)
    GemvMat dm = mat_of(L.down, res_out(), h);
    if ((rc = gemv_plan(&p, &dm, 1, res_epi, B))) return rc;
    p.error_flag = m->be->d_err;
    p.x = m->act;
    p.x_ld = I;
    if (L.down.cols != I) {
      LRS_CUDA(launch_pad_copy(m->act, I, m->act_pad, L.down.cols, L.d_lo, B, st));
      p.x = m->act_pad;
      p.x_ld = L.down.cols;
    }
    LRS_CUDA(model_gemv(m, p, st, sms));
    if ((rc = allreduce_residual())) return rc;
  }
  if (lm_item == -2) return LRS_OK;
  // final norm + lm_head (src/model.rs:263-268) fused with the greedy argmax
  const int nb = lm_item >= 0 ? 1 : B;
  const float* xin = m->residual + (lm_item >= 0 ? (size_t)lm_item * h : 0);
  GemvMat lmm = mat_of(m->lm, want_logits ? m->logits : nullptr, c.vocab_size);
  GemvParams p;
  if ((rc = gemv_plan(&p, &lmm, 1, EPI_ARGMAX, nb))) return rc;
  p.error_flag = m->be->d_err;
  p.argmax_keys = m->keys + (lm_item >= 0 ? lm_item : 0);
  if (nb == 1 || gemm_supported(p)) {
    p.x = xin;
    p.norm_w = m->final_norm;
    p.norm_eps = c.rms_norm_eps;
  } else {
    LRS_CUDA(launch_rmsnorm(xin, m->final_norm, c.rms_norm_eps, h, nb, m->xn, st));
    p.x = m->xn;
  }
  p.x_ld = h;
  LRS_CUDA(model_gemv(m, p, st, sms));
  if (tp) {
    // shard rows -> vocabulary ids, then the shard argmaxes meet in one MAX
    // all-reduce of the packed keys
    LRS_CUDA(launch_key_offset(p.argmax_keys, nb, (uint32_t)m->vocab0, st));
    LRS_NCCL(nccl().AllReduce(p.argmax_keys, p.argmax_keys, (size_t)nb, ncclUint64, ncclMax,
                              m->comm, st));
    if (want_logits)
      LRS_NCCL(nccl().AllGather(m->logits, m->logits_full, (size_t)c.vocab_size, ncclFloat32,
                                m->comm, st));
  }
  if (greedy_advance)
    LRS_CUDA(launch_advance(m->keys, m->d_tok, m->d_pos, B, m->d_step, n_steps_cap,
                            m->d_tokens_out, m->d_last, st));
  return LRS_OK;
}

// The batch-1 decode step of step1.cu: the layer table, the chunk plans and
// the shared-memory plan, uploaded once.  Models it cannot serve (tensor
// parallel, head_dim other than 64/128, more than 8 query heads per KV head,
// or x rows wider than shared memory) keep the per-kernel step.
int32_t setup_step1(lrs_model* m) {
  const lrs_config& c = m->c;
  if (m->tp_world != 1 || !m->opt.persistent_decode) return LRS_OK;
  if ((c.head_dim != 64 && c.head_dim != 128) || c.num_attention_heads / c.num_key_value_heads > 8)
    return LRS_OK;
  int coop = 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->be->device) != cudaSuccess || !coop)
    return LRS_OK;
  const int G = m->be->sms;
  S1Model& s = m->s1;
  s = S1Model{};
  s.L = (int)m->layers.size();
  s.h = (int)c.hidden_size;
  s.nh = (int)c.num_attention_heads;
  s.nkv = (int)c.num_key_value_heads;
  s.hd = (int)c.head_dim;
  s.inter = (int)c.intermediate_size;
  s.vocab = (int)c.vocab_size;
  s.eps = c.rms_norm_eps;
  s.attn_scale = 1.0f / sqrtf((float)c.head_dim);
  s.kv_bf16 = m->opt.kv_dtype == LRS_KV_BF16;
  int cols[3] = {0, 0, 0};
  auto mat = [&](const DevTensor& t, const DevTensor* t2, const float* bias, float* out, int epi,
                 S1Mat* o) -> bool {
    *o = S1Mat{};
    o->w = t.d;
    o->w2 = t2 ? t2->d : nullptr;
    o->bias = bias;
    o->out = out;
    o->type = (int)t.type;
    o->rows = t.rows;
    o->cols = t.cols;
    o->epi = epi;
    if (!s1_plan_mat(o, t2 ? 2 : 1, G)) return false;
    int& w = cols[s1_xclass(o->type)];
    w = std::max(w, o->cols);
    return true;
  };
  std::vector<S1Layer> layers(s.L);
  for (int l = 0; l < s.L; l++) {
    const Layer& L = m->layers[l];
    S1Layer& y = layers[l];
    bool ok = mat(L.q, nullptr, L.qb, m->q, EPI_STORE, &y.qkv[0]) &&
              mat(L.k, nullptr, L.kb, m->k, EPI_STORE, &y.qkv[1]) &&
              mat(L.v, nullptr, L.vb, m->v, EPI_STORE, &y.qkv[2]) &&
              mat(L.o, nullptr, nullptr, m->residual, EPI_ADD, &y.o) &&
              mat(L.down, nullptr, nullptr, m->residual, EPI_ADD, &y.down);
    if (L.gate.type == L.up.type) {
      y.ngu = 1;
      ok = ok && mat(L.gate, &L.up, nullptr, m->act, EPI_SWIGLU, &y.gu[0]);
    } else {
      y.ngu = 2;
      ok = ok && mat(L.gate, nullptr, nullptr, m->act, EPI_STORE, &y.gu[0]) &&
           mat(L.up, nullptr, nullptr, m->act2, EPI_STORE, &y.gu[1]);
    }
    if (!ok || L.o.cols != (int)(c.num_attention_heads * c.head_dim)) return LRS_OK;
    y.in_norm = L.in_norm;
    y.post_norm = L.post_norm;
    y.kpool = L.kpool;
    y.vpool = L.vpool;
  }
  if (!mat(m->lm, nullptr, nullptr, nullptr, EPI_ARGMAX, &s.lm)) return LRS_OK;
  s.embed = m->embed.d;
  s.embed_type = (int)m->embed.type;
  s.final_norm = m->final_norm;
  s.rope_cos = m->rope_cos;
  s.rope_sin = m->rope_sin;
  s.residual = m->residual;
  s.q = m->q;
  s.k = m->k;
  s.v = m->v;
  s.att = m->att;
  s.act = m->act;
  s.act2 = m->act2;
  s.part = m->part;
  s.max_split = std::max(1, std::min(G / s.nkv, m->max_split * (s.nh / s.nkv)));
  s.split_cap = std::max(64, (int)((m->opt.max_seq_len + s.max_split - 1) / s.max_split));
  const int work = std::max(s.h, kS1MaxGroup * s.hd + kS1MaxGroup * s.split_cap + 2 * s.hd + 2 * kS1MaxGroup);
  if (!s1_plan_smem(&s.sm, cols[0], cols[1], cols[2], work)) return LRS_OK;
  if (s1_occupancy(s.sm.total) < 1) return LRS_OK;
  int32_t rc;
  unsigned* sync = nullptr;
  S1Layer* d_layers = nullptr;
  if ((rc = model_alloc(m, (void**)&sync, (1 + (size_t)s.nkv) * 4)) ||
      (rc = model_alloc(m, (void**)&d_layers, layers.size() * sizeof(S1Layer))) ||
      (rc = model_alloc(m, (void**)&m->d_s1, sizeof(S1Model))))
    return rc;
  LRS_CUDA(cudaMemset(sync, 0, (1 + (size_t)s.nkv) * 4));
  LRS_CUDA(cudaMemcpy(d_layers, layers.data(), layers.size() * sizeof(S1Layer), cudaMemcpyHostToDevice));
  s.layers = d_layers;
  s.bar_ctr = sync;
  s.attn_cnt = sync + 1;
  s.keys = m->keys;
  s.tok = m->d_tok;
  s.pos = m->d_pos;
  s.seq = m->d_seq;
  s.pages = m->d_pages;
  s.max_pages = m->pages_per_seq;
  s.step = m->d_step;
  s.last = m->d_last;
  s.error_flag = m->be->d_err;
  s.tokens_out = nullptr;
  s.n_steps_cap = 0;
  LRS_CUDA(cudaMemcpy(m->d_s1, &s, sizeof(S1Model), cudaMemcpyHostToDevice));
  m->s1_tokens = nullptr;
  m->s1_cap = 0;
  m->s1_ok = true;
  return LRS_OK;
}

// Queues one greedy decode step of item 0 through the step kernel (the
// device copy of the model table must name the current token buffer).
int32_t enqueue_step1(lrs_model* m) {
  LRS_CUDA(s1_launch_step(m->s1, m->d_s1, m->be->sms, m->be->stream));
  return LRS_OK;
}

int32_t set_items(lrs_model* m, int n, const int* tok, const int* pos, const int* seq) {
  cudaStream_t st = m->be->stream;
  LRS_CUDA(cudaMemcpyAsync(m->d_tok, tok, n * sizeof(int), cudaMemcpyHostToDevice, st));
  LRS_CUDA(cudaMemcpyAsync(m->d_pos, pos, n * sizeof(int), cudaMemcpyHostToDevice, st));
  LRS_CUDA(cudaMemcpyAsync(m->d_seq, seq, n * sizeof(int), cudaMemcpyHostToDevice, st));
  // the host arrays may go out of scope: make the copies complete
  LRS_CUDA(cudaStreamSynchronize(st));
  return LRS_OK;
}

int32_t read_argmax(lrs_model* m, int item, uint32_t* out) {
  unsigned long long key = 0;
  LRS_CUDA(cudaMemcpy(&key, m->keys + item, sizeof(key), cudaMemcpyDeviceToHost));
  *out = (uint32_t)(key & 0xffffffffull);
  return LRS_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Row window [r0, r0 + n) of a tensor (rows are contiguous: no copy).
lrs_tensor_desc rows_of(const lrs_tensor_desc& d, size_t r0, size_t n) {
  lrs_tensor_desc o = d;
  const size_t rb = d.rows ? d.nbytes / d.rows : 0;
  o.data = static_cast<const uint8_t*>(d.data) + r0 * rb;
  o.rows = n;
  o.nbytes = n * rb;
  return o;
}

// Column window [c0, c0 + n) of a tensor, copied into `buf` as the whole
// blocks that cover it: columns [c0 - *lo, c0 - *lo + out->cols).  The
// blocks' values outside the window meet zeros in x, so the shard's dot
// equals the window's (blocks are never re-encoded: the bytes stay the
// reference's).
int32_t cols_of(const lrs_tensor_desc& d, size_t c0, size_t n, const char* what,
                std::vector<uint8_t>* buf, lrs_tensor_desc* out, int* lo) {
  uint32_t bv = 0, bb = 0;
  if (!type_geometry(d.ggml_type, &bv, &bb))
    return fail(LRS_ERR_UNSUPPORTED, std::string("unknown ggml type of ") + what);
  const size_t a0 = c0 / bv * bv, a1 = (c0 + n + bv - 1) / bv * bv;
  *lo = (int)(c0 - a0);
  n = a1 - a0;
  const size_t rb = d.rows ? d.nbytes / d.rows : 0, off = a0 / bv * bb, len = n / bv * bb;
  buf->resize(d.rows * len);
  for (size_t r = 0; r < d.rows; r++)
    memcpy(buf->data() + r * len, static_cast<const uint8_t*>(d.data) + r * rb + off, len);
  *out = d;
  out->data = buf->data();
  out->cols = n;
  out->nbytes = buf->size();
  return LRS_OK;
}

// maybe_quantize on the device (src/loader.rs:406-447): a float matrix of the
// description (full shape) is uploaded, widened to f32 and encoded with the
// recipe's type for `name` (lrs_quantize_matrix_device: the host encoders'
// bytes); then rows [r0, r0 + nr) and the whole blocks covering columns
// [c0, c0 + nc) (*lo as in cols_of) become `out`.  Encoding the full matrix
// first keeps the reference's per-matrix choices (fallbacks on cols) and bytes
// under tensor parallelism.  *done = false for other types (host path).
int32_t device_encode_mat(lrs_model* m, uint32_t recipe, const lrs_tensor_desc& d,
                          const std::string& name, size_t r0, size_t nr, size_t c0, size_t nc,
                          DevTensor* out, int* lo, bool* done) {
  *done = false;
  const uint32_t t = d.ggml_type;
  if (recipe == LRS_RECIPE_NONE || (t != LRS_GGML_F32 && t != LRS_GGML_F16 && t != LRS_GGML_BF16))
    return LRS_OK;
  const size_t R = d.rows, C = d.cols, n = R * C;
  cudaStream_t st = m->be->stream;
  uint8_t* raw = nullptr;
  float* f32 = nullptr;
  uint8_t* enc = nullptr;
  auto release = [&]() {
    cudaFree(raw);
    if ((void*)f32 != (void*)raw) cudaFree(f32);
    cudaFree(enc);
  };
  if (cudaMalloc(&raw, d.nbytes) != cudaSuccess) return fail(LRS_ERR_OOM, "upload of " + name);
  // on the stream the encoder runs on: a cudaMemcpy from pageable memory may
  // return before its DMA lands, and the backend's stream does not wait for it
  if (cudaMemcpyAsync(raw, d.data, d.nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    release();
    return fail(LRS_ERR_CUDA, "upload copy of " + name + " failed");
  }
  if (t == LRS_GGML_F32) {
    f32 = reinterpret_cast<float*>(raw);
  } else if (cudaMalloc(&f32, n * 4) != cudaSuccess || launch_widen(raw, t, n, f32, st) != cudaSuccess) {
    release();
    return fail(LRS_ERR_OOM, "widening " + name);
  }
  const uint32_t qt = lrs_recipe_type(recipe, name.c_str(), R, C);
  const size_t cap = lrs_quantized_size(qt, R, C);
  if (cudaMalloc(&enc, cap + 256) != cudaSuccess) {
    release();
    return fail(LRS_ERR_OOM, "encoded buffer of " + name);
  }
  uint32_t made;
  size_t len;
  int32_t rc = lrs_quantize_matrix_device(m->be, qt, f32, R, C, enc, cap, &made, &len);
  if (rc) {
    release();
    return rc;
  }
  uint32_t bv, bb;
  type_geometry(made, &bv, &bb);
  const size_t rb = len / R, a0 = c0 / bv * bv, a1 = (c0 + nc + bv - 1) / bv * bv;
  const size_t off = a0 / bv * bb, w = (a1 - a0) / bv * bb;
  *lo = (int)(c0 - a0);
  uint8_t* dst = nullptr;
  if (r0 == 0 && nr == R && a0 == 0 && a1 == C) {  // the whole matrix: keep the buffer
    dst = enc;
    enc = nullptr;
    cudaMemsetAsync(dst + len, 0, 256, st);
  } else {
    if (cudaMalloc(&dst, nr * w + 256) != cudaSuccess) {
      release();
      return fail(LRS_ERR_OOM, "shard of " + name);
    }
    cudaMemsetAsync(dst + nr * w, 0, 256, st);
    if (cudaMemcpy2DAsync(dst, w, enc + r0 * rb + off, rb, w, nr, cudaMemcpyDeviceToDevice, st) !=
        cudaSuccess) {
      cudaFree(dst);
      release();
      return fail(LRS_ERR_CUDA, "shard copy of " + name);
    }
  }
  cudaStreamSynchronize(st);
  release();
  out->d = dst;
  out->nbytes = nr * w;
  out->rows = (int)nr;
  out->cols = (int)(a1 - a0);
  out->type = made;
  *done = true;
  return LRS_OK;
}

int32_t check_shape(const lrs_tensor_desc& d, size_t rows, size_t cols, const char* what) {
  if (d.rows != rows || d.cols != cols)
    return fail(LRS_ERR_INVALID, std::string("tensor ") + what + " has shape [" +
                                     std::to_string(d.rows) + ", " + std::to_string(d.cols) +
                                     "], expected [" + std::to_string(rows) + ", " +
                                     std::to_string(cols) + "]");
  return validate_tensor(d.nbytes, d.rows, d.cols, d.ggml_type);
}

int32_t create_model(lrs_backend* be, const lrs_model_desc* d, const lrs_model_options* options,
                     int rank, int world, ncclComm_t comm, lrs_model** out) {
  if (!be || !d || !out) return fail(LRS_ERR_INVALID, "null argument");
  const lrs_config& c = d->config;
  // LlamaConfig::validate, src/config.rs:57-89
  if (!c.hidden_size || !c.intermediate_size || !c.num_attention_heads ||
      !c.num_key_value_heads || !c.num_hidden_layers || !c.vocab_size || !c.head_dim)
    return fail(LRS_ERR_INVALID, "invalid Qwen2 config: dimensions must be non-zero");
  if (c.num_attention_heads % c.num_key_value_heads)
    return fail(LRS_ERR_INVALID, "num_attention_heads must be divisible by num_key_value_heads");
  if (c.num_attention_heads * c.head_dim != c.hidden_size)
    return fail(LRS_ERR_INVALID, "num_attention_heads * head_dim must equal hidden_size");
  if (c.head_dim % 2) return fail(LRS_ERR_INVALID, "Qwen2 RoPE requires an even head_dim");
  if (!(c.rms_norm_eps > 0.0f) || !std::isfinite(c.rms_norm_eps))
    return fail(LRS_ERR_INVALID, "rms_norm_eps must be finite and positive");
  if (!(c.rope_theta > 0.0f) || !std::isfinite(c.rope_theta))
    return fail(LRS_ERR_INVALID, "rope_theta must be finite and positive");
  if (c.head_dim != 64 && c.head_dim != 128)
    return fail(LRS_ERR_UNSUPPORTED, "the CUDA attention kernel supports head_dim 64 or 128");
  if (c.num_attention_heads / c.num_key_value_heads > 8)
    return fail(LRS_ERR_UNSUPPORTED, "the CUDA attention kernel supports up to 8 query heads per KV head");
  lrs_model_options opt{};
  opt.max_seq_len = 4096;
  opt.max_sequences = 1;
  opt.kv_dtype = LRS_KV_F32;
  opt.use_graph = 1;
  if (options) opt = *options;
  if (opt.max_seq_len == 0 || opt.max_seq_len > c.max_position_embeddings)
    return fail(LRS_ERR_INVALID, "requested context " + std::to_string(opt.max_seq_len) +
                                     " exceeds model limit " +
                                     std::to_string(c.max_position_embeddings));
  if (opt.max_sequences == 0) opt.max_sequences = 1;
  if (opt.device_recipe > LRS_RECIPE_Q4KM) return fail(LRS_ERR_INVALID, "unknown device recipe");
  LRS_CUDA(cudaSetDevice(be->device));

  // Tensor parallelism (world > 1): heads, the MLP width and the LM-head rows
  // are split evenly; q/k/v/gate/up/lm_head by rows, o/down by columns.
  if (world > 1 && (c.num_key_value_heads % world || c.intermediate_size % world ||
                    c.vocab_size % world))
    return fail(LRS_ERR_UNSUPPORTED, "tensor-parallel degree " + std::to_string(world) +
                                         " does not divide the KV heads, the MLP width and the vocabulary");
  lrs_config cl = c;
  cl.num_attention_heads /= world;
  cl.num_key_value_heads /= world;
  cl.intermediate_size /= world;
  cl.vocab_size /= world;

  auto m = std::make_unique<lrs_model>();
  m->be = be;
  m->c = cl;
  m->opt = opt;
  m->tp_rank = rank;
  m->tp_world = world;
  m->comm = comm;
  m->vocab_full = c.vocab_size;
  m->vocab0 = rank * (int)cl.vocab_size;
  const size_t h = c.hidden_size, I = cl.intermediate_size, kvw = (size_t)cl.num_key_value_heads * c.head_dim,
               qw = (size_t)cl.num_attention_heads * c.head_dim, V = cl.vocab_size;
  const size_t kvw_full = (size_t)c.num_key_value_heads * c.head_dim;
  int32_t rc;
  auto cleanup = [&](int32_t code) {
    if (m->comm == comm) m->comm = nullptr;  // the caller owns a communicator it passed in
    lrs_model_destroy(m.release());
    return code;
  };
  // a matrix: encoded on the device when opt.device_recipe asks for it (float
  // types), else uploaded as given; rows [r0, r0 + nr), columns [c0, c0 + nc)
  // of the full tensor (column windows: whole blocks, *lo as cols_of)
  const uint32_t drec = opt.device_recipe;
  std::vector<uint8_t> colbuf;
  auto load_mat = [&](const lrs_tensor_desc& full, const std::string& name, size_t r0, size_t nr,
                      size_t c0, size_t nc, DevTensor* dt, int* lo) -> int32_t {
    bool done = false;
    int32_t r2 = device_encode_mat(m.get(), drec, full, name, r0, nr, c0, nc, dt, lo, &done);
    if (r2 || done) return r2;
    *lo = 0;
    lrs_tensor_desc part = rows_of(full, r0, nr);
    if (c0 != 0 || nc != full.cols) {
      if ((r2 = cols_of(part, c0, nc, name.c_str(), &colbuf, &part, lo))) return r2;
    }
    return upload_mat(part, nr, part.cols, name.c_str(), dt);
  };
  int lo_unused = 0;
  if ((rc = check_shape(d->embed_tokens, c.vocab_size, h, "model.embed_tokens.weight")) ||
      (rc = load_mat(d->embed_tokens, "model.embed_tokens.weight", 0, c.vocab_size, 0, h,
                     &m->embed, &lo_unused)))
    return cleanup(rc);
  const bool head_is_embed = d->lm_head.data == d->embed_tokens.data;
  if (head_is_embed && world == 1) {
    m->tied = true;
    m->lm = m->embed;
  } else if ((rc = check_shape(d->lm_head, c.vocab_size, h, "lm_head.weight")) ||
             (rc = load_mat(d->lm_head, head_is_embed ? "model.embed_tokens.weight" : "lm_head.weight",
                            m->vocab0, V, 0, h, &m->lm, &lo_unused))) {
    return cleanup(rc);
  }
  if ((rc = upload_vec(m.get(), d->final_norm, h, &m->final_norm))) return cleanup(rc);
  if (!m->final_norm) return cleanup(fail(LRS_ERR_INVALID, "missing model.norm.weight"));
  m->weight_bytes = m->lm.nbytes + m->embed.nbytes / c.vocab_size;
  m->layers.resize(c.num_hidden_layers);
  for (uint32_t i = 0; i < c.num_hidden_layers; i++) {
    const lrs_layer_desc& s = d->layers[i];
    Layer& L = m->layers[i];
    if ((rc = check_shape(s.q_proj, h, h, "q_proj")) ||
        (rc = check_shape(s.k_proj, kvw_full, h, "k_proj")) ||
        (rc = check_shape(s.v_proj, kvw_full, h, "v_proj")) ||
        (rc = check_shape(s.o_proj, h, h, "o_proj")) ||
        (rc = check_shape(s.gate_proj, (size_t)c.intermediate_size, h, "gate_proj")) ||
        (rc = check_shape(s.up_proj, (size_t)c.intermediate_size, h, "up_proj")) ||
        (rc = check_shape(s.down_proj, h, (size_t)c.intermediate_size, "down_proj")))
      return cleanup(rc);
    const std::string pre = "model.layers." + std::to_string(i);
    if ((rc = load_mat(s.q_proj, pre + ".self_attn.q_proj.weight", rank * qw, qw, 0, h, &L.q, &lo_unused)) ||
        (rc = load_mat(s.k_proj, pre + ".self_attn.k_proj.weight", rank * kvw, kvw, 0, h, &L.k, &lo_unused)) ||
        (rc = load_mat(s.v_proj, pre + ".self_attn.v_proj.weight", rank * kvw, kvw, 0, h, &L.v, &lo_unused)) ||
        (rc = load_mat(s.o_proj, pre + ".self_attn.o_proj.weight", 0, h, rank * qw, qw, &L.o, &L.o_lo)) ||
        (rc = load_mat(s.gate_proj, pre + ".mlp.gate_proj.weight", rank * I, I, 0, h, &L.gate, &lo_unused)) ||
        (rc = load_mat(s.up_proj, pre + ".mlp.up_proj.weight", rank * I, I, 0, h, &L.up, &lo_unused)) ||
        (rc = load_mat(s.down_proj, pre + ".mlp.down_proj.weight", 0, h, rank * I, I, &L.down, &L.d_lo)))
      return cleanup(rc);
    if ((rc = upload_vec(m.get(), s.input_layernorm, h, &L.in_norm)) ||
        (rc = upload_vec(m.get(), s.post_attention_layernorm, h, &L.post_norm)) ||
        (rc = upload_vec(m.get(), s.q_bias ? s.q_bias + rank * qw : nullptr, qw, &L.qb)) ||
        (rc = upload_vec(m.get(), s.k_bias ? s.k_bias + rank * kvw : nullptr, kvw, &L.kb)) ||
        (rc = upload_vec(m.get(), s.v_bias ? s.v_bias + rank * kvw : nullptr, kvw, &L.vb)))
      return cleanup(rc);
    if (!L.in_norm || !L.post_norm) return cleanup(fail(LRS_ERR_INVALID, "missing layer norm weight"));
    m->weight_bytes += L.q.nbytes + L.k.nbytes + L.v.nbytes + L.o.nbytes + L.gate.nbytes +
                       L.up.nbytes + L.down.nbytes;
  }
  // RoPE table: prepare_rope (src/model.rs:76-84) for every position, on the
  // host with the same libm calls, so device and reference agree bit for bit.
  {
    const size_t half = c.head_dim / 2;
    std::vector<float> cs(opt.max_seq_len * half), sn(opt.max_seq_len * half);
    for (size_t pos = 0; pos < opt.max_seq_len; pos++)
      for (size_t i = 0; i < half; i++) {
        float inv_freq = 1.0f / powf(c.rope_theta, 2.0f * (float)i / (float)c.head_dim);
        float angle = (float)pos * inv_freq;
        sn[pos * half + i] = sinf(angle);
        cs[pos * half + i] = cosf(angle);
      }
    if ((rc = upload_vec(m.get(), cs.data(), cs.size(), &m->rope_cos)) ||
        (rc = upload_vec(m.get(), sn.data(), sn.size(), &m->rope_sin)))
      return cleanup(rc);
  }
  // Paged KV pools.
  m->kv_elem = opt.kv_dtype == LRS_KV_BF16 ? 2 : 4;
  m->pages_per_seq = (int)((opt.max_seq_len + kPageSize - 1) / kPageSize);
  m->total_pages = m->pages_per_seq * (int)opt.max_sequences;
  const size_t page_elems = (size_t)cl.num_key_value_heads * kPageSize * c.head_dim;
  for (auto& L : m->layers) {
    if ((rc = model_alloc(m.get(), &L.kpool, (size_t)m->total_pages * page_elems * m->kv_elem)) ||
        (rc = model_alloc(m.get(), &L.vpool, (size_t)m->total_pages * page_elems * m->kv_elem)))
      return cleanup(rc);
  }
  for (int pg = m->total_pages - 1; pg >= 0; pg--) m->free_pages.push_back(pg);
  m->seq_pages.resize(opt.max_sequences);
  if ((rc = model_alloc(m.get(), (void**)&m->d_pages,
                        (size_t)m->total_pages * sizeof(int))))
    return cleanup(rc);
  LRS_CUDA(cudaMemset(m->d_pages, 0, (size_t)m->total_pages * sizeof(int)));
  // Activations (InferenceBuffers, src/cache.rs:79-101) for up to max_items items.
  m->max_items = std::max<int>(64, (int)opt.max_sequences);
  const size_t B = m->max_items;
  if ((rc = model_alloc(m.get(), (void**)&m->residual, B * h * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->xn, B * h * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->q, B * h * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->k, B * kvw * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->v, B * kvw * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->att, B * h * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->act, B * I * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->logits, (size_t)c.vocab_size * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->part,
                        B * c.num_attention_heads * m->max_split * (c.head_dim + 2) * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->keys, B * 8)) ||
      (rc = model_alloc(m.get(), (void**)&m->d_tok, B * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->d_pos, B * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->d_seq, B * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->d_step, 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->d_last, B * 4)) ||
      (rc = model_alloc(m.get(), (void**)&m->d_attn_cnt, B * c.num_key_value_heads * 4)))
    return cleanup(rc);
  LRS_CUDA(cudaMemset(m->d_attn_cnt, 0, B * c.num_key_value_heads * 4));
  LRS_CUDA(cudaStreamCreateWithFlags(&m->side, cudaStreamNonBlocking));
  LRS_CUDA(cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming));
  LRS_CUDA(cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming));
  {
    size_t ow = 0, dw = 0;
    for (const auto& L : m->layers) {
      if (L.o.cols != (int)(cl.num_attention_heads * c.head_dim)) ow = std::max(ow, (size_t)L.o.cols);
      if (L.down.cols != (int)cl.intermediate_size) dw = std::max(dw, (size_t)L.down.cols);
    }
    if ((ow && (rc = model_alloc(m.get(), (void**)&m->att_pad, B * ow * 4))) ||
        (dw && (rc = model_alloc(m.get(), (void**)&m->act_pad, B * dw * 4))))
      return cleanup(rc);
  }
  for (const auto& L : m->layers)
    if (L.gate.type != L.up.type && !m->act2 &&
        (rc = model_alloc(m.get(), (void**)&m->act2, B * I * 4)))
      return cleanup(rc);
  m->gemm_scratch_bytes = gemm_scratch_bytes((int)B, std::max(h, I), m->be->sms);
  {
    // the tcgen05 path keeps all K-group partials of a launch: size for the
    // largest one at 64 items (q/k/v, o, gate+up, down, LM head)
    const Layer& L0 = m->layers[0];
    GemvMat mats[][3] = {{mat_of(L0.q, nullptr, 1), mat_of(L0.k, nullptr, 1), mat_of(L0.v, nullptr, 1)},
                         {mat_of(L0.o, nullptr, 1)},
                         {mat_of(L0.gate, nullptr, 1, nullptr, &L0.up)},
                         {mat_of(L0.down, nullptr, 1)},
                         {mat_of(m->lm, nullptr, 1)}};
    const int nm[] = {3, 1, 1, 1, 1}, epis[] = {EPI_STORE, EPI_ADD, EPI_SWIGLU, EPI_ADD, EPI_ARGMAX};
    for (int i = 0; i < 5; i++) {
      GemvParams p;
      if (gemv_plan(&p, mats[i], nm[i], epis[i], (int)std::min<size_t>(B, 64)) == LRS_OK)
        m->gemm_scratch_bytes = std::max(m->gemm_scratch_bytes, gemm_tc_scratch_bytes(p, m->be->sms));
    }
  }
  if ((rc = model_alloc(m.get(), &m->gemm_scratch, m->gemm_scratch_bytes))) return cleanup(rc);
  if (world > 1 && opt.tp_allreduce == LRS_TP_ALLREDUCE_P2P && (rc = setup_tp_p2p(m.get(), h)))
    return cleanup(rc);
  if (world > 1 &&
      (rc = model_alloc(m.get(), (void**)&m->logits_full, (size_t)c.vocab_size * 4)))
    return cleanup(rc);
  if ((rc = setup_step1(m.get()))) return cleanup(rc);
  LRS_CUDA(cudaDeviceSynchronize());
  *out = m.release();
  return LRS_OK;
}

}  // namespace

extern "C" {

lrs_status lrs_model_create(lrs_backend* be, const lrs_model_desc* d,
                            const lrs_model_options* options, lrs_model** out) try {
  return create_model(be, d, options, 0, 1, nullptr, out);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_tp_unique_id(uint8_t* id_out) try {
  if (!id_out) return fail(LRS_ERR_INVALID, "null argument");
  const NcclApi& n = nccl();
  if (!n.ok) return fail(LRS_ERR_UNSUPPORTED, n.err);
  static_assert(sizeof(ncclUniqueId) == LRS_TP_ID_BYTES, "NCCL unique id size");
  ncclUniqueId id;
  LRS_NCCL(n.GetUniqueId(&id));
  memcpy(id_out, &id, sizeof id);
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_create_tp(lrs_backend* be, const lrs_model_desc* d,
                               const lrs_model_options* options, uint32_t rank, uint32_t world,
                               const uint8_t* id, lrs_model** out) try {
  if (!be || !d || !id || !out) return fail(LRS_ERR_INVALID, "null argument");
  if (world < 1 || rank >= world) return fail(LRS_ERR_INVALID, "tensor-parallel rank out of range");
  if (world == 1) return create_model(be, d, options, 0, 1, nullptr, out);
  const NcclApi& n = nccl();
  if (!n.ok) return fail(LRS_ERR_UNSUPPORTED, n.err);
  LRS_CUDA(cudaSetDevice(be->device));
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclComm_t comm = nullptr;
  LRS_NCCL(n.CommInitRank(&comm, (int)world, uid, (int)rank));
  int32_t rc = create_model(be, d, options, (int)rank, (int)world, comm, out);
  if (rc) n.CommDestroy(comm);
  return rc;
} catch (...) {
  return lrs::status_of_current_exception();
}

uint32_t lrs_model_tp_world(const lrs_model* m) { return m ? (uint32_t)m->tp_world : 0; }

void lrs_model_destroy(lrs_model* m) {
  if (!m) return;
  cudaSetDevice(m->be->device);
  cudaStreamSynchronize(m->be->stream);
  for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
  for (auto& L : m->layers) {
    cudaFree(L.q.d);
    cudaFree(L.k.d);
    cudaFree(L.v.d);
    cudaFree(L.o.d);
    cudaFree(L.gate.d);
    cudaFree(L.up.d);
    cudaFree(L.down.d);
  }
  if (m->tp_p2p && m->comm) {
    // Peers may still be reading this rank's exchange buffer in their last
    // all-reduce: one collective (which starts on every rank only after its
    // earlier kernels finished) before the buffers are unmapped and freed.
    const NcclApi& n = nccl();
    if (n.ok && n.AllReduce(m->tp_sig, m->tp_sig, 1, ncclInt32, ncclMax, m->comm, m->be->stream) ==
                    ncclSuccess)
      cudaStreamSynchronize(m->be->stream);
  }
  for (void* p : m->ipc_opened) cudaIpcCloseMemHandle(p);
  if (m->side) cudaStreamDestroy(m->side);
  if (m->ev_fork) cudaEventDestroy(m->ev_fork);
  if (m->ev_join) cudaEventDestroy(m->ev_join);
  cudaFree(m->embed.d);
  if (!m->tied) cudaFree(m->lm.d);
  for (void* p : m->allocs) cudaFree(p);
  cudaFree(m->d_tokens_out);
  if (m->comm) nccl().CommDestroy(m->comm);
  delete m;
}

uint64_t lrs_model_weight_bytes(const lrs_model* m) { return m ? m->weight_bytes : 0; }

lrs_status lrs_model_weights_digest(lrs_model* m, uint64_t* out) try {
  if (!m || !out) return fail(LRS_ERR_INVALID, "null argument");
  LRS_CUDA(cudaSetDevice(m->be->device));
  LRS_CUDA(cudaStreamSynchronize(m->be->stream));
  uint64_t h = 1469598103934665603ull;
  std::vector<uint8_t> buf;
  auto eat = [&](const DevTensor& t) -> int32_t {
    buf.resize(t.nbytes);
    if (t.nbytes) LRS_CUDA(cudaMemcpy(buf.data(), t.d, t.nbytes, cudaMemcpyDeviceToHost));
    for (uint8_t b : buf) h = (h ^ b) * 1099511628211ull;
    return LRS_OK;
  };
  int32_t rc;
  if ((rc = eat(m->embed))) return rc;
  for (const auto& L : m->layers)
    for (const DevTensor* t : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down})
      if ((rc = eat(*t))) return rc;
  if ((rc = eat(m->lm))) return rc;
  *out = h;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_reset(lrs_model* m, uint32_t seq) try {
  if (!m) return fail(LRS_ERR_INVALID, "null model");
  if (seq >= m->opt.max_sequences) return fail(LRS_ERR_INVALID, "sequence slot out of range");
  // KVCache::reset is a no-op in the reference (positions are overwritten
  // before they are read); here the slot's pages go back to the pool.
  for (int pg : m->seq_pages[seq]) m->free_pages.push_back(pg);
  m->seq_pages[seq].clear();
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_forward_token(lrs_model* m, uint32_t seq, uint32_t token, uint32_t pos,
                                   int logits_mode, float* logits_out, uint32_t* argmax_out) try {
  if (!m) return fail(LRS_ERR_INVALID, "null model");
  return lrs_model_prefill(m, seq, &token, 1, pos, logits_mode == LRS_LOGITS_COMPUTE ? logits_out : nullptr,
                           logits_mode == LRS_LOGITS_COMPUTE ? argmax_out : nullptr) ;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_prefill(lrs_model* m, uint32_t seq, const uint32_t* tokens, size_t n,
                             uint32_t start_pos, float* logits_out, uint32_t* argmax_out) try {
  if (!m || !tokens) return fail(LRS_ERR_INVALID, "null argument");
  if (n == 0) return fail(LRS_ERR_INVALID, "prefill requires at least one token");
  if (seq >= m->opt.max_sequences) return fail(LRS_ERR_INVALID, "sequence slot out of range");
  if ((size_t)start_pos + n > m->opt.max_seq_len)
    return fail(LRS_ERR_INVALID, "position " + std::to_string(start_pos + n - 1) +
                                     " exceeds configured context " + std::to_string(m->opt.max_seq_len));
  for (size_t i = 0; i < n; i++)
    if (tokens[i] >= m->vocab_full)
      return fail(LRS_ERR_INVALID, "token id " + std::to_string(tokens[i]) + " is outside vocabulary");
  LRS_CUDA(cudaSetDevice(m->be->device));
  int32_t rc = ensure_pages(m, (int)seq, start_pos + (uint32_t)n - 1);
  if (rc) return rc;
  const bool want = logits_out != nullptr || argmax_out != nullptr;
  const size_t chunk = 64;
  std::vector<int> tok(chunk), pos(chunk), sq(chunk, (int)seq);
  for (size_t c0 = 0; c0 < n; c0 += chunk) {
    const int nb = (int)std::min(chunk, n - c0);
    for (int i = 0; i < nb; i++) {
      tok[i] = (int)tokens[c0 + i];
      pos[i] = (int)(start_pos + c0 + i);
    }
    if ((rc = set_items(m, nb, tok.data(), pos.data(), sq.data()))) return rc;
    const bool last = c0 + nb == n;
    rc = enqueue_step(m, nb, last && want ? nb - 1 : -2, logits_out != nullptr, false, 0);
    if (rc) return rc;
  }
  if (logits_out)
    LRS_CUDA(cudaMemcpyAsync(logits_out, m->tp_world > 1 ? m->logits_full : m->logits,
                             (size_t)m->vocab_full * 4,
                             cudaMemcpyDeviceToHost, m->be->stream));
  LRS_CUDA(cudaStreamSynchronize(m->be->stream));
  if ((rc = check_device_error(m->be))) return rc;
  if (argmax_out) {
    int item = (int)((n - 1) % chunk);
    if ((rc = read_argmax(m, item, argmax_out))) return rc;
  }
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_forward_sample(lrs_model* m, uint32_t seq, uint32_t token, uint32_t pos,
                                    const lrs_sampler* params, const uint32_t* recent,
                                    size_t n_recent, float u, uint32_t* next_out) try {
  // InferenceEngine::forward_step, src/engine.rs:96-106: forward_token with
  // LogitsMode::Compute, then sample_current_logits on the device logits
  if (!m || !next_out || (n_recent && !recent)) return fail(LRS_ERR_INVALID, "null argument");
  int32_t rc = lrs_sampler_check(params, m->vocab_full);
  if (rc) return rc;
  if (!(u >= 0.0f && u < 1.0f)) return fail(LRS_ERR_INVALID, "u must be in [0, 1)");
  if (seq >= m->opt.max_sequences) return fail(LRS_ERR_INVALID, "sequence slot out of range");
  if ((size_t)pos + 1 > m->opt.max_seq_len)
    return fail(LRS_ERR_INVALID, "position " + std::to_string(pos) + " exceeds configured context " +
                                     std::to_string(m->opt.max_seq_len));
  if (token >= m->vocab_full)
    return fail(LRS_ERR_INVALID, "token id " + std::to_string(token) + " is outside vocabulary");
  LRS_CUDA(cudaSetDevice(m->be->device));
  if ((rc = ensure_pages(m, (int)seq, pos))) return rc;
  int t = (int)token, p = (int)pos, s = (int)seq;
  if ((rc = set_items(m, 1, &t, &p, &s))) return rc;
  if ((rc = enqueue_step(m, 1, 0, true, false, 0))) return rc;
  uint32_t *d_recent, *d_out;
  if ((rc = sample_buffers(m->be, recent, n_recent, &d_recent, &d_out))) return rc;
  LRS_CUDA(launch_sample(m->tp_world > 1 ? m->logits_full : m->logits, (int)m->vocab_full,
                         d_recent, (int)n_recent, *params, u, d_out, m->be->stream));
  LRS_CUDA(cudaMemcpyAsync(next_out, d_out, 4, cudaMemcpyDeviceToHost, m->be->stream));
  LRS_CUDA(cudaStreamSynchronize(m->be->stream));
  return check_device_error(m->be);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_decode_enqueue(lrs_model* m, size_t n_seqs, const uint32_t* seqs,
                                    const uint32_t* first_tokens, const uint32_t* start_pos,
                                    size_t n_steps) try {
  if (!m || !seqs || !first_tokens || !start_pos) return fail(LRS_ERR_INVALID, "null argument");
  if (n_seqs == 0 || n_seqs > (size_t)m->max_items)
    return fail(LRS_ERR_INVALID, "n_seqs out of range");
  if (n_steps == 0) return LRS_OK;
  LRS_CUDA(cudaSetDevice(m->be->device));
  const int B = (int)n_seqs;
  std::vector<int> tok(B), pos(B), sq(B);
  for (int i = 0; i < B; i++) {
    if (seqs[i] >= m->opt.max_sequences) return fail(LRS_ERR_INVALID, "sequence slot out of range");
    if (first_tokens[i] >= m->vocab_full) return fail(LRS_ERR_INVALID, "token id is outside vocabulary");
    if ((size_t)start_pos[i] + n_steps > m->opt.max_seq_len)
      return fail(LRS_ERR_INVALID, "decode steps exceed configured context");
    for (int j = 0; j < i; j++)
      if (seqs[j] == seqs[i]) return fail(LRS_ERR_INVALID, "duplicate sequence slot in batch");
    tok[i] = (int)first_tokens[i];
    pos[i] = (int)start_pos[i];
    sq[i] = (int)seqs[i];
    int32_t rc = ensure_pages(m, sq[i], start_pos[i] + (uint32_t)n_steps - 1);
    if (rc) return rc;
  }
  // tokens_out: [n_steps][B]; row s holds the token step s produced.
  size_t need = n_steps * (size_t)B;
  if (need > m->tokens_out_cap) {
    for (auto it = m->graphs.begin(); it != m->graphs.end();) {
      cudaGraphExecDestroy(it->second);
      it = m->graphs.erase(it);
    }
    cudaFree(m->d_tokens_out);
    m->d_tokens_out = nullptr;
    size_t cap = std::max(need, (size_t)4096);
    if (cudaMalloc(&m->d_tokens_out, cap * 4) != cudaSuccess)
      return fail(LRS_ERR_OOM, "token buffer allocation failed");
    m->tokens_out_cap = cap;
  }
  int32_t rc = set_items(m, B, tok.data(), pos.data(), sq.data());
  if (rc) return rc;
  cudaStream_t st = m->be->stream;
  LRS_CUDA(cudaMemsetAsync(m->d_step, 0, 4, st));
  const int cap_steps = (int)(m->tokens_out_cap / B);
  const bool step1 = B == 1 && m->s1_ok;
  if (step1 && (m->s1_tokens != m->d_tokens_out || m->s1_cap != cap_steps)) {
    m->s1.tokens_out = m->d_tokens_out;
    m->s1.n_steps_cap = cap_steps;
    LRS_CUDA(cudaMemcpyAsync(m->d_s1, &m->s1, sizeof(S1Model), cudaMemcpyHostToDevice, st));
    LRS_CUDA(cudaStreamSynchronize(st));
    m->s1_tokens = m->d_tokens_out;
    m->s1_cap = cap_steps;
  }
  if (m->opt.use_graph) {
    GraphKey key{B, m->d_tokens_out};
    auto it = m->graphs.find(key);
    cudaGraphExec_t exec = nullptr;
    if (it == m->graphs.end()) {
      cudaGraph_t graph;
      LRS_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      rc = step1 ? enqueue_step1(m) : enqueue_step(m, B, -1, false, true, cap_steps);
      cudaError_t e = cudaStreamEndCapture(st, &graph);
      if (rc) return rc;
      if (e != cudaSuccess) return fail(LRS_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
      size_t nn = 0;
      cudaGraphGetNodes(graph, nullptr, &nn);
      std::vector<cudaGraphNode_t> nodes(nn);
      uint32_t nk = 0;
      if (nn && cudaGraphGetNodes(graph, nodes.data(), &nn) == cudaSuccess)
        for (auto nd : nodes) {
          cudaGraphNodeType ty;
          if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) nk++;
        }
      m->graph_kernels[key] = nk;
      e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess)
        return fail(LRS_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
      m->graphs[key] = exec;
    } else {
      exec = it->second;
    }
    m->last_step_kernels = m->graph_kernels[key];
    for (size_t s = 0; s < n_steps; s++) LRS_CUDA(cudaGraphLaunch(exec, st));
  } else {
    for (size_t s = 0; s < n_steps; s++)
      if ((rc = step1 ? enqueue_step1(m) : enqueue_step(m, B, -1, false, true, cap_steps))) return rc;
  }
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

uint32_t lrs_model_step_kernels(const lrs_model* m) { return m ? m->last_step_kernels : 0; }

lrs_status lrs_model_read_tokens(lrs_model* m, size_t n_seqs, size_t n_steps, uint32_t* out) try {
  if (!m || !out) return fail(LRS_ERR_INVALID, "null argument");
  if (n_seqs * n_steps > m->tokens_out_cap) return fail(LRS_ERR_INVALID, "token range out of bounds");
  LRS_CUDA(cudaSetDevice(m->be->device));
  LRS_CUDA(cudaMemcpyAsync(out, m->d_tokens_out, n_seqs * n_steps * 4, cudaMemcpyDeviceToHost,
                           m->be->stream));
  LRS_CUDA(cudaStreamSynchronize(m->be->stream));
  return check_device_error(m->be);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_profile_step(lrs_model* m, size_t n_seqs, const uint32_t* seqs,
                                  const uint32_t* tokens, const uint32_t* pos, float* gemv_ms,
                                  uint32_t* gemv_launches, float* step_ms, float* attn_ms) try {
  if (!m || !seqs || !tokens || !pos) return fail(LRS_ERR_INVALID, "null argument");
  if (n_seqs == 0 || n_seqs > (size_t)m->max_items) return fail(LRS_ERR_INVALID, "n_seqs out of range");
  LRS_CUDA(cudaSetDevice(m->be->device));
  const int B = (int)n_seqs;
  std::vector<int> tok(B), ps(B), sq(B);
  for (int i = 0; i < B; i++) {
    if (seqs[i] >= m->opt.max_sequences || tokens[i] >= m->vocab_full ||
        pos[i] >= m->opt.max_seq_len)
      return fail(LRS_ERR_INVALID, "profile_step: item out of range");
    for (size_t j = 0; j < i; j++)
      if (seqs[j] == seqs[i]) return fail(LRS_ERR_INVALID, "duplicate sequence slot in batch");
    tok[i] = (int)tokens[i];
    ps[i] = (int)pos[i];
    sq[i] = (int)seqs[i];
    int32_t rc = ensure_pages(m, sq[i], pos[i]);
    if (rc) return rc;
  }
  int32_t rc = set_items(m, B, tok.data(), ps.data(), sq.data());
  if (rc) return rc;
  cudaStream_t st = m->be->stream;
  std::vector<cudaEvent_t> ev, aev;
  cudaEvent_t s0, s1;
  cudaEventCreate(&s0);
  cudaEventCreate(&s1);
  cudaEventRecord(s0, st);
  m->prof = &ev;
  m->prof_attn = &aev;
  rc = enqueue_step(m, B, -1, false, true, 0);
  m->prof = nullptr;
  m->prof_attn = nullptr;
  cudaEventRecord(s1, st);
  cudaError_t e = cudaStreamSynchronize(st);
  float total = 0.0f, step = 0.0f;
  for (size_t i = 0; i + 1 < ev.size(); i += 2) {
    float t = 0.0f;
    cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
    total += t;
  }
  cudaEventElapsedTime(&step, s0, s1);
  float atotal = 0.0f;
  for (size_t i = 0; i + 1 < aev.size(); i += 2) {
    float t = 0.0f;
    cudaEventElapsedTime(&t, aev[i], aev[i + 1]);
    atotal += t;
  }
  for (auto x : aev) cudaEventDestroy(x);
  if (attn_ms) *attn_ms = atotal;
  for (auto x : ev) cudaEventDestroy(x);
  cudaEventDestroy(s0);
  cudaEventDestroy(s1);
  if (rc) return rc;
  if (e != cudaSuccess) return fail(LRS_ERR_CUDA, cudaGetErrorString(e));
  if (gemv_ms) *gemv_ms = total;
  if (gemv_launches) *gemv_launches = (uint32_t)(ev.size() / 2);
  if (step_ms) *step_ms = step;
  return check_device_error(m->be);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_model_decode_greedy(lrs_model* m, size_t n_seqs, const uint32_t* seqs,
                                   const uint32_t* first_tokens, const uint32_t* start_pos,
                                   size_t n_steps, uint32_t* tokens_out) try {
  int32_t rc = lrs_model_decode_enqueue(m, n_seqs, seqs, first_tokens, start_pos, n_steps);
  if (rc) return rc;
  if (!tokens_out || n_steps == 0) return lrs_backend_synchronize(m->be);
  return lrs_model_read_tokens(m, n_seqs, n_steps, tokens_out);
} catch (...) {
  return lrs::status_of_current_exception();
}

}  // extern "C"

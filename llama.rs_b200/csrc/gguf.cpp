// gguf.cpp -- GGUF model files (host): the reader of src/gguf.rs and the
// Qwen2 loader of src/loader.rs:231-398, producing an lrs_model_desc whose
// pre-quantized tensors point into the memory-mapped file.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/llamars.h"
#include "../../include/llamars_gguf.h"
#include "../../include/llamars_synth.h"
#include "common.h"
#include "load_common.h"

namespace {

using lrs::fail;

// MetadataValue (src/gguf.rs:13-57): arrays keep only their length.
struct Meta {
  enum Kind { U64, I64, F64, BOOL, STR, ARR } kind = U64;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint32_t elem = 0;
  uint64_t len = 0;
  bool as_u64(uint64_t* out) const {
    if (kind == U64) return *out = u, true;
    if (kind == I64 && i >= 0) return *out = (uint64_t)i, true;
    return false;
  }
  bool as_f32(float* out) const {
    if (kind == F64) return *out = (float)f, true;
    if (kind == U64) return *out = (float)u, true;
    if (kind == I64) return *out = (float)i, true;
    return false;
  }
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // GGML order: dims[0] is the row width
  uint32_t type = 0;
  uint64_t offset = 0;
};

bool known_type(uint32_t t) {
  uint32_t bv, bb;
  return lrs::type_geometry(t, &bv, &bb);
}

std::string unsupported_type(uint32_t t) {
  return "unsupported GGML tensor type " + std::to_string(t) +
         "; supported: F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K";
}

// Reader (src/gguf.rs:238-330): little-endian fields with bounds checks.
struct Reader {
  const uint8_t* d;
  size_t n, pos = 0;
  int32_t err = LRS_OK;
  bool take(size_t len, const uint8_t** out) {
    if (pos > n || len > n - pos) {
      err = fail(LRS_ERR_INVALID, "truncated GGUF file at byte " + std::to_string(pos));
      return false;
    }
    *out = d + pos;
    pos += len;
    return true;
  }
  template <typename T>
  bool get(T* v) {
    const uint8_t* p;
    if (!take(sizeof(T), &p)) return false;
    memcpy(v, p, sizeof(T));
    return true;
  }
  bool str(std::string* s) {
    uint64_t len;
    if (!get(&len)) return false;
    if (len > (1ull << 30)) {
      err = fail(LRS_ERR_INVALID, "unreasonable GGUF string length " + std::to_string(len));
      return false;
    }
    const uint8_t* p;
    if (!take((size_t)len, &p)) return false;
    if (!lrs::valid_utf8(p, (size_t)len)) {
      err = fail(LRS_ERR_INVALID, "invalid UTF-8 in GGUF string");
      return false;
    }
    s->assign(reinterpret_cast<const char*>(p), (size_t)len);
    return true;
  }
  // metadata_value (src/gguf.rs:313-343)
  bool value(uint32_t ty, Meta* m) {
    switch (ty) {
      case 0: { uint8_t v; if (!get(&v)) return false; m->kind = Meta::U64; m->u = v; return true; }
      case 1: { int8_t v; if (!get(&v)) return false; m->kind = Meta::I64; m->i = v; return true; }
      case 2: { uint16_t v; if (!get(&v)) return false; m->kind = Meta::U64; m->u = v; return true; }
      case 3: { int16_t v; if (!get(&v)) return false; m->kind = Meta::I64; m->i = v; return true; }
      case 4: { uint32_t v; if (!get(&v)) return false; m->kind = Meta::U64; m->u = v; return true; }
      case 5: { int32_t v; if (!get(&v)) return false; m->kind = Meta::I64; m->i = v; return true; }
      case 6: { float v; if (!get(&v)) return false; m->kind = Meta::F64; m->f = v; return true; }
      case 7: { uint8_t v; if (!get(&v)) return false; m->kind = Meta::BOOL; m->u = v != 0; return true; }
      case 8: m->kind = Meta::STR; return str(&m->s);
      case 9: {
        uint32_t et;
        uint64_t len;
        if (!get(&et)) return false;
        if (et == 9) {
          err = fail(LRS_ERR_INVALID, "nested GGUF arrays are not supported by the format");
          return false;
        }
        if (!get(&len)) return false;
        if (len > 100000000ull) {
          err = fail(LRS_ERR_INVALID, "unreasonable GGUF array length " + std::to_string(len));
          return false;
        }
        Meta tmp;
        for (uint64_t k = 0; k < len; k++)
          if (!value(et, &tmp)) return false;
        m->kind = Meta::ARR;
        m->elem = et;
        m->len = len;
        return true;
      }
      case 10: { uint64_t v; if (!get(&v)) return false; m->kind = Meta::U64; m->u = v; return true; }
      case 11: { int64_t v; if (!get(&v)) return false; m->kind = Meta::I64; m->i = v; return true; }
      case 12: { double v; if (!get(&v)) return false; m->kind = Meta::F64; m->f = v; return true; }
    }
    err = fail(LRS_ERR_INVALID, "unknown GGUF metadata type " + std::to_string(ty));
    return false;
  }
};

// Exact f16 -> f32 (`half` crate semantics: every f16 value is exact in f32).
}  // namespace

struct lrs_gguf {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  std::map<std::string, Meta> meta;
  std::map<std::string, TensorInfo> tensors;
  size_t data_offset = 0;
  // owned by a built description
  lrs::Blobs blobs;
  std::vector<std::unique_ptr<std::vector<float>>> vecs;
  std::vector<lrs_layer_desc> layers;
  lrs_model_desc desc{};

  ~lrs_gguf() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
    if (fd >= 0) close(fd);
  }

  // tensor_range (src/gguf.rs:217-252)
  int32_t range(const TensorInfo& t, size_t* start, size_t* len) const {
    uint32_t bv, bb;
    if (!lrs::type_geometry(t.type, &bv, &bb))
      return fail(LRS_ERR_UNSUPPORTED, "tensor " + t.name + ": " + unsupported_type(t.type));
    uint64_t el = 1;
    for (uint64_t d : t.dims) {
      if (d != 0 && el > UINT64_MAX / d)
        return fail(LRS_ERR_INVALID, "tensor " + t.name + " element count overflow");
      el *= d;
    }
    if (el % bv)
      return fail(LRS_ERR_INVALID, "tensor " + t.name + " element count is incompatible with " +
                                       lrs::type_name(t.type));
    if (t.dims[0] % bv)
      return fail(LRS_ERR_INVALID, "tensor " + t.name + " row width " + std::to_string(t.dims[0]) +
                                       " is incompatible with " + lrs::type_name(t.type));
    const uint64_t l = el / bv * bb;
    if (t.offset > UINT64_MAX - data_offset)
      return fail(LRS_ERR_INVALID, "tensor " + t.name + " offset overflow");
    const uint64_t s = data_offset + t.offset;
    if (s > size || l > size - s)
      return fail(LRS_ERR_INVALID, "tensor " + t.name + " is outside the GGUF file");
    *start = (size_t)s;
    *len = (size_t)l;
    return LRS_OK;
  }
};

namespace {

int32_t parse(lrs_gguf* g, const char* path) {
  Reader r{g->map, g->size};
  const uint8_t* magic;
  if (!r.take(4, &magic)) return r.err;
  if (memcmp(magic, "GGUF", 4) != 0) return fail(LRS_ERR_INVALID, std::string(path) + " is not a GGUF file");
  if (!r.get(&g->version)) return r.err;
  if (g->version < 2 || g->version > 3)
    return fail(LRS_ERR_INVALID, "unsupported GGUF version " + std::to_string(g->version) +
                                     "; versions 2 and 3 are supported");
  uint64_t nt, nm;
  if (!r.get(&nt) || !r.get(&nm)) return r.err;
  if (nt > 1000000 || nm > 1000000) return fail(LRS_ERR_INVALID, "unreasonable GGUF header counts");
  for (uint64_t k = 0; k < nm; k++) {
    std::string key;
    uint32_t ty;
    Meta m;
    if (!r.str(&key) || !r.get(&ty) || !r.value(ty, &m)) return r.err;
    if (!g->meta.emplace(key, m).second)
      return fail(LRS_ERR_INVALID, "duplicate GGUF metadata key " + key);
  }
  for (uint64_t k = 0; k < nt; k++) {
    TensorInfo t;
    uint32_t nd;
    if (!r.str(&t.name) || !r.get(&nd)) return r.err;
    if (nd < 1 || nd > 4)
      return fail(LRS_ERR_INVALID, "tensor " + t.name + " has invalid dimension count " +
                                       std::to_string(nd));
    t.dims.resize(nd);
    for (auto& d : t.dims)
      if (!r.get(&d)) return r.err;
    if (!r.get(&t.type) || !r.get(&t.offset)) return r.err;
    const std::string name = t.name;
    if (!g->tensors.emplace(name, std::move(t)).second)
      return fail(LRS_ERR_INVALID, "duplicate GGUF tensor " + name);
  }
  uint64_t align = 32;
  auto it = g->meta.find("general.alignment");
  if (it != g->meta.end()) {
    uint64_t a;
    if (it->second.as_u64(&a)) align = a;
  }
  if (align == 0 || (align & (align - 1)) || align > (1u << 20))
    return fail(LRS_ERR_INVALID, "invalid GGUF alignment " + std::to_string(align));
  g->data_offset = (r.pos + (size_t)align - 1) & ~((size_t)align - 1);
  if (g->data_offset > g->size)
    return fail(LRS_ERR_INVALID, "GGUF tensor data offset is outside the file");
  // validate every range eagerly (src/gguf.rs:162-166)
  for (auto& kv : g->tensors) {
    size_t s, l;
    int32_t rc = g->range(kv.second, &s, &l);
    if (rc) return rc;
  }
  return LRS_OK;
}

// GgufFile::tensor (src/gguf.rs:196-215) as a desc: rows x cols (1-D: 1 x len).
int32_t tensor_desc(const lrs_gguf* g, const std::string& name, lrs_tensor_desc* out, bool* one_d) {
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return fail(LRS_ERR_INVALID, "missing GGUF tensor " + name);
  const TensorInfo& t = it->second;
  if (t.dims.size() > 2)
    return fail(LRS_ERR_INVALID, "tensor " + name + " has " + std::to_string(t.dims.size()) +
                                     " dimensions; Qwen2 loader supports 1D/2D weights");
  size_t s, l;
  int32_t rc = g->range(t, &s, &l);
  if (rc) return rc;
  memset(out, 0, sizeof(*out));
  out->data = g->map + s;
  out->nbytes = l;
  out->cols = t.dims[0];
  out->rows = t.dims.size() == 2 ? t.dims[1] : 1;
  out->ggml_type = t.type;
  if (one_d) *one_d = t.dims.size() == 1;
  return LRS_OK;
}

std::string shape_str(const lrs_tensor_desc& d, bool one_d) {
  return one_d ? "[" + std::to_string(d.cols) + "]"
               : "[" + std::to_string(d.rows) + ", " + std::to_string(d.cols) + "]";
}

}  // namespace

extern "C" {

lrs_status lrs_gguf_open(const char* path, lrs_gguf** out) try {
  if (!path || !out) return fail(LRS_ERR_INVALID, "null argument");
  auto g = std::make_unique<lrs_gguf>();
  g->fd = open(path, O_RDONLY);
  if (g->fd < 0) return fail(LRS_ERR_INVALID, std::string("failed to open ") + path);
  struct stat st;
  if (fstat(g->fd, &st) != 0) return fail(LRS_ERR_INVALID, std::string("failed to open ") + path);
  g->size = (size_t)st.st_size;
  if (g->size) {
    void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) return fail(LRS_ERR_INVALID, std::string("failed to map ") + path);
    g->map = static_cast<const uint8_t*>(m);
  }
  int32_t rc = parse(g.get(), path);
  if (rc) return rc;
  *out = g.release();
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

void lrs_gguf_close(lrs_gguf* g) { delete g; }
uint32_t lrs_gguf_version(const lrs_gguf* g) { return g ? g->version : 0; }
size_t lrs_gguf_tensor_count(const lrs_gguf* g) { return g ? g->tensors.size() : 0; }

lrs_status lrs_gguf_metadata_u64(const lrs_gguf* g, const char* key, uint64_t* out) try {
  if (!g || !key || !out) return fail(LRS_ERR_INVALID, "null argument");
  auto it = g->meta.find(key);
  if (it == g->meta.end() || !it->second.as_u64(out))
    return fail(LRS_ERR_INVALID, std::string("missing or non-integer GGUF metadata ") + key);
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_gguf_metadata_f32(const lrs_gguf* g, const char* key, float* out) try {
  if (!g || !key || !out) return fail(LRS_ERR_INVALID, "null argument");
  auto it = g->meta.find(key);
  if (it == g->meta.end() || !it->second.as_f32(out))
    return fail(LRS_ERR_INVALID, std::string("missing or non-numeric GGUF metadata ") + key);
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_gguf_metadata_str(const lrs_gguf* g, const char* key, const char** out) try {
  if (!g || !key || !out) return fail(LRS_ERR_INVALID, "null argument");
  auto it = g->meta.find(key);
  if (it == g->meta.end() || it->second.kind != Meta::STR)
    return fail(LRS_ERR_INVALID, std::string("missing or non-string GGUF metadata ") + key);
  *out = it->second.s.c_str();
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_gguf_tensor(const lrs_gguf* g, const char* name, lrs_tensor_desc* out) try {
  if (!g || !name || !out) return fail(LRS_ERR_INVALID, "null argument");
  return tensor_desc(g, name, out, nullptr);
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_gguf_qwen2_desc(lrs_gguf* g, uint32_t recipe, const lrs_model_desc** out) try {
  if (!g || !out) return fail(LRS_ERR_INVALID, "null argument");
  if (recipe > LRS_RECIPE_Q4KM) return fail(LRS_ERR_INVALID, "unknown load quantization");
  const char* arch;
  int32_t rc = lrs_gguf_metadata_str(g, "general.architecture", &arch);
  if (rc) return rc;
  if (std::string(arch) != "qwen2")
    return fail(LRS_ERR_UNSUPPORTED, std::string("unsupported GGUF architecture \"") + arch + "\"");
  auto tok = g->tensors.find("token_embd.weight");
  if (tok == g->tensors.end()) return fail(LRS_ERR_INVALID, "missing GGUF tensor token_embd.weight");
  if (tok->second.dims.size() != 2) return fail(LRS_ERR_INVALID, "token_embd.weight must be 2D");
  uint64_t hidden, inter, heads, kv, layers, ctx;
  float eps, theta = 10000.0f;
  if ((rc = lrs_gguf_metadata_u64(g, "qwen2.embedding_length", &hidden)) ||
      (rc = lrs_gguf_metadata_u64(g, "qwen2.feed_forward_length", &inter)) ||
      (rc = lrs_gguf_metadata_u64(g, "qwen2.attention.head_count", &heads)) ||
      (rc = lrs_gguf_metadata_u64(g, "qwen2.attention.head_count_kv", &kv)) ||
      (rc = lrs_gguf_metadata_u64(g, "qwen2.block_count", &layers)) ||
      (rc = lrs_gguf_metadata_f32(g, "qwen2.attention.layer_norm_rms_epsilon", &eps)) ||
      (rc = lrs_gguf_metadata_u64(g, "qwen2.context_length", &ctx)))
    return rc;
  auto th = g->meta.find("qwen2.rope.freq_base");
  if (th != g->meta.end()) {
    float v;
    if (th->second.as_f32(&v)) theta = v;
  }
  if (!heads || hidden % heads)
    return fail(LRS_ERR_INVALID, "hidden_size must be divisible by num_attention_heads");
  if (hidden > UINT32_MAX || inter > UINT32_MAX || heads > UINT32_MAX || kv > UINT32_MAX ||
      layers > UINT32_MAX || ctx > UINT32_MAX || tok->second.dims[1] > UINT32_MAX)
    return fail(LRS_ERR_INVALID, "GGUF model dimensions do not fit 32 bits");
  if (tok->second.dims[0] != hidden) return fail(LRS_ERR_INVALID, "GGUF embedding width/config mismatch");
  lrs_config c{};
  c.hidden_size = (uint32_t)hidden;
  c.intermediate_size = (uint32_t)inter;
  c.num_attention_heads = (uint32_t)heads;
  c.num_key_value_heads = (uint32_t)kv;
  c.num_hidden_layers = (uint32_t)layers;
  c.vocab_size = (uint32_t)tok->second.dims[1];
  c.head_dim = (uint32_t)(hidden / heads);
  c.max_position_embeddings = (uint32_t)ctx;
  c.rms_norm_eps = eps;
  c.rope_theta = theta;
  const size_t kvw = (size_t)kv * c.head_dim;

  g->blobs.clear();
  g->vecs.clear();
  // load_gguf_matrix + maybe_quantize (src/loader.rs:497-507, 406-447)
  auto matrix = [&](const std::string& name, size_t rows, size_t cols, lrs_tensor_desc* d) -> int32_t {
    bool one_d;
    int32_t r2 = tensor_desc(g, name, d, &one_d);
    if (r2) return r2;
    if (one_d || d->rows != rows || d->cols != cols)
      return fail(LRS_ERR_INVALID, "tensor " + name + " has shape " + shape_str(*d, one_d) +
                                       ", expected [" + std::to_string(rows) + ", " +
                                       std::to_string(cols) + "]");
    return lrs::maybe_quantize_desc(recipe, name, rows, cols, d, &g->blobs, "GGUF");
  };
  // load_gguf_vector (src/loader.rs:509-517)
  auto vector = [&](const std::string& name, size_t len, const float** outp) -> int32_t {
    lrs_tensor_desc d;
    bool one_d;
    int32_t r2 = tensor_desc(g, name, &d, &one_d);
    if (r2) return r2;
    if (!one_d || d.cols != len)
      return fail(LRS_ERR_INVALID, "tensor " + name + " has shape " + shape_str(d, one_d) +
                                       ", expected [" + std::to_string(len) + "]");
    auto v = std::make_unique<std::vector<float>>();
    if ((r2 = lrs::desc_to_f32(d, name, v.get(), "GGUF"))) return r2;
    *outp = v->data();
    g->vecs.push_back(std::move(v));
    return LRS_OK;
  };
  // optional bias: missing = zeros (src/loader.rs:528-532)
  auto bias = [&](const std::string& name, size_t len, const float** outp) -> int32_t {
    *outp = nullptr;
    if (!g->tensors.count(name)) return LRS_OK;
    return vector(name, len, outp);
  };

  lrs_model_desc& d = g->desc;
  memset(&d, 0, sizeof(d));
  d.config = c;
  if ((rc = matrix("token_embd.weight", c.vocab_size, hidden, &d.embed_tokens)) ||
      (rc = vector("output_norm.weight", hidden, &d.final_norm)))
    return rc;
  // one layer at a time: a corrupt block count fails at its first missing
  // tensor (the reference's error) instead of allocating for it up front
  g->layers.clear();
  for (uint64_t i = 0; i < layers; i++) {
    const std::string p = "blk." + std::to_string(i);
    g->layers.push_back(lrs_layer_desc{});
    lrs_layer_desc& L = g->layers.back();
    if ((rc = vector(p + ".attn_norm.weight", hidden, &L.input_layernorm)) ||
        (rc = matrix(p + ".attn_q.weight", hidden, hidden, &L.q_proj)) ||
        (rc = bias(p + ".attn_q.bias", hidden, &L.q_bias)) ||
        (rc = matrix(p + ".attn_k.weight", kvw, hidden, &L.k_proj)) ||
        (rc = bias(p + ".attn_k.bias", kvw, &L.k_bias)) ||
        (rc = matrix(p + ".attn_v.weight", kvw, hidden, &L.v_proj)) ||
        (rc = bias(p + ".attn_v.bias", kvw, &L.v_bias)) ||
        (rc = matrix(p + ".attn_output.weight", hidden, hidden, &L.o_proj)) ||
        (rc = vector(p + ".ffn_norm.weight", hidden, &L.post_attention_layernorm)) ||
        (rc = matrix(p + ".ffn_gate.weight", inter, hidden, &L.gate_proj)) ||
        (rc = matrix(p + ".ffn_up.weight", inter, hidden, &L.up_proj)) ||
        (rc = matrix(p + ".ffn_down.weight", hidden, inter, &L.down_proj)))
      return rc;
  }
  // output.weight present: its own head; absent: the embedding (tied)
  if (g->tensors.count("output.weight")) {
    if ((rc = matrix("output.weight", c.vocab_size, hidden, &d.lm_head))) return rc;
  } else {
    d.lm_head = d.embed_tokens;
  }
  d.layers = g->layers.data();
  *out = &d;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

}  // extern "C"

// safetensors.cpp -- SafeTensors checkpoints and ModelLoader::load's format
// dispatch (host).  See include/llamars_safetensors.h.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/llamars.h"
#include "../../include/llamars_gguf.h"
#include "../../include/llamars_safetensors.h"
#include "../../include/llamars_synth.h"
#include "common.h"
#include "json.h"
#include "load_common.h"

using lrs::fail;
using lrs::JValue;

namespace {

constexpr uint64_t kMaxHeader = 100000000;  // the crate's MAX_HEADER_SIZE

struct Mapped {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  ~Mapped() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
    if (fd >= 0) close(fd);
  }
};

struct StTensor {
  std::string dtype;
  std::vector<uint64_t> shape;
  size_t start = 0, len = 0;  // absolute byte range in the file
  int file = -1;
};

bool is_file(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}
bool is_dir(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}
std::string join(const std::string& dir, const std::string& name) {
  return dir.empty() || dir.back() == '/' ? dir + name : dir + "/" + name;
}
bool ends_with(const std::string& s, const std::string& suffix) {
  return s.size() >= suffix.size() && s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0;
}
// Files of `dir` whose names end with `ext`, sorted.
std::vector<std::string> list_ext(const std::string& dir, const std::string& ext) {
  std::vector<std::string> out;
  DIR* d = opendir(dir.c_str());
  if (!d) return out;
  while (dirent* e = readdir(d)) {
    const std::string n = e->d_name;
    if (n.size() > ext.size() && ends_with(n, ext) && is_file(join(dir, n))) out.push_back(join(dir, n));
  }
  closedir(d);
  std::sort(out.begin(), out.end());
  return out;
}
bool read_text(const std::string& path, std::string* out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[65536];
  size_t n;
  out->clear();
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
  const bool ok = !ferror(f);
  fclose(f);
  return ok;
}

// Element size of a safetensors dtype; 0 for an unknown name.
size_t dtype_size(const std::string& t) {
  static const std::map<std::string, size_t> sizes = {
      {"BOOL", 1}, {"U8", 1},  {"I8", 1},  {"F8_E5M2", 1}, {"F8_E4M3", 1},
      {"I16", 2},  {"U16", 2}, {"F16", 2}, {"BF16", 2},    {"I32", 4},
      {"U32", 4},  {"F32", 4}, {"F64", 8}, {"I64", 8},     {"U64", 8}};
  auto it = sizes.find(t);
  return it == sizes.end() ? 0 : it->second;
}

std::string shape_str(const std::vector<uint64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); i++) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

}  // namespace

struct lrs_safetensors {
  std::string dir;
  std::vector<std::unique_ptr<Mapped>> files;
  std::vector<std::string> paths;
  std::map<std::string, StTensor> tensors;
  // listed by the shard index but absent from their shard (an error on use)
  std::map<std::string, std::string> unresolved;
  bool contains(const std::string& n) const { return tensors.count(n) || unresolved.count(n); }
  // owned by a built description
  lrs::Blobs blobs;
  std::vector<std::unique_ptr<std::vector<float>>> vecs;
  std::vector<lrs_layer_desc> layers;
  lrs_model_desc desc{};
};

namespace {

// SafeTensors::deserialize: the header of file `fi` into its tensor list.
int32_t parse_file(lrs_safetensors* st, int fi, std::map<std::string, StTensor>* out) {
  const Mapped& m = *st->files[fi];
  const std::string& path = st->paths[fi];
  auto bad = [&](const std::string& why) {
    return fail(LRS_ERR_INVALID, "invalid safetensors file " + path + ": " + why);
  };
  if (m.size < 8) return bad("header too small");
  uint64_t n;
  memcpy(&n, m.map, 8);
  if (n > kMaxHeader) return bad("header too large");
  if (n > m.size - 8) return bad("invalid header length");
  const char* h = reinterpret_cast<const char*>(m.map + 8);
  if (n == 0 || h[0] != '{') return bad("invalid header start");
  // the header is a str (safetensors' from_utf8 before the JSON parse)
  if (!lrs::valid_utf8(reinterpret_cast<const uint8_t*>(h), (size_t)n))
    return bad("invalid header: not UTF-8");
  JValue root;
  std::string err;
  if (!lrs::JsonParser(h, n).parse(&root, &err)) return bad("invalid header: " + err);
  if (root.kind != JValue::Obj) return bad("the header is not a JSON object");
  const size_t data0 = 8 + (size_t)n, buf_len = m.size - data0;
  std::vector<std::pair<uint64_t, uint64_t>> spans;
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind != JValue::Obj) return bad("__metadata__ is not a string map");
      for (const auto& mv : kv.second.obj)
        if (mv.second.kind != JValue::Str) return bad("__metadata__ is not a string map");
      continue;
    }
    const JValue& t = kv.second;
    const JValue* dt = t.get("dtype");
    const JValue* sh = t.get("shape");
    const JValue* off = t.get("data_offsets");
    if (t.kind != JValue::Obj || !dt || dt->kind != JValue::Str || !sh || sh->kind != JValue::Arr ||
        !off || off->kind != JValue::Arr || off->arr.size() != 2)
      return bad("invalid tensor entry " + kv.first);
    StTensor info;
    info.dtype = dt->s;
    const size_t es = dtype_size(info.dtype);
    if (!es) return bad("unknown dtype " + info.dtype + " for tensor " + kv.first);
    uint64_t numel = 1;
    for (const JValue& d : sh->arr) {
      if (d.kind != JValue::Num || !d.is_uint) return bad("invalid shape of tensor " + kv.first);
      if (d.u && numel > UINT64_MAX / d.u) return bad("shape overflow of tensor " + kv.first);
      numel *= d.u;
      info.shape.push_back(d.u);
    }
    for (const JValue& o : off->arr)
      if (o.kind != JValue::Num || !o.is_uint) return bad("invalid data_offsets of tensor " + kv.first);
    const uint64_t b = off->arr[0].u, e = off->arr[1].u;
    if (b > e || e > buf_len) return bad("data_offsets of tensor " + kv.first + " out of range");
    if (numel > UINT64_MAX / es || e - b != numel * es)
      return bad("data_offsets of tensor " + kv.first + " do not match its dtype and shape");
    info.start = data0 + (size_t)b;
    info.len = (size_t)(e - b);
    info.file = fi;
    spans.emplace_back(b, e);
    (*out)[kv.first] = info;
  }
  // the offsets tile the byte buffer: no gap, no overlap, nothing left over
  std::sort(spans.begin(), spans.end());
  uint64_t at = 0;
  for (const auto& sp : spans) {
    if (sp.first != at) return bad("data_offsets leave a gap or overlap");
    at = sp.second;
  }
  if (at != buf_len) return bad("data_offsets do not cover the byte buffer");
  return LRS_OK;
}

int32_t map_file(const std::string& path, std::unique_ptr<Mapped>* out) {
  auto m = std::make_unique<Mapped>();
  m->fd = open(path.c_str(), O_RDONLY);
  if (m->fd < 0) return fail(LRS_ERR_INVALID, "failed to open " + path);
  struct stat sb;
  if (fstat(m->fd, &sb) != 0) return fail(LRS_ERR_INVALID, "failed to open " + path);
  m->size = (size_t)sb.st_size;
  if (m->size) {
    void* p = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, m->fd, 0);
    if (p == MAP_FAILED) return fail(LRS_ERR_INVALID, "failed to map " + path);
    m->map = static_cast<const uint8_t*>(p);
  }
  *out = std::move(m);
  return LRS_OK;
}

// LlamaConfig::from_json + validate (src/config.rs:18-93).
int32_t parse_config(const std::string& text, lrs_config* c) {
  JValue root;
  std::string err;
  if (!lrs::JsonParser(text.data(), text.size()).parse(&root, &err))
    return fail(LRS_ERR_INVALID, "invalid config.json: " + err);
  if (root.kind != JValue::Obj) return fail(LRS_ERR_INVALID, "invalid config.json: not an object");
  auto need_usize = [&](const char* key, uint64_t* v) -> int32_t {
    const JValue* j = root.get(key);
    if (!j) return fail(LRS_ERR_INVALID, std::string("missing field `") + key + "`");
    if (j->kind != JValue::Num || !j->is_uint)
      return fail(LRS_ERR_INVALID, std::string("invalid type for `") + key + "`, expected usize");
    *v = j->u;
    return LRS_OK;
  };
  auto opt_f32 = [&](const char* key, float dflt, float* v) -> int32_t {
    const JValue* j = root.get(key);
    *v = dflt;
    if (!j) return LRS_OK;
    if (j->kind != JValue::Num)
      return fail(LRS_ERR_INVALID, std::string("invalid type for `") + key + "`, expected f32");
    *v = (float)j->num;
    return LRS_OK;
  };
  uint64_t hidden, inter, heads, kv, layers, vocab, ctx = 32768, hd = 0;
  float eps, theta;
  int32_t rc;
  if ((rc = need_usize("hidden_size", &hidden)) || (rc = need_usize("intermediate_size", &inter)) ||
      (rc = need_usize("num_attention_heads", &heads)) ||
      (rc = need_usize("num_key_value_heads", &kv)) ||
      (rc = need_usize("num_hidden_layers", &layers)) || (rc = need_usize("vocab_size", &vocab)) ||
      (rc = opt_f32("rms_norm_eps", 1e-6f, &eps)) || (rc = opt_f32("rope_theta", 10000.0f, &theta)))
    return rc;
  if (root.get("max_position_embeddings") && (rc = need_usize("max_position_embeddings", &ctx)))
    return rc;
  const JValue* hdj = root.get("head_dim");
  const bool has_hd = hdj && hdj->kind != JValue::Null;
  if (has_hd && (rc = need_usize("head_dim", &hd))) return rc;
  const JValue* tie = root.get("tie_word_embeddings");
  if (tie && tie->kind != JValue::Bool && tie->kind != JValue::Null)
    return fail(LRS_ERR_INVALID, "invalid type for `tie_word_embeddings`, expected a boolean");
  // LlamaConfig::validate
  if (!hidden || !inter || !heads || !kv || !layers || !vocab)
    return fail(LRS_ERR_INVALID, "invalid Qwen2 config: dimensions must be non-zero");
  if (hidden % heads && !has_hd)
    return fail(LRS_ERR_INVALID, "hidden_size must be divisible by num_attention_heads");
  if (heads % kv) return fail(LRS_ERR_INVALID, "num_attention_heads must be divisible by num_key_value_heads");
  if (!has_hd) hd = hidden / heads;
  if (heads * hd != hidden) return fail(LRS_ERR_INVALID, "num_attention_heads * head_dim must equal hidden_size");
  if (hd % 2) return fail(LRS_ERR_INVALID, "Qwen2 RoPE requires an even head_dim");
  if (!std::isfinite(eps) || eps <= 0.0f) return fail(LRS_ERR_INVALID, "rms_norm_eps must be finite and positive");
  if (!std::isfinite(theta) || theta <= 0.0f)
    return fail(LRS_ERR_INVALID, "rope_theta must be finite and positive");
  if (hidden > UINT32_MAX || inter > UINT32_MAX || heads > UINT32_MAX || kv > UINT32_MAX ||
      layers > UINT32_MAX || vocab > UINT32_MAX || ctx > UINT32_MAX || hd > UINT32_MAX)
    return fail(LRS_ERR_INVALID, "model dimensions do not fit 32 bits");
  memset(c, 0, sizeof(*c));
  c->hidden_size = (uint32_t)hidden;
  c->intermediate_size = (uint32_t)inter;
  c->num_attention_heads = (uint32_t)heads;
  c->num_key_value_heads = (uint32_t)kv;
  c->num_hidden_layers = (uint32_t)layers;
  c->vocab_size = (uint32_t)vocab;
  c->head_dim = (uint32_t)hd;
  c->max_position_embeddings = (uint32_t)ctx;
  c->rms_norm_eps = eps;
  c->rope_theta = theta;
  return LRS_OK;
}

}  // namespace

extern "C" {

lrs_status lrs_st_open(const char* model_dir, lrs_safetensors** out) try {
  if (!model_dir || !out) return fail(LRS_ERR_INVALID, "null argument");
  *out = nullptr;
  auto st = std::make_unique<lrs_safetensors>();
  st->dir = model_dir;
  const std::string index_path = join(st->dir, "model.safetensors.index.json");
  const bool indexed = is_file(index_path);
  std::map<std::string, std::string> weight_map;
  if (indexed) {
    std::string text;
    if (!read_text(index_path, &text)) return fail(LRS_ERR_INVALID, "failed to read " + index_path);
    JValue root;
    std::string err;
    if (!lrs::JsonParser(text.data(), text.size()).parse(&root, &err))
      return fail(LRS_ERR_INVALID, "invalid " + index_path + ": " + err);
    const JValue* wm = root.get("weight_map");
    if (!wm || wm->kind != JValue::Obj)
      return fail(LRS_ERR_INVALID, "invalid " + index_path + ": missing field `weight_map`");
    for (const auto& kv : wm->obj) {
      if (kv.second.kind != JValue::Str)
        return fail(LRS_ERR_INVALID, "invalid " + index_path + ": weight_map values must be strings");
      weight_map[kv.first] = join(st->dir, kv.second.s);
      st->paths.push_back(join(st->dir, kv.second.s));
    }
    std::sort(st->paths.begin(), st->paths.end());
    st->paths.erase(std::unique(st->paths.begin(), st->paths.end()), st->paths.end());
  } else {
    st->paths = list_ext(st->dir, ".safetensors");
    if (st->paths.empty()) return fail(LRS_ERR_INVALID, "no .safetensors files in " + st->dir);
  }
  for (size_t i = 0; i < st->paths.size(); i++) {
    std::unique_ptr<Mapped> m;
    int32_t rc = map_file(st->paths[i], &m);
    if (rc) return rc;
    st->files.push_back(std::move(m));
    std::map<std::string, StTensor> found;
    if ((rc = parse_file(st.get(), (int)i, &found))) return rc;
    if (indexed) {  // the index names the shard of each tensor
      for (auto& kv : found) {
        auto w = weight_map.find(kv.first);
        if (w != weight_map.end() && w->second == st->paths[i]) st->tensors[kv.first] = kv.second;
      }
    } else {
      for (auto& kv : found)
        if (!st->tensors.emplace(kv.first, kv.second).second)
          return fail(LRS_ERR_INVALID, "duplicate safetensors tensor " + kv.first);
    }
  }
  if (indexed)
    for (const auto& kv : weight_map)
      if (!st->tensors.count(kv.first)) st->unresolved[kv.first] = kv.second;
  *out = st.release();
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

void lrs_st_close(lrs_safetensors* st) { delete st; }
size_t lrs_st_tensor_count(const lrs_safetensors* st) { return st ? st->tensors.size() : 0; }

lrs_status lrs_st_tensor(const lrs_safetensors* st, const char* name_c, lrs_tensor_desc* out) try {
  if (!st || !name_c || !out) return fail(LRS_ERR_INVALID, "null argument");
  const std::string name = name_c;
  auto it = st->tensors.find(name);
  if (it == st->tensors.end()) {
    auto u = st->unresolved.find(name);
    if (u != st->unresolved.end())
      return fail(LRS_ERR_INVALID, "invalid safetensors tensor " + name + ": not in " + u->second);
    return fail(LRS_ERR_INVALID, "missing safetensors tensor " + name);
  }
  const StTensor& t = it->second;
  uint32_t ty;
  if (t.dtype == "F32") {
    ty = LRS_GGML_F32;
  } else if (t.dtype == "F16") {
    ty = LRS_GGML_F16;
  } else if (t.dtype == "BF16") {
    ty = LRS_GGML_BF16;
  } else {
    return fail(LRS_ERR_UNSUPPORTED, "unsupported safetensors dtype " + t.dtype + "; use F32/F16/BF16");
  }
  if (t.shape.size() > 2)
    return fail(LRS_ERR_INVALID, "invalid safetensors tensor " + name + ": " +
                                     std::to_string(t.shape.size()) + " dimensions");
  memset(out, 0, sizeof(*out));
  out->data = st->files[t.file]->map + t.start;
  out->nbytes = t.len;
  out->rows = t.shape.size() == 2 ? t.shape[0] : 1;
  out->cols = t.shape.empty() ? 1 : t.shape.back();
  out->ggml_type = ty;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

lrs_status lrs_st_qwen2_desc(lrs_safetensors* st, uint32_t recipe, const lrs_model_desc** out) try {
  if (!st || !out) return fail(LRS_ERR_INVALID, "null argument");
  if (recipe > LRS_RECIPE_Q4KM) return fail(LRS_ERR_INVALID, "unknown load quantization");
  // SafetensorsLoader::load, src/loader.rs:83-100
  const std::string config_path = join(st->dir, "config.json");
  std::string text;
  // fs::read_to_string: unreadable or not UTF-8 is a read failure
  if (!read_text(config_path, &text) ||
      !lrs::valid_utf8(reinterpret_cast<const uint8_t*>(text.data()), text.size()))
    return fail(LRS_ERR_INVALID, "failed to read " + config_path);
  {
    JValue root;
    std::string err;
    if (!lrs::JsonParser(text.data(), text.size()).parse(&root, &err))
      return fail(LRS_ERR_INVALID, "invalid config.json: " + err);
    const JValue* mt = root.get("model_type");
    if (!mt || mt->kind != JValue::Str) return fail(LRS_ERR_INVALID, "config.json is missing model_type");
    if (mt->s != "qwen2")
      return fail(LRS_ERR_UNSUPPORTED, "unsupported Hugging Face model_type \"" + mt->s + "\"");
  }
  lrs_config c;
  int32_t rc = parse_config(text, &c);
  if (rc) return rc;
  const size_t hidden = c.hidden_size, inter = c.intermediate_size;
  const size_t kvw = (size_t)c.num_key_value_heads * c.head_dim;
  st->blobs.clear();
  st->vecs.clear();

  auto dims_of = [&](const std::string& name) { return st->tensors.at(name).shape; };
  // load_st_matrix (src/loader.rs:458-468): shape check, then maybe_quantize
  auto matrix = [&](const std::string& name, size_t rows, size_t cols, lrs_tensor_desc* d) -> int32_t {
    int32_t r2 = lrs_st_tensor(st, name.c_str(), d);
    if (r2) return r2;
    const auto dims = dims_of(name);
    if (dims.size() != 2 || dims[0] != rows || dims[1] != cols)
      return fail(LRS_ERR_INVALID, "tensor " + name + " has shape " + shape_str(dims) + ", expected [" +
                                       std::to_string(rows) + ", " + std::to_string(cols) + "]");
    return lrs::maybe_quantize_desc(recipe, name, rows, cols, d, &st->blobs, "SafeTensors");
  };
  // load_st_vector (src/loader.rs:470-478)
  auto vector = [&](const std::string& name, size_t len, const float** outp) -> int32_t {
    lrs_tensor_desc d;
    int32_t r2 = lrs_st_tensor(st, name.c_str(), &d);
    if (r2) return r2;
    const auto dims = dims_of(name);
    if (dims.size() != 1 || dims[0] != len)
      return fail(LRS_ERR_INVALID, "tensor " + name + " has shape " + shape_str(dims) +
                                       ", expected [" + std::to_string(len) + "]");
    auto v = std::make_unique<std::vector<float>>();
    if ((r2 = lrs::desc_to_f32(d, name, v.get(), "SafeTensors"))) return r2;
    *outp = v->data();
    st->vecs.push_back(std::move(v));
    return LRS_OK;
  };
  // load_st_linear's bias: present -> loaded, absent -> zeros (src/loader.rs:480-495)
  auto bias = [&](const std::string& name, size_t len, const float** outp) -> int32_t {
    *outp = nullptr;
    if (!st->contains(name)) return LRS_OK;
    return vector(name, len, outp);
  };

  lrs_model_desc& d = st->desc;
  memset(&d, 0, sizeof(d));
  d.config = c;
  if ((rc = matrix("model.embed_tokens.weight", c.vocab_size, hidden, &d.embed_tokens)) ||
      (rc = vector("model.norm.weight", hidden, &d.final_norm)))
    return rc;
  // one layer at a time: a corrupt layer count fails at its first missing
  // tensor (the reference's error) instead of allocating for it up front
  st->layers.clear();
  for (uint32_t i = 0; i < c.num_hidden_layers; i++) {
    const std::string p = "model.layers." + std::to_string(i);
    st->layers.push_back(lrs_layer_desc{});
    lrs_layer_desc& L = st->layers.back();
    if ((rc = vector(p + ".input_layernorm.weight", hidden, &L.input_layernorm)) ||
        (rc = vector(p + ".post_attention_layernorm.weight", hidden, &L.post_attention_layernorm)) ||
        (rc = matrix(p + ".self_attn.q_proj.weight", hidden, hidden, &L.q_proj)) ||
        (rc = bias(p + ".self_attn.q_proj.bias", hidden, &L.q_bias)) ||
        (rc = matrix(p + ".self_attn.k_proj.weight", kvw, hidden, &L.k_proj)) ||
        (rc = bias(p + ".self_attn.k_proj.bias", kvw, &L.k_bias)) ||
        (rc = matrix(p + ".self_attn.v_proj.weight", kvw, hidden, &L.v_proj)) ||
        (rc = bias(p + ".self_attn.v_proj.bias", kvw, &L.v_bias)) ||
        (rc = matrix(p + ".self_attn.o_proj.weight", hidden, hidden, &L.o_proj)) ||
        (rc = matrix(p + ".mlp.gate_proj.weight", inter, hidden, &L.gate_proj)) ||
        (rc = matrix(p + ".mlp.up_proj.weight", inter, hidden, &L.up_proj)) ||
        (rc = matrix(p + ".mlp.down_proj.weight", hidden, inter, &L.down_proj)))
      return rc;
  }
  // lm_head.weight present: its own head; absent: tied to the embedding
  if (st->contains("lm_head.weight")) {
    if ((rc = matrix("lm_head.weight", c.vocab_size, hidden, &d.lm_head))) return rc;
  } else {
    d.lm_head = d.embed_tokens;
  }
  d.layers = st->layers.data();
  *out = &d;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

}  // extern "C"

struct lrs_loaded {
  lrs_gguf* gguf = nullptr;
  lrs_safetensors* st = nullptr;
  ~lrs_loaded() {
    if (gguf) lrs_gguf_close(gguf);
    if (st) lrs_st_close(st);
  }
};

extern "C" {

lrs_status lrs_model_load(const char* path_c, uint32_t recipe, lrs_loaded** out,
                          const lrs_model_desc** desc) try {
  if (!path_c || !out || !desc) return fail(LRS_ERR_INVALID, "null argument");
  *out = nullptr;
  const std::string path = path_c;
  auto l = std::make_unique<lrs_loaded>();
  int32_t rc;
  auto load_gguf = [&](const std::string& p) -> int32_t {
    if ((rc = lrs_gguf_open(p.c_str(), &l->gguf))) return rc;
    return lrs_gguf_qwen2_desc(l->gguf, recipe, desc);
  };
  auto load_st = [&](const std::string& dir) -> int32_t {
    if ((rc = lrs_st_open(dir.c_str(), &l->st))) return rc;
    return lrs_st_qwen2_desc(l->st, recipe, desc);
  };
  // ModelLoader::load, src/loader.rs:46-79
  if (is_file(path) && ends_with(path, ".gguf")) {
    rc = load_gguf(path);
  } else if (is_file(path) && ends_with(path, ".safetensors")) {
    const size_t slash = path.find_last_of('/');
    rc = load_st(slash == std::string::npos ? "." : path.substr(0, slash == 0 ? 1 : slash));
  } else if (is_dir(path)) {
    const auto ggufs = list_ext(path, ".gguf");
    if (is_file(join(path, "model.safetensors")) || is_file(join(path, "model.safetensors.index.json"))) {
      rc = load_st(path);
    } else if (ggufs.size() == 1) {
      rc = load_gguf(ggufs[0]);
    } else if (ggufs.size() > 1) {
      rc = fail(LRS_ERR_INVALID, path + " contains multiple GGUF files; pass the desired file explicitly");
    } else {
      rc = fail(LRS_ERR_INVALID, "cannot detect model format at " + path);
    }
  } else {
    rc = fail(LRS_ERR_INVALID, "cannot detect model format at " + path);
  }
  if (rc) return rc;
  *out = l.release();
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

void lrs_loaded_close(lrs_loaded* l) { delete l; }

}  // extern "C"

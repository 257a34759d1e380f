// synth.cpp -- seeded synthetic Qwen2 models (host).
//
// Builds, in memory, the model a reference user would get from a one-file F32
// SafeTensors checkpoint loaded with `--quantize q4k|q4km`
// (SafetensorsLoader::load, src/loader.rs:83-227, then maybe_quantize,
// :406-447): weights and biases N(0, std), RMSNorm weights 1.0, tensor names of
// the Hugging Face Qwen2 layout, and an lm_head that reuses the quantized
// embedding when the embeddings are tied (src/loader.rs:205-216).
//
// Values are counter-based: element i of tensor `name` under `seed` is a
// Box-Muller normal of two SplitMix64 draws keyed by (seed, FNV-1a(name), i/2),
// so any row range can be generated and quantized independently, on any number
// of threads, with the same result.
#include <algorithm>
#include <cmath>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/llamars_synth.h"
#include "common.h"

namespace lrs {
uint32_t effective_type(uint32_t t, size_t cols);
void quantize_row(uint32_t t, const float* v, size_t cols, uint8_t* out);

namespace {

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
inline uint64_t fnv1a(const char* s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (; *s; s++) h = (h ^ (uint8_t)*s) * 0x100000001b3ull;
  return h;
}

struct NormalStream {
  uint64_t key;
  NormalStream(uint64_t seed, const char* name) : key(splitmix64(seed ^ splitmix64(fnv1a(name)))) {}
  // Writes values offset..offset+n-1 scaled by stddev.
  void fill(float stddev, uint64_t offset, size_t n, float* out) const {
    const float two_pi = 6.28318530717958647692f;
    size_t k = 0;
    while (k < n) {
      uint64_t i = offset + k;
      uint64_t pair = i >> 1;
      uint64_t a = splitmix64(key + 2 * pair), b = splitmix64(key + 2 * pair + 1);
      float u1 = (float)((a >> 40) + 1) * (1.0f / 16777216.0f);  // (0, 1]
      float u2 = (float)(b >> 40) * (1.0f / 16777216.0f);        // [0, 1)
      float r = sqrtf(-2.0f * logf(u1));
      float th = two_pi * u2;
      float z0 = r * cosf(th), z1 = r * sinf(th);
      if ((i & 1) == 0) {
        out[k++] = stddev * z0;
        if (k < n) out[k++] = stddev * z1;
      } else {
        out[k++] = stddev * z1;
      }
    }
  }
};

template <typename F>
void parallel_rows(size_t rows, int threads, F&& fn) {
  int nt = (int)std::min<size_t>(rows, (size_t)std::max(1, threads));
  if (nt <= 1) {
    fn(0, rows);
    return;
  }
  std::vector<std::thread> ts;
  for (int t = 0; t < nt; t++) {
    size_t b = rows * t / nt, e = rows * (t + 1) / nt;
    ts.emplace_back([&fn, b, e] { fn(b, e); });
  }
  for (auto& t : ts) t.join();
}

}  // namespace
}  // namespace lrs

using namespace lrs;

struct lrs_synth_model {
  lrs_model_desc desc;
  std::vector<lrs_layer_desc> layers;
  std::vector<std::unique_ptr<std::vector<uint8_t>>> blobs;
  std::vector<std::unique_ptr<std::vector<float>>> vecs;
};

namespace {

lrs_tensor_desc make_matrix(lrs_synth_model* m, const lrs_synth_spec& s, const std::string& name,
                            size_t rows, size_t cols, int threads) {
  uint32_t t = lrs_recipe_type(s.recipe, name.c_str(), rows, cols);
  size_t rb = row_bytes(t, cols);
  m->blobs.emplace_back(new std::vector<uint8_t>(rows * rb + 64));
  uint8_t* out = m->blobs.back()->data();
  NormalStream ns(s.seed, name.c_str());
  float sd = s.init_std;
  parallel_rows(rows, threads, [&](size_t b, size_t e) {
    std::vector<float> row(cols);
    for (size_t r = b; r < e; r++) {
      ns.fill(sd, (uint64_t)r * cols, cols, row.data());
      quantize_row(t, row.data(), cols, out + r * rb);
    }
  });
  lrs_tensor_desc d{};
  d.data = out;
  d.nbytes = rows * rb;
  d.rows = rows;
  d.cols = cols;
  d.ggml_type = t;
  return d;
}

const float* make_vector(lrs_synth_model* m, const lrs_synth_spec& s, const std::string& name,
                         size_t n, bool ones) {
  m->vecs.emplace_back(new std::vector<float>(n, 1.0f));
  float* p = m->vecs.back()->data();
  if (!ones) NormalStream(s.seed, name.c_str()).fill(s.init_std, 0, n, p);
  return p;
}

}  // namespace

extern "C" {

void lrs_synth_fill(uint64_t seed, const char* name, float stddev, uint64_t offset, size_t n,
                    float* out) {
  NormalStream(seed, name).fill(stddev, offset, n, out);
}

lrs_status lrs_synth_model_create(const lrs_synth_spec* spec, lrs_synth_model** out) try {
  if (!spec || !out) return fail(LRS_ERR_INVALID, "null argument");
  const lrs_config& c = spec->config;
  if (!c.hidden_size || !c.intermediate_size || !c.num_attention_heads ||
      !c.num_key_value_heads || !c.num_hidden_layers || !c.vocab_size || !c.head_dim)
    return fail(LRS_ERR_INVALID, "invalid Qwen2 config: dimensions must be non-zero");
  if (c.num_attention_heads % c.num_key_value_heads)
    return fail(LRS_ERR_INVALID, "num_attention_heads must be divisible by num_key_value_heads");
  if (c.num_attention_heads * c.head_dim != c.hidden_size)
    return fail(LRS_ERR_INVALID, "num_attention_heads * head_dim must equal hidden_size");
  if (c.head_dim % 2) return fail(LRS_ERR_INVALID, "Qwen2 RoPE requires an even head_dim");
  int threads = spec->threads ? (int)spec->threads : (int)std::thread::hardware_concurrency();
  auto* m = new lrs_synth_model();
  m->desc.config = c;
  size_t h = c.hidden_size, I = c.intermediate_size, kv = (size_t)c.num_key_value_heads * c.head_dim;
  m->desc.embed_tokens = make_matrix(m, *spec, "model.embed_tokens.weight", c.vocab_size, h, threads);
  m->desc.final_norm = make_vector(m, *spec, "model.norm.weight", h, true);
  m->layers.resize(c.num_hidden_layers);
  for (uint32_t i = 0; i < c.num_hidden_layers; i++) {
    std::string p = "model.layers." + std::to_string(i);
    lrs_layer_desc& L = m->layers[i];
    L.input_layernorm = make_vector(m, *spec, p + ".input_layernorm.weight", h, true);
    L.post_attention_layernorm = make_vector(m, *spec, p + ".post_attention_layernorm.weight", h, true);
    L.q_proj = make_matrix(m, *spec, p + ".self_attn.q_proj.weight", h, h, threads);
    L.k_proj = make_matrix(m, *spec, p + ".self_attn.k_proj.weight", kv, h, threads);
    L.v_proj = make_matrix(m, *spec, p + ".self_attn.v_proj.weight", kv, h, threads);
    L.o_proj = make_matrix(m, *spec, p + ".self_attn.o_proj.weight", h, h, threads);
    L.gate_proj = make_matrix(m, *spec, p + ".mlp.gate_proj.weight", I, h, threads);
    L.up_proj = make_matrix(m, *spec, p + ".mlp.up_proj.weight", I, h, threads);
    L.down_proj = make_matrix(m, *spec, p + ".mlp.down_proj.weight", h, I, threads);
    L.q_bias = make_vector(m, *spec, p + ".self_attn.q_proj.bias", h, false);
    L.k_bias = make_vector(m, *spec, p + ".self_attn.k_proj.bias", kv, false);
    L.v_bias = make_vector(m, *spec, p + ".self_attn.v_proj.bias", kv, false);
  }
  m->desc.layers = m->layers.data();
  if (spec->tie_word_embeddings)
    m->desc.lm_head = m->desc.embed_tokens;
  else
    m->desc.lm_head = make_matrix(m, *spec, "lm_head.weight", c.vocab_size, h, threads);
  *out = m;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

const lrs_model_desc* lrs_synth_model_desc(const lrs_synth_model* m) { return m ? &m->desc : nullptr; }

void lrs_synth_model_destroy(lrs_synth_model* m) { delete m; }

}  // extern "C"

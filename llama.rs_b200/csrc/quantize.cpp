// quantize.cpp -- the load-time encoders on the host: the q4k / q4km recipe
// and multithreaded matrix encoding (the encoders are in encoders.h).  Compiled
// with -ffp-contract=off (Rust never fuses a*b+c).
#include <algorithm>
#include <string>
#include <thread>
#include <vector>

#include "../../include/llamars_synth.h"
#include "common.h"
#include "encoders.h"

namespace lrs {
uint32_t effective_type(uint32_t t, size_t cols) { return enc::effective_type(t, cols); }
void quantize_row(uint32_t t, const float* v, size_t cols, uint8_t* out) {
  enc::quantize_row(t, v, cols, out);
}
}  // namespace lrs

using namespace lrs;

extern "C" {

uint32_t lrs_recipe_type(uint32_t recipe, const char* name_c, size_t rows, size_t cols) {
  // maybe_quantize, src/loader.rs:406-447 (applies to F32/F16/BF16 2-D tensors).
  (void)rows;
  std::string name(name_c ? name_c : "");
  if (recipe == LRS_RECIPE_NONE) return LRS_GGML_F32;
  uint32_t t;
  if (recipe == LRS_RECIPE_Q4K) {
    t = LRS_GGML_Q4_K;
  } else if (name.find("embed_tokens") != std::string::npos || name == "token_embd.weight" ||
             name == "lm_head.weight" || name == "output.weight" ||
             name.find("attn.v_proj.weight") != std::string::npos ||
             name.find("attn_v.weight") != std::string::npos) {
    t = LRS_GGML_Q8_0;
  } else if (name.find("mlp.down_proj.weight") != std::string::npos ||
             name.find("ffn_down.weight") != std::string::npos) {
    t = LRS_GGML_Q6_K;
  } else {
    t = LRS_GGML_Q4_K;
  }
  return effective_type(t, cols);
}

size_t lrs_quantized_size(uint32_t t, size_t rows, size_t cols) {
  uint32_t e = effective_type(t, cols);
  uint32_t bv, bb;
  if (!type_geometry(e, &bv, &bb)) return 0;
  return rows * (cols / bv) * bb;
}

lrs_status lrs_quantize_matrix(uint32_t t, const float* values, size_t rows, size_t cols,
                               void* out, size_t out_cap, uint32_t* out_type, size_t* out_len) try {
  uint32_t bv, bb;
  if (!type_geometry(t, &bv, &bb)) return fail(LRS_ERR_UNSUPPORTED, "unsupported GGML type");
  uint32_t e = effective_type(t, cols);
  size_t need = lrs_quantized_size(t, rows, cols);
  if (out_cap < need) return fail(LRS_ERR_INVALID, "output buffer too small");
  size_t rb = row_bytes(e, cols);
  // Rows are independent: split them over the host threads.
  size_t nt = std::min<size_t>(std::max(1u, std::thread::hardware_concurrency()),
                               std::max<size_t>(1, rows * cols / (1u << 16)));
  auto work = [&](size_t b, size_t e2) {
    for (size_t r = b; r < e2; r++) quantize_row(e, values + r * cols, cols, (uint8_t*)out + r * rb);
  };
  if (nt <= 1) {
    work(0, rows);
  } else {
    std::vector<std::thread> ts;
    for (size_t t2 = 0; t2 < nt; t2++) ts.emplace_back(work, rows * t2 / nt, rows * (t2 + 1) / nt);
    for (auto& th : ts) th.join();
  }
  if (out_type) *out_type = e;
  if (out_len) *out_len = need;
  return LRS_OK;
} catch (...) {
  return lrs::status_of_current_exception();
}

}  // extern "C"

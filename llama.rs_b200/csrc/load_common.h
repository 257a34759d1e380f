// load_common.h -- pieces the GGUF and SafeTensors loaders share (host):
// QuantTensor::to_vec_f32 for float tensors, and maybe_quantize
// (src/loader.rs:406-447) applied to a float matrix descriptor.
#pragma once
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/llamars.h"
#include "../../include/llamars_synth.h"
#include "common.h"

namespace lrs {

// Owned buffers a built model description points into.
using Blobs = std::vector<std::unique_ptr<std::vector<uint8_t>>>;

inline float f16_to_f32_host(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      uint32_t m = man;
      do {
        e++;
        m <<= 1;
      } while ((m & 0x400) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// QuantTensor::to_vec_f32 for F32/F16/BF16 (value_at, src/quant.rs:349-360).
inline int32_t desc_to_f32(const lrs_tensor_desc& d, const std::string& name,
                           std::vector<float>* out, const char* loader) {
  const size_t n = d.rows * d.cols;
  out->resize(n);
  const uint8_t* p = static_cast<const uint8_t*>(d.data);
  switch (d.ggml_type) {
    case LRS_GGML_F32:
      memcpy(out->data(), p, n * 4);
      return LRS_OK;
    case LRS_GGML_F16:
      for (size_t i = 0; i < n; i++) {
        uint16_t h;
        memcpy(&h, p + 2 * i, 2);
        (*out)[i] = f16_to_f32_host(h);
      }
      return LRS_OK;
    case LRS_GGML_BF16:
      for (size_t i = 0; i < n; i++) {
        uint16_t h;
        memcpy(&h, p + 2 * i, 2);
        const uint32_t b = (uint32_t)h << 16;
        memcpy(&(*out)[i], &b, 4);
      }
      return LRS_OK;
  }
  return fail(LRS_ERR_UNSUPPORTED, "tensor " + name + ": " + type_name(d.ggml_type) +
                                       " vectors are not supported by the CUDA backend's " +
                                       loader + " loader");
}

// maybe_quantize: F32/F16/BF16 matrices are encoded with the recipe's type for
// `name`; other types (and recipe none) keep the descriptor as it is.
inline int32_t maybe_quantize_desc(uint32_t recipe, const std::string& name, size_t rows,
                                   size_t cols, lrs_tensor_desc* d, Blobs* blobs,
                                   const char* loader) {
  const uint32_t t = d->ggml_type;
  if (recipe == LRS_RECIPE_NONE || (t != LRS_GGML_F32 && t != LRS_GGML_F16 && t != LRS_GGML_BF16))
    return LRS_OK;
  std::vector<float> v;
  int32_t rc = desc_to_f32(*d, name, &v, loader);
  if (rc) return rc;
  const uint32_t qt = lrs_recipe_type(recipe, name.c_str(), rows, cols);
  if (qt == LRS_GGML_F32) {  // the encoders' fallback keeps f32
    auto buf = std::make_unique<std::vector<uint8_t>>(v.size() * 4);
    memcpy(buf->data(), v.data(), buf->size());
    d->data = buf->data();
    d->nbytes = buf->size();
    d->ggml_type = LRS_GGML_F32;
    blobs->push_back(std::move(buf));
    return LRS_OK;
  }
  auto buf = std::make_unique<std::vector<uint8_t>>(lrs_quantized_size(qt, rows, cols));
  uint32_t made;
  size_t len;
  if ((rc = lrs_quantize_matrix(qt, v.data(), rows, cols, buf->data(), buf->size(), &made, &len)))
    return rc;
  d->data = buf->data();
  d->nbytes = len;
  d->ggml_type = made;
  blobs->push_back(std::move(buf));
  return LRS_OK;
}

// Strict UTF-8 check (Rust's str::from_utf8).
inline bool valid_utf8(const uint8_t* p, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = p[i];
    size_t len;
    uint32_t cp;
    if (c < 0x80) {
      i++;
      continue;
    } else if ((c & 0xE0) == 0xC0) {
      len = 2, cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      len = 3, cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      len = 4, cp = c & 0x07;
    } else {
      return false;
    }
    if (i + len > n) return false;
    for (size_t k = 1; k < len; k++) {
      if ((p[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
        cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    i += len;
  }
  return true;
}

}  // namespace lrs

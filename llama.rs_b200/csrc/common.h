// common.h -- shared host helpers of the llama.rs CUDA backend library.
#pragma once
#include <cstdint>
#include <cstring>
#include <exception>
#include <new>
#include <string>

#include "../../include/llamars.h"

namespace lrs {

// Sets the thread's last-error message and returns `code`.
int32_t fail(int32_t code, const std::string& msg);
void clear_error();

// The status of the exception being handled, for the function-try-blocks of
// the C entry points: no C++ exception crosses the C ABI.  A failed host
// allocation (a corrupt file or an argument asking for too much) is
// LRS_ERR_OOM, any other exception LRS_ERR_INVALID.
inline int32_t status_of_current_exception() {
  try {
    throw;
  } catch (const std::bad_alloc&) {
    return fail(LRS_ERR_OOM, "out of host memory");
  } catch (const std::exception& e) {
    return fail(LRS_ERR_INVALID, e.what());
  } catch (...) {
    return fail(LRS_ERR_INVALID, "unexpected host error");
  }
}

// QuantType::block_size / type_size (src/quant.rs:46-67).
inline bool type_geometry(uint32_t t, uint32_t* bv, uint32_t* bb) {
  switch (t) {
    case LRS_GGML_F32: *bv = 1; *bb = 4; return true;
    case LRS_GGML_F16:
    case LRS_GGML_BF16: *bv = 1; *bb = 2; return true;
    case LRS_GGML_Q4_0: *bv = 32; *bb = 18; return true;
    case LRS_GGML_Q4_1: *bv = 32; *bb = 20; return true;
    case LRS_GGML_Q5_0: *bv = 32; *bb = 22; return true;
    case LRS_GGML_Q5_1: *bv = 32; *bb = 24; return true;
    case LRS_GGML_Q8_0: *bv = 32; *bb = 34; return true;
    case LRS_GGML_Q4_K: *bv = 256; *bb = 144; return true;
    case LRS_GGML_Q5_K: *bv = 256; *bb = 176; return true;
    case LRS_GGML_Q6_K: *bv = 256; *bb = 210; return true;
  }
  return false;
}

inline const char* type_name(uint32_t t) {
  switch (t) {
    case LRS_GGML_F32: return "F32";
    case LRS_GGML_F16: return "F16";
    case LRS_GGML_BF16: return "BF16";
    case LRS_GGML_Q4_0: return "Q4_0";
    case LRS_GGML_Q4_1: return "Q4_1";
    case LRS_GGML_Q5_0: return "Q5_0";
    case LRS_GGML_Q5_1: return "Q5_1";
    case LRS_GGML_Q8_0: return "Q8_0";
    case LRS_GGML_Q4_K: return "Q4_K";
    case LRS_GGML_Q5_K: return "Q5_K";
    case LRS_GGML_Q6_K: return "Q6_K";
  }
  return "?";
}

inline size_t row_bytes(uint32_t t, size_t cols) {
  uint32_t bv = 1, bb = 4;
  type_geometry(t, &bv, &bb);
  return cols / bv * bb;
}

}  // namespace lrs

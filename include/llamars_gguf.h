/*
 * llamars_gguf.h -- GGUF model files for the CUDA backend (host side).
 *
 * Restates the reference's GGUF reader (GgufFile, src/gguf.rs:72-230) and
 * its Qwen2 loader (GgufLoader::load, src/loader.rs:231-398) so that a .gguf
 * file feeds lrs_model_create directly: tensors that are already quantized
 * are views into the memory-mapped file (uploaded to HBM without any f32
 * expansion), F32/F16/BF16 matrices go through the same load-time recipe as
 * the reference (maybe_quantize, src/loader.rs:406-447).  Errors carry the
 * reference's messages.
 */
#ifndef LLAMARS_GGUF_H
#define LLAMARS_GGUF_H
#include "llamars.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lrs_gguf lrs_gguf;

/* GgufFile::open (src/gguf.rs:80-170): maps the file and checks the magic,
 * version (2 or 3), header counts, metadata, tensor infos, the alignment and
 * every tensor's byte range. */
lrs_status lrs_gguf_open(const char* path, lrs_gguf** out);
void lrs_gguf_close(lrs_gguf* gguf);
uint32_t lrs_gguf_version(const lrs_gguf* gguf);
size_t lrs_gguf_tensor_count(const lrs_gguf* gguf);

/* GgufFile::metadata_u64 / metadata_f32 / metadata_str (src/gguf.rs:172-191).
 * The string stays valid while the handle lives. */
lrs_status lrs_gguf_metadata_u64(const lrs_gguf* gguf, const char* key, uint64_t* out);
lrs_status lrs_gguf_metadata_f32(const lrs_gguf* gguf, const char* key, float* out);
lrs_status lrs_gguf_metadata_str(const lrs_gguf* gguf, const char* key, const char** out);

/* GgufFile::tensor (src/gguf.rs:196-215): a QuantTensor view.  GGML order
 * [cols, rows] becomes rows x cols; a 1-D tensor is 1 x len. */
lrs_status lrs_gguf_tensor(const lrs_gguf* gguf, const char* name, lrs_tensor_desc* out);

/* GgufLoader::load (src/loader.rs:233-398) for "qwen2": the config from the
 * qwen2.* metadata, the blk.N.* tensors, F32/F16/BF16 matrices encoded with
 * `recipe` (LRS_RECIPE_*, llamars_synth.h), norm vectors as f32, missing
 * q/k/v biases as zeros (NULL), and no output.weight = tied head.  The
 * description (and any encoded or converted buffers) belongs to the handle. */
lrs_status lrs_gguf_qwen2_desc(lrs_gguf* gguf, uint32_t recipe, const lrs_model_desc** out);

#ifdef __cplusplus
}
#endif
#endif /* LLAMARS_GGUF_H */

/*
 * llamars_safetensors.h -- Hugging Face SafeTensors checkpoints for the CUDA
 * backend (host side), and the format dispatch of ModelLoader::load.
 *
 * Restates SafetensorStore (src/loader.rs:535-645) and SafetensorsLoader::load
 * (src/loader.rs:80-230) so that a model directory (config.json plus
 * model.safetensors, or shards listed by model.safetensors.index.json) feeds
 * lrs_model_create directly: F32/F16/BF16 matrices go through the load-time
 * recipe (maybe_quantize, src/loader.rs:406-447), norms and biases become f32,
 * missing q/k/v biases are zeros (NULL) and a missing lm_head.weight ties the
 * head to the embedding.  The file format is the one of the `safetensors`
 * crate 0.4 the reference depends on (Cargo.toml): an 8-byte little-endian
 * header length (at most 100,000,000), a JSON object header naming each
 * tensor's dtype, shape and data_offsets, then the tensor bytes, which the
 * offsets must cover exactly.  Errors carry the reference's messages.
 */
#ifndef LLAMARS_SAFETENSORS_H
#define LLAMARS_SAFETENSORS_H
#include "llamars.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lrs_safetensors lrs_safetensors;

/* SafetensorStore::open (src/loader.rs:541-600): the shards of `model_dir`. */
lrs_status lrs_st_open(const char* model_dir, lrs_safetensors** out);
void lrs_st_close(lrs_safetensors* st);
size_t lrs_st_tensor_count(const lrs_safetensors* st);

/* SafetensorStore::tensor (src/loader.rs:606-623): a view of an F32, F16 or
 * BF16 tensor (1-D tensors are 1 x len). */
lrs_status lrs_st_tensor(const lrs_safetensors* st, const char* name, lrs_tensor_desc* out);

/* SafetensorsLoader::load (src/loader.rs:83-230) on the store's directory:
 * config.json (LlamaConfig::from_json, src/config.rs) and the Qwen2 tensors,
 * matrices encoded with `recipe` (LRS_RECIPE_*).  The description (and any
 * encoded or converted buffers) belongs to the store. */
lrs_status lrs_st_qwen2_desc(lrs_safetensors* st, uint32_t recipe, const lrs_model_desc** out);

/* ModelLoader::load (src/loader.rs:46-79): `path` is a .gguf file, a
 * .safetensors file (its directory is loaded) or a directory (SafeTensors when
 * it holds model.safetensors or its index, else its single .gguf file).  The
 * description lives until lrs_loaded_close. */
typedef struct lrs_loaded lrs_loaded;
lrs_status lrs_model_load(const char* path, uint32_t recipe, lrs_loaded** out,
                          const lrs_model_desc** desc);
void lrs_loaded_close(lrs_loaded* loaded);

#ifdef __cplusplus
}
#endif
#endif /* LLAMARS_SAFETENSORS_H */

/*
 * gfxinfer-b200 `.gfxi` artifact container (version 1).
 *
 * The on-disk format is the reference engine's (src/artifact.cpp:27-64,
 * docs/ARTIFACT_FORMAT.md): a 256-byte little-endian header, 128-byte tensor
 * directory entries, a string table of tensor names, then payloads aligned to
 * powers of two of at least 256 bytes. CRC64-ECMA (polynomial
 * 0x42F0E1EBA9EA3693, initial value 0, no reflection) covers the directory
 * plus string table, and every tensor's primary payload. Files written here
 * open with the reference's ArtifactView and the other way round.
 *
 * Recipes (identity.recipe_id) this library writes and reads:
 *  - "b200-v1": 2-D low-bit tensors in the B200 GEMV layout (gfxb.h), fp16
 *    tiled scales in the auxiliary plane; the embedding row-major with
 *    row-major fp16 scales; everything else bf16.
 *  - the reference's tiled recipes (recipe_id containing "tiled-v"): 2-D
 *    low-bit tensors in the gfx12 tiled layout (quantization.cpp:253-318),
 *    W3 only in the sequential 3-bit form ("w3seq"); repacked to the B200
 *    layout while loading.
 */
#ifndef GFXB_ARTIFACT_H
#define GFXB_ARTIFACT_H

#include <stddef.h>
#include <stdint.h>

#include "gfxb/gfxb.h"

#ifdef __cplusplus
extern "C" {
#endif

/* DType and Quantization values of the reference (artifact.h:18-34). */
enum {
  GFXB_DTYPE_U8 = 1,
  GFXB_DTYPE_I32 = 2,
  GFXB_DTYPE_F16 = 3,
  GFXB_DTYPE_BF16 = 4,
  GFXB_DTYPE_F32 = 5
};
enum {
  GFXB_QUANT_NONE = 0,
  GFXB_QUANT_W2G128 = 1,
  GFXB_QUANT_W3G128 = 2,
  GFXB_QUANT_W4G128 = 3,
  GFXB_QUANT_W8G128 = 4,
  GFXB_QUANT_FP8_ROW = 5
};

/* ArtifactIdentity (artifact.h:36-41): NUL-terminated, non-empty strings. */
typedef struct {
  char target_arch[16];
  char model_id[32];
  char weights_id[32];
  char recipe_id[64];
} gfxb_artifact_identity;

/* TensorDescriptor (artifact.h:43-56) plus host pointers into the mapping. */
typedef struct {
  const char* name; /* NUL-terminated, owned by the artifact */
  uint16_t dtype, quantization, rank, flags;
  uint32_t alignment;
  uint64_t dimensions[4];
  const void* data;
  uint64_t data_bytes;
  const void* aux; /* NULL when aux_bytes == 0 */
  uint64_t aux_bytes;
  uint64_t data_offset, aux_offset, data_crc64;
} gfxb_tensor_view;

/* TensorWriteRequest (artifact.h:58-66). alignment 0 means 256. */
typedef struct {
  const char* name;
  uint16_t dtype, quantization, rank;
  uint64_t dimensions[4];
  const void* data;
  uint64_t data_bytes;
  const void* aux;
  uint64_t aux_bytes;
  uint32_t alignment;
} gfxb_tensor_write;

typedef struct gfxb_artifact gfxb_artifact;

/* crc64_ecma_update (artifact.cpp:192-214): *out = CRC of `bytes` continued from `state`. */
int gfxb_crc64_ecma(uint64_t state, const void* bytes, size_t size, uint64_t* out);

/* ArtifactView::open (artifact.cpp:274-407): mmap + validation; with
 * verify_checksums the manifest and every payload CRC are checked. Errors:
 * GFXB_IO_ERROR (open/stat/mmap), GFXB_CORRUPT_ARTIFACT (bounds, names,
 * checksums, overlaps), GFXB_UNSUPPORTED (version, byte order). */
int gfxb_artifact_open(const char* path, int verify_checksums, gfxb_artifact** artifact);
int gfxb_artifact_close(gfxb_artifact* artifact);
int gfxb_artifact_identity_of(const gfxb_artifact* artifact, gfxb_artifact_identity* identity);
int gfxb_artifact_file_bytes(const gfxb_artifact* artifact, uint64_t* bytes);
int gfxb_artifact_tensor_count(const gfxb_artifact* artifact, size_t* count);
int gfxb_artifact_tensor_at(const gfxb_artifact* artifact, size_t index, gfxb_tensor_view* tensor);
/* Exact-name lookup (an index built at open, so names appended after a
 * sorted inventory are found too). *found = 0 when absent. */
int gfxb_artifact_find(const gfxb_artifact* artifact, const char* name, gfxb_tensor_view* tensor, int* found);

/* ArtifactWriter::write (artifact.cpp:426-562): writes a temporary file next
 * to `path`, fsyncs and renames it into place. Names must be unique, relative
 * and use [A-Za-z0-9_./-] without "..", data non-empty, rank <= 4, alignment
 * a power of two >= 256. */
int gfxb_artifact_write(const char* path, const gfxb_artifact_identity* identity, const gfxb_tensor_write* tensors,
                        size_t count);

/* ---- conversion (the reference's converter, src/converter.cpp) ---------------- */

/* One source tensor: fp32 or bf16 values in HOST memory, row-major. */
typedef struct {
  const char* name;      /* the reference tensor name (qwen38_spec.cpp:32-102) */
  uint16_t dtype;        /* GFXB_DTYPE_F32 or GFXB_DTYPE_BF16 */
  uint16_t rank;         /* 1..4 */
  uint64_t dimensions[4];
  const void* data;
  uint64_t data_bytes;
} gfxb_convert_source;

typedef struct {
  uint32_t layout;         /* GFXB_LAYOUT_B200 (recipe "b200-v1") or GFXB_LAYOUT_GFX12 (a "tiled-v" recipe) */
  uint32_t mlp_bits;       /* Qwen38ConversionOptions::mlp_bits: 2, 3 or 4 */
  uint32_t w3_start_layer; /* with mlp_bits 3, the MLPs of earlier layers are W2 */
  uint32_t w4_tail_layers; /* the MLPs of the last w4_tail_layers decoder layers are W4 */
  uint32_t head_bits;      /* lm_head.weight: 2, 3 or 4 */
  uint32_t layers;         /* decoder layers of the model */
  uint32_t chunk_rows;     /* rows converted per device step: a multiple of 16, at most 4096 */
} gfxb_convert_options;

/* convert_qwen38's plan and write (converter.cpp:98-119, 186-330, 345-393)
 * for tensors already in memory (the safetensors reader is not part of this
 * library): choose_quantization's rules pick W2/W3/W4 per 2-D tensor (N % 16
 * == 0, K % 128 == 0), other tensors are stored as bf16 (fp32 rounded to
 * nearest even); quantized tensors run through gfxb_convert_group128 on
 * `device` in chunks of chunk_rows rows and are streamed to the file with
 * fp16 scales. With GFXB_LAYOUT_B200 the embedding is stored row-major (the
 * b200-v1 recipe). The recipe id in `identity` must name the layout, and a
 * tiled recipe holding W3 tensors must name the sequential form ("w3seq"). */
int gfxb_convert_to_artifact(const char* path, const gfxb_artifact_identity* identity,
                             const gfxb_convert_source* sources, size_t count, const gfxb_convert_options* options,
                             int device);

/* ---- engine <-> artifact ---------------------------------------------------- */

typedef struct {
  uint32_t activation_bits;  /* 4 (A4) or 8 (A8) */
  uint32_t max_context;      /* KV capacity sessions may request */
  uint32_t draft_vocab;      /* MTP draft rows (0: min(98304, vocab)) */
  uint32_t include_mtp;      /* load the MTP layer (the artifact must carry it) */
  uint32_t verify_checksums; /* verify every CRC while opening */
} gfxb_artifact_load_options;

/* Engine::create from an artifact (engine.cpp:62-216): model shape from the
 * tensor shapes (qwen38_spec.cpp:32-102 naming), weights uploaded shard by
 * shard (tensor parallelism as in gfxb_engine_create_synthetic) and repacked
 * to the B200 layout when the recipe is a reference gfx12 one. */
int gfxb_engine_create_from_artifact(const char* path, const gfxb_artifact_load_options* options, int device,
                                     int tp_rank, int tp_size, const void* nccl_id128, gfxb_engine** engine);
/* The model configuration an engine was built with. */
int gfxb_engine_config(const gfxb_engine* engine, gfxb_model_config* config);
/* Writes a single-GPU engine's weights as a "b200-v1" artifact with the
 * reference tensor names (a converter from seeded random weights). */
int gfxb_engine_export_artifact(gfxb_engine* engine, const char* path, const char* weights_id);

#ifdef __cplusplus
}
#endif
#endif

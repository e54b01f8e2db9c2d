/*
 * b2loader.h -- reader of the reference engine's single-file model format
 * (the format ModelLoader parses, src/model_loader.cpp:20-68):
 *
 *   char magic[4] = "LFM2"; uint32 version; uint32 num_tensors;
 *   num_tensors x { uint32 name_len; char name[name_len]; uint32 ndim;
 *                   uint32 dims[ndim]; uint64 offset; }
 *   fp32 data of each tensor at its byte offset from the start of the file
 *   (little-endian throughout).
 *
 * The file is memory-mapped read-only; tensors are returned as pointers into
 * the mapping (zero copy; a tensor whose offset is not 4-byte aligned is
 * copied once into an aligned buffer).  Every index entry is bounds-checked
 * against the file size.  Host-only: no device work, no CUDA calls.
 */
#ifndef B2LOADER_H
#define B2LOADER_H

#include <stdint.h>

#include "b2moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2_loader b2_loader;

/* Replaces ModelLoader::ModelLoader + build_index (include/model_loader.h:11-13,
 * src/model_loader.cpp:8-60).  B2_ERR_INVALID for a missing file, a bad
 * magic, or an index that runs past the end of the file. */
b2_status b2_loader_open(const char *path, b2_loader **out);

/* Number of tensors in the index. */
int64_t b2_loader_num_tensors(const b2_loader *loader);

/* Name of tensor i (0 <= i < num_tensors) in index order, or NULL. */
const char *b2_loader_name(const b2_loader *loader, int64_t i);

/* Replaces ModelLoader::load_tensor / has_tensor / get_shape
 * (include/model_loader.h:15-22, src/model_loader.cpp:62-87): *data points
 * at the tensor's fp32 values (valid until b2_loader_close), *numel their
 * count, shape[0..*ndim) the dimensions (at most 8).  Any output may be
 * NULL.  B2_ERR_INVALID if the tensor does not exist. */
b2_status b2_loader_tensor(const b2_loader *loader, const char *name, const float **data,
                           int64_t *numel, int64_t *shape, int *ndim);

/* The weight-source callback type of include/b2lfm2.h over an open loader (ctx = the
 * b2_loader*): the tensor's data if it exists and holds `numel` values, else
 * NULL.  Lets b2_lfm2_create read a model file directly. */
const float *b2_loader_weight(void *loader, const char *name, int64_t numel);

b2_status b2_loader_close(b2_loader *loader);

#ifdef __cplusplus
}
#endif

#endif /* B2LOADER_H */

/*
 * nvfp4_loader.h -- safetensors reader of libnvfp4.so: NVFP4 checkpoints
 * straight into device memory (the reference's nvfp4/weight_loader.mojo,
 * safetensors part, restated in C++ with a direct host -> device upload).
 *
 * The reference reads each tensor into a host List[UInt8] and leaves the
 * copy to the device to the caller (nvfp4/weight_loader.mojo:614-675).  Here
 * a tensor is read from the file through pinned staging buffers (two of
 * 32 MiB; the read of one, split over four threads, overlaps the copy of the
 * other) into caller-owned device memory.
 * Handles are not thread-safe: use one handle from one thread at a time.
 * Conventions as in nvfp4.h (0 or a negative nvfp4_status, message in
 * nvfp4_last_error_string()).
 */
#ifndef NVFP4_LOADER_H
#define NVFP4_LOADER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nvfp4_st_file nvfp4_st_file;   /* one opened .safetensors file */
typedef struct nvfp4_st_model nvfp4_st_model; /* the shards of a model directory */

/* struct TensorInfo (nvfp4/weight_loader.mojo:190-238). */
typedef struct nvfp4_st_tensor_info {
  char dtype[16];       /* "U8", "F8_E4M3", "F32", "BF16", ... ("" if absent) */
  int32_t ndim;         /* 0 for a scalar or a missing shape */
  int64_t shape[8];
  int64_t data_offset;  /* bytes from the start of the data region */
  int64_t data_size;    /* data_offsets[1] - data_offsets[0] (0 if absent) */
} nvfp4_st_tensor_info;

/*
 * Replaces open_safetensors (nvfp4/weight_loader.mojo:366-410) and
 * _parse_safetensors_header (:292-363): 8-byte little-endian header size
 * (0 < size <= file size - 8, else NVFP4_ERR_INVALID_ARG), JSON header of
 * name -> {dtype, shape, data_offsets}; `__metadata__` is skipped; tensors
 * keep the header's order.  Stricter than the reference: malformed JSON and
 * data offsets outside the file are errors.
 */
int nvfp4_st_open(const char *path, nvfp4_st_file **out);
void nvfp4_st_close(nvfp4_st_file *file);
int64_t nvfp4_st_num_tensors(const nvfp4_st_file *file);
/* Name of tensor i (owned by the handle), NULL if i is out of range. */
const char *nvfp4_st_tensor_name(const nvfp4_st_file *file, int64_t i);
/* find_tensor (:269-274): index of the first tensor of that name, or -1. */
int64_t nvfp4_st_find(const nvfp4_st_file *file, const char *name);
int nvfp4_st_get_tensor_info(const nvfp4_st_file *file, int64_t i, nvfp4_st_tensor_info *out);
/*
 * read_tensor_into (:285-289) into host memory: the tensor's bytes into dst
 * (capacity cap bytes, at least data_size); returns the bytes read or a
 * negative status.
 */
int64_t nvfp4_st_read_host(const nvfp4_st_file *file, int64_t i, void *dst, int64_t cap);
/*
 * The tensor's bytes into device memory dst (data_size bytes), copied on
 * `stream` through the file's pinned staging buffers; returns once the
 * copies have completed.
 */
int nvfp4_st_read_device(nvfp4_st_file *file, int64_t i, void *dst, void *stream);

/*
 * Replaces _read_f32_from_bytes (:678-700): the first 4 bytes of buf as a
 * little-endian float32, with the reference's rules: fewer than 4 bytes ->
 * 1.0; exponent field 0 (zero and subnormals) -> +-0.0; exponent field 255
 * (inf, NaN) -> 1.0; every other value exactly.
 */
float nvfp4_st_f32_from_bytes(const uint8_t *buf, int64_t len);

/*
 * Replaces discover_safetensor_shards / open_model_shards (:909-954):
 * `model_dir/model.safetensors` if it exists, else the shards
 * `model-NNNNN-of-TTTTT.safetensors`, i = 1, 2, ... up to the first missing
 * one, TTTTT taken from shard 1 (the smallest total that has a shard 1).
 * Differs from the reference where the reference stops early: its probe
 * loop finds only shard 1 of a model with three or more shards (after the
 * first hit it tries total = i only) and starts from shard 2 when shard 1 is
 * missing; here every shard of the set is opened and a missing shard 1 is an
 * error.
 */
int nvfp4_st_open_model(const char *model_dir, nvfp4_st_model **out);
/* A shard set from an explicit list of files (opened in that order); one
 * file gives the single-file form open_safetensors returns. */
int nvfp4_st_open_files(const char *const *paths, int32_t n, nvfp4_st_model **out);
void nvfp4_st_close_model(nvfp4_st_model *model);
int32_t nvfp4_st_model_num_shards(const nvfp4_st_model *model);
const char *nvfp4_st_model_shard_path(const nvfp4_st_model *model, int32_t shard);
nvfp4_st_file *nvfp4_st_model_shard(nvfp4_st_model *model, int32_t shard);
/* _find_load_raw (:839-847): first shard holding `name`; -1 if none. */
int nvfp4_st_model_find(const nvfp4_st_model *model, const char *name, int32_t *shard,
                        int64_t *index);

/* What load_linear_safetensors (:703-760) finds for `prefix`. */
typedef struct nvfp4_st_linear_info {
  int64_t out_features;     /* shape[0] of {prefix}.weight */
  int64_t in_features;      /* 2 * shape[1] */
  float weight_scale_2;     /* first value of {prefix}.weight_scale_2 (f32 rules), 1.0 if absent */
  float input_scale;        /* {prefix}.input_scale (f32 rules), 1.0 if absent */
  int32_t weight_scale_2_rows;  /* nonzero: weight_scale_2 holds one F32 per output row */
  int32_t shard;            /* shard holding {prefix}.weight */
} nvfp4_st_linear_info;

/*
 * _find_load_linear (:828-836) + load_linear_safetensors (:703-760): the
 * first shard with {prefix}.weight, {prefix}.weight_scale from the same
 * shard (both required), weight at least 2-D with data_size = out * in/2,
 * weight_scale data_size = out * (in/16), else NVFP4_ERR_INVALID_ARG.
 */
int nvfp4_st_get_linear_info(const nvfp4_st_model *model, const char *prefix,
                             nvfp4_st_linear_info *out);

#define NVFP4_ST_FOLD_INPUT_SCALE 0x1u  /* weight_scale_2_rows *= input_scale */

/*
 * Loads one linear into device memory: packed_weights [out, in/2],
 * blockscales [out, in/16] and, if weight_scale_2_rows is non-NULL, fp32
 * [out] per-row second-level scales (the per-row tensor, or the scalar
 * repeated; each value by the f32 rules above), times input_scale with
 * NVFP4_ST_FOLD_INPUT_SCALE (one fp32 product, as the kernels form alpha).
 */
int nvfp4_st_load_linear(nvfp4_st_model *model, const char *prefix, uint8_t *packed_weights,
                         uint8_t *blockscales, float *weight_scale_2_rows, uint32_t flags,
                         void *stream);

/*
 * Experts [first, first + count) of `layer_prefix` (e.g. "model.layers.3")
 * into the stacked layout of nvfp4_moe_weights: gate_up rows [e * 2I, e * 2I
 * + I) from `.mlp.experts.{e}.gate_proj`, [e * 2I + I, (e + 1) * 2I) from
 * `.up_proj`, down rows [e * H, (e + 1) * H) from `.down_proj`
 * (nvfp4/weight_loader.mojo:770-771, :875-878); each linear's input_scale is
 * folded into its rows' weight_scale_2, so the expert input scales are 1.
 * shared != 0 loads `.mlp.shared_expert.*` instead (count must be 1;
 * :881-884).  All experts must have the same shapes.
 */
int nvfp4_st_load_experts(nvfp4_st_model *model, const char *layer_prefix, int32_t first,
                          int32_t count, int32_t shared, uint8_t *gate_up,
                          uint8_t *gate_up_scale, float *gate_up_scale_2, uint8_t *down,
                          uint8_t *down_scale, float *down_scale_2, void *stream);

/*
 * The router `{layer_prefix}.mlp.gate.weight` (:769, :887; BF16 [E, H], or F32)
 * as the fp32 [H, E] matrix nvfp4_moe_weights.router takes; E and H are
 * returned through num_experts / hidden when non-NULL.  router_out NULL: only
 * the shape is returned.
 */
int nvfp4_st_load_router(nvfp4_st_model *model, const char *layer_prefix, float *router_out,
                         int32_t *num_experts, int32_t *hidden, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_LOADER_H */

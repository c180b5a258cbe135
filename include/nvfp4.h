/*
 * nvfp4.h -- C ABI of libnvfp4.so, the B200 (sm_100a) NVFP4 kernels.
 *
 * This is the drop-in boundary for the reference's NVFP4 hot path
 * (MikkoParkkola/nvfp4-mojo).  The reference's Mojo host code would bind
 * these symbols with external_call / DLHandle, the same FFI style its
 * safetensors loader uses for libc (nvfp4/weight_loader.mojo:51-73).
 *
 * Conventions (all entry points):
 *   - Every buffer is a DEVICE pointer owned by the caller; nothing is
 *     retained after return (nvfp4/config.mojo:64-69: "weight pointers are
 *     passed to forward functions separately").
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Work is enqueued asynchronously on it; no hidden streams.
 *   - Return 0 on success or a negative nvfp4_status; never exit/abort.
 *     nvfp4_last_error_string() describes the last failure of this thread
 *     (the reference raises a Mojo Error with a message instead).
 *   - There is no CPU fallback: every compute entry point launches CUDA
 *     kernels built for sm_100a.
 *
 * Layout (nvfp4/config.mojo:13-35, nvfp4/weight_loader.mojo:614-760):
 *   packed weight  uint8  [out_features, in_features/2], low nibble = even k
 *   blockscales    e4m3fn [out_features, in_features/16] (raw bytes)
 *   weight_scale_2 fp32 scalar (reference) or per-row [out_features]
 *   input_scale    fp32 scalar
 *   value(n, k) = LUT[code] * float(blockscale); y = alpha * sum_k value * x
 *   with alpha = input_scale * weight_scale_2 (nvfp4/config.mojo:93-95).
 * Naming: M = tokens, N = out_features, K = in_features.
 */
#ifndef NVFP4_H
#define NVFP4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4_ABI_VERSION 1

/* nvfp4/config.mojo:13-14 */
#define NVFP4_GROUP_SIZE 16
#define NVFP4_PACK_FACTOR 2

typedef enum nvfp4_status {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID_ARG = -1, /* null pointer, bad shape, misalignment */
  NVFP4_ERR_UNSUPPORTED = -2, /* valid request this build does not serve */
  NVFP4_ERR_CUDA = -3,        /* a CUDA runtime call or launch failed */
  NVFP4_ERR_WORKSPACE = -4,   /* caller workspace too small */
  NVFP4_ERR_TIMEOUT = -5,     /* a bounded device wait gave up */
} nvfp4_status;

typedef enum nvfp4_dtype {
  NVFP4_DTYPE_F32 = 0,
  NVFP4_DTYPE_BF16 = 1,
} nvfp4_dtype;

/* Flags of nvfp4_linear_forward. */
#define NVFP4_FLAG_W4A4 0x1u         /* quantize activations with input_scale, FP4 MMA */
#define NVFP4_FLAG_FORCE_SKINNY 0x2u /* dispatch override (tests/bench): decode GEMV path */
#define NVFP4_FLAG_FORCE_TC 0x4u     /* dispatch override (tests/bench): tcgen05 GEMM path */
#define NVFP4_FLAG_FORCE_F32 0x8u    /* dispatch override: CUDA-core fp32 path */

/*
 * Mirrors struct NvFp4Linear (nvfp4/config.mojo:64-103): in/out features,
 * scalar input_scale and weight_scale_2 (default 1.0, :78-79).  The optional
 * device array weight_scale_2_rows [out_features] replaces the scalar per
 * output row (per-row second-level scales); NULL keeps the reference scalar.
 */
typedef struct nvfp4_linear_desc {
  int64_t in_features;
  int64_t out_features;
  float input_scale;
  float weight_scale_2;
  const float *weight_scale_2_rows;
} nvfp4_linear_desc;

/* ABI version (NVFP4_ABI_VERSION of the built library). */
int nvfp4_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char *nvfp4_last_error_string(void);

/*
 * Status word of the tensor-core kernels, read (synchronously) and cleared:
 * 0 = no failure; > 0 = a kernel abandoned a bounded wait (1 TMA stage,
 * 2 decoded operands, 3 stage release, 4 accumulator) and returned early,
 * its output then being undefined; < 0 = the status could not be read.
 * No reference counterpart (the reference has no GPU kernel that runs).
 */
int nvfp4_device_status(void);

/*
 * Replaces nvfp4_linear_forward (nvfp4/nvfp4_gemm_gpu.mojo:185-224), whose
 * launch the reference leaves as a placeholder (:219-224).
 * activations [batch_seq_len, in_features] (act_dtype bf16 or f32), output
 * [batch_seq_len, out_features] (out_dtype bf16 or f32): token-major, as the
 * reference's docstring states (:203-206).
 * Dispatch: M <= 64 tokens -> tensor-core decode GEMV (HBM-bound), larger M ->
 * tcgen05 W4A16 GEMM; fp32 activations with M <= 8 -> the CUDA-core fp32 path
 * (nvfp4_matvec arithmetic).  NVFP4_FLAG_W4A4 -> block-scaled FP4 MMA.
 */
int nvfp4_linear_forward(const nvfp4_linear_desc *linear, const uint8_t *packed_weights,
                         const uint8_t *blockscales, const void *activations,
                         int act_dtype, void *output, int out_dtype,
                         int64_t batch_seq_len, uint32_t flags, void *stream);

/*
 * Replaces nvfp4_gemm_kernel (nvfp4/nvfp4_gemm_gpu.mojo:99-182) in the
 * reference kernel's own layout: activations K-major [K, N_tok], output
 * [M_out, N_tok]; out = alpha * dequant(W[M_out, K/2]) @ act (fp32 accumulate).
 * (Reference naming here: M_out = out_features, N_tok = tokens.)
 */
int nvfp4_gemm_kernel(int64_t M_out, int64_t N_tok, int64_t K,
                      const uint8_t *packed_weights, const uint8_t *blockscales,
                      const void *activations, int act_dtype, void *output,
                      int out_dtype, float alpha, void *stream);

/*
 * Replaces nvfp4_matvec (nvfp4/deltanet.mojo:549-584): result[out] =
 * alpha * dequant(W) @ input_vec[in], fp32 in, fp32 out, fp32 accumulation.
 */
int nvfp4_matvec(const nvfp4_linear_desc *linear, const uint8_t *packed_weights,
                 const uint8_t *blockscales, const float *input_vec, float *result,
                 void *stream);

/*
 * Replaces load_and_dequant_fp4_tile (nvfp4/nvfp4_gemm_gpu.mojo:44-96):
 * out[m * tile_k + k] (fp32) = LUT[code(start_row+m, start_col+k)] * float(scale).
 */
int nvfp4_dequant_tile(const uint8_t *packed_weights, const uint8_t *blockscales,
                       float *output, int64_t weight_stride, int64_t scale_stride,
                       int64_t start_row, int64_t start_col, int64_t tile_m,
                       int64_t tile_k, void *stream);

/*
 * Whole-matrix dequant (dequant_fp4 over every element, nvfp4/config.mojo:
 * 117-135): out [rows, K] fp32, or bf16 (exact: E2M1 x E4M3 fits bf16).
 * The bf16 form runs the same decode the tensor-core kernels feed their MMAs.
 */
int nvfp4_dequant(const uint8_t *packed_weights, const uint8_t *blockscales, int64_t rows,
                  int64_t K, void *output, int out_dtype, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* NVFP4_H */

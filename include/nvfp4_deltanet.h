/*
 * nvfp4_deltanet.h -- gated DeltaNet decode step of libnvfp4.so with NVFP4
 * projections (the reference's deltanet_forward, nvfp4/deltanet.mojo:335-546,
 * with its fp32 weight matrices replaced by NVFP4 linears as nvfp4_matvec,
 * :549-584, computes them).
 *
 * One call advances B independent sequences by one token: the five
 * projections (qkv, z, beta, alpha, out) run on the NVFP4 linear path of
 * nvfp4.h (decode GEMV for B <= 8), the causal conv1d + SiLU and the
 * per-head recurrence (decay, delta rule, state update, output, RMS norm,
 * SiLU gate) in CUDA kernels, the state staying in device memory.
 * Conventions as in nvfp4.h: device pointers owned by the caller, 0 or a
 * negative nvfp4_status, work enqueued on `stream`.
 */
#ifndef NVFP4_DELTANET_H
#define NVFP4_DELTANET_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* struct DeltaNetConfig (nvfp4/deltanet.mojo:87-178). */
typedef struct nvfp4_deltanet_desc {
  int32_t d_model;          /* multiple of 16 */
  int32_t num_key_heads;
  int32_t num_value_heads;  /* a multiple of num_key_heads */
  int32_t key_dim;          /* <= 256 */
  int32_t value_dim;        /* a power of two, 4 .. 256 */
  int32_t conv_kernel;      /* 1 .. 8 */
  float rms_eps;
} nvfp4_deltanet_desc;

/* One NVFP4 projection [out_features, in_features] in the layout of nvfp4.h. */
typedef struct nvfp4_deltanet_proj {
  const uint8_t *packed_weights;      /* [out, in/2] */
  const uint8_t *blockscales;         /* [out, in/16] e4m3 */
  float input_scale;
  float weight_scale_2;
  const float *weight_scale_2_rows;   /* [out] or NULL */
} nvfp4_deltanet_proj;

/* The arguments of deltanet_forward (:335-352), projections in NVFP4. */
typedef struct nvfp4_deltanet_weights {
  nvfp4_deltanet_proj qkv;  /* [2 nkh kd + nvh vd, d_model] */
  nvfp4_deltanet_proj z;    /* [nvh vd, d_model] */
  nvfp4_deltanet_proj b;    /* [nvh, d_model] (beta) */
  nvfp4_deltanet_proj a;    /* [nvh, d_model] (alpha) */
  nvfp4_deltanet_proj out;  /* [d_model, nvh vd] */
  /* Optional (packed_weights NULL: unused): the rows of qkv, z, b and a
   * concatenated in that order, one NVFP4 matrix [2 nkh kd + 2 nvh vd +
   * 2 nvh, d_model] with one input_scale (nvfp4_stack_rows builds it); one
   * projection launch instead of four.  qkv, z, b, a are then ignored. */
  nvfp4_deltanet_proj in_proj;
  const float *a_log;       /* [nvh] */
  const float *dt_bias;     /* [nvh] */
  const float *conv_q, *conv_k, *conv_v;                /* [dim, conv_kernel] */
  const float *conv_bias_q, *conv_bias_k, *conv_bias_v; /* [dim] each, or all NULL */
} nvfp4_deltanet_weights;

/* struct DeltaNetState (:181-218) for B sequences, fp32, updated in place. */
typedef struct nvfp4_deltanet_state {
  float *s;       /* [B, nvh, kd, vd] */
  float *conv_q;  /* [B, nkh kd, conv_kernel - 1], oldest first */
  float *conv_k;  /* [B, nkh kd, conv_kernel - 1] */
  float *conv_v;  /* [B, nvh vd, conv_kernel - 1] */
} nvfp4_deltanet_state;

size_t nvfp4_deltanet_workspace_size(const nvfp4_deltanet_desc *desc, int64_t B);

/*
 * deltanet_forward for B sequences: hidden [B, d_model] (hidden_dtype bf16
 * or f32) -> output [B, d_model] (out_dtype).  proj_dtype chooses the
 * activations the projections take: NVFP4_DTYPE_F32 keeps the reference's
 * fp32 arithmetic (the CUDA-core fp32 linear path), NVFP4_DTYPE_BF16 rounds
 * the hidden state and the gated output to bf16 and takes the decode GEMV.
 * The recurrence is fp32 either way.  Workspace: 256-byte aligned, at least
 * nvfp4_deltanet_workspace_size(desc, B) bytes.
 */
int nvfp4_deltanet_forward(const nvfp4_deltanet_desc *desc, const nvfp4_deltanet_weights *w,
                           const void *hidden, int hidden_dtype, void *output, int out_dtype,
                           int64_t B, const nvfp4_deltanet_state *state, int proj_dtype,
                           void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_DELTANET_H */

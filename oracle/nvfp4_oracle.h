/*
 * nvfp4_oracle.h -- CPU restatement of the reference's NVFP4 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code: it is the checker that tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference leg compare the CUDA path with.
 *
 * Parity status (what pins this restatement):
 *   - LUT, nibble pack/unpack, scalar dequant and config constants are pinned
 *     by the reference's own known-answer tests (tests/test_nvfp4.mojo:44-115),
 *     re-stated as golden vectors in tests/golden/reference_kats.json.
 *   - sigmoid / silu are pinned by tests/test_deltanet.mojo:65-76.
 *   - E4M3 decoding is pinned against ml_dtypes' float8_e4m3fn on all 256
 *     codes (tests/golden/e4m3_table.json).
 *   - The matvec / GEMM loop (nvfp4/deltanet.mojo:549-584) has NO reference
 *     test or fixture: it is a loop-order-faithful restatement, cross-checked
 *     against an independent numpy float64 evaluation.  "GEMM parity pinned at
 *     the helper level only".
 *   - The MoE layer and the W4A4 activation quantizer have no counterpart in
 *     the reference at all: their semantics are defined here (parity unpinned).
 *
 * Naming: M = tokens, N = out_features, K = in_features, except where a
 * function mirrors a reference function whose names differ.
 */
#ifndef NVFP4_ORACLE_H
#define NVFP4_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* nvfp4/config.mojo:13-14 */
#define ORACLE_GROUP_SIZE 16
#define ORACLE_PACK_FACTOR 2

/* nvfp4/config.mojo:18-35 */
float oracle_lut(int code);
/* nvfp4/config.mojo:106-114 */
void oracle_unpack_fp4_pair(uint8_t packed, uint8_t *lo, uint8_t *hi);
/* nvfp4/config.mojo:138-140 */
uint8_t oracle_pack_fp4_pair(uint8_t lo, uint8_t hi);
/* nvfp4/config.mojo:117-121 */
float oracle_dequant_fp4(uint8_t v, float scale);
/* nvfp4/config.mojo:143-149 */
float oracle_compute_effective_scale(float blockscale, float ws2, float input_scale);
/* Float8_e4m3fn -> Float32 cast used at nvfp4/deltanet.mojo:574-576 (OCP FP8 E4M3FN). */
float oracle_e4m3_to_f32(uint8_t b);
/* Float32 -> E4M3FN, round-to-nearest-even, saturating to +-448 (NaN stays NaN). */
uint8_t oracle_f32_to_e4m3_satfinite(float x);
/* Float32 -> E2M1 code, round-to-nearest-even, saturating to +-6. */
uint8_t oracle_f32_to_e2m1_satfinite(float x);
/* bf16 <-> f32 helpers (bf16 -> f32 is exact; f32 -> bf16 is RNE). */
float oracle_bf16_to_f32(uint16_t b);
uint16_t oracle_f32_to_bf16(float x);

/* nvfp4/deltanet.mojo:66-80 */
float oracle_sigmoid(float x);
float oracle_silu(float x);

/*
 * nvfp4/nvfp4_gemm_gpu.mojo:44-96 (load_and_dequant_fp4_tile):
 * out[m*tile_k + k] = LUT[nib(start_row+m, start_col+k)] * float(sf[...]).
 */
void oracle_dequant_tile(const uint8_t *packed, const uint8_t *scales, float *out,
                         int64_t weight_stride, int64_t scale_stride,
                         int64_t start_row, int64_t start_col,
                         int64_t tile_m, int64_t tile_k);

/*
 * nvfp4/deltanet.mojo:549-584 (nvfp4_matvec), loop-order faithful: for each
 * output row, fp32 sequential sum over k of LUT*float(sf)*x[k], then *alpha.
 * alpha_n = input_scale * (ws2_rows ? ws2_rows[n] : ws2).  With ws2_rows ==
 * NULL this is exactly the reference (scalar weight_scale_2, config.mojo:93-95).
 */
void oracle_matvec(int64_t K, int64_t N, float input_scale, float ws2,
                   const float *ws2_rows, const uint8_t *packed,
                   const uint8_t *scales, const float *x, float *y);

/*
 * Token-major linear (nvfp4/nvfp4_gemm_gpu.mojo:185-206 docstring layout):
 * y[m, n] for m < M, one oracle_matvec per token row.  `rows`/`cols`, when
 * non-NULL, restrict the work to n_rows tokens x n_cols outputs (sampled
 * checking of large shapes); y is then [n_rows, n_cols].
 * n_threads > 1 parallelises over output rows with OpenMP (timing only).
 */
void oracle_linear(int64_t M, int64_t K, int64_t N, float input_scale, float ws2,
                   const float *ws2_rows, const uint8_t *packed,
                   const uint8_t *scales, const float *x, float *y,
                   const int64_t *rows, int64_t n_rows,
                   const int64_t *cols, int64_t n_cols, int n_threads);

/*
 * nvfp4/nvfp4_gemm_gpu.mojo:99-182 (nvfp4_gemm_kernel) in the reference's
 * own layout: out[M_out, N_tok] = alpha * dequant(W[M_out, K/2]) @ act[K, N_tok].
 */
void oracle_gemm_kernel(int64_t M_out, int64_t N_tok, int64_t K,
                        const uint8_t *packed, const uint8_t *scales,
                        const float *act_kmajor, float *out, float alpha);

/*
 * W4A4 activation quantizer (no reference counterpart; NVFP4 convention):
 * per 16-element group g of row m, amax -> sf = e4m3(amax / (6*input_scale)),
 * q = e2m1(x / (float(sf) * input_scale)); codes packed low nibble = even k.
 */
void oracle_quantize_act(int64_t M, int64_t K, const float *x, float input_scale,
                         uint8_t *q_packed, uint8_t *q_scales);

/*
 * One MoE FFN layer (no reference counterpart).  router [H, E] fp32,
 * logits = x @ router (fp32, sequential h), softmax over E, top-k with ties
 * to the lower expert index, optional renormalisation, then per selected
 * expert: h = gate_up(x) [2I] (oracle_matvec), a = silu(h[:I]) * h[I:],
 * y_e = down(a) [H], out = sum_j w_j * y_e_j (j in selection order).
 * Expert weights are stacked: gate_up [E, 2I, H/2] / [E, 2I, H/16] / ws2 [E, 2I],
 * down [E, H, I/2] / [E, H, I/16] / ws2 [E, H]; input scales per expert.
 * `tokens` (optional) restricts the work to n_tok selected tokens, out is
 * then [n_tok, H].  topk_ids/topk_w (optional) receive the routing
 * decisions [n_tok, k].  force_ids (optional, [n_tok, k]) overrides the
 * selection (used to replay the GPU's choice on near-ties).
 */
void oracle_moe(int64_t T, int64_t H, int64_t I, int64_t E, int64_t top_k,
                int renormalize, const float *x, const float *router,
                const uint8_t *gu_w, const uint8_t *gu_sf, const float *gu_ws2,
                const float *gu_in_scale, const uint8_t *dn_w,
                const uint8_t *dn_sf, const float *dn_ws2,
                const float *dn_in_scale, float *out,
                const int64_t *tokens, int64_t n_tok, int32_t *topk_ids,
                float *topk_w, const int32_t *force_ids, int n_threads);

/* Router only: fp32 logits [T, E] and softmax probabilities [T, E]. */
void oracle_router(int64_t T, int64_t H, int64_t E, const float *x,
                   const float *router, float *logits, float *probs);

/* Gated DeltaNet decode step (nvfp4/deltanet.mojo:51-542), fp32.  Shapes:
 * hidden/out [d]; w_qkv [(2 nkh kd + nvh vd), d]; w_z [nvh vd, d]; w_b, w_a
 * [nvh, d]; w_out [d, nvh vd]; a_log, dt_bias [nvh]; conv weights [dim,
 * conv_k]; conv biases [dim] or NULL; state s_matrix [nvh, kd, vd] and conv
 * windows [dim, conv_k - 1], both updated in place. */
float oracle_softplus(float x);
void oracle_dn_matvec(const float *mat, const float *vec, float *result, int64_t rows,
                      int64_t cols);
void oracle_dn_matvec_t(const float *mat, const float *vec, float *result, int64_t rows,
                        int64_t cols);
void oracle_rms_norm(float *x, int64_t n, float eps);
void oracle_conv1d_step(const float *new_input, float *buf, const float *w, float *result,
                        int64_t channels, int64_t kernel, const float *bias);
void oracle_deltanet_forward(int64_t d, int64_t nkh, int64_t nvh, int64_t kd, int64_t vd,
                             int64_t conv_k, float eps, const float *hidden, float *out,
                             const float *w_qkv, const float *w_z, const float *w_b,
                             const float *w_a, const float *w_out, const float *a_log,
                             const float *dt_bias, const float *wc_q, const float *wc_k,
                             const float *wc_v, const float *cb_q, const float *cb_k,
                             const float *cb_v, float *s_matrix, float *buf_q, float *buf_k,
                             float *buf_v);

#ifdef __cplusplus
}
#endif
#endif

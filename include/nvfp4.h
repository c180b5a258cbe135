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
#define NVFP4_FLAG_TS_GEMV 0x10u /* M <= 8 on the tcgen05 decode GEMV (decoded weights in
                                    tensor memory) instead of the mma.sync one */
#define NVFP4_FLAG_DIGIT_GEMV 0x20u /* M <= 8: activations as four NVFP4 digits, weights as
                                       stored into block-scaled FP4 MMAs (~5e-4 x RMS of the
                                       bf16-operand result; K <= 16384) */

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
 * 2 decoded operands or blockscales, 3 stage release, 4 accumulator) or
 * found its share of the work larger than its launch was sized for (5) and
 * returned early,
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
 * Dispatch: M <= 8 tokens -> decode GEMV, M <= 64 -> tensor-core skinny GEMM
 * (both HBM-bound), larger M -> tcgen05 W4A16 GEMM; fp32 activations -> the
 * CUDA-core fp32 path (nvfp4_matvec arithmetic).  NVFP4_FLAG_W4A4 -> the
 * activations are quantized to NVFP4 with input_scale (nvfp4_quantize_act,
 * into stream-ordered scratch from cudaMallocAsync) and multiplied on the
 * block-scaled FP4 tensor cores (nvfp4_linear_w4a4); in_features % 256 == 0.
 * The decode GEMV is launched with programmatic dependent launch and starts
 * reading the weights, blockscales and weight_scale_2 before the preceding
 * kernel in the stream has finished (activations and output only after it):
 * do not write those weight buffers with the kernel launched immediately
 * before this call on the same stream.
 */
int nvfp4_linear_forward(const nvfp4_linear_desc *linear, const uint8_t *packed_weights,
                         const uint8_t *blockscales, const void *activations,
                         int act_dtype, void *output, int out_dtype,
                         int64_t batch_seq_len, uint32_t flags, void *stream);

/*
 * W4A4 activation quantizer (no reference counterpart: the reference stores
 * input_scale, nvfp4/weight_loader.mojo:713-758, but never quantizes
 * activations).  x [M, K] (x_dtype bf16 or f32, row stride x_ld elements,
 * 16-byte aligned rows) -> codes [M, K/2] (E2M1, low nibble = even k) and
 * blockscales [M, K/16] (E4M3): per 16-group, sf = e4m3(amax / (6 *
 * input_scale)), code = e2m1(x / (float(sf) * input_scale)), both
 * round-to-nearest-even with saturation; a zero scale gives zero codes.
 */
int nvfp4_quantize_act(const void *x, int x_dtype, int64_t M, int64_t K, int64_t x_ld,
                       float input_scale, uint8_t *codes, uint8_t *scales, void *stream);

/*
 * W4A4 GEMM on the block-scaled FP4 tensor cores (tcgen05 kind::mxf4nvf4):
 * y[M, N] = input_scale * weight_scale_2[n] * sum_k W~[n, k] * X~[m, k],
 * W~ / X~ = e2m1 code * e4m3 blockscale of the weights / of the activations
 * from nvfp4_quantize_act; fp32 accumulation; y token-major (bf16 or f32).
 * in_features % 256 == 0; all buffers 16-byte aligned.
 */
int nvfp4_linear_w4a4(const nvfp4_linear_desc *linear, const uint8_t *packed_weights,
                      const uint8_t *blockscales, const uint8_t *act_codes,
                      const uint8_t *act_scales, void *output, int out_dtype, int64_t M,
                      void *stream);

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

/* ------------------------------------------------------------------------
 * MoE expert path.  No counterpart in the reference, which only defines the
 * per-expert NVFP4 weight layout (nvfp4/weight_loader.mojo:767-793,
 * :873-887: expert gate/up/down linears and the router `mlp.gate.weight`)
 * and SiLU (nvfp4/deltanet.mojo:66-80).  Experts are stacked: expert e's
 * fused gate_up linear is rows [e*2I, (e+1)*2I) (gate rows first, then up),
 * its down linear rows [e*H, (e+1)*H); each in the layout above.
 * ---------------------------------------------------------------------- */
typedef struct nvfp4_moe_desc {
  int32_t num_experts;   /* E (local experts, <= 256) */
  int32_t top_k;         /* k (<= 32) */
  int32_t hidden;        /* H (multiple of 128) */
  int32_t intermediate;  /* I (multiple of 128) */
  int32_t renormalize;   /* nonzero: the k routing weights are renormalised to sum 1 */
} nvfp4_moe_desc;

typedef struct nvfp4_moe_weights {
  const float *router;                /* [H, E] fp32 (logits = x @ router) */
  const uint8_t *gate_up;             /* [E, 2I, H/2] packed E2M1 */
  const uint8_t *gate_up_scale;       /* [E, 2I, H/16] e4m3 */
  const float *gate_up_scale_2;       /* [E, 2I] fp32, or NULL (1.0) */
  const float *gate_up_input_scale;   /* [E] fp32, or NULL (1.0) */
  const uint8_t *down;                /* [E, H, I/2] */
  const uint8_t *down_scale;          /* [E, H, I/16] */
  const float *down_scale_2;          /* [E, H], or NULL */
  const float *down_input_scale;      /* [E], or NULL */
} nvfp4_moe_weights;

/* Bytes of caller-provided device workspace nvfp4_moe_forward needs for T tokens. */
size_t nvfp4_moe_workspace_size(const nvfp4_moe_desc *desc, int64_t T);
/* Bytes of workspace nvfp4_moe_experts needs for R rows. */
size_t nvfp4_moe_experts_workspace_size(const nvfp4_moe_desc *desc, int64_t R);

/*
 * One MoE FFN layer: y[T, H] = sum_j w_j * expert_{e_j}(x) (+ residual if
 * non-NULL, bf16 [T, H]); x bf16 [T, H]; y bf16 or fp32 (y_dtype).
 * Workspace: device memory of at least nvfp4_moe_workspace_size() bytes,
 * 256-byte aligned, owned by the caller; its contents on entry do not
 * matter.  If topk_ids / topk_w are non-NULL they receive the routing
 * decisions (int32 / fp32 [T, k]).
 */
int nvfp4_moe_forward(const nvfp4_moe_desc *desc, const nvfp4_moe_weights *weights,
                      const void *x, const void *residual, void *y, int y_dtype, int64_t T,
                      int32_t *topk_ids, float *topk_w, void *workspace,
                      size_t workspace_bytes, void *stream);

/*
 * No counterpart in the reference.  nvfp4_moe_forward for callers that cannot
 * allocate device memory: a caller with no device allocator of its own (such
 * as foreign-function host code that only holds the pointers it was given) or
 * a serving loop that must not call cudaMalloc once it runs (it synchronises
 * the device and is not allowed during stream capture).  The workspace is a
 * static device array of NVFP4_NOALLOC_SCRATCH_BYTES inside the library,
 * which every GPU that loads the library holds until the process exits; the
 * call allocates nothing.  Layers whose workspace would exceed it
 * (nvfp4_moe_workspace_size(desc, T) > NVFP4_NOALLOC_SCRATCH_BYTES) are
 * rejected with NVFP4_ERR_WORKSPACE.  The first call on each device looks up
 * the array's device address (with that device current): make it before any
 * stream capture.  All calls on a device share the array, so calls that
 * overlap on the GPU race and must be serialised by the caller; nothing in it
 * has to start at zero.  Arguments as nvfp4_moe_forward, minus the workspace.
 */
#define NVFP4_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int nvfp4_moe_forward_noalloc(const nvfp4_moe_desc *desc, const nvfp4_moe_weights *weights,
                              const void *x, const void *residual, void *y, int y_dtype,
                              int64_t T, int32_t *topk_ids, float *topk_w, void *stream);

/*
 * Shared expert.  The reference loads it
 * (`model.layers.{l}.mlp.shared_expert.{gate,up,down}_proj`,
 * nvfp4/weight_loader.mojo:771, :788-790, :881-884) but computes nothing with
 * it.  nvfp4_moe_forward_shared is nvfp4_moe_forward plus one always-on
 * expert: y = sum_j w_j * expert_{e_j}(x) + shared(x) (+ residual), the
 * shared expert's output added with weight 1 after the routed sum.  `shared`
 * describes a one-expert stack (E = 1) in the layout above, gate_up rows
 * [0, 2*shared_intermediate), down rows [0, H); its router is ignored.  The
 * workspace is nvfp4_moe_shared_workspace_size() bytes (more than
 * nvfp4_moe_workspace_size: the shared expert's rows and fp32 output).
 */
size_t nvfp4_moe_shared_workspace_size(const nvfp4_moe_desc *desc, int32_t shared_intermediate,
                                       int64_t T);
int nvfp4_moe_forward_shared(const nvfp4_moe_desc *desc, const nvfp4_moe_weights *weights,
                             const nvfp4_moe_weights *shared, int32_t shared_intermediate,
                             const void *x, const void *residual, void *y, int y_dtype,
                             int64_t T, int32_t *topk_ids, float *topk_w, void *workspace,
                             size_t workspace_bytes, void *stream);

/*
 * Row-concatenation prepack: dst = srcs[0] rows ++ srcs[1] rows ++ ..., each
 * source rows[i] rows of row_bytes bytes (device or host memory; one
 * stream-ordered copy per source).  Turns the reference's separate per-expert
 * gate_proj / up_proj linears (nvfp4/weight_loader.mojo:876-877) into the
 * stacked gate_up layout above: for each expert, gate rows then up rows, for
 * the packed codes (row_bytes K/2), the block scales (K/16) and the per-row
 * weight_scale_2 (4).
 */
int nvfp4_stack_rows(const void *const *srcs, const int64_t *rows, int32_t n,
                     int64_t row_bytes, void *dst, void *stream);

/* Router alone: topk_ids int32 [T, k], topk_w fp32 [T, k]; logits fp32
 * [T, E] is caller memory the router writes (and the caller may read).  The
 * arithmetic is that of nvfp4_moe_forward's router (same logits bit for
 * bit); its split-H partial sums go to stream-ordered scratch
 * (cudaMallocAsync on `stream`) when the split is used. */
int nvfp4_moe_route(const nvfp4_moe_desc *desc, const float *router, const void *x, int64_t T,
                    int32_t *topk_ids, float *topk_w, float *logits, void *stream);

/*
 * Expert FFNs over R rows, each assigned one expert: y_rows[r] ([R, H],
 * y_dtype fp32 or bf16) = down_e(silu(gate_e(x)) * up_e(x)) with e =
 * row_expert[r] and x = x[x_row_index[r]] (or x[r] when x_row_index is
 * NULL); x is bf16 [*, H]; rows whose expert id is outside [0, E) are left
 * untouched.  The building block of the expert-parallel layer (rows
 * received from other ranks).
 */
int nvfp4_moe_experts(const nvfp4_moe_desc *desc, const nvfp4_moe_weights *weights,
                      const void *x, const int32_t *x_row_index, const int32_t *row_expert,
                      int64_t R, void *y_rows, int y_dtype, void *workspace,
                      size_t workspace_bytes, void *stream);

/* y[t] = sum_j topk_w[t, j] * y_slots[row(t*k + j)] (+ residual[t]) with
 * row(s) = slot_pos ? slot_pos[s] : s: fp32 sums in j order; residual bf16;
 * y_slots and y fp32 or bf16 (slot_dtype, y_dtype). */
int nvfp4_moe_combine(const void *y_slots, int slot_dtype, const float *topk_w,
                      const int32_t *slot_pos, const void *residual, void *y, int y_dtype,
                      int64_t T, int32_t k, int32_t hidden, void *stream);

/*
 * Expert-parallel dispatch plan (the exchange itself is NCCL all-to-all over
 * NVLink, driven by the host): slot s = t*k + j with global expert
 * e = topk_ids[s] goes to rank e / experts_per_rank as local expert
 * e % experts_per_rank.  Writes send_counts [world], and in send order
 * (grouped by rank; slot order within a rank) send_token [T*k] and
 * send_expert [T*k]; slot_pos [T*k] = send position of each slot.
 */
int nvfp4_ep_dispatch_plan(const int32_t *topk_ids, int64_t T, int32_t k,
                           int32_t experts_per_rank, int32_t world, int32_t *send_counts,
                           int32_t *send_token, int32_t *send_expert, int32_t *slot_pos,
                           void *stream);

/*
 * Fixed-capacity form of the dispatch (after nvfp4_ep_dispatch_plan): lays
 * the send order out as `world` blocks of `cap` rows (cap >= T*k), block r =
 * the token rows x[send_token[i]] bound for rank r followed by zero rows;
 * send_expert_padded [world*cap] = local expert id or -1 for padding;
 * slot_padded [T*k] = padded position of each slot (-1 if none).  Every
 * exchange then has the same sizes (cap rows per peer), so a step needs no
 * host-side count and can be captured in a CUDA graph.
 */
int nvfp4_ep_dispatch_padded(const int32_t *send_counts, const int32_t *send_token,
                             const int32_t *send_expert, const int32_t *slot_pos, int64_t T,
                             int32_t k, int32_t world, int64_t cap, const void *x,
                             int64_t row_bytes, void *send_rows, int32_t *send_expert_padded,
                             int32_t *slot_padded, void *stream);

/* dst[i] = src[row_index[i]] for n rows of row_bytes bytes (multiple of 16). */
int nvfp4_gather_rows(const void *src, const int32_t *row_index, int64_t n, int64_t row_bytes,
                      void *dst, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* NVFP4_H */

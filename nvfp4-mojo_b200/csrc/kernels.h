// kernels.h -- host-side launchers of the NVFP4 kernels (internal to libnvfp4).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4 {

enum DType : int { kF32 = 0, kBF16 = 1 };

// alpha_n = input_scale[g] * (ws2_rows ? ws2_rows[g][n] : ws2)
struct AlphaSpec {
  float input_scale = 1.0f;           // used when input_scales == nullptr
  const float *input_scales = nullptr;  // per group [G]
  float ws2 = 1.0f;                   // used when ws2_rows == nullptr
  const float *ws2_rows = nullptr;      // [G][N]
  int64_t ws2_group_stride = 0;         // elements
};

#ifdef __CUDACC__
__device__ __forceinline__ float alpha_of(const AlphaSpec &al, int g, int n) {
  const float ins = al.input_scales ? al.input_scales[g] : al.input_scale;
  const float w2 = al.ws2_rows ? al.ws2_rows[(int64_t)g * al.ws2_group_stride + n] : al.ws2;
  return ins * w2;
}
#endif

// Grouped NVFP4 weights: group g has rows [N, K/2] at w + g*w_group_stride.
struct WeightSpec {
  const uint8_t *w = nullptr;
  const uint8_t *sf = nullptr;
  int64_t w_group_stride = 0;   // bytes
  int64_t sf_group_stride = 0;  // bytes
  int N = 0;                    // rows (output features)
  int K = 0;                    // in features
};

// Full-matrix dequant: out[r, k] = LUT * float(sf) (fp32), or the bf16 of it.
cudaError_t launch_dequant(const uint8_t *w, const uint8_t *sf, int64_t rows, int64_t K,
                           void *out, int out_dtype, cudaStream_t s);

// Reference tile form (nvfp4/nvfp4_gemm_gpu.mojo:44-96), fp32 out [tile_m, tile_k].
cudaError_t launch_dequant_tile(const uint8_t *w, const uint8_t *sf, float *out,
                                int64_t weight_stride, int64_t scale_stride,
                                int64_t start_row, int64_t start_col, int64_t tile_m,
                                int64_t tile_k, cudaStream_t s);

// CUDA-core fp32 linear, any layout by strides (x: [M,K] via xs_m/xs_k,
// y: [M,N] via ys_m/ys_n).  Faithful to nvfp4_matvec's fp32 arithmetic.
cudaError_t launch_linear_f32(const WeightSpec &ws, const AlphaSpec &al, const void *x,
                              int x_dtype, int64_t xs_m, int64_t xs_k, void *y,
                              int y_dtype, int64_t ys_m, int64_t ys_n, int M,
                              cudaStream_t s);

// Work item of the grouped skinny kernel: (group, first token slot, tokens).
struct SkinnyWork {
  int group;
  int slot0;
  int count;
};

// Tensor-core skinny GEMM (mma.sync m16n8k16, decode in registers).
// Tokens: for plain linear, slot = token row (x row = slot, y row = slot).
// For grouped use: `work`/`n_work` list the (group, slot range) items and
// x_rows / y_rows map a slot to its activation / output row (nullable).
// silu_gate: W has 2*Nout rows, output n = silu(h[n]) * h[Nout + n].
struct SkinnyArgs {
  WeightSpec ws;
  AlphaSpec al;
  const uint16_t *x = nullptr;  // bf16 rows of length K, ld x_ld
  const uint16_t *x_lo = nullptr;  // optional bf16 low parts (x = x + x_lo), same layout
  int64_t x_ld = 0;
  const int32_t *x_rows = nullptr;
  void *y = nullptr;
  int y_dtype = kBF16;
  int64_t y_ld = 0;
  const int32_t *y_rows = nullptr;
  uint16_t *y_lo = nullptr;     // silu_gate only: bf16 low parts of the outputs
  int M = 0;                    // tokens (plain mode)
  const SkinnyWork *work = nullptr;
  const int *n_work = nullptr;  // device count of work items
  int work_capacity = 0;        // host upper bound of n_work
  bool silu_gate = false;
  int tokens_per_item = 8;      // 8, 16 or 32
};
cudaError_t launch_skinny(const SkinnyArgs &a, cudaStream_t s);

// Decode GEMV for M <= 8 tokens (token-major bf16 x, K % 256 == 0, 32-byte
// aligned weights, 4-byte aligned blockscales, 16-byte aligned x rows).
bool gemv_supported(int M, int K, const void *w, const void *sf, const void *x, int64_t x_ld);
cudaError_t launch_gemv(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                        int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                        cudaStream_t st);

// Decode GEMV for M <= 8 tokens on tcgen05 with the decoded weights in TMEM
// (A operand) and the activations in shared memory (B), K % 256 == 0,
// 16-byte aligned weights, scales and x rows.
bool gemv_ts_supported(int M, int N, int K, const void *w, const void *sf, const void *x,
                       int64_t x_ld);
cudaError_t launch_gemv_ts(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                           int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                           cudaStream_t st);
int read_gemv_ts_device_status();

// Decode GEMV for M <= 8 tokens on the block-scaled FP4 tensor cores: the
// activations as four NVFP4 digits (computed into `scratch`, of
// gemv_dg_scratch_bytes(K)), the weights fed to the MMA as stored.
// K % 256 == 0, K <= 16384, 16-byte aligned weights, scales and x rows.
bool gemv_dg_supported(int M, int N, int K, const void *w, const void *sf, const void *x,
                       int64_t x_ld);
size_t gemv_dg_scratch_bytes(int K);
cudaError_t launch_gemv_dg(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                           int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                           uint8_t *scratch, size_t scratch_bytes, cudaStream_t st);
int read_gemv_dg_device_status();

// Grouped MoE expert GEMMs on the decode GEMV kernel (work items of at most
// 8 token slots): gate_up -> silu(gate) * up as bf16 hi + lo [R, I] (rows in
// slot order), down on those hi + lo rows -> y rows (dst_row scatter).
struct MoeGemvLaunch {
  const uint8_t *w = nullptr;   // stacked [groups * N, K/2]
  const uint8_t *sf = nullptr;  // stacked [groups * N, K/16]
  AlphaSpec al;                 // per group: input_scales[g], ws2_rows + g * N
  const uint16_t *x = nullptr;
  const uint16_t *x_lo = nullptr;  // down: low parts
  int64_t x_ld = 0;
  void *y = nullptr;
  uint16_t *y_lo = nullptr;        // gate_up: low parts
  int y_dtype = kBF16;
  int64_t y_ld = 0;
  int N = 0, K = 0, groups = 0;
  int items = 0;                   // host upper bound of the work items
  const SkinnyWork *work = nullptr;
  const int *n_work = nullptr;
  const int32_t *x_rows = nullptr;  // gate_up: slot -> x row
  const int32_t *y_rows = nullptr;  // down: slot -> y row
  bool gate_up = false;
};
bool moe_gemv_supported(int H, int I, const void *gate_up, const void *gate_up_sf,
                        const void *down, const void *down_sf);
cudaError_t launch_moe_gemv(const MoeGemvLaunch &m, cudaStream_t st);

// tcgen05 W4A16 GEMM (token-major x [M, K] bf16 with row stride x_ld).
bool tc_gemm_supported(int K, const void *w, const void *x, int64_t x_ld);
cudaError_t launch_w4a16_tc(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                            int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                            cudaStream_t st);
// Return and clear the device status word of the tensor-core GEMM, the
// decode GEMV, the grouped MoE tensor-core kernels and the W4A4 GEMM
// (-1: not readable).
int read_gemm_device_status();
int read_gemv_device_status();
int read_moe_tc_device_status();
int read_w4a4_device_status();

// W4A4: activation quantizer and block-scaled FP4 GEMM (tcgen05 mxf4nvf4).
cudaError_t launch_quantize_act(const void *x, int x_dtype, int64_t x_ld, int64_t M, int64_t K,
                                float input_scale, uint8_t *q, uint8_t *qsf, cudaStream_t st);
bool w4a4_supported(int K, const void *w, const void *sf, const void *xq, const void *xsf);
cudaError_t launch_w4a4_gemm(const WeightSpec &ws, const AlphaSpec &al, const uint8_t *xq,
                             const uint8_t *xsf, int M, void *y, int y_dtype, int64_t y_ld,
                             cudaStream_t st);

}  // namespace nvfp4

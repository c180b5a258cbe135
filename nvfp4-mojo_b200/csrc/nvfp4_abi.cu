// nvfp4_abi.cu -- extern "C" entry points of libnvfp4.so (include/nvfp4.h).
//
// Validation, dispatch and error reporting.  Every compute entry point ends
// in a CUDA launch on the caller's stream; there is no host compute path.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/nvfp4.h"
#include "abi_util.h"
#include "kernels.h"

namespace nvfp4 {

static thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(cudaError_t e, const char *what) {
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return NVFP4_OK;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace nvfp4

using namespace nvfp4;

extern "C" int nvfp4_abi_version(void) { return NVFP4_ABI_VERSION; }

extern "C" const char *nvfp4_last_error_string(void) { return g_last_error.c_str(); }

static int valid_dtype(int dt) { return dt == NVFP4_DTYPE_F32 || dt == NVFP4_DTYPE_BF16; }

// Linear over token-major x [M, K] -> y [M, N] (shared by linear_forward and
// the reference-layout gemm entry, which passes its own strides).
static int run_linear(const WeightSpec &ws, const AlphaSpec &al, const void *x, int x_dt,
                      int64_t xs_m, int64_t xs_k, void *y, int y_dt, int64_t ys_m,
                      int64_t ys_n, int64_t M, uint32_t flags, cudaStream_t st) {
  if (M == 0) return NVFP4_OK;
  if (M > INT32_MAX / 2) return fail(NVFP4_ERR_INVALID_ARG, "too many tokens: %lld", (long long)M);
  const bool token_major = (xs_k == 1 && ys_n == 1);
  const bool force_f32 = flags & NVFP4_FLAG_FORCE_F32;
  // Decode GEMV: 16-byte code chunks and 4-byte scale words stream through
  // cp.async, hence K % 64 (scale rows of whole 4-byte words) and alignment.
  const bool skinny_ok = token_major && x_dt == kBF16 && (ws.K % 64) == 0 &&
                         aligned(ws.w, 16) && aligned(ws.sf, 4) && aligned(x, 16) &&
                         (xs_m % 8) == 0;
  const bool tc_ok = token_major && x_dt == kBF16 && !force_f32 &&
                     tc_gemm_supported(ws.K, ws.w, x, xs_m);
  if ((flags & NVFP4_FLAG_FORCE_TC) && !tc_ok)
    return fail(NVFP4_ERR_UNSUPPORTED,
                "tcgen05 GEMM path needs bf16 token-major activations, K %% 64 == 0 and "
                "16-byte aligned weights/activations");
  if (tc_ok && ((flags & NVFP4_FLAG_FORCE_TC) || (M > 64 && !(flags & NVFP4_FLAG_FORCE_SKINNY))))
    return check_launch(launch_w4a16_tc(ws, al, reinterpret_cast<const uint16_t *>(x), xs_m, y,
                                        y_dt, ys_m, (int)M, st),
                        "tcgen05 GEMM launch");
  // M <= 8 with NVFP4_FLAG_DIGIT_GEMV: the activations as four NVFP4 digits
  // (stream-ordered scratch, so the call stays asynchronous and capturable),
  // the weights straight into block-scaled FP4 MMAs.
  if (!force_f32 && token_major && x_dt == kBF16 && (flags & NVFP4_FLAG_DIGIT_GEMV) &&
      gemv_dg_supported((int)M, ws.N, ws.K, ws.w, ws.sf, x, xs_m)) {
    const size_t bytes = gemv_dg_scratch_bytes(ws.K);
    void *buf = nullptr;
    cudaError_t e = cudaMallocAsync(&buf, bytes, st);
    if (e != cudaSuccess) return check_launch(e, "digit GEMV scratch (cudaMallocAsync)");
    const int rc = check_launch(launch_gemv_dg(ws, al, reinterpret_cast<const uint16_t *>(x), xs_m,
                                               y, y_dt, ys_m, (int)M, static_cast<uint8_t *>(buf),
                                               bytes, st),
                                "digit GEMV launch");
    e = cudaFreeAsync(buf, st);
    if (rc == NVFP4_OK && e != cudaSuccess) return check_launch(e, "digit GEMV scratch release");
    return rc;
  }
  // M <= 8 with NVFP4_FLAG_TS_GEMV: the decode GEMV on tcgen05 (decoded
  // weights in tensor memory, K split across a thread-block cluster when the
  // tiles do not fill the GPU).  Exact like the default below, but slower on
  // B200 as measured: the 128 x 16 x 16 MMAs it issues cost about as much as
  // full-width ones.
  if (!force_f32 && token_major && x_dt == kBF16 && (flags & NVFP4_FLAG_TS_GEMV) &&
      gemv_ts_supported((int)M, ws.N, ws.K, ws.w, ws.sf, x, xs_m))
    return check_launch(launch_gemv_ts(ws, al, reinterpret_cast<const uint16_t *>(x), xs_m, y,
                                       y_dt, ys_m, (int)M, st),
                        "decode GEMV launch");
  // M <= 8: the decode GEMV on register-fragment mma.sync tensor-core
  // instructions fed by the hardware FP4 / FP8 conversions.
  if (!force_f32 && token_major && x_dt == kBF16 &&
      gemv_supported((int)M, ws.K, ws.w, ws.sf, x, xs_m))
    return check_launch(launch_gemv(ws, al, reinterpret_cast<const uint16_t *>(x), xs_m, y, y_dt,
                                    ys_m, (int)M, st),
                        "decode GEMV launch");
  if (!force_f32 && skinny_ok && (M <= 64 || !tc_ok || (flags & NVFP4_FLAG_FORCE_SKINNY))) {
    SkinnyArgs a;
    a.ws = ws;
    a.al = al;
    a.x = reinterpret_cast<const uint16_t *>(x);
    a.x_ld = xs_m;
    a.y = y;
    a.y_dtype = y_dt;
    a.y_ld = ys_m;
    a.M = (int)M;
    a.tokens_per_item = M <= 8 ? 8 : (M <= 16 ? 16 : 32);
    return check_launch(launch_skinny(a, st), "skinny GEMM launch");
  }
  if ((flags & NVFP4_FLAG_FORCE_SKINNY) && !skinny_ok)
    return fail(NVFP4_ERR_UNSUPPORTED,
                "decode GEMV path needs bf16 token-major activations, K %% 64 == 0 and "
                "16-byte aligned weights/activations");
  return check_launch(
      launch_linear_f32(ws, al, x, x_dt, xs_m, xs_k, y, y_dt, ys_m, ys_n, (int)M, st),
      "fp32 linear launch");
}

static int check_weights(const uint8_t *w, const uint8_t *sf, int64_t N, int64_t K) {
  if (!w || !sf) return fail(NVFP4_ERR_INVALID_ARG, "null weight or blockscale pointer");
  if (N <= 0 || K <= 0) return fail(NVFP4_ERR_INVALID_ARG, "bad shape N=%lld K=%lld", (long long)N, (long long)K);
  if (K % NVFP4_GROUP_SIZE)
    return fail(NVFP4_ERR_INVALID_ARG, "in_features %lld is not a multiple of %d", (long long)K,
                NVFP4_GROUP_SIZE);
  if (N > INT32_MAX || K > INT32_MAX) return fail(NVFP4_ERR_INVALID_ARG, "shape too large");
  return NVFP4_OK;
}

extern "C" int nvfp4_quantize_act(const void *x, int x_dt, int64_t M, int64_t K, int64_t x_ld,
                                  float input_scale, uint8_t *codes, uint8_t *scales,
                                  void *stream) {
  NVFP4_ABI_RANGE();
  if (!valid_dtype(x_dt)) return fail(NVFP4_ERR_INVALID_ARG, "bad dtype");
  if (M < 0 || K <= 0 || K % NVFP4_GROUP_SIZE || x_ld < K)
    return fail(NVFP4_ERR_INVALID_ARG, "bad shape M=%lld K=%lld ld=%lld", (long long)M,
                (long long)K, (long long)x_ld);
  if (M == 0) return NVFP4_OK;
  if (!x || !codes || !scales) return fail(NVFP4_ERR_INVALID_ARG, "null pointer");
  const int esize = x_dt == kBF16 ? 2 : 4;
  if (!aligned(x, 16) || (x_ld * esize) % 16 || !aligned(codes, 8))
    return fail(NVFP4_ERR_INVALID_ARG,
                "activation rows must be 16-byte aligned and codes 8-byte aligned");
  if (!(input_scale > 0.0f) || !isfinite(input_scale))
    return fail(NVFP4_ERR_INVALID_ARG, "input_scale must be positive and finite");
  return check_launch(launch_quantize_act(x, x_dt, x_ld, M, K, input_scale, codes, scales,
                                          static_cast<cudaStream_t>(stream)),
                      "activation quantizer launch");
}

extern "C" int nvfp4_linear_w4a4(const nvfp4_linear_desc *lin, const uint8_t *w,
                                 const uint8_t *sf, const uint8_t *xq, const uint8_t *xsf,
                                 void *y, int y_dt, int64_t M, void *stream) {
  NVFP4_ABI_RANGE();
  if (!lin) return fail(NVFP4_ERR_INVALID_ARG, "null linear descriptor");
  int rc = check_weights(w, sf, lin->out_features, lin->in_features);
  if (rc) return rc;
  if (!valid_dtype(y_dt)) return fail(NVFP4_ERR_INVALID_ARG, "bad dtype");
  if (M < 0 || M > INT32_MAX) return fail(NVFP4_ERR_INVALID_ARG, "bad token count");
  if (M == 0) return NVFP4_OK;
  if (!xq || !xsf || !y) return fail(NVFP4_ERR_INVALID_ARG, "null activation or output pointer");
  if (!w4a4_supported((int)lin->in_features, w, sf, xq, xsf))
    return fail(NVFP4_ERR_UNSUPPORTED,
                "W4A4 GEMM needs in_features %% 256 == 0 and 16-byte aligned operands");
  WeightSpec ws;
  ws.w = w;
  ws.sf = sf;
  ws.N = (int)lin->out_features;
  ws.K = (int)lin->in_features;
  AlphaSpec al;
  al.input_scale = lin->input_scale;
  al.ws2 = lin->weight_scale_2;
  al.ws2_rows = lin->weight_scale_2_rows;
  return check_launch(launch_w4a4_gemm(ws, al, xq, xsf, (int)M, y, y_dt, ws.N,
                                       static_cast<cudaStream_t>(stream)),
                      "W4A4 GEMM launch");
}

// nvfp4_linear_forward with NVFP4_FLAG_W4A4: quantized activations live in
// stream-ordered scratch (cudaMallocAsync / cudaFreeAsync on the caller's
// stream, so the call stays asynchronous and capturable).
static int run_w4a4_with_scratch(const nvfp4_linear_desc *lin, const uint8_t *w,
                                 const uint8_t *sf, const void *x, int x_dt, void *y, int y_dt,
                                 int64_t M, void *stream) {
  if (M == 0) return NVFP4_OK;
  const int64_t K = lin->in_features;
  const size_t codes = (size_t)M * (size_t)(K / 2), scales = (size_t)M * (size_t)(K / 16);
  const size_t off = (codes + 255) & ~(size_t)255;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void *buf = nullptr;
  cudaError_t e = cudaMallocAsync(&buf, off + scales, st);
  if (e != cudaSuccess) return check_launch(e, "W4A4 activation scratch (cudaMallocAsync)");
  uint8_t *q = static_cast<uint8_t *>(buf), *qsf = q + off;
  int rc = nvfp4_quantize_act(x, x_dt, M, K, K, lin->input_scale, q, qsf, stream);
  if (rc == NVFP4_OK) rc = nvfp4_linear_w4a4(lin, w, sf, q, qsf, y, y_dt, M, stream);
  e = cudaFreeAsync(buf, st);
  if (rc == NVFP4_OK && e != cudaSuccess) return check_launch(e, "W4A4 scratch release");
  return rc;
}

extern "C" int nvfp4_linear_forward(const nvfp4_linear_desc *lin, const uint8_t *w,
                                    const uint8_t *sf, const void *x, int x_dt, void *y,
                                    int y_dt, int64_t M, uint32_t flags, void *stream) {
  NVFP4_ABI_RANGE();
  if (!lin) return fail(NVFP4_ERR_INVALID_ARG, "null linear descriptor");
  int rc = check_weights(w, sf, lin->out_features, lin->in_features);
  if (rc) return rc;
  if (!valid_dtype(x_dt) || !valid_dtype(y_dt)) return fail(NVFP4_ERR_INVALID_ARG, "bad dtype");
  if (M < 0) return fail(NVFP4_ERR_INVALID_ARG, "negative batch_seq_len");
  if (M > 0 && (!x || !y)) return fail(NVFP4_ERR_INVALID_ARG, "null activation or output pointer");
  if (flags & NVFP4_FLAG_W4A4) return run_w4a4_with_scratch(lin, w, sf, x, x_dt, y, y_dt, M, stream);
  WeightSpec ws;
  ws.w = w;
  ws.sf = sf;
  ws.N = (int)lin->out_features;
  ws.K = (int)lin->in_features;
  AlphaSpec al;
  al.input_scale = lin->input_scale;
  al.ws2 = lin->weight_scale_2;
  al.ws2_rows = lin->weight_scale_2_rows;
  return run_linear(ws, al, x, x_dt, ws.K, 1, y, y_dt, ws.N, 1, M, flags,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int nvfp4_gemm_kernel(int64_t M_out, int64_t N_tok, int64_t K, const uint8_t *w,
                                 const uint8_t *sf, const void *act, int act_dt, void *out,
                                 int out_dt, float alpha, void *stream) {
  NVFP4_ABI_RANGE();
  int rc = check_weights(w, sf, M_out, K);
  if (rc) return rc;
  if (!valid_dtype(act_dt) || !valid_dtype(out_dt)) return fail(NVFP4_ERR_INVALID_ARG, "bad dtype");
  if (N_tok < 0) return fail(NVFP4_ERR_INVALID_ARG, "negative N");
  if (N_tok > 0 && (!act || !out)) return fail(NVFP4_ERR_INVALID_ARG, "null activation or output pointer");
  WeightSpec ws;
  ws.w = w;
  ws.sf = sf;
  ws.N = (int)M_out;
  ws.K = (int)K;
  AlphaSpec al;
  al.input_scale = alpha;
  al.ws2 = 1.0f;
  // act[k, n] at k*N_tok + n; out[m, n] at m*N_tok + n.
  return run_linear(ws, al, act, act_dt, 1, N_tok, out, out_dt, 1, N_tok, N_tok, 0,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int nvfp4_matvec(const nvfp4_linear_desc *lin, const uint8_t *w, const uint8_t *sf,
                            const float *x, float *y, void *stream) {
  NVFP4_ABI_RANGE();
  if (!lin) return fail(NVFP4_ERR_INVALID_ARG, "null linear descriptor");
  int rc = check_weights(w, sf, lin->out_features, lin->in_features);
  if (rc) return rc;
  if (!x || !y) return fail(NVFP4_ERR_INVALID_ARG, "null input or result pointer");
  WeightSpec ws;
  ws.w = w;
  ws.sf = sf;
  ws.N = (int)lin->out_features;
  ws.K = (int)lin->in_features;
  AlphaSpec al;
  al.input_scale = lin->input_scale;
  al.ws2 = lin->weight_scale_2;
  al.ws2_rows = lin->weight_scale_2_rows;
  return check_launch(launch_linear_f32(ws, al, x, kF32, ws.K, 1, y, kF32, ws.N, 1, 1,
                                        static_cast<cudaStream_t>(stream)),
                      "matvec launch");
}

extern "C" int nvfp4_dequant_tile(const uint8_t *w, const uint8_t *sf, float *out,
                                  int64_t weight_stride, int64_t scale_stride, int64_t start_row,
                                  int64_t start_col, int64_t tile_m, int64_t tile_k,
                                  void *stream) {
  NVFP4_ABI_RANGE();
  if (!w || !sf || !out) return fail(NVFP4_ERR_INVALID_ARG, "null pointer");
  if (tile_m < 0 || tile_k < 0 || start_row < 0 || start_col < 0)
    return fail(NVFP4_ERR_INVALID_ARG, "negative tile geometry");
  if (tile_k % NVFP4_PACK_FACTOR || start_col % NVFP4_PACK_FACTOR)
    return fail(NVFP4_ERR_INVALID_ARG, "tile_k and start_col must be even");
  return check_launch(launch_dequant_tile(w, sf, out, weight_stride, scale_stride, start_row,
                                          start_col, tile_m, tile_k,
                                          static_cast<cudaStream_t>(stream)),
                      "dequant tile launch");
}

extern "C" int nvfp4_device_status(void) {
  const int words[6] = {read_gemm_device_status(), read_gemv_device_status(),
                        read_moe_tc_device_status(), read_w4a4_device_status(),
                        read_gemv_ts_device_status(), read_gemv_dg_device_status()};
  int v = 0;
  for (int w : words) {
    if (w < 0) return fail(NVFP4_ERR_CUDA, "could not read the device status word");
    if (!v) v = w;
  }
  return v;
}

extern "C" int nvfp4_dequant(const uint8_t *w, const uint8_t *sf, int64_t rows, int64_t K,
                             void *out, int out_dt, void *stream) {
  NVFP4_ABI_RANGE();
  int rc = check_weights(w, sf, rows, K);
  if (rc) return rc;
  if (!out) return fail(NVFP4_ERR_INVALID_ARG, "null output pointer");
  if (!valid_dtype(out_dt)) return fail(NVFP4_ERR_INVALID_ARG, "bad dtype");
  if (!aligned(w, 4) || !aligned(out, 16))
    return fail(NVFP4_ERR_INVALID_ARG, "weights must be 4-byte and output 16-byte aligned");
  return check_launch(launch_dequant(w, sf, rows, K, out, out_dt, static_cast<cudaStream_t>(stream)),
                      "dequant launch");
}

/*
 * nvfp4_oracle.c -- CPU restatement of the reference's NVFP4 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  See nvfp4_oracle.h for what pins
 * each function.  Every function cites the reference file:line it restates.
 * Built by oracle/Makefile into oracle/_build/liboracle.so (scalar, -O2,
 * no fast-math so fp32 evaluation order is the one written here).
 */
#include "nvfp4_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* nvfp4/config.mojo:18-35 -- E2M1 code -> value; code 8 is -0.0. */
static const float k_lut[16] = {
    0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

float oracle_lut(int code) { return k_lut[code & 15]; }

/* nvfp4/config.mojo:106-114 -- lo = b & 0xF (even k), hi = (b >> 4) & 0xF. */
void oracle_unpack_fp4_pair(uint8_t packed, uint8_t *lo, uint8_t *hi) {
  *lo = (uint8_t)(packed & 0x0F);
  *hi = (uint8_t)((packed >> 4) & 0x0F);
}

/* nvfp4/config.mojo:138-140 */
uint8_t oracle_pack_fp4_pair(uint8_t lo, uint8_t hi) {
  return (uint8_t)((hi << 4) | (lo & 0x0F));
}

/* nvfp4/config.mojo:117-121 -- LUT[v] * scale in fp32. */
float oracle_dequant_fp4(uint8_t v, float scale) { return k_lut[v & 15] * scale; }

/* nvfp4/config.mojo:143-149 -- left-to-right fp32 products. */
float oracle_compute_effective_scale(float blockscale, float ws2, float input_scale) {
  float t = blockscale * ws2;
  return t * input_scale;
}

/*
 * Float8_e4m3fn -> Float32 (the `.cast[DType.float32]()` at
 * nvfp4/deltanet.mojo:574-576 and nvfp4/nvfp4_gemm_gpu.mojo:167-169).
 * OCP FP8 E4M3FN: bias 7, subnormals m*2^-9, S.1111.111 is NaN, no Inf.
 */
float oracle_e4m3_to_f32(uint8_t b) {
  int s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0)
    v = ldexpf((float)m, -9);
  else
    v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

/* Round-to-nearest-even of a non-negative value onto a sorted code table. */
static int rne_on_table(double a, const double *vals, int n) {
  if (a >= vals[n - 1]) return n - 1; /* saturate */
  int lo = 0;
  while (lo + 1 < n && vals[lo + 1] <= a) lo++;
  if (vals[lo] == a) return lo;
  double dl = a - vals[lo], dh = vals[lo + 1] - a;
  if (dl < dh) return lo;
  if (dh < dl) return lo + 1;
  return (lo & 1) ? lo + 1 : lo; /* tie: even mantissa (even code) */
}

uint8_t oracle_f32_to_e4m3_satfinite(float x) {
  static double vals[127];
  static int init = 0;
  if (!init) {
    for (int c = 0; c < 127; ++c) vals[c] = (double)oracle_e4m3_to_f32((uint8_t)c);
    init = 1;
  }
  if (isnan(x)) return 0x7F;
  int s = signbit(x) ? 0x80 : 0;
  int c = rne_on_table(fabs((double)x), vals, 127);
  return (uint8_t)(s | c);
}

uint8_t oracle_f32_to_e2m1_satfinite(float x) {
  static const double vals[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};
  int s = signbit(x) ? 8 : 0;
  int c = rne_on_table(fabs((double)x), vals, 8);
  return (uint8_t)(s | c);
}

float oracle_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t oracle_f32_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if (isnan(x)) return (uint16_t)((u >> 16) | 0x40);
  uint32_t r = 0x7FFF + ((u >> 16) & 1);
  return (uint16_t)((u + r) >> 16);
}

/* nvfp4/deltanet.mojo:66-74 -- sign-split logistic. */
float oracle_sigmoid(float x) {
  if (x >= 0.0f) {
    float e = expf(-x);
    return 1.0f / (1.0f + e);
  } else {
    float e = expf(x);
    return e / (1.0f + e);
  }
}

/* nvfp4/deltanet.mojo:77-80 */
float oracle_silu(float x) { return x * oracle_sigmoid(x); }

/* nvfp4/nvfp4_gemm_gpu.mojo:44-96 */
void oracle_dequant_tile(const uint8_t *packed, const uint8_t *scales, float *out,
                         int64_t weight_stride, int64_t scale_stride,
                         int64_t start_row, int64_t start_col,
                         int64_t tile_m, int64_t tile_k) {
  int64_t packed_col = start_col / ORACLE_PACK_FACTOR;
  for (int64_t m = 0; m < tile_m; ++m) {
    int64_t row = start_row + m;
    for (int64_t k = 0; k < tile_k / ORACLE_PACK_FACTOR; ++k) {
      int64_t col = packed_col + k;
      uint8_t p = packed[row * weight_stride + col];
      int64_t scale_col = (start_col + k * ORACLE_PACK_FACTOR) / ORACLE_GROUP_SIZE;
      float scale = oracle_e4m3_to_f32(scales[row * scale_stride + scale_col]);
      uint8_t lo, hi;
      oracle_unpack_fp4_pair(p, &lo, &hi);
      out[m * tile_k + k * 2] = oracle_dequant_fp4(lo, scale);
      out[m * tile_k + k * 2 + 1] = oracle_dequant_fp4(hi, scale);
    }
  }
}

/* One output row of nvfp4/deltanet.mojo:569-584. */
static float matvec_row(int64_t K, int64_t m, float alpha, const uint8_t *packed,
                        const uint8_t *scales, const float *x) {
  int64_t packed_stride = K / ORACLE_PACK_FACTOR;
  int64_t scale_stride = K / ORACLE_GROUP_SIZE;
  float acc = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    int64_t packed_k = k / ORACLE_PACK_FACTOR;
    uint8_t packed_byte = packed[m * packed_stride + packed_k];
    uint8_t lo, hi;
    oracle_unpack_fp4_pair(packed_byte, &lo, &hi);
    int64_t scale_k = k / ORACLE_GROUP_SIZE;
    float scale = oracle_e4m3_to_f32(scales[m * scale_stride + scale_k]);
    uint8_t fp4_val = (k % 2 == 0) ? lo : hi;
    float weight = oracle_dequant_fp4(fp4_val, scale);
    acc += weight * x[k];
  }
  return acc * alpha;
}

/* nvfp4/deltanet.mojo:549-584; alpha from nvfp4/config.mojo:93-95. */
void oracle_matvec(int64_t K, int64_t N, float input_scale, float ws2,
                   const float *ws2_rows, const uint8_t *packed,
                   const uint8_t *scales, const float *x, float *y) {
  for (int64_t m = 0; m < N; ++m) {
    float alpha = input_scale * (ws2_rows ? ws2_rows[m] : ws2);
    y[m] = matvec_row(K, m, alpha, packed, scales, x);
  }
}

void oracle_linear(int64_t M, int64_t K, int64_t N, float input_scale, float ws2,
                   const float *ws2_rows, const uint8_t *packed,
                   const uint8_t *scales, const float *x, float *y,
                   const int64_t *rows, int64_t n_rows,
                   const int64_t *cols, int64_t n_cols, int n_threads) {
  int64_t R = rows ? n_rows : M;
  int64_t C = cols ? n_cols : N;
  int64_t total = R * C;
#ifdef _OPENMP
  if (n_threads < 1) n_threads = 1;
#pragma omp parallel for schedule(static) num_threads(n_threads)
#endif
  for (int64_t i = 0; i < total; ++i) {
    int64_t r = i / C, c = i % C;
    int64_t tok = rows ? rows[r] : r;
    int64_t n = cols ? cols[c] : c;
    float alpha = input_scale * (ws2_rows ? ws2_rows[n] : ws2);
    y[r * C + c] = matvec_row(K, n, alpha, packed, scales, x + tok * K);
  }
  (void)n_threads;
}

/* nvfp4/nvfp4_gemm_gpu.mojo:148-182 (reference kernel body, [K, N] activations). */
void oracle_gemm_kernel(int64_t M_out, int64_t N_tok, int64_t K,
                        const uint8_t *packed, const uint8_t *scales,
                        const float *act, float *out, float alpha) {
  for (int64_t gm = 0; gm < M_out; ++gm) {
    for (int64_t gn = 0; gn < N_tok; ++gn) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        int64_t packed_k = k / ORACLE_PACK_FACTOR;
        uint8_t p = packed[gm * (K / ORACLE_PACK_FACTOR) + packed_k];
        uint8_t lo, hi;
        oracle_unpack_fp4_pair(p, &lo, &hi);
        int64_t scale_k = k / ORACLE_GROUP_SIZE;
        float scale = oracle_e4m3_to_f32(scales[gm * (K / ORACLE_GROUP_SIZE) + scale_k]);
        uint8_t v = (k % 2 == 0) ? lo : hi;
        float w = oracle_dequant_fp4(v, scale);
        acc += w * act[k * N_tok + gn];
      }
      out[gm * N_tok + gn] = acc * alpha;
    }
  }
}

void oracle_quantize_act(int64_t M, int64_t K, const float *x, float input_scale,
                         uint8_t *q_packed, uint8_t *q_scales) {
  float denom = 6.0f * input_scale;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t g = 0; g < K / ORACLE_GROUP_SIZE; ++g) {
      const float *xs = x + m * K + g * ORACLE_GROUP_SIZE;
      float amax = 0.0f;
      for (int i = 0; i < ORACLE_GROUP_SIZE; ++i) {
        float a = fabsf(xs[i]);
        if (a > amax) amax = a;
      }
      uint8_t sf = oracle_f32_to_e4m3_satfinite(amax / denom);
      q_scales[m * (K / ORACLE_GROUP_SIZE) + g] = sf;
      float sdeq = oracle_e4m3_to_f32(sf) * input_scale;
      for (int i = 0; i < ORACLE_GROUP_SIZE; i += 2) {
        uint8_t c0 = 0, c1 = 0;
        if (sdeq != 0.0f) {
          c0 = oracle_f32_to_e2m1_satfinite(xs[i] / sdeq);
          c1 = oracle_f32_to_e2m1_satfinite(xs[i + 1] / sdeq);
        }
        q_packed[m * (K / 2) + g * 8 + i / 2] = oracle_pack_fp4_pair(c0, c1);
      }
    }
  }
}

void oracle_router(int64_t T, int64_t H, int64_t E, const float *x,
                   const float *router, float *logits, float *probs) {
  for (int64_t t = 0; t < T; ++t) {
    float mx = -INFINITY;
    for (int64_t e = 0; e < E; ++e) {
      float acc = 0.0f;
      for (int64_t h = 0; h < H; ++h) acc += x[t * H + h] * router[h * E + e];
      logits[t * E + e] = acc;
      if (acc > mx) mx = acc;
    }
    float sum = 0.0f;
    for (int64_t e = 0; e < E; ++e) {
      float p = expf(logits[t * E + e] - mx);
      probs[t * E + e] = p;
      sum += p;
    }
    for (int64_t e = 0; e < E; ++e) probs[t * E + e] = probs[t * E + e] / sum;
  }
}

/* Top-k by descending probability, ties to the lower index. */
static void select_topk(const float *p, int64_t E, int64_t k, int32_t *ids) {
  for (int64_t j = 0; j < k; ++j) {
    int64_t best = -1;
    for (int64_t e = 0; e < E; ++e) {
      int taken = 0;
      for (int64_t i = 0; i < j; ++i)
        if (ids[i] == e) taken = 1;
      if (taken) continue;
      if (best < 0 || p[e] > p[best]) best = e;
    }
    ids[j] = (int32_t)best;
  }
}

void oracle_moe(int64_t T, int64_t H, int64_t I, int64_t E, int64_t top_k,
                int renormalize, const float *x, const float *router,
                const uint8_t *gu_w, const uint8_t *gu_sf, const float *gu_ws2,
                const float *gu_in_scale, const uint8_t *dn_w,
                const uint8_t *dn_sf, const float *dn_ws2,
                const float *dn_in_scale, float *out,
                const int64_t *tokens, int64_t n_tok, int32_t *topk_ids,
                float *topk_w, const int32_t *force_ids, int n_threads) {
  int64_t R = tokens ? n_tok : T;
#ifdef _OPENMP
  if (n_threads < 1) n_threads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(n_threads)
#endif
  for (int64_t r = 0; r < R; ++r) {
    int64_t t = tokens ? tokens[r] : r;
    const float *xt = x + t * H;
    float *logits = (float *)malloc(sizeof(float) * E);
    float *probs = (float *)malloc(sizeof(float) * E);
    float *h = (float *)malloc(sizeof(float) * 2 * I);
    float *a = (float *)malloc(sizeof(float) * I);
    float *y = (float *)malloc(sizeof(float) * H);
    int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * top_k);
    float *w = (float *)malloc(sizeof(float) * top_k);
    oracle_router(1, H, E, xt, router, logits, probs);
    if (force_ids)
      memcpy(ids, force_ids + r * top_k, sizeof(int32_t) * top_k);
    else
      select_topk(probs, E, top_k, ids);
    float wsum = 0.0f;
    for (int64_t j = 0; j < top_k; ++j) {
      w[j] = probs[ids[j]];
      wsum += w[j];
    }
    if (renormalize)
      for (int64_t j = 0; j < top_k; ++j) w[j] = w[j] / wsum;
    float *o = out + r * H;
    for (int64_t i = 0; i < H; ++i) o[i] = 0.0f;
    for (int64_t j = 0; j < top_k; ++j) {
      int64_t e = ids[j];
      float gis = gu_in_scale ? gu_in_scale[e] : 1.0f;
      float dis = dn_in_scale ? dn_in_scale[e] : 1.0f;
      oracle_matvec(H, 2 * I, gis, 1.0f, gu_ws2 + e * 2 * I,
                    gu_w + e * (2 * I) * (H / 2), gu_sf + e * (2 * I) * (H / 16), xt, h);
      for (int64_t i = 0; i < I; ++i) a[i] = oracle_silu(h[i]) * h[I + i];
      oracle_matvec(I, H, dis, 1.0f, dn_ws2 + e * H, dn_w + e * H * (I / 2),
                    dn_sf + e * H * (I / 16), a, y);
      for (int64_t i = 0; i < H; ++i) o[i] += w[j] * y[i];
    }
    if (topk_ids) memcpy(topk_ids + r * top_k, ids, sizeof(int32_t) * top_k);
    if (topk_w) memcpy(topk_w + r * top_k, w, sizeof(float) * top_k);
    free(logits); free(probs); free(h); free(a); free(y); free(ids); free(w);
  }
  (void)n_threads;
}

/* ------------------------------------------------------------------------
 * Gated DeltaNet decode step (nvfp4/deltanet.mojo:51-542), fp32, the
 * reference's loops as written.
 * ---------------------------------------------------------------------- */

/* nvfp4/deltanet.mojo:56-63 */
float oracle_softplus(float x) {
  if (x > 20.0f) return x;
  if (x < -20.0f) return 0.0f;
  return logf(1.0f + expf(x));
}

/* matvec (:239-254): result[r] = sum_c mat[r, c] * vec[c], sequential c. */
void oracle_dn_matvec(const float *mat, const float *vec, float *result, int64_t rows,
                      int64_t cols) {
  for (int64_t r = 0; r < rows; ++r) {
    float acc = 0.0f;
    for (int64_t c = 0; c < cols; ++c) acc += mat[r * cols + c] * vec[c];
    result[r] = acc;
  }
}

/* matvec_transposed (:221-236): result[c] = sum_r mat[r, c] * vec[r], sequential r. */
void oracle_dn_matvec_t(const float *mat, const float *vec, float *result, int64_t rows,
                        int64_t cols) {
  for (int64_t c = 0; c < cols; ++c) {
    float acc = 0.0f;
    for (int64_t r = 0; r < rows; ++r) acc += mat[r * cols + c] * vec[r];
    result[c] = acc;
  }
}

/* rms_norm_inplace (:270-284) */
void oracle_rms_norm(float *x, int64_t n, float eps) {
  float sum_sq = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
  const float scale = 1.0f / sqrtf(sum_sq / (float)n + eps);
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] * scale;
}

/* conv1d_step (:287-328): history oldest first, weight[:, kernel-1] on the
 * new input, then the window shifts by one. */
void oracle_conv1d_step(const float *new_input, float *buf, const float *w, float *result,
                        int64_t channels, int64_t kernel, const float *bias) {
  const int64_t hist = kernel - 1;
  for (int64_t ch = 0; ch < channels; ++ch) {
    float acc = 0.0f;
    for (int64_t t = 0; t < hist; ++t) acc += buf[ch * hist + t] * w[ch * kernel + t];
    acc += new_input[ch] * w[ch * kernel + hist];
    if (bias) acc += bias[ch];
    result[ch] = acc;
  }
  for (int64_t ch = 0; ch < channels; ++ch) {
    for (int64_t t = 0; t < hist - 1; ++t) buf[ch * hist + t] = buf[ch * hist + t + 1];
    if (hist > 0) buf[ch * hist + hist - 1] = new_input[ch];
  }
}

/* deltanet_forward (:335-542), one token. */
void oracle_deltanet_forward(int64_t d, int64_t nkh, int64_t nvh, int64_t kd, int64_t vd,
                             int64_t conv_k, float eps, const float *hidden, float *out,
                             const float *w_qkv, const float *w_z, const float *w_b,
                             const float *w_a, const float *w_out, const float *a_log,
                             const float *dt_bias, const float *wc_q, const float *wc_k,
                             const float *wc_v, const float *cb_q, const float *cb_k,
                             const float *cb_v, float *s_matrix, float *buf_q, float *buf_k,
                             float *buf_v) {
  const int64_t vg = nvh / nkh, q_dim = nkh * kd, k_dim = nkh * kd, v_dim = nvh * vd;
  const int64_t qkv_dim = q_dim + k_dim + v_dim, z_dim = nvh * vd;
  float *qkv = (float *)calloc((size_t)qkv_dim, sizeof(float));
  float *z = (float *)calloc((size_t)z_dim, sizeof(float));
  float *braw = (float *)calloc((size_t)nvh, sizeof(float));
  float *araw = (float *)calloc((size_t)nvh, sizeof(float));
  float *q = (float *)calloc((size_t)q_dim, sizeof(float));
  float *k = (float *)calloc((size_t)k_dim, sizeof(float));
  float *v = (float *)calloc((size_t)v_dim, sizeof(float));
  float *beta = (float *)calloc((size_t)nvh, sizeof(float));
  float *decay = (float *)calloc((size_t)nvh, sizeof(float));
  float *o = (float *)calloc((size_t)z_dim, sizeof(float));
  float *vc = (float *)calloc((size_t)vd, sizeof(float));
  float *stk = (float *)calloc((size_t)vd, sizeof(float));
  /* Step 1: projections (:404-426). */
  oracle_dn_matvec(w_qkv, hidden, qkv, qkv_dim, d);
  oracle_dn_matvec(w_z, hidden, z, z_dim, d);
  oracle_dn_matvec(w_b, hidden, braw, nvh, d);
  oracle_dn_matvec(w_a, hidden, araw, nvh, d);
  /* Step 2: causal conv1d on q, k, v (:431-469). */
  oracle_conv1d_step(qkv, buf_q, wc_q, q, q_dim, conv_k, cb_q);
  oracle_conv1d_step(qkv + q_dim, buf_k, wc_k, k, k_dim, conv_k, cb_k);
  oracle_conv1d_step(qkv + q_dim + k_dim, buf_v, wc_v, v, v_dim, conv_k, cb_v);
  /* Step 3: SiLU (:471-479). */
  for (int64_t i = 0; i < q_dim; ++i) q[i] = oracle_silu(q[i]);
  for (int64_t i = 0; i < k_dim; ++i) k[i] = oracle_silu(k[i]);
  for (int64_t i = 0; i < v_dim; ++i) v[i] = oracle_silu(v[i]);
  /* Step 4: beta, decay, per-head recurrence (:481-532). */
  for (int64_t h = 0; h < nvh; ++h) beta[h] = oracle_sigmoid(braw[h]);
  for (int64_t h = 0; h < nvh; ++h) {
    const float a_val = oracle_softplus(a_log[h]);
    const float dt_val = oracle_softplus(araw[h] + dt_bias[h]);
    decay[h] = expf(-a_val * dt_val);
  }
  for (int64_t h = 0; h < nvh; ++h) {
    const int64_t kh = h / vg;
    const float *q_h = q + kh * kd, *k_h = k + kh * kd, *v_h = v + h * vd;
    float *o_h = o + h * vd, *s_h = s_matrix + h * kd * vd;
    oracle_dn_matvec_t(s_h, k_h, stk, kd, vd);
    for (int64_t i = 0; i < vd; ++i) vc[i] = v_h[i] - stk[i];
    const float d_h = decay[h], b_h = beta[h];
    for (int64_t r = 0; r < kd; ++r) {
      const float k_r = k_h[r];
      for (int64_t c = 0; c < vd; ++c) {
        const int64_t idx = r * vd + c;
        s_h[idx] = d_h * s_h[idx] + b_h * k_r * vc[c];
      }
    }
    oracle_dn_matvec_t(s_h, q_h, o_h, kd, vd);
  }
  /* Step 5: output gate (:534-541). */
  for (int64_t h = 0; h < nvh; ++h) oracle_rms_norm(o + h * vd, vd, eps);
  for (int64_t i = 0; i < z_dim; ++i) o[i] = oracle_silu(z[i]) * o[i];
  /* Step 6: output projection (:543-546). */
  oracle_dn_matvec(w_out, o, out, d, z_dim);
  free(qkv); free(z); free(braw); free(araw); free(q); free(k); free(v);
  free(beta); free(decay); free(o); free(vc); free(stk);
}

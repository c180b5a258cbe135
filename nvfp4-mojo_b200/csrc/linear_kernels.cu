// linear_kernels.cu -- NVFP4 dequant, decode-GEMV/skinny GEMM and the
// CUDA-core fp32 linear (sm_100a).
//
// Reference behaviour these kernels reproduce:
//   * dequant: nvfp4/nvfp4_gemm_gpu.mojo:44-96 (load_and_dequant_fp4_tile),
//     nvfp4/config.mojo:106-121 (unpack_fp4_pair, dequant_fp4);
//   * linear: nvfp4/deltanet.mojo:549-584 (nvfp4_matvec) and the kernel body
//     nvfp4/nvfp4_gemm_gpu.mojo:148-182: y = alpha * dequant(W) @ x with fp32
//     accumulation, alpha = input_scale * weight_scale_2 applied at the end.
#include "kernels.h"
#include "nvfp4_common.cuh"

namespace nvfp4 {

// ---------------------------------------------------------------------------
// Dequant.  One thread per 8 codes (one 32-bit word).  HBM-bound: reads
// 4 B codes + 1/2 B scale, writes 32 B (fp32) or 16 B (bf16) per thread.
// ---------------------------------------------------------------------------
__global__ void dequant_f32_kernel(const uint32_t *__restrict__ w,
                                   const uint8_t *__restrict__ sf, int64_t n_words,
                                   int64_t words_per_row, int64_t K, float4 *__restrict__ out) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  int64_t row = i / words_per_row, wi = i % words_per_row;
  uint32_t v = w[i];
  float s = e4m3_to_f32(sf[row * (K / kGroup) + (wi * 8) / kGroup]);
  float f[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = e2m1_to_f32((v >> (4 * j)) & 15u) * s;
  out[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
  out[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
}

// bf16 output through the exact tensor-core decode (decode8_natural), then
// * 2^7: this is the operand the GEMM/GEMV kernels feed their MMAs, so its
// bit-exactness test covers theirs.
__global__ void dequant_bf16_kernel(const uint32_t *__restrict__ w,
                                    const uint8_t *__restrict__ sf, int64_t n_words,
                                    int64_t words_per_row, int64_t K, uint4 *__restrict__ out) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  int64_t row = i / words_per_row, wi = i % words_per_row;
  uint32_t s2 = scale_to_bf16x2_2p119(sf[row * (K / kGroup) + (wi * 8) / kGroup]);
  uint32_t d[4];
  decode8_natural(w[i], s2, d);
  const uint32_t two7 = 0x43004300u;  // bf16x2(128, 128)
  out[i] = make_uint4(bf16x2_mul(d[0], two7), bf16x2_mul(d[1], two7),
                      bf16x2_mul(d[2], two7), bf16x2_mul(d[3], two7));
}

cudaError_t launch_dequant(const uint8_t *w, const uint8_t *sf, int64_t rows, int64_t K,
                           void *out, int out_dtype, cudaStream_t s) {
  int64_t words_per_row = K / 8;
  int64_t n = rows * words_per_row;
  if (n == 0) return cudaSuccess;
  int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (out_dtype == kF32)
    dequant_f32_kernel<<<(unsigned)blocks, threads, 0, s>>>(
        reinterpret_cast<const uint32_t *>(w), sf, n, words_per_row, K,
        reinterpret_cast<float4 *>(out));
  else
    dequant_bf16_kernel<<<(unsigned)blocks, threads, 0, s>>>(
        reinterpret_cast<const uint32_t *>(w), sf, n, words_per_row, K,
        reinterpret_cast<uint4 *>(out));
  return cudaGetLastError();
}

// nvfp4/nvfp4_gemm_gpu.mojo:44-96 -- one thread per packed byte of the tile.
__global__ void dequant_tile_kernel(const uint8_t *__restrict__ w, const uint8_t *__restrict__ sf,
                                    float *__restrict__ out, int64_t weight_stride,
                                    int64_t scale_stride, int64_t start_row, int64_t start_col,
                                    int64_t tile_m, int64_t tile_k) {
  int64_t half = tile_k / kPack;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= tile_m * half) return;
  int64_t m = i / half, k = i % half;
  int64_t row = start_row + m;
  uint32_t p = w[row * weight_stride + start_col / kPack + k];
  float s = e4m3_to_f32(sf[row * scale_stride + (start_col + k * kPack) / kGroup]);
  out[m * tile_k + 2 * k] = e2m1_to_f32(p & 15u) * s;
  out[m * tile_k + 2 * k + 1] = e2m1_to_f32((p >> 4) & 15u) * s;
}

cudaError_t launch_dequant_tile(const uint8_t *w, const uint8_t *sf, float *out,
                                int64_t weight_stride, int64_t scale_stride,
                                int64_t start_row, int64_t start_col, int64_t tile_m,
                                int64_t tile_k, cudaStream_t s) {
  int64_t n = tile_m * (tile_k / kPack);
  if (n == 0) return cudaSuccess;
  int threads = 256;
  dequant_tile_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, s>>>(
      w, sf, out, weight_stride, scale_stride, start_row, start_col, tile_m, tile_k);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// CUDA-core fp32 linear: one warp per output row, 8 tokens per warp, lanes
// stride over the 16-element groups; fp32 products LUT*scale*x exactly as
// nvfp4_matvec forms them, summed per lane then by warp shuffle.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_act(const void *x, int dt, int64_t idx) {
  if (dt == kF32) return reinterpret_cast<const float *>(x)[idx];
  return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(x)[idx] << 16);
}

__device__ __forceinline__ void store_out(void *y, int dt, int64_t idx, float v) {
  if (dt == kF32)
    reinterpret_cast<float *>(y)[idx] = v;
  else
    reinterpret_cast<uint16_t *>(y)[idx] = f32_to_bf16_bits(v);
}

__global__ void __launch_bounds__(256) linear_f32_kernel(WeightSpec ws, AlphaSpec al,
                                                         const void *x, int x_dt, int64_t xs_m,
                                                         int64_t xs_k, void *y, int y_dt,
                                                         int64_t ys_m, int64_t ys_n, int M) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = blockIdx.x * 8 + warp;
  const int m0 = blockIdx.y * 8;
  if (n >= ws.N) return;
  const int K = ws.K;
  const int groups = K / kGroup;
  const uint8_t *wr = ws.w + (int64_t)n * (K / kPack);
  const uint8_t *sr = ws.sf + (int64_t)n * groups;
  const int mcount = min(8, M - m0);
  float acc[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) acc[m] = 0.0f;
  for (int gi = lane; gi < groups; gi += 32) {
    float s = e4m3_to_f32(sr[gi]);
    const uint8_t *wb = wr + gi * (kGroup / kPack);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      uint32_t p = wb[b];
      int64_t k = (int64_t)gi * kGroup + 2 * b;
      float w0 = e2m1_to_f32(p & 15u) * s;
      float w1 = e2m1_to_f32((p >> 4) & 15u) * s;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        if (m < mcount) {
          int64_t base = (int64_t)(m0 + m) * xs_m;
          acc[m] += w0 * load_act(x, x_dt, base + k * xs_k);
          acc[m] += w1 * load_act(x, x_dt, base + (k + 1) * xs_k);
        }
      }
    }
  }
  float alpha = alpha_of(al, 0, n);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = acc[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && m < mcount) store_out(y, y_dt, (int64_t)(m0 + m) * ys_m + (int64_t)n * ys_n, v * alpha);
  }
}

cudaError_t launch_linear_f32(const WeightSpec &ws, const AlphaSpec &al, const void *x,
                              int x_dtype, int64_t xs_m, int64_t xs_k, void *y, int y_dtype,
                              int64_t ys_m, int64_t ys_n, int M, cudaStream_t s) {
  if (M == 0 || ws.N == 0) return cudaSuccess;
  dim3 grid((ws.N + 7) / 8, (M + 7) / 8);
  linear_f32_kernel<<<grid, 256, 0, s>>>(ws, al, x, x_dtype, xs_m, xs_k, y, y_dtype, ys_m,
                                         ys_n, M);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Skinny tensor-core GEMM (decode GEMV for M <= 8; grouped expert GEMMs with
// few tokens per expert).  HBM-bound on the weights: every weight byte is
// streamed once per CTA with 128-bit non-allocating loads.
//
// CTA = 16 output features x (8*NT) token slots; its warps split K in rounds
// of 128.  In a round, lane (g = lane/4, c = lane%4) loads 16 bytes (32 codes)
// of rows g and g+8 at k = k0 + 32c, decodes them in registers to bf16
// (LUT*scale*2^-7) and issues 8 mma.m16n8k16 per token tile.  The MMA's 16
// logical k slots are a permutation of physical k; the activation fragments
// use the same permutation (prmt of the token's 32 activations), so the sum is
// unchanged.  Partial sums of the warps are reduced in shared memory in a
// fixed order, then scaled by alpha*2^7 and stored.
// ---------------------------------------------------------------------------
// Warps per CTA (they split K) and rounds of codes/scales kept in flight per
// warp ahead of the one being decoded.
#ifndef NVFP4_SKINNY_WARPS
#define NVFP4_SKINNY_WARPS 4
#endif
#ifndef NVFP4_SKINNY_PIPE
#define NVFP4_SKINNY_PIPE 4
#endif
constexpr int kSkinnyWarps = NVFP4_SKINNY_WARPS;
constexpr int kSkinnyPipe = NVFP4_SKINNY_PIPE;

// Per-round operands of one lane: 16 bytes of codes and 2 scales for each of
// its rows (g, g+8, and their `up` rows for the SiLU-gated form), plus the
// token tiles' 32 activations each.
template <int NT, bool SILU>
struct SkinnyRound {
  static constexpr int R = SILU ? 4 : 2;
  uint4 w[R];
  uint32_t s[R];
  int kc;
};

// Full rounds (k0 + 128 <= K): unpredicated loads.  Token slots past the
// item's count read the first slot's row; their columns are never stored.
template <int NT, bool SILU>
__device__ __forceinline__ void skinny_load(SkinnyRound<NT, SILU> &d,
                                            const uint8_t *const (&wp)[SkinnyRound<NT, SILU>::R],
                                            const uint8_t *const (&sp)[SkinnyRound<NT, SILU>::R],
                                            const uint16_t *const (&xrow)[NT], int kc) {
#pragma unroll
  for (int i = 0; i < SkinnyRound<NT, SILU>::R; ++i) {
    d.w[i] = ldg_nc_v4(wp[i] + kc / 2);
    d.s[i] = (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(sp[i] + kc / kGroup));
  }
  d.kc = kc;
  (void)xrow;
}

// Tail round (K % 128 != 0): lanes whose 32-element chunk is past K load
// nothing and contribute zero codes with unit scales.
template <int NT, bool SILU>
__device__ __forceinline__ void skinny_load_tail(SkinnyRound<NT, SILU> &d,
                                                 const uint8_t *const (&wp)[SkinnyRound<NT, SILU>::R],
                                                 const uint8_t *const (&sp)[SkinnyRound<NT, SILU>::R],
                                                 const uint16_t *const (&xrow)[NT], int kc,
                                                 bool kval) {
  if (kval) {
    skinny_load(d, wp, sp, xrow, kc);
  } else {
#pragma unroll
    for (int i = 0; i < SkinnyRound<NT, SILU>::R; ++i) {
      d.w[i] = make_uint4(0, 0, 0, 0);
      d.s[i] = 0x3838u;  // e4m3 1.0, 1.0
    }
    d.kc = -1;  // activations read as zero
  }
}

template <int NT, bool SILU, bool SPLIT, bool TAIL = false>
__device__ __forceinline__ void skinny_compute(const SkinnyRound<NT, SILU> &d,
                                               const uint16_t *const (&xrow)[NT],
                                               const uint16_t *const (&xrow_lo)[NT],
                                               float (&acc)[NT][4], float (&accu)[NT][4],
                                               const uint32_t *slut) {
  constexpr int R = SkinnyRound<NT, SILU>::R;
  // Activations are small and shared by every CTA on the SM: L1-resident.
  // SPLIT: the activations are hi + lo bf16 parts (x = hi + lo to ~2^-16);
  // both multiply the same decoded weights into the same accumulator.
  uint4 xv[NT][4], xl[SPLIT ? NT : 1][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      xv[t][q] = (!TAIL || d.kc >= 0) ? __ldg(reinterpret_cast<const uint4 *>(xrow[t] + d.kc + 8 * q))
                                      : make_uint4(0, 0, 0, 0);
      if (SPLIT)
        xl[SPLIT ? t : 0][q] = (!TAIL || d.kc >= 0)
                                   ? __ldg(reinterpret_cast<const uint4 *>(xrow_lo[t] + d.kc + 8 * q))
                                   : make_uint4(0, 0, 0, 0);
    }
  // e4m3 -> bf16x2 (scale * 2^119) through the CTA's 256-entry table.
  uint32_t sc[R][2];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    sc[i][0] = slut[d.s[i] & 0xffu];
    sc[i][1] = slut[(d.s[i] >> 8) & 0xffu];
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int gsel = q >> 1;
    uint32_t dec[R][4];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const uint32_t wq = q == 0 ? d.w[i].x : q == 1 ? d.w[i].y : q == 2 ? d.w[i].z : d.w[i].w;
      decode8_raw_pairs(wq, dec[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) dec[i][j] = bf16x2_mul(dec[i][j], sc[i][gsel]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t A[4] = {dec[0][2 * h], dec[1][2 * h], dec[0][2 * h + 1], dec[1][2 * h + 1]};
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint32_t x0 = h ? xv[t][q].y : xv[t][q].x;
        const uint32_t x1 = h ? xv[t][q].w : xv[t][q].z;
        const uint32_t b0 = prmt(x0, x1, 0x5410u), b1 = prmt(x0, x1, 0x7632u);
        mma_bf16_16816(acc[t], A, b0, b1);
        if (SPLIT) {
          const uint32_t l0 = h ? xl[SPLIT ? t : 0][q].y : xl[SPLIT ? t : 0][q].x;
          const uint32_t l1 = h ? xl[SPLIT ? t : 0][q].w : xl[SPLIT ? t : 0][q].z;
          mma_bf16_16816(acc[t], A, prmt(l0, l1, 0x5410u), prmt(l0, l1, 0x7632u));
        }
        if (SILU) {
          const uint32_t AU[4] = {dec[2 % R][2 * h], dec[3 % R][2 * h], dec[2 % R][2 * h + 1],
                                  dec[3 % R][2 * h + 1]};
          mma_bf16_16816(accu[t], AU, b0, b1);
        }
      }
    }
  }
}

template <int NT, bool SILU, bool SPLIT>
__global__ void __launch_bounds__(32 * kSkinnyWarps,
                                  (NT == 1 && !SILU && !SPLIT) ? 7
                                  : (NT == 4 ? 2 : ((SILU || SPLIT) ? 3 : 4)) * 4 / kSkinnyWarps)
    skinny_kernel(SkinnyArgs a) {
  constexpr int NACC = NT * 4 * (SILU ? 2 : 1);
  constexpr int RR = SILU ? 4 : 2;
  // The cp.async ring and, after the main loop, the cross-warp reduction
  // share one buffer.
  constexpr int RING_BYTES = kSkinnyWarps * kSkinnyPipe * (RR * 512 + RR * 128);
  constexpr int RED_BYTES = kSkinnyWarps * NACC * 32 * 4;
  __shared__ uint32_t slut[256];
  __shared__ __align__(16) uint8_t skinny_smem[RING_BYTES > RED_BYTES ? RING_BYTES : RED_BYTES];
  float(*red)[NACC][32] = reinterpret_cast<float(*)[NACC][32]>(skinny_smem);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) slut[i] = scale_to_bf16x2_2p119(i);
  __syncthreads();

  int group = 0, slot0, count;
  if (a.work) {
    if ((int)blockIdx.y >= *a.n_work) return;
    SkinnyWork wk = a.work[blockIdx.y];
    group = wk.group;
    slot0 = wk.slot0;
    count = wk.count;
  } else {
    slot0 = blockIdx.y * (8 * NT);
    count = min(8 * NT, a.M - slot0);
  }
  const int Nout = SILU ? a.ws.N / 2 : a.ws.N;
  const int row0 = blockIdx.x * 16;
  const int K = a.ws.K;
  const int64_t wld = K / kPack, sld = K / kGroup;
  const uint8_t *W = a.ws.w + (int64_t)group * a.ws.w_group_stride;
  const uint8_t *SF = a.ws.sf + (int64_t)group * a.ws.sf_group_stride;
  // Rows past N are clamped for loading (always valid memory), never stored.
  const int ra = min(row0 + g, Nout - 1), rb = min(row0 + g + 8, Nout - 1);
  const int rows[4] = {ra, rb, ra + Nout, rb + Nout};
  constexpr int R = SkinnyRound<NT, SILU>::R;
  const uint8_t *wp[R];
  const uint8_t *sp[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    wp[i] = W + rows[i] * wld;
    sp[i] = SF + rows[i] * sld;
  }

  const uint16_t *xrow[NT];
  const uint16_t *xrow_lo[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int sl = 8 * t + g;
    const int slot = slot0 + (sl < count ? sl : 0);
    const int64_t r = a.x_rows ? a.x_rows[slot] : slot;
    xrow[t] = a.x + r * a.x_ld;
    xrow_lo[t] = SPLIT ? a.x_lo + r * a.x_ld : nullptr;
  }

  float acc[NT][4], accu[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = accu[t][i] = 0.0f;

  // Software pipeline over this warp's full rounds r = warp + i * nwarps:
  // cp.async streams each lane's 16-byte code chunks (and the 4 scale bytes
  // holding its two blockscales) into a per-warp shared-memory ring that is
  // kSkinnyPipe rounds deep, so the HBM latency is covered without holding
  // the data in registers.  Each lane reads back only what it copied itself.
  constexpr int PD = kSkinnyPipe;
  constexpr int WSTAGE = R * 512;       // bytes of codes per round per warp
  constexpr int SSTAGE = R * 32 * 4;    // bytes of scales per round per warp
  uint8_t *wring = skinny_smem + warp * PD * (WSTAGE + SSTAGE);
  uint8_t *sring = wring + PD * WSTAGE;
  const uint32_t wr0 = smem_addr(wring) + g * 64 + c * 16;
  const uint32_t sr0 = smem_addr(sring) + lane * 4;
  const int full = K / 128;
  const int cbyte = 4 * (c >> 1);         // this lane's 4-byte scale word within the 8
  const int cshift = 16 * (c & 1);        // and its two bytes within that word
#pragma unroll
  for (int i = 0; i < PD; ++i) {
    const int rr = warp + i * nwarps;
    if (rr < full) {
      const int kc = rr * 128 + 32 * c;
#pragma unroll
      for (int q = 0; q < R; ++q) {
        cp_async_16(wr0 + i * WSTAGE + q * 512, wp[q] + kc / 2);
        cp_async_4(sr0 + i * SSTAGE + q * 128, sp[q] + rr * 8 + cbyte);
      }
    }
    cp_async_commit();
  }
  int stage = 0;
  for (int i = 0;; ++i) {
    const int rr = warp + i * nwarps;
    if (rr >= full) break;
    cp_async_wait<PD - 1>();
    SkinnyRound<NT, SILU> d;
#pragma unroll
    for (int q = 0; q < R; ++q) {
      d.w[q] = lds_v4(wr0 + stage * WSTAGE + q * 512);
      d.s[q] = (lds_u32(sr0 + stage * SSTAGE + q * 128) >> cshift) & 0xffffu;
    }
    d.kc = rr * 128 + 32 * c;
    skinny_compute<NT, SILU, SPLIT>(d, xrow, xrow_lo, acc, accu, slut);
    const int rl = rr + PD * nwarps;
    if (rl < full) {
      const int kc = rl * 128 + 32 * c;
#pragma unroll
      for (int q = 0; q < R; ++q) {
        cp_async_16(wr0 + stage * WSTAGE + q * 512, wp[q] + kc / 2);
        cp_async_4(sr0 + stage * SSTAGE + q * 128, sp[q] + rl * 8 + cbyte);
      }
    }
    cp_async_commit();
    stage = stage + 1 == PD ? 0 : stage + 1;
  }
  cp_async_wait<0>();
  SkinnyRound<NT, SILU> buf[1];
  if ((K % 128) != 0 && warp == (full % nwarps)) {
    const int kc = full * 128 + 32 * c;
    skinny_load_tail(buf[0], wp, sp, xrow, kc, kc < K);
    skinny_compute<NT, SILU, SPLIT, true>(buf[0], xrow, xrow_lo, acc, accu, slut);
  }

  // Cross-warp reduction in a fixed order (the ring's memory is reused).
  __syncthreads();
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      red[warp][t * 4 + i][lane] = acc[t][i];
      if (SILU) red[warp][NT * 4 + t * 4 + i][lane] = accu[t][i];
    }
  __syncthreads();

  // Output o = token_local * 16 + row_local; consecutive threads write
  // consecutive features of one token.
  const int n_out = 16 * 8 * NT;
  for (int o = threadIdx.x; o < n_out; o += blockDim.x) {
    const int tl = o >> 4, rl = o & 15;
    const int t = tl >> 3, tt = tl & 7;
    const int cc = tt >> 1, lo = tt & 1;
    const int gg = rl & 7, reg = (rl >> 3) * 2 + lo;
    const int ln = gg * 4 + cc;
    const int n = row0 + rl;
    if (tl >= count || n >= Nout) continue;
    float v = 0.0f, vu = 0.0f;
    for (int w = 0; w < nwarps; ++w) {
      v += red[w][t * 4 + reg][ln];
      if (SILU) vu += red[w][NT * 4 + t * 4 + reg][ln];
    }
    float out;
    if (SILU) {
      float hg = v * (alpha_of(a.al, group, n) * kDecodeUnscale);
      float hu = vu * (alpha_of(a.al, group, n + Nout) * kDecodeUnscale);
      out = silu_f32(hg) * hu;
    } else {
      out = v * (alpha_of(a.al, group, n) * kDecodeUnscale);
    }
    const int slot = slot0 + tl;
    const int64_t yr = a.y_rows ? a.y_rows[slot] : slot;
    if (a.y_lo) {
      // bf16 hi part and the bf16 of the remainder: hi + lo == out to ~2^-16.
      const uint16_t hb = f32_to_bf16_bits(out);
      reinterpret_cast<uint16_t *>(a.y)[yr * a.y_ld + n] = hb;
      a.y_lo[yr * a.y_ld + n] = f32_to_bf16_bits(out - __uint_as_float((uint32_t)hb << 16));
    } else {
      store_out(a.y, a.y_dtype, yr * a.y_ld + n, out);
    }
  }
}

cudaError_t launch_skinny(const SkinnyArgs &a, cudaStream_t s) {
  const int Nout = a.silu_gate ? a.ws.N / 2 : a.ws.N;
  if (Nout == 0) return cudaSuccess;
  const int tpi = a.tokens_per_item;
  const int items = a.work ? a.work_capacity : (a.M + tpi - 1) / tpi;
  if (items == 0) return cudaSuccess;
  const int rounds = (a.ws.K + 127) / 128;
  const int nwarps = rounds < kSkinnyWarps ? rounds : kSkinnyWarps;
  dim3 grid((Nout + 15) / 16, items);
  dim3 block(32 * nwarps);
#define NVFP4_SKINNY(NT_)                                                  \
  do {                                                                     \
    if (a.silu_gate)                                                       \
      skinny_kernel<NT_, true, false><<<grid, block, 0, s>>>(a);           \
    else if (a.x_lo)                                                       \
      skinny_kernel<NT_, false, true><<<grid, block, 0, s>>>(a);           \
    else                                                                   \
      skinny_kernel<NT_, false, false><<<grid, block, 0, s>>>(a);          \
  } while (0)
  if (tpi == 8)
    NVFP4_SKINNY(1);
  else if (tpi == 16)
    NVFP4_SKINNY(2);
  else if (tpi == 32)
    NVFP4_SKINNY(4);
  else
    return cudaErrorInvalidValue;
#undef NVFP4_SKINNY
  return cudaGetLastError();
}

}  // namespace nvfp4

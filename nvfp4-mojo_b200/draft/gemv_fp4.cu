// gemv_fp4.cu -- DRAFT, not part of libnvfp4.so: it compiles for sm_100a
// beside the sources in ../csrc (copy it there to build it) but has not yet
// run on a GPU, so nothing calls it.  To wire it in: an opt-in flag of
// nvfp4_linear_forward for M <= 8, K % 256 == 0, K <= 8192, its scratch
// (digits, scales, partial sums: gemv_fp4_scratch_bytes) taken from
// stream-ordered memory as the W4A4 path does.  Decode GEMV y[M, N] =
// alpha[n] * x[M, K] . W[N, K]^T (M <= 8) on the block-scaled FP4 tensor
// cores, with no per-weight decode.
//
// The weights go to tcgen05.mma kind::mxf4nvf4 exactly as stored (E2M1
// codes, E4M3 scales per 16).  The bf16 activations are written as a sum of
// kDg FP4 "digits": digit d of token t is the NVFP4 quantization of the
// residual left by digits 0..d-1, under a per-(token, digit) fp32 scale
// s[t][d] = amax(residual) / (6 * 448) so that every block scale fits E4M3.
// B = the M * kDg digit rows (row t * kDg + d); the token's output is
// sum_d s[t][d] * acc[t * kDg + d].
//
// Kernels (chained by programmatic dependent launch):
//   fp4_digits_kernel  one CTA per token: kDg rounds of (row amax, per-16
//                      E4M3 scale, E2M1 codes RNE, residual update);
//   fp4_gemv_kernel    persistent, one CTA per SM, stream-K: the N/128 x
//                      K/256 (tile, chunk) units split evenly over the CTAs;
//                      a CTA's units form at most a few tile segments, each
//                      accumulated in TMEM (double-buffered) and written,
//                      digit-summed, to a partial-sum workspace;
//                      warp 0 TMA (weights 128 x 128 B + scales, digits
//                      32 x 128 B + scales), warp 1 TMEM + MMA issue (N = 128
//                      instruction shape of the W4A4 kernel; B rows >= 32 are
//                      never written and their accumulator columns never
//                      read), warps 2-5 scale movers, warps 6-9 epilogue;
//   fp4_finalize_kernel  y[t][n] = alpha[n] * the partial sums of the CTAs
//                      that covered tile n / 128, in CTA order.
#include <cuda.h>

#include "../../include/nvfp4.h"
#include "abi_util.h"
#include "kernels.h"
#include "nvfp4_common.cuh"
#include "tc_common.cuh"

namespace nvfp4 {

bool make_tmap_2d(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base,
                  int64_t rows, int64_t cols, int64_t ld_elems, int box_cols, int box_rows,
                  CUtensorMapSwizzle sw);
int tc_sm_count();

namespace {

static __device__ int g_fp4gv_status;

constexpr int kDg = 4;                     // digits per token
constexpr int kDgTok = 8;                  // tokens per call (M <= 8)
constexpr int kDgRows = kDg * kDgTok;      // B rows loaded per chunk
constexpr int kDgMaxK = 8192;              // digits kernel: 2 groups of 16 per thread
constexpr int kGvBM = 128;                 // weight rows per tile (MMA M)
constexpr int kGvBN = 128;                 // MMA N (only kDgRows columns are used)
constexpr int kGvBK = 256;                 // k per chunk
constexpr int kGvStages = 5;
constexpr int kGvSfCols = 32;              // TMEM scale columns per stage (A 16 + B 16)
constexpr int kGvThreads = 10 * 32;
constexpr int kGvTmemCols = 512;           // 2 x 128 accumulators + 5 x 32 scale columns

struct GvSmem {
  static constexpr int kA = kGvBM * kGvBK / 2;    // 16 KB
  static constexpr int kB = kGvBN * kGvBK / 2;    // 16 KB region, first 4 KB loaded
  static constexpr int kSA = kGvBM * kGvBK / 16;  // 2 KB
  static constexpr int kSB = kGvBN * kGvBK / 16;  // 2 KB region, first 512 B loaded
  static constexpr int kStage = kA + kB + kSA + kSB;
  static constexpr int kTx = kA + kDgRows * (kGvBK / 2) + kSA + kDgRows * (kGvBK / 16);
  static constexpr int offBar = kGvStages * kStage;
  static constexpr int nBars = 3 * kGvStages + 4;
  static constexpr int offTmem = offBar + nBars * 8;
  static constexpr int bytes = offTmem + 16;
  static constexpr int alloc = bytes + 1024;
  static_assert(kStage % 1024 == 0, "stages stay 1024-byte aligned");
  static_assert(alloc <= 227 * 1024, "shared memory per CTA");
};
static_assert(2 * kGvBN + kGvStages * kGvSfCols <= kGvTmemCols, "TMEM columns");

__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}

// Adds `bytes` to the phase's expected transaction count without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tmem_st_wait_all() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t e2m1x2_rn(float even_k, float odd_k) {
  uint32_t r;
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; cvt.u32.u8 %0, t; }"
      : "=r"(r)
      : "f"(odd_k), "f"(even_k));
  return r;
}

__device__ __forceinline__ uint32_t e4m3_rn(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xFFu;
}

// ---------------------------------------------------------------------------
// Digits: CTA t quantizes token t's row into kDg NVFP4 digit rows.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fp4_digits_kernel(const uint16_t *__restrict__ x,
                                                         int64_t x_ld, int K,
                                                         uint8_t *__restrict__ q,
                                                         uint8_t *__restrict__ qsf,
                                                         float *__restrict__ sd) {
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = K / kGroup;
  pdl_wait();  // x comes from the previous kernel
  pdl_trigger();
  float v[2][16];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int g = tid + 256 * i;
    if (g < G) {
      const uint4 *p = reinterpret_cast<const uint4 *>(x + (int64_t)t * x_ld + g * kGroup);
      const uint4 a = __ldcg(p), b = __ldcg(p + 1);
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][2 * j] = bf16lo(w[j]);
        v[i][2 * j + 1] = bf16hi(w[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[i][j] = 0.0f;
    }
  }
  for (int d = 0; d < kDg; ++d) {
    float ga[2];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      ga[i] = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) ga[i] = fmaxf(ga[i], fabsf(v[i][j]));
      m = fmaxf(m, ga[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();  // red[] of the previous digit has been read
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float amax = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
    const float s = amax / (6.0f * 448.0f);  // 0 for an all-zero residual
    const int row = t * kDg + d;
    if (tid == 0) sd[row] = s;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int g = tid + 256 * i;
      if (g >= G) continue;
      const uint32_t sf = s > 0.0f ? e4m3_rn(ga[i] / (6.0f * s)) : 0u;
      const float sff = e4m3_to_f32(sf);
      const float sdeq = sff * s;
      uint32_t packed[2] = {0u, 0u};
      if (sdeq != 0.0f) {
        // Residual as the oracle forms it: (LUT * scale, exact) * s, then
        // the subtraction, each rounded once (no contraction into an FMA).
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t c = e2m1x2_rn(v[i][2 * j] / sdeq, v[i][2 * j + 1] / sdeq);
          packed[j >> 2] |= c << (8 * (j & 3));
          v[i][2 * j] = __fsub_rn(v[i][2 * j], __fmul_rn(e2m1_to_f32(c & 15u) * sff, s));
          v[i][2 * j + 1] = __fsub_rn(v[i][2 * j + 1], __fmul_rn(e2m1_to_f32(c >> 4) * sff, s));
        }
      }
      *reinterpret_cast<uint2 *>(q + (int64_t)row * (K / 2) + g * 8) =
          make_uint2(packed[0], packed[1]);
      qsf[(int64_t)row * G + g] = (uint8_t)sf;
    }
  }
}

// ---------------------------------------------------------------------------
// Stream-K FP4 GEMV.
// ---------------------------------------------------------------------------
struct GvArgs {
  int M, N, K;
  int KB;        // chunks per row
  int n_tiles;   // N / 128 (rounded up)
  int64_t U;     // units = n_tiles * KB
  int segs;      // workspace segments per CTA
  const float *sd;  // [M * kDg] digit scales
  float *ws;        // [grid][segs][kDgTok][128] partial sums
};

__device__ __forceinline__ int64_t unit_lo(int64_t U, int G, int b) { return U * b / G; }

__global__ void __launch_bounds__(kGvThreads, 1)
    fp4_gemv_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmSA,
                    const __grid_constant__ CUtensorMap tmSB, GvArgs a) {
  using L = GvSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::offBar;
  const uint32_t bar_sf = bar_full + 8 * kGvStages;
  const uint32_t bar_empty = bar_sf + 8 * kGvStages;
  const uint32_t bar_tfull = bar_empty + 8 * kGvStages;
  const uint32_t bar_tempty = bar_tfull + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::offTmem);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t lo = unit_lo(a.U, gridDim.x, blockIdx.x);
  const int64_t hi = unit_lo(a.U, gridDim.x, blockIdx.x + 1);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kGvStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_sf + 8 * s, 4);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_tfull + 8 * b, 1);
      mbar_init(bar_tempty + 8 * b, 4);
    }
    mbar_fence_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmSA);
    prefetch_tmap(&tmSB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kGvTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_sf = tmem + 2 * kGvBN;
  volatile int *abort = &abort_flag;
  // Programmatic dependent launch: the digits (B, their scales, sd) come
  // from the previous kernel, the weights do not.  The producer issues the
  // first stages' weight loads before griddepcontrol.wait (their phases
  // cannot complete before the digit loads' arrive.expect_tx); every other
  // thread waits first.  The weight buffers must therefore not be written by
  // the kernel launched just before this one.
  const bool pre_issue = warp == 0 && lane == 0;
  if (!pre_issue) {
    pdl_wait();
    pdl_trigger();
  }

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      constexpr int kTxA = L::kA + L::kSA;
      // Weights of the first stages, before the wait.
      const int pre = hi - lo < kGvStages ? (int)(hi - lo) : kGvStages;
      for (int g = 0; g < pre; ++g) {
        const int64_t u = lo + g;
        const int tile = (int)(u / a.KB), kb = (int)(u % a.KB);
        const uint32_t st = sbase + g * L::kStage;
        mbar_expect_tx(bar_full + 8 * g, kTxA);
        tma_load_2d(st, &tmA, kb * (kGvBK / 2), tile * kGvBM, bar_full + 8 * g);
        tma_load_2d(st + L::kA + L::kB, &tmSA, kb * (kGvBK / 16), tile * kGvBM,
                    bar_full + 8 * g);
      }
      pdl_wait();
      pdl_trigger();
      int g = 0, issued = 0;
      for (int64_t u = lo; u < hi; ++u, ++g) {
        const int tile = (int)(u / a.KB), kb = (int)(u % a.KB);
        const int s = g % kGvStages, ph = g / kGvStages;
        if (ph > 0 && !mbar_wait(bar_empty + 8 * s, (ph - 1) & 1, &g_fp4gv_status,
                                 kDevTimeoutEmpty, abort))
          break;
        const uint32_t st = sbase + s * L::kStage;
        if (g < pre) {
          mbar_arrive_expect_tx(bar_full + 8 * s, L::kTx - kTxA);
        } else {
          mbar_arrive_expect_tx(bar_full + 8 * s, L::kTx);
          tma_load_2d(st, &tmA, kb * (kGvBK / 2), tile * kGvBM, bar_full + 8 * s);
          tma_load_2d(st + L::kA + L::kB, &tmSA, kb * (kGvBK / 16), tile * kGvBM,
                      bar_full + 8 * s);
        }
        tma_load_2d(st + L::kA, &tmB, kb * (kGvBK / 2), 0, bar_full + 8 * s);
        tma_load_2d(st + L::kA + L::kB + L::kSA, &tmSB, kb * (kGvBK / 16), 0, bar_full + 8 * s);
        issued = g + 1;
      }
      // (The loop cannot stop before `pre`: its first waits come at g >= S.)
      for (int qq = issued - kGvStages > 0 ? issued - kGvStages : 0; qq < issued; ++qq) {
        volatile int no_abort = 0;
        mbar_wait(bar_full + 8 * (qq % kGvStages), (qq / kGvStages) & 1, &g_fp4gv_status,
                  kDevTimeoutFull, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kGvBM, kGvBN);
      int g = 0, i = 0;
      bool ok = true;
      for (int64_t u = lo; u < hi && ok; ++i) {
        const int tile = (int)(u / a.KB);
        const int64_t seg_end = min(hi, (int64_t)(tile + 1) * a.KB);
        const int b = i & 1, ub = i >> 1;
        if (ub > 0 && !mbar_wait(bar_tempty + 8 * b, (ub - 1) & 1, &g_fp4gv_status,
                                 kDevTimeoutAcc, abort))
          break;
        tc_fence_after();
        const uint32_t d = tmem + b * kGvBN;
        for (int64_t uu = u; uu < seg_end; ++uu, ++g) {
          const int s = g % kGvStages, ph = g / kGvStages;
          if (!mbar_wait(bar_full + 8 * s, ph & 1, &g_fp4gv_status, kDevTimeoutFull, abort) ||
              !mbar_wait(bar_sf + 8 * s, ph & 1, &g_fp4gv_status, kDevTimeoutDec, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * L::kStage, sb = sa + L::kA;
          const uint32_t sf = tmem_sf + s * kGvSfCols;
#pragma unroll
          for (int j = 0; j < kGvBK / 64; ++j)
            mma_nvf4(d, sw128_kmajor_desc(sa + 32 * j), sw128_kmajor_desc(sb + 32 * j), idesc,
                     sf + 4 * j, sf + 16 + 4 * j, (uu != u || j != 0) ? 1u : 0u);
          tc_commit(bar_empty + 8 * s);
        }
        tc_commit(bar_tfull + 8 * b);
        u = seg_end;
      }
    }
  } else if (warp < 6) {
    // ---------------- blockscale movers (as in the W4A4 kernel) ----------------
    const int q = warp & 3;
    int g = 0;
    for (int64_t u = lo; u < hi; ++u, ++g) {
      const int s = g % kGvStages, ph = g / kGvStages;
      const bool w_ok =
          mbar_wait(bar_full + 8 * s, ph & 1, &g_fp4gv_status, kDevTimeoutFull, abort);
      if (!__all_sync(0xffffffffu, w_ok)) break;
      const uint8_t *sfa = smem + s * L::kStage + L::kA + L::kB;
      const uint8_t *sfb = sfa + L::kSA;
      const uint32_t col = tmem_sf + s * kGvSfCols + (static_cast<uint32_t>(32 * q) << 16);
#pragma unroll
      for (int op = 0; op < 2; ++op) {
        const uint8_t *src = op == 0 ? sfa : sfb;
        uint32_t v[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 r = *reinterpret_cast<const uint4 *>(src + 16 * (lane + 32 * c));
          v[c] = r.x;
          v[4 + c] = r.y;
          v[8 + c] = r.z;
          v[12 + c] = r.w;
        }
        tmem_st_x16(col + 16 * op, v);
      }
      tmem_st_wait_all();
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sf + 8 * s);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    int i = 0;
    for (int64_t u = lo; u < hi; ++i) {
      const int tile = (int)(u / a.KB);
      const int64_t seg_end = min(hi, (int64_t)(tile + 1) * a.KB);
      const int b = i & 1, ub = i >> 1;
      const bool w_ok =
          mbar_wait(bar_tfull + 8 * b, ub & 1, &g_fp4gv_status, kDevTimeoutAcc, abort);
      if (!__all_sync(0xffffffffu, w_ok && !*abort)) break;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * kGvBN, v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty + 8 * b);
      float *wsp = a.ws + (((int64_t)blockIdx.x * a.segs + i) * kDgTok) * kGvBM + 32 * q + lane;
#pragma unroll
      for (int t = 0; t < kDgTok; ++t) {
        float p = 0.0f;
        if (t < a.M) {
#pragma unroll
          for (int d = 0; d < kDg; ++d)
            p = fmaf(__ldcg(a.sd + t * kDg + d), __uint_as_float(v[t * kDg + d]), p);
        }
        wsp[t * kGvBM] = p;
      }
      u = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kGvTmemCols);
  }
}

// y[t][n] = alpha[n] * sum over the CTAs that covered n's tile, in CTA order.
template <typename OutT>
__global__ void fp4_finalize_kernel(GvArgs a, int grid, AlphaSpec al, OutT *__restrict__ y,
                                    int64_t y_ld) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  if (i >= (int64_t)a.M * a.N) return;
  const int t = (int)(i / a.N), n = (int)(i % a.N);
  const int tile = n / kGvBM, r = n % kGvBM;
  const int64_t u0 = (int64_t)tile * a.KB, u1 = u0 + a.KB;
  // First CTA whose range contains u0.
  int b = (int)((u0 * grid) / a.U);
  while (b + 1 < grid && unit_lo(a.U, grid, b + 1) <= u0) ++b;
  while (b > 0 && unit_lo(a.U, grid, b) > u0) --b;
  float acc = 0.0f;
  for (; b < grid && unit_lo(a.U, grid, b) < u1; ++b) {
    const int64_t lo = unit_lo(a.U, grid, b);
    if (unit_lo(a.U, grid, b + 1) <= u0) continue;  // empty range before the tile
    const int seg = tile - (int)(lo / a.KB) > 0 ? tile - (int)(lo / a.KB) : 0;
    acc += __ldcg(a.ws + (((int64_t)b * a.segs + seg) * kDgTok + t) * kGvBM + r);
  }
  const float o = acc * alpha_of(al, 0, n);
  if constexpr (sizeof(OutT) == 4)
    y[(int64_t)t * y_ld + n] = o;
  else
    y[(int64_t)t * y_ld + n] = f32_to_bf16_bits(o);
}

struct ScratchLayout {
  size_t q, qsf, sd, ws, total;
};

size_t sup(size_t v) { return (v + 255) & ~size_t(255); }

ScratchLayout scratch_layout(int M, int K, int grid, int segs) {
  ScratchLayout L;
  size_t o = 0;
  L.q = o;
  o = sup(o + (size_t)M * kDg * (K / 2));
  L.qsf = o;
  o = sup(o + (size_t)M * kDg * (K / 16));
  L.sd = o;
  o = sup(o + sizeof(float) * kDgRows);
  L.ws = o;
  o = sup(o + sizeof(float) * (size_t)grid * segs * kDgTok * kGvBM);
  L.total = o;
  return L;
}

void plan(int N, int K, int *grid, int *segs, int64_t *U) {
  const int KB = K / kGvBK, nt = (N + kGvBM - 1) / kGvBM;
  *U = (int64_t)nt * KB;
  const int sms = tc_sm_count();
  *grid = (int)(*U < sms ? *U : sms);
  const int64_t per = (*U + *grid - 1) / *grid;  // most units of one CTA
  *segs = (int)((per + KB - 1) / KB) + 1;
}

}  // namespace

size_t gemv_fp4_scratch_bytes(int M, int N, int K) {
  int grid, segs;
  int64_t U;
  plan(N, K, &grid, &segs, &U);
  return scratch_layout(M, K, grid, segs).total;
}

cudaError_t launch_gemv_fp4(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                            int64_t x_ld, int M, void *y, int y_dtype, int64_t y_ld,
                            uint8_t *scratch, size_t scratch_bytes, cudaStream_t st) {
  if (M <= 0 || M > kDgTok || ws.K % kGvBK || ws.K > kDgMaxK) return cudaErrorInvalidValue;
  int grid, segs;
  int64_t U;
  plan(ws.N, ws.K, &grid, &segs, &U);
  const ScratchLayout SL = scratch_layout(M, ws.K, grid, segs);
  if (scratch_bytes < SL.total) return cudaErrorInvalidValue;
  uint8_t *q = scratch + SL.q, *qsf = scratch + SL.qsf;
  float *sd = reinterpret_cast<float *>(scratch + SL.sd);
  float *part = reinterpret_cast<float *>(scratch + SL.ws);
  cudaError_t e = launch_pdl(fp4_digits_kernel, dim3(M), dim3(256), 0, st, x, x_ld, ws.K, q, qsf,
                             sd);
  if (e != cudaSuccess) return e;
  CUtensorMap tmA, tmB, tmSA, tmSB;
  if (!make_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.w, ws.N, ws.K / 2, ws.K / 2,
                    kGvBK / 2, kGvBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, M * kDg, ws.K / 2, ws.K / 2,
                    kGvBK / 2, kDgRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmSA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.sf, ws.N, ws.K / 16, ws.K / 16,
                    kGvBK / 16, kGvBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tmap_2d(&tmSB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qsf, M * kDg, ws.K / 16, ws.K / 16,
                    kGvBK / 16, kDgRows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    e = cudaFuncSetAttribute(fp4_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GvSmem::alloc);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  GvArgs a;
  a.M = M;
  a.N = ws.N;
  a.K = ws.K;
  a.KB = ws.K / kGvBK;
  a.n_tiles = (ws.N + kGvBM - 1) / kGvBM;
  a.U = U;
  a.segs = segs;
  a.sd = sd;
  a.ws = part;
  e = launch_pdl(fp4_gemv_kernel, dim3(grid), dim3(kGvThreads), (size_t)GvSmem::alloc, st, tmA,
                 tmB, tmSA, tmSB, a);
  if (e != cudaSuccess) return e;
  const int64_t n = (int64_t)M * ws.N;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (y_dtype == kF32)
    return launch_pdl(fp4_finalize_kernel<float>, dim3(blocks), dim3(256), 0, st, a, grid, al,
                      static_cast<float *>(y), y_ld);
  return launch_pdl(fp4_finalize_kernel<uint16_t>, dim3(blocks), dim3(256), 0, st, a, grid, al,
                    static_cast<uint16_t *>(y), y_ld);
}

}  // namespace nvfp4

// Test hook of the draft (no header declaration).
extern "C" size_t nvfp4_draft_fp4gemv_scratch(int M, int N, int K) {
  return nvfp4::gemv_fp4_scratch_bytes(M, N, K);
}

extern "C" int nvfp4_draft_fp4gemv(const uint8_t *w, const uint8_t *sf, const float *ws2_rows,
                                   float input_scale, const void *x, int M, int N, int K,
                                   void *y, int y_dtype, void *scratch, size_t scratch_bytes,
                                   void *stream) {
  nvfp4::WeightSpec ws;
  ws.w = w;
  ws.sf = sf;
  ws.N = N;
  ws.K = K;
  nvfp4::AlphaSpec al;
  al.input_scale = input_scale;
  al.ws2_rows = ws2_rows;
  cudaError_t e = nvfp4::launch_gemv_fp4(ws, al, static_cast<const uint16_t *>(x), K, M, y,
                                         y_dtype, N, static_cast<uint8_t *>(scratch),
                                         scratch_bytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : -3;
}

// gemv_dg.cu -- decode GEMV for M <= 8 tokens on the block-scaled FP4 tensor
// cores, the weights fed to the MMA exactly as stored (no per-weight decode).
//
//   y[t, n] = alpha[n] * sum_k x[t, k] * LUT[code(n, k)] * float(sf(n, k / 16))
//
// (nvfp4_matvec, nvfp4/deltanet.mojo:549-584, for M tokens; alpha applied
// after accumulation, nvfp4/config.mojo:93-95.)
//
// The activations are written as a sum of kDg FP4 "digits": digit d of token
// t is the NVFP4 quantization (per-16 E4M3 scale, E2M1 codes) of the residual
// that digits 0..d-1 leave, under a per-(token, digit) fp32 scale
// s[t][d] = max|residual| / (6 * 448), so every block scale fits E4M3.  Four
// digits rebuild x to ~1e-4 of each 16-block's largest element; the GEMV
// then differs from the exact bf16-operand result by ~5e-4 of RMS, well
// inside the 2e-2 x RMS tolerance of the bf16 paths.  The weights (E2M1
// codes, E4M3 scales per 16) are already the A operand format of
// tcgen05.mma kind::mxf4nvf4.block_scale.block16; the digits are its B
// operand (N = 8 tokens x 4 digits = 32 rows); token t's output is
// sum_d s[t][d] * acc[t * 4 + d].
//
// Why this shape.  On B200 one thread's tcgen05.mma stream completes about
// one instruction per ~480 SM cycles whatever its M x N x K (measured: f16
// K=16 and FP4 K=64 alike, N from 8 to 256), and per-SM MMA throughput grows
// with the number of CTAs issuing.  At 0.5625 bytes per weight the HBM rate
// is ~40 weights per SM cycle: one K=16 f16 MMA (2048 weights) per issuer
// cannot keep up; an M=128, K=64 FP4 MMA carries 8192 weights, and with four
// CTAs per SM (~68 weights per cycle measured) the weight stream, not the
// tensor core, is the bound.  So the CTA is small: 6 warps, <= 56 KB of
// shared memory, 128 TMEM columns.
//
// Kernels (chained by programmatic dependent launch):
//   dg_digits_kernel  one CTA per token: kDg rounds of (row amax -> digit
//                     scale, per-16 E4M3 scales, E2M1 codes round-to-nearest-
//                     even, residual update) into scratch;
//   dg_gemv_kernel    grid (C, tiles): cluster of C CTAs per 128-row weight
//                     tile splits K; warp 4 = TMA producer (weights 128 x
//                     256-k codes + scales, the digit rows 32 x 256-k codes
//                     + scales) through a two-stage ring, warp 5 = TMEM
//                     allocator and MMA issuer, warps 0-3 = blockscale
//                     movers (shared memory -> TMEM in the scale-factor
//                     layout) and the epilogue; the cluster's partial sums
//                     meet in the leader CTA's shared memory (DSMEM), added in
//                     rank order.
// The producer issues the first stages' weight loads before
// griddepcontrol.wait (weights are constant and must not be written by the
// kernel launched just before); the digits are read after it.
#include <cuda.h>

#include <map>
#include <mutex>
#include <tuple>

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

static __device__ int g_gemv_dg_status;

constexpr int kDg = 4;                   // digits per token
constexpr int kDgTok = 8;                // tokens per call
constexpr int kDgRows = kDg * kDgTok;    // B rows (MMA N)
constexpr int kDgMaxK = 16384;           // digits kernel: <= 4 groups of 16 per thread
constexpr int kBM = 128;                 // weight rows per tile (MMA M)
constexpr int kBK = 256;                 // k per stage
constexpr int kStages = 2;
constexpr int kThreads = 192;            // warps 0-3 movers/epilogue, 4 producer, 5 MMA
constexpr int kTmemCols = 128;
// Stage: weight codes (SW128) 16 KB | digit codes (SW128) 4 KB | weight
// scales 2 KB | digit scales 512 B.
constexpr int kOffB = kBM * kBK / 2;                 // 16384
constexpr int kOffSA = kOffB + kDgRows * kBK / 2;    // 20480
constexpr int kOffSB = kOffSA + kBM * kBK / 16;      // 22528
constexpr int kStageTx = kOffSB + kDgRows * kBK / 16;  // 23040 bytes landed per stage
constexpr int kStage = 23552;                        // stride (1024-aligned)
constexpr int kTxA = kBM * kBK / 2 + kBM * kBK / 16;  // weight part of a stage
// TMEM columns: accumulator [0, 32), weight scales 16 per stage, digit
// scales 16 per stage (a 4-column group per MMA, as the scale-factor
// operand address of each MMA is 4-column aligned; the 32 digit rows use the
// group's first column).
constexpr int kColD = 0, kColSA = 32, kColSB = 32 + 16 * kStages;
static_assert(kColSB + 16 * kStages <= kTmemCols, "TMEM columns");
constexpr int kSmemBytes = kStages * kStage + 256;   // + barriers and misc
constexpr int kMaxC = 8;

// Instruction descriptor, kind::mxf4nvf4: E2M1 x E2M1, UE4M3 scales per 16,
// fp32 accumulate, both operands K-major, scale-factor ids 0.
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kDgRows >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(sfa), "r"(sfb)
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

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void st_cluster_f32(uint32_t local_addr, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// E2M1 pair (even k in the low nibble), round-to-nearest-even, saturating.
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
// Digits: CTA t turns token t's row into kDg NVFP4 digit rows t*kDg + d.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dg_digits_kernel(const uint16_t *__restrict__ x,
                                                        int64_t x_ld, int K,
                                                        uint8_t *__restrict__ q,
                                                        uint8_t *__restrict__ qsf,
                                                        float *__restrict__ sd) {
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = K / kGroup;
  pdl_wait();  // x comes from the previous kernel
  pdl_trigger();
  constexpr int kGpt = kDgMaxK / kGroup / 256;  // groups per thread (4)
  float v[kGpt][16];
#pragma unroll
  for (int i = 0; i < kGpt; ++i) {
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
    float ga[kGpt];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < kGpt; ++i) {
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
    for (int i = 0; i < kGpt; ++i) {
      const int g = tid + 256 * i;
      if (g >= G) continue;
      const uint32_t sf = s > 0.0f ? e4m3_rn(ga[i] / (6.0f * s)) : 0u;
      const float sff = e4m3_to_f32(sf);
      const float sdeq = sff * s;
      uint32_t packed[2] = {0u, 0u};
      if (sdeq != 0.0f) {
        const float inv = 1.0f / sdeq;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t c = e2m1x2_rn(v[i][2 * j] * inv, v[i][2 * j + 1] * inv);
          packed[j >> 2] |= c << (8 * (j & 3));
          // The residual keeps exactly what the digit did not represent:
          // (LUT * scale, exact) * s, subtracted in fp32.
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
// GEMV on the block-scaled FP4 tensor cores.
// ---------------------------------------------------------------------------
struct DgArgs {
  AlphaSpec al;
  const float *sd;  // [M * kDg] digit scales
  void *y;
  int y_dtype;
  int64_t y_ld;
  int M, N, K;
  int C;   // CTAs per cluster (K split)
  int ks;  // K per CTA
};

__global__ void __launch_bounds__(kThreads, 4)
    dg_gemv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmSA,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmSB,
                   DgArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + kStages * kStage;
  const uint32_t bar_sf = bar_full + 8 * kStages;
  const uint32_t bar_empty = bar_sf + 8 * kStages;
  const uint32_t bar_dfull = bar_empty + 8 * kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kStages * kStage + 128);
  __shared__ int abort_flag;
  volatile int *abort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int part = a.C > 1 ? (int)cluster_ctarank() : 0;
  const int row0 = blockIdx.y * kBM;
  const int k0 = part * a.ks;
  const int nst = a.ks / kBK;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_sf + 8 * s, 4);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_dfull, 1);
    mbar_fence_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmSA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmSB);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      const int pre = nst < kStages ? nst : kStages;
      // The weights of the first stages stream before the wait (constant).
      for (int g = 0; g < pre; ++g) {
        const uint32_t st = sbase + g * kStage;
        const int kx = k0 + g * kBK;
        mbar_arrive_expect_tx(bar_full + 8 * g, kStageTx);
        tma_load_2d_hint(st, &tmA, kx / 2, row0, bar_full + 8 * g, pol);
        tma_load_2d_hint(st + kOffSA, &tmSA, kx / kGroup, row0, bar_full + 8 * g, pol);
      }
      pdl_wait();  // the digits come from the kernel before
      pdl_trigger();
      for (int g = 0; g < pre; ++g) {
        const uint32_t st = sbase + g * kStage;
        const int kx = k0 + g * kBK;
        tma_load_2d(st + kOffB, &tmB, kx / 2, 0, bar_full + 8 * g);
        tma_load_2d(st + kOffSB, &tmSB, kx / kGroup, 0, bar_full + 8 * g);
      }
      int issued = pre;
      for (int g = pre; g < nst; ++g) {
        const int s = g % kStages;
        if (!mbar_wait(bar_empty + 8 * s, ((g / kStages) - 1) & 1, &g_gemv_dg_status,
                       kDevTimeoutEmpty, abort))
          break;
        const uint32_t st = sbase + s * kStage;
        const int kx = k0 + g * kBK;
        mbar_arrive_expect_tx(bar_full + 8 * s, kStageTx);
        tma_load_2d_hint(st, &tmA, kx / 2, row0, bar_full + 8 * s, pol);
        tma_load_2d_hint(st + kOffSA, &tmSA, kx / kGroup, row0, bar_full + 8 * s, pol);
        tma_load_2d(st + kOffB, &tmB, kx / 2, 0, bar_full + 8 * s);
        tma_load_2d(st + kOffSB, &tmSB, kx / kGroup, 0, bar_full + 8 * s);
        issued = g + 1;
      }
      // No load may still be in flight when the CTA exits.
      for (int g = issued - kStages > 0 ? issued - kStages : 0; g < issued; ++g) {
        volatile int no_abort = 0;
        mbar_wait(bar_full + 8 * (g % kStages), (g / kStages) & 1, &g_gemv_dg_status,
                  kDevTimeoutFull, &no_abort);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    pdl_wait();
    if (lane == 0) {
      for (int g = 0; g < nst; ++g) {
        const int s = g % kStages;
        if (!mbar_wait(bar_sf + 8 * s, (g / kStages) & 1, &g_gemv_dg_status, kDevTimeoutDec,
                       abort))
          break;
        tc_fence_after();
        const uint32_t st = sbase + s * kStage;
#pragma unroll
        for (int j = 0; j < kBK / 64; ++j)
          mma_nvf4(tmem + kColD, sw128_kmajor_desc(st + 32 * j),
                   sw128_kmajor_desc(st + kOffB + 32 * j), tmem + kColSA + 16 * s + 4 * j,
                   tmem + kColSB + 16 * s + 4 * j, (g | j) != 0 ? 1u : 0u);
        tc_commit(bar_empty + 8 * s);
      }
      tc_commit(bar_dfull);  // also after an abort: the epilogue waits for every MMA
    }
    __syncwarp();
  } else {
    // ---------------- blockscale movers (warps 0-3), then the epilogue ----------------
    const int q = warp;  // TMEM lane quarter
    pdl_wait();
    pdl_trigger();
    for (int g = 0; g < nst; ++g) {
      const int s = g % kStages;
      const bool ok =
          mbar_wait(bar_full + 8 * s, (g / kStages) & 1, &g_gemv_dg_status, kDevTimeoutFull, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint8_t *sa = smem + s * kStage + kOffSA;
      const uint8_t *sb = smem + s * kStage + kOffSB;
      // Scale-factor layout (M = 128, and the digit rows): for the MMA j of
      // the stage, row r's four scales (one word) sit in lane r % 32 of
      // column base + 4j + r / 32 (B: rows < 32, so column base + 4j), the
      // 32-lane pattern repeated in each lane quarter.
      uint32_t va[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 r = *reinterpret_cast<const uint4 *>(sa + 16 * (lane + 32 * c));
        va[c] = r.x;
        va[4 + c] = r.y;
        va[8 + c] = r.z;
        va[12 + c] = r.w;
      }
      const uint4 rb = *reinterpret_cast<const uint4 *>(sb + 16 * lane);
      const uint32_t vb[16] = {rb.x, 0u, 0u, 0u, rb.y, 0u, 0u, 0u,
                               rb.z, 0u, 0u, 0u, rb.w, 0u, 0u, 0u};
      const uint32_t lq = static_cast<uint32_t>(32 * q) << 16;
      tmem_st_x16(tmem + lq + kColSA + 16 * s, va);
      tmem_st_x16(tmem + lq + kColSB + 16 * s, vb);
      tmem_st_wait();
      tc_fence_before();
      fence_proxy_async_smem();  // these reads before the next TMA write of the stage
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sf + 8 * s);
    }

    // Epilogue: row r = 32q + lane; column t*4 + d of the accumulator.
    const int r = 32 * q + lane;
    float acc[kDgTok];
#pragma unroll
    for (int t = 0; t < kDgTok; ++t) acc[t] = 0.0f;
    bool have = false;
    {
      volatile int no_abort = 0;
      const bool okd = mbar_wait(bar_dfull, 0, &g_gemv_dg_status, kDevTimeoutAcc, &no_abort);
      if (__all_sync(0xffffffffu, okd) && !*abort) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + kColD, v);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < kDgTok; ++t) {
          if (t < a.M) {
            float p = 0.0f;
#pragma unroll
            for (int d = 0; d < kDg; ++d)
              p = fmaf(__ldcg(a.sd + t * kDg + d), __uint_as_float(v[t * kDg + d]), p);
            acc[t] = p;
          }
        }
        have = true;
      }
    }
    if (a.C > 1) {
      // Partial sums meet in the leader's shared memory, in the stage ring
      // (free once every CTA of the cluster is past its main loop).
      cluster_sync_all();
      if (part != 0) {
        const uint32_t red = sbase + (((part - 1) * kDgTok) * kBM + r) * 4;
#pragma unroll
        for (int t = 0; t < kDgTok; ++t)
          if (t < a.M) st_cluster_f32(red + t * kBM * 4, 0, have ? acc[t] : 0.0f);
      }
      cluster_sync_all();
    }
    if (part == 0 && have) {
      const int n = row0 + r;
      if (n < a.N) {
        const float al = alpha_of(a.al, 0, n);
        const float *red = reinterpret_cast<const float *>(smem);
#pragma unroll
        for (int t = 0; t < kDgTok; ++t) {
          if (t >= a.M) break;
          float v = acc[t];
          for (int c = 1; c < a.C; ++c) v += red[((c - 1) * kDgTok + t) * kBM + r];
          v *= al;
          if (a.y_dtype == kBF16)
            reinterpret_cast<uint16_t *>(a.y)[(int64_t)t * a.y_ld + n] = f32_to_bf16_bits(v);
          else
            reinterpret_cast<float *>(a.y)[(int64_t)t * a.y_ld + n] = v;
        }
      }
    }
  }
  if (a.C > 1 && warp >= 4) {
    cluster_sync_all();
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

struct DgScratch {
  size_t q, qsf, sd, total;
};

size_t dup(size_t v) { return (v + 255) & ~size_t(255); }

DgScratch dg_scratch(int K) {
  DgScratch L;
  size_t o = 0;
  L.q = o;
  o = dup(o + (size_t)kDgRows * (K / 2));
  L.qsf = o;
  o = dup(o + (size_t)kDgRows * (K / kGroup));
  L.sd = o;
  o = dup(o + sizeof(float) * kDgRows);
  L.total = o;
  return L;
}

std::mutex g_dg_mu;
bool g_dg_attr[64] = {};

cudaError_t dg_set_attr() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_dg_mu);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!g_dg_attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(dg_gemv_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes + 1024);
    if (e != cudaSuccess) return e;
    g_dg_attr[dev] = true;
  }
  return cudaSuccess;
}

// Clusters of C CTAs the GPU holds at once (occupancy query, cached).
int dg_cluster_capacity(int C) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(dev, C);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (dg_set_attr() == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes + 1024;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, dg_gemv_kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

// K split C: a divisor of the stage count, at most 8, whose partial buffer
// fits the stage ring.  Cost = waves of clusters x K per CTA, with a premium
// on plans that leave SMs without their four MMA issuers (the per-SM MMA rate
// grows with the CTAs issuing); ties go to the smaller C.
int dg_plan(int N, int K) {
  const int tiles = (N + kBM - 1) / kBM;
  const int nst = K / kBK;
  const int sms = tc_sm_count();
  int bestC = 0;
  double best = 0.0;
  for (int C = 1; C <= kMaxC; ++C) {
    if (nst % C || (C - 1) * kDgTok * kBM * 4 > kStages * kStage) continue;
    const int held = dg_cluster_capacity(C);
    if (held <= 0) continue;
    const int64_t waves = ((int64_t)tiles + held - 1) / held;
    const double per_sm = (double)tiles * C / sms;  // issuers per SM in the wave
    const double mma_slow = per_sm < 4.0 ? 4.0 / (per_sm > 0.25 ? per_sm : 0.25) : 1.0;
    const double cost = (double)waves * (K / C) * (mma_slow > 1.6 ? mma_slow / 1.6 : 1.0);
    if (bestC == 0 || cost < best * 0.999) {
      bestC = C;
      best = cost;
    }
  }
  return bestC;
}

}  // namespace

size_t gemv_dg_scratch_bytes(int K) { return dg_scratch(K).total; }

bool gemv_dg_supported(int M, int N, int K, const void *w, const void *sf, const void *x,
                       int64_t x_ld) {
  return M >= 1 && M <= kDgTok && N >= 1 && K > 0 && K % kBK == 0 && K <= kDgMaxK &&
         ((uintptr_t)w & 15) == 0 && ((uintptr_t)sf & 15) == 0 && ((uintptr_t)x & 15) == 0 &&
         x_ld % 8 == 0 && (N + kBM - 1) / kBM <= 65535;
}

int read_gemv_dg_device_status() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_dg_status, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_gemv_dg_status, &zero, sizeof(int));
  return v;
}

cudaError_t launch_gemv_dg(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                           int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                           uint8_t *scratch, size_t scratch_bytes, cudaStream_t st) {
  if (M == 0 || ws.N == 0) return cudaSuccess;
  const DgScratch SL = dg_scratch(ws.K);
  if (scratch_bytes < SL.total || !scratch) return cudaErrorInvalidValue;
  const int C = dg_plan(ws.N, ws.K);
  if (C == 0) return cudaErrorInvalidValue;
  uint8_t *q = scratch + SL.q, *qsf = scratch + SL.qsf;
  float *sd = reinterpret_cast<float *>(scratch + SL.sd);
  cudaError_t e = launch_pdl(dg_digits_kernel, dim3(M), dim3(256), 0, st, x, x_ld, ws.K, q, qsf, sd);
  if (e != cudaSuccess) return e;
  CUtensorMap tmA, tmSA, tmB, tmSB;
  if (!make_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.w, ws.N, ws.K / 2, ws.K / 2,
                    kBK / 2, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmSA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.sf, ws.N, ws.K / kGroup,
                    ws.K / kGroup, kBK / kGroup, kBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, M * kDg, ws.K / 2, ws.K / 2,
                    kBK / 2, kDgRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmSB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qsf, M * kDg, ws.K / kGroup,
                    ws.K / kGroup, kBK / kGroup, kDgRows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  e = dg_set_attr();
  if (e != cudaSuccess) return e;
  DgArgs a;
  a.al = al;
  a.sd = sd;
  a.y = y;
  a.y_dtype = y_dtype;
  a.y_ld = y_ld;
  a.M = M;
  a.N = ws.N;
  a.K = ws.K;
  a.C = C;
  a.ks = ws.K / C;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, (ws.N + kBM - 1) / kBM, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes + 1024;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, dg_gemv_kernel, tmA, tmSA, tmB, tmSB, a);
}

}  // namespace nvfp4

// w4a4.cu -- W4A4 mode: NVFP4 activations (quantized with input_scale) times
// NVFP4 weights on the block-scaled FP4 tensor cores.
//
//   nvfp4_quantize_act: x [M, K] (bf16 or fp32) -> codes [M, K/2] (E2M1, low
//     nibble = even k) and blockscales [M, K/16] (E4M3): per 16-group,
//     sf = e4m3(amax / (6 * input_scale)) and q = e2m1(x / (float(sf) *
//     input_scale)), both round-to-nearest-even with saturation (the NVFP4
//     convention for activations; the reference only defines the weight
//     side, nvfp4/config.mojo:13-35, and the input_scale it stores,
//     nvfp4/weight_loader.mojo:713-758).
//   W4A4 GEMM: y[M, N] = input_scale * ws2[n] * sum_k W~[n, k] * X~[m, k]
//     with W~ = e2m1 * e4m3 (weights), X~ = e2m1 * e4m3 (activations):
//     tcgen05.mma kind::mxf4nvf4 with 16-element block scales (E4M3), A =
//     weight codes, B = activation codes, both straight from TMA (no decode).
//
// GEMM kernel: persistent, one CTA per SM, tiles of 128 weight rows x 128
// tokens; 256-k stages (one 128-byte swizzle row of codes per matrix row):
//   warp 0      TMA producer: A codes [128 x 128 B], B codes [128 x 128 B]
//               (128-byte swizzle), blockscales [128 x 16 B] of each;
//   warp 1      TMEM owner and the MMA-issuing thread (4 MMAs of K = 64 per
//               stage, accumulators double-buffered in TMEM);
//   warps 2-5   scale movers: blockscales from shared memory into TMEM in
//               the tensor cores' scale-factor layout (tcgen05.st);
//   warps 6-9   epilogue: tcgen05.ld, * alpha, store.
// Scale-factor layout in TMEM (per MMA of K = 64, i.e. 4 blockscales per
// row): row r of the operand is in lane r % 32, column (base + r / 32), byte
// j = its blockscale j; the 32-lane pattern is repeated in all four lane
// quarters (each mover warp writes its own quarter).
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

static __device__ int g_w4a4_status;  // DeviceStatus of the last failing CTA

// ---------------------------------------------------------------------------
// Activation quantizer: one thread per 16-element group.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e2m1x2_rn_sat(float even_k, float odd_k) {
  uint32_t r;
  // The first source goes to the high nibble.
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; cvt.u32.u8 %0, t; }"
      : "=r"(r)
      : "f"(odd_k), "f"(even_k));
  return r;
}

__device__ __forceinline__ uint32_t e4m3_rn_sat(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xFFu;
}

template <typename XT>
__global__ void quantize_act_kernel(const XT *__restrict__ x, int64_t x_ld, int64_t M, int64_t K,
                                    float input_scale, uint8_t *__restrict__ q,
                                    uint8_t *__restrict__ qsf) {
  const int64_t groups = K / kGroup;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= M * groups) return;
  const int64_t m = gid / groups, g = gid - m * groups;
  float v[16];
  if constexpr (sizeof(XT) == 2) {
    const uint4 *p = reinterpret_cast<const uint4 *>(x + m * x_ld + g * kGroup);
    const uint4 a = p[0], b = p[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = bf16lo(w[i]);
      v[2 * i + 1] = bf16hi(w[i]);
    }
  } else {
    const float4 *p = reinterpret_cast<const float4 *>(x + m * x_ld + g * kGroup);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = p[i];
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));  // NaN elements ignored
  const uint32_t sf = e4m3_rn_sat(amax / (6.0f * input_scale));
  const float sdeq = e4m3_to_f32(sf) * input_scale;
  uint32_t packed[2] = {0u, 0u};
  if (sdeq != 0.0f) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      packed[i >> 2] |= e2m1x2_rn_sat(v[2 * i] / sdeq, v[2 * i + 1] / sdeq) << (8 * (i & 3));
  }
  *reinterpret_cast<uint2 *>(q + m * (K / 2) + g * 8) = make_uint2(packed[0], packed[1]);
  qsf[m * groups + g] = (uint8_t)sf;
}

// ---------------------------------------------------------------------------
// Block-scaled FP4 GEMM.
// ---------------------------------------------------------------------------
constexpr int kFqBM = 128;      // weight rows per tile (MMA M)
constexpr int kFqBN = 128;      // tokens per tile (MMA N)
constexpr int kFqBK = 256;      // k per stage (128 bytes of codes per row)
constexpr int kFqStages = 4;
constexpr int kFqSfCols = 32;   // TMEM columns of blockscales per stage (A 16 + B 16)
constexpr int kFqThreads = 10 * 32;
constexpr int kFqTmemCols = 512;  // 2 x 128 accumulator + 4 x 32 blockscale columns

struct FqSmem {
  static constexpr int kA = kFqBM * kFqBK / 2;   // 16 KB
  static constexpr int kB = kFqBN * kFqBK / 2;   // 16 KB
  static constexpr int kSA = kFqBM * kFqBK / 16;  // 2 KB
  static constexpr int kSB = kFqBN * kFqBK / 16;  // 2 KB
  static constexpr int kStage = kA + kB + kSA + kSB;
  static constexpr int offBar = kFqStages * kStage;
  static constexpr int nBars = 3 * kFqStages + 4;
  static constexpr int offTmem = offBar + nBars * 8;
  static constexpr int bytes = offTmem + 16;
  static constexpr int alloc = bytes + 1024;
  static_assert(kStage % 1024 == 0, "stages stay 1024-byte aligned");
  static_assert(alloc <= 227 * 1024, "shared memory per CTA");
};
static_assert(2 * kFqBN + kFqStages * kFqSfCols <= kFqTmemCols, "TMEM columns");

// Instruction descriptor, kind::mxf4nvf4: E2M1 x E2M1, UE4M3 scales per 16,
// fp32 accumulate, both operands K-major, scale-factor ids 0.
__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
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

struct FqArgs {
  int M, N, K;
  AlphaSpec al;
  void *y;
  int y_dtype;
  int64_t y_ld;
};

__global__ void __launch_bounds__(kFqThreads, 1)
    w4a4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmSA,
                     const __grid_constant__ CUtensorMap tmSB, FqArgs a) {
  using L = FqSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::offBar;             // [S] TMA stage landed
  const uint32_t bar_sf = bar_full + 8 * kFqStages;        // [S] blockscales in TMEM
  const uint32_t bar_empty = bar_sf + 8 * kFqStages;       // [S] MMAs done with stage
  const uint32_t bar_tfull = bar_empty + 8 * kFqStages;    // [2] accumulator ready
  const uint32_t bar_tempty = bar_tfull + 16;              // [2] accumulator drained
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::offTmem);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.K / kFqBK;
  const int n_tiles_n = (a.N + kFqBM - 1) / kFqBM;
  const int n_tiles = n_tiles_n * ((a.M + kFqBN - 1) / kFqBN);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kFqStages; ++s) {
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
    tmem_alloc(smem_u32(tmem_slot), kFqTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_sf = tmem + 2 * kFqBN;  // blockscale columns, kFqSfCols per stage
  volatile int *abort = &abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const int n0 = (t % n_tiles_n) * kFqBM, m0 = (t / n_tiles_n) * kFqBN;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % kFqStages, u = g / kFqStages;
          if (u > 0 && !mbar_wait(bar_empty + 8 * s, (u - 1) & 1, &g_w4a4_status,
                                  kDevTimeoutEmpty, abort)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + s * L::kStage;
          mbar_arrive_expect_tx(bar_full + 8 * s, L::kStage);
          tma_load_2d(st, &tmA, kb * (kFqBK / 2), n0, bar_full + 8 * s);
          tma_load_2d(st + L::kA, &tmB, kb * (kFqBK / 2), m0, bar_full + 8 * s);
          tma_load_2d(st + L::kA + L::kB, &tmSA, kb * (kFqBK / 16), n0, bar_full + 8 * s);
          tma_load_2d(st + L::kA + L::kB + L::kSA, &tmSB, kb * (kFqBK / 16), m0,
                      bar_full + 8 * s);
          issued = g + 1;
        }
      }
      // Drain: the CTA never exits with a TMA copy still writing its memory.
      for (int q = issued - kFqStages > 0 ? issued - kFqStages : 0; q < issued; ++q) {
        volatile int no_abort = 0;
        mbar_wait(bar_full + 8 * (q % kFqStages), (q / kFqStages) & 1, &g_w4a4_status,
                  kDevTimeoutFull, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kFqBM, kFqBN);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++i) {
        const int b = i & 1, ub = i >> 1;
        if (ub > 0 && !mbar_wait(bar_tempty + 8 * b, (ub - 1) & 1, &g_w4a4_status,
                                 kDevTimeoutAcc, abort))
          break;
        tc_fence_after();
        const uint32_t d = tmem + b * kFqBN;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % kFqStages, u = g / kFqStages;
          if (!mbar_wait(bar_full + 8 * s, u & 1, &g_w4a4_status, kDevTimeoutFull, abort) ||
              !mbar_wait(bar_sf + 8 * s, u & 1, &g_w4a4_status, kDevTimeoutDec, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * L::kStage, sb = sa + L::kA;
          const uint32_t sf = tmem_sf + s * kFqSfCols;
#pragma unroll
          for (int j = 0; j < kFqBK / 64; ++j)
            tc_mma_nvf4(d, sw128_kmajor_desc(sa + 32 * j), sw128_kmajor_desc(sb + 32 * j), idesc,
                        sf + 4 * j, sf + 16 + 4 * j, (kb | j) != 0);
          tc_commit(bar_empty + 8 * s);
        }
        tc_commit(bar_tfull + 8 * b);  // issued on abort too: marks the MMAs done
      }
    }
  } else if (warp < 6) {
    // ---------------- blockscale movers ----------------
    // Lane l of the warp with lane quarter q writes, per stage, TMEM lane
    // 32 q + l: columns [4j + c] = blockscales 4j..4j+3 of row l + 32c (A,
    // then B at +16), j = MMA of the stage, c = row group.
    const int q = warp & 3;
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++g) {
        const int s = g % kFqStages, u = g / kFqStages;
        // Stage s was refilled only after the MMAs of its previous use (which
        // read these TMEM columns) completed, so full[s] also frees them.
        const bool w_ok =
            mbar_wait(bar_full + 8 * s, u & 1, &g_w4a4_status, kDevTimeoutFull, abort);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        const uint8_t *sfa = smem + s * L::kStage + L::kA + L::kB;
        const uint8_t *sfb = sfa + L::kSA;
        const uint32_t col = tmem_sf + s * kFqSfCols + (static_cast<uint32_t>(32 * q) << 16);
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
          tmem_st_32x32b_x16(col + 16 * op, v);
        }
        tmem_st_wait();
        tc_fence_before();
        // The stage's scale factors were read through the generic proxy and
        // the stage is refilled by TMA (async proxy) after the MMAs: order
        // the reads before that write.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sf + 8 * s);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter of this warp
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1, ub = i >> 1;
      const bool w_ok = mbar_wait(bar_tfull + 8 * b, ub & 1, &g_w4a4_status, kDevTimeoutAcc, abort);
      if (!__all_sync(0xffffffffu, w_ok && !*abort)) break;
      tc_fence_after();
      const int n0 = (t % n_tiles_n) * kFqBM, m0 = (t / n_tiles_n) * kFqBN;
      const int n = n0 + 32 * q + lane;
      const bool nval = n < a.N;
      const float alpha = nval ? alpha_of(a.al, 0, n) : 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < kFqBN; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * kFqBN + c0, v);
        tmem_ld_wait();
        if (nval) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            if (m < a.M) {
              const float o = __uint_as_float(v[j]) * alpha;
              if (a.y_dtype == kF32)
                reinterpret_cast<float *>(a.y)[(int64_t)m * a.y_ld + n] = o;
              else
                reinterpret_cast<uint16_t *>(a.y)[(int64_t)m * a.y_ld + n] = f32_to_bf16_bits(o);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty + 8 * b);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kFqTmemCols);
  }
}

}  // namespace

cudaError_t launch_quantize_act(const void *x, int x_dtype, int64_t x_ld, int64_t M, int64_t K,
                                float input_scale, uint8_t *q, uint8_t *qsf, cudaStream_t st) {
  const int64_t n = M * (K / kGroup);
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const unsigned blocks = (unsigned)((n + threads - 1) / threads);
  if (x_dtype == kBF16)
    quantize_act_kernel<uint16_t><<<blocks, threads, 0, st>>>(
        static_cast<const uint16_t *>(x), x_ld, M, K, input_scale, q, qsf);
  else
    quantize_act_kernel<float><<<blocks, threads, 0, st>>>(static_cast<const float *>(x), x_ld, M,
                                                           K, input_scale, q, qsf);
  return cudaGetLastError();
}

bool w4a4_supported(int K, const void *w, const void *sf, const void *xq, const void *xsf) {
  return K % kFqBK == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)sf & 15) == 0 &&
         ((uintptr_t)xq & 15) == 0 && ((uintptr_t)xsf & 15) == 0;
}

cudaError_t launch_w4a4_gemm(const WeightSpec &ws, const AlphaSpec &al, const uint8_t *xq,
                             const uint8_t *xsf, int M, void *y, int y_dtype, int64_t y_ld,
                             cudaStream_t st) {
  if (M == 0 || ws.N == 0) return cudaSuccess;
  CUtensorMap tmA, tmB, tmSA, tmSB;
  if (!make_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.w, ws.N, ws.K / 2, ws.K / 2,
                    kFqBK / 2, kFqBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xq, M, ws.K / 2, ws.K / 2, kFqBK / 2,
                    kFqBN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmSA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.sf, ws.N, ws.K / 16, ws.K / 16,
                    kFqBK / 16, kFqBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tmap_2d(&tmSB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xsf, M, ws.K / 16, ws.K / 16,
                    kFqBK / 16, kFqBN, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(w4a4_gemm_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, FqSmem::alloc);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  FqArgs a;
  a.M = M;
  a.N = ws.N;
  a.K = ws.K;
  a.al = al;
  a.y = y;
  a.y_dtype = y_dtype;
  a.y_ld = y_ld;
  const int tiles = ((ws.N + kFqBM - 1) / kFqBM) * ((M + kFqBN - 1) / kFqBN);
  const int grid = tiles < tc_sm_count() ? tiles : tc_sm_count();
  w4a4_gemm_kernel<<<grid, kFqThreads, FqSmem::alloc, st>>>(tmA, tmB, tmSA, tmSB, a);
  return cudaGetLastError();
}

int read_w4a4_device_status() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_w4a4_status, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_w4a4_status, &zero, sizeof(int));
  return v;
}

}  // namespace nvfp4

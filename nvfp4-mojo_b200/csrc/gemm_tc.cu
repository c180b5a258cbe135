// gemm_tc.cu -- W4A16 prefill GEMM on the 5th-generation tensor cores.
//
// y[M, N] = alpha_n * (x[M, K] (bf16) @ dequant(W)[N, K]^T), fp32 accumulation:
// the arithmetic of nvfp4/nvfp4_gemm_gpu.mojo:148-182 (dequant fused into the
// GEMM, alpha applied after accumulation) at tensor-core speed.
//
// Persistent kernel, one CTA per SM, tiles of 128 weight rows x BN tokens
// visited round-robin (n-tile fastest, so the CTAs in flight share one
// activation tile and the whole weight matrix stays L2-resident).  Roles:
//   warp 0       TMA producer: per 64-k stage the packed FP4 tile [128 x 32 B]
//                and the bf16 activation tile [BN x 64] (128-byte swizzle);
//                every 4th stage also the blockscale tile [128 x 16 B];
//   warp 1       TMEM owner (2 x BN columns: double-buffered accumulator) and
//                the single MMA-issuing thread: tcgen05.mma kind::f16,
//                A = decoded weights (M = 128), B = activations (N = BN);
//   warps 4-11   decoders: E2M1 x E4M3 -> bf16 (LUT*scale*2^-7, exact) from
//                the staged codes into the swizzled A tile of the stage;
//   warps 12-15  epilogue: tcgen05.ld of the finished accumulator,
//                * alpha_n * 2^7, store; overlaps the next tile's main loop.
// Stages and accumulators are handed over with mbarriers; every wait is
// bounded (tc_common.cuh) so a fault in one role cannot hang the GPU.
#include <cstdio>
#include <cuda.h>

#include "../../include/nvfp4.h"
#include "abi_util.h"
#include "kernels.h"
#include "nvfp4_common.cuh"
#include "tc_common.cuh"

namespace nvfp4 {

static __device__ int g_gemm_status;  // DeviceStatus of the last failing CTA

constexpr int kTcBM = 128;  // weight rows per tile (MMA M)
constexpr int kTcBK = 64;   // K per stage (128 B of bf16 per row)
constexpr int kTcStages = 4;
constexpr int kTcScaleChunk = 4;  // stages per blockscale tile (16 B per row)
constexpr int kTcDecWarps = 8;
constexpr int kTcEpiWarps = 4;
constexpr int kTcThreads = (4 + kTcDecWarps + kTcEpiWarps) * 32;
static_assert(kTcStages % kTcScaleChunk == 0, "scale chunks must start on stage 0");

template <int BN>
struct TcSmem {
  static constexpr int kA = kTcBM * kTcBK * 2;  // 16 KB decoded weights
  static constexpr int kB = BN * kTcBK * 2;     // activations
  static constexpr int kR = kTcBM * kTcBK / 2;  // 4 KB packed codes
  static constexpr int kS = kTcBM * 16;         // 2 KB blockscales (4 stages)
  static constexpr int offA = 0;
  static constexpr int offB = offA + kTcStages * kA;
  static constexpr int offR = offB + kTcStages * kB;
  static constexpr int offS = offR + kTcStages * kR;
  static constexpr int offLut = offS + 2 * kS;  // 256 x u32 scale table
  static constexpr int offBar = offLut + 256 * 4;
  static constexpr int nBars = 3 * kTcStages + 4;
  static constexpr int offTmem = offBar + nBars * 8;
  static constexpr int bytes = offTmem + 16;
  static constexpr int alloc = bytes + 1024;  // slack for 1024-byte alignment
};

struct TcArgs {
  int M, N, K;
  AlphaSpec al;
  void *y;
  int y_dtype;
  int64_t y_ld;
};

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmS, TcArgs a) {
  using L = TcSmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L::offBar;           // [S] TMA stage landed
  const uint32_t bar_dec = bar_full + 8 * kTcStages;     // [S] A tile decoded
  const uint32_t bar_empty = bar_dec + 8 * kTcStages;    // [S] MMAs done with stage
  const uint32_t bar_tfull = bar_empty + 8 * kTcStages;  // [2] accumulator ready
  const uint32_t bar_tempty = bar_tfull + 16;            // [2] accumulator drained
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::offTmem);
  uint32_t *lut = reinterpret_cast<uint32_t *>(smem + L::offLut);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.K / kTcBK;
  const int n_tiles_n = (a.N + kTcBM - 1) / kTcBM;
  const int n_tiles = n_tiles_n * ((a.M + BN - 1) / BN);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_dec + 8 * s, kTcDecWarps);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_tfull + 8 * b, 1);
      mbar_init(bar_tempty + 8 * b, kTcEpiWarps);
    }
    mbar_fence_init();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
  }
  if (threadIdx.x >= 128 && threadIdx.x < 384) {
    // e4m3 code -> bf16x2 of float(code) * 2^119 (exact, NaN and zero included).
    lut[threadIdx.x - 128] = scale_to_bf16x2_2p119(threadIdx.x - 128);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int *abort = &abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const int n0 = (t % n_tiles_n) * kTcBM, m0 = (t / n_tiles_n) * BN;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % kTcStages, u = g / kTcStages;
          if (u > 0 && !mbar_wait(bar_empty + 8 * s, (u - 1) & 1, &g_gemm_status,
                                  kDevTimeoutEmpty, abort)) {
            ok = false;
            break;
          }
          const bool with_scales = (kb % kTcScaleChunk) == 0;
          mbar_arrive_expect_tx(bar_full + 8 * s, L::kB + L::kR + (with_scales ? L::kS : 0));
          tma_load_2d(sbase + L::offB + s * L::kB, &tmX, kb * kTcBK, m0, bar_full + 8 * s);
          tma_load_2d(sbase + L::offR + s * L::kR, &tmW, kb * (kTcBK / 2), n0, bar_full + 8 * s);
          // Scale buffers alternate on the global chunk count (g / 4; K % 256 == 0
          // so chunks never straddle tiles): the buffer reused here last held
          // chunk g/4 - 2, whose stages the MMA (hence the decoders) finished
          // before bar_empty of stage g - 4 completed.
          if (with_scales)
            tma_load_2d(sbase + L::offS + ((g / kTcScaleChunk) & 1) * L::kS, &tmS,
                        (kb / kTcScaleChunk) * 16, n0, bar_full + 8 * s);
          issued = g + 1;
        }
      }
      // Drain: the CTA never exits with a TMA copy still writing its memory.
      for (int q = issued - kTcStages > 0 ? issued - kTcStages : 0; q < issued; ++q) {
        volatile int no_abort = 0;
        mbar_wait(bar_full + 8 * (q % kTcStages), (q / kTcStages) & 1, &g_gemm_status,
                  kDevTimeoutFull, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kTcBM, BN);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++i) {
        const int b = i & 1, ub = i >> 1;
        if (ub > 0 && !mbar_wait(bar_tempty + 8 * b, (ub - 1) & 1, &g_gemm_status,
                                 kDevTimeoutAcc, abort))
          break;
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % kTcStages, u = g / kTcStages;
          if (!mbar_wait(bar_full + 8 * s, u & 1, &g_gemm_status, kDevTimeoutFull, abort) ||
              !mbar_wait(bar_dec + 8 * s, u & 1, &g_gemm_status, kDevTimeoutDec, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + L::offA + s * L::kA;
          const uint32_t sb = sbase + L::offB + s * L::kB;
#pragma unroll
          for (int k = 0; k < kTcBK / 16; ++k)
            tc_mma_f16(d, sw128_kmajor_desc(sa + 32 * k), sw128_kmajor_desc(sb + 32 * k), idesc,
                       (kb | k) != 0);
          tc_commit(bar_empty + 8 * s);
        }
        tc_commit(bar_tfull + 8 * b);  // issued on abort too: marks the MMAs done
      }
    }
  } else if (warp >= 4 && warp < 4 + kTcDecWarps) {
    // ---------------- decoders ----------------
    // Thread dt decodes, per stage, words wi and wi+1 (16 codes = one 16-group,
    // one blockscale) of rows rbase and rbase + 64.
    const int dt = threadIdx.x - 128;  // 0..255
    const int wi = 2 * (dt & 3);       // even 8-code word within the 64-k row
    const int rbase = dt >> 2;         // 0..63
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++g) {
        const int s = g % kTcStages, u = g / kTcStages;
        // Every lane waits; the decision to go on is made warp-uniform so the
        // warp-synchronous steps below never run with a partial warp.
        bool w_ok = u == 0 || mbar_wait(bar_empty + 8 * s, (u - 1) & 1, &g_gemm_status,
                                        kDevTimeoutEmpty, abort);
        w_ok = w_ok && mbar_wait(bar_full + 8 * s, u & 1, &g_gemm_status, kDevTimeoutFull, abort);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        const uint8_t *R = smem + L::offR + s * L::kR;
        const uint8_t *S = smem + L::offS + ((g / kTcScaleChunk) & 1) * L::kS;
        uint8_t *A = smem + L::offA + s * L::kA;
        const int scol = (kb % kTcScaleChunk) * 4 + (wi >> 1);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int row = rbase + 64 * j;
          const uint2 w2 = *reinterpret_cast<const uint2 *>(R + row * 32 + wi * 4);
          const uint32_t s2 = lut[S[row * 16 + scol]];
          uint32_t d0[4], d1[4];
          decode8_natural(w2.x, s2, d0);
          decode8_natural(w2.y, s2, d1);
          *reinterpret_cast<uint4 *>(A + row * 128 + ((wi ^ (row & 7)) << 4)) =
              make_uint4(d0[0], d0[1], d0[2], d0[3]);
          *reinterpret_cast<uint4 *>(A + row * 128 + (((wi + 1) ^ (row & 7)) << 4)) =
              make_uint4(d1[0], d1[1], d1[2], d1[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_dec + 8 * s);
      }
    }
  } else if (warp >= 4 + kTcDecWarps) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter of this warp
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1, ub = i >> 1;
      const bool w_ok = mbar_wait(bar_tfull + 8 * b, ub & 1, &g_gemm_status, kDevTimeoutAcc, abort);
      if (!__all_sync(0xffffffffu, w_ok && !*abort)) break;
      tc_fence_after();
      const int n0 = (t % n_tiles_n) * kTcBM, m0 = (t / n_tiles_n) * BN;
      const int n = n0 + 32 * q + lane;
      const bool nval = n < a.N;
      const float alpha = nval ? alpha_of(a.al, 0, n) * kDecodeUnscale : 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * BN + c0, v);
        tmem_ld_wait();
        if (nval) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            if (m < a.M) {
              const float o = __uint_as_float(v[j]) * alpha;
              if (a.y_dtype == kF32)
                reinterpret_cast<float *>(a.y)[m * a.y_ld + n] = o;
              else
                reinterpret_cast<uint16_t *>(a.y)[m * a.y_ld + n] = f32_to_bf16_bits(o);
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
    tmem_dealloc(tmem, 2 * BN);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor map: rows x cols elements, box box_rows x box_cols.
bool make_tmap_2d(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base,
                  int64_t rows, int64_t cols, int64_t ld_elems, int box_cols, int box_rows,
                  CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_gemm_supported(int K, const void *w, const void *x, int64_t x_ld) {
  // K % 256: whole blockscale tiles (16 B per row per 4 stages, 16-byte strides).
  return (K % (kTcBK * kTcScaleChunk)) == 0 && aligned(w, 16) && aligned(x, 16) &&
         (x_ld % 8) == 0 && encode_fn() != nullptr;
}

int tc_sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN>
static cudaError_t launch_tc_bn(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                                int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                                cudaStream_t st) {
  using L = TcSmem<BN>;
  CUtensorMap tmX, tmW, tmS;
  if (!make_tmap_2d(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, M, ws.K, x_ld, kTcBK, BN,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.w, ws.N, ws.K / 2, ws.K / 2,
                kTcBK / 2, kTcBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tmap_2d(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.sf, ws.N, ws.K / 16, ws.K / 16, 16,
                kTcBM, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(w4a16_tc_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::alloc);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  TcArgs a;
  a.M = M;
  a.N = ws.N;
  a.K = ws.K;
  a.al = al;
  a.y = y;
  a.y_dtype = y_dtype;
  a.y_ld = y_ld;
  const int tiles = ((ws.N + kTcBM - 1) / kTcBM) * ((M + BN - 1) / BN);
  const int grid = tiles < tc_sm_count() ? tiles : tc_sm_count();
  w4a16_tc_kernel<BN><<<grid, kTcThreads, L::alloc, st>>>(tmX, tmW, tmS, a);
  return cudaGetLastError();
}

cudaError_t launch_w4a16_tc(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                            int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                            cudaStream_t st) {
  // Smaller token tiles when 256-token tiles would leave SMs idle.
  const int tiles256 = ((ws.N + kTcBM - 1) / kTcBM) * ((M + 255) / 256);
  if (tiles256 < 4 * tc_sm_count())
    return launch_tc_bn<128>(ws, al, x, x_ld, y, y_dtype, y_ld, M, st);
  return launch_tc_bn<256>(ws, al, x, x_ld, y, y_dtype, y_ld, M, st);
}

int read_gemm_device_status() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
  return v;
}

}  // namespace nvfp4

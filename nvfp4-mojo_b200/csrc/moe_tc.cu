// moe_tc.cu -- grouped NVFP4 expert GEMMs on the 5th-generation tensor cores,
// for MoE batches with many rows per expert (prefill).
//
// Rows are sorted by expert (moe_permute_kernel) into items of at most 256
// rows; a tile is (item, 128 weight rows).  Persistent CTAs walk the tile list
// (its length is read from device memory), one CTA per SM.  Roles as in
// gemm_tc.cu: warp 0 TMA producer, warp 1 TMEM owner + single MMA thread,
// warps 4-11 E2M1 x E4M3 -> bf16 decoders, warps 12-15 epilogue.
//
//   kGateUp: A = gate rows and up rows of the expert (two 128-row tiles, two
//            128 x 256 accumulators), B = the expert's activation rows (gathered into
//            sorted order); epilogue h_g, h_u -> silu(h_g) * h_u written as bf16
//            hi + lo parts (nvfp4/deltanet.mojo:66-80 for SiLU).
//   kDown:   A = down rows, B = the SiLU*up rows as hi and lo bf16 tiles (two
//            MMAs into one accumulator, so the activations enter to ~2^-16);
//            epilogue scatters fp32 rows to their token slots.
#include <cuda.h>

#include "../../include/nvfp4.h"
#include "abi_util.h"
#include "kernels.h"
#include "moe.h"
#include "nvfp4_common.cuh"
#include "tc_common.cuh"

namespace nvfp4 {

static __device__ int g_moe_tc_status;

constexpr int kMtBM = 128, kMtBN = 256, kMtBK = 64;
constexpr int kMtDecWarps = 8, kMtEpiWarps = 4;
constexpr int kMtThreads = (4 + kMtDecWarps + kMtEpiWarps) * 32;
enum MoeTcMode { kGateUp = 0, kDown = 1 };

// 256-token tiles: the weight decode per MMA flop is halved against 128.
// kGateUp: two 128x256 accumulators fill TMEM (512 columns, one buffer: the
// epilogue of a tile runs before the next tile's first MMA); kDown: one
// accumulator, double-buffered.
template <int MODE>
struct MtCfg {
  static constexpr int NA = MODE == kGateUp ? 2 : 1;   // A tiles (weight row sets)
  static constexpr int NB = MODE == kGateUp ? 1 : 2;   // B tiles (activation parts)
  static constexpr int S = MODE == kGateUp ? 3 : 2;    // pipeline stages
  static constexpr int NBUF = MODE == kGateUp ? 1 : 2; // TMEM accumulator buffers
  static constexpr int kA = kMtBM * kMtBK * 2;         // 16 KB
  static constexpr int kB = kMtBN * kMtBK * 2;         // 32 KB
  static constexpr int kR = kMtBM * kMtBK / 2;         // 4 KB
  static constexpr int kS = kMtBM * 16;                // 2 KB per 4 stages
  static constexpr int offA = 0;
  static constexpr int offB = offA + S * NA * kA;
  static constexpr int offR = offB + S * NB * kB;
  static constexpr int offS = offR + S * NA * kR;
  static constexpr int offLut = offS + 2 * NA * kS;
  static constexpr int offBar = offLut + 1024;
  static constexpr int nBars = 3 * S + 4;
  static constexpr int offTmem = offBar + nBars * 8;
  static constexpr int alloc = offTmem + 16 + 1024;
  static constexpr int tmem_cols = NBUF * NA * kMtBN;
  static_assert(tmem_cols <= 512, "TMEM has 512 columns");
  static_assert(alloc <= 232448, "dynamic shared memory per CTA");
};

struct MoeTcArgs {
  const SkinnyWork *work;  // items: (expert, first sorted row, rows)
  const int *n_work;
  int n_tiles_n;           // weight-row tiles per item
  int K;                   // reduction length
  int Nw;                  // weight rows per expert (2I for gate_up, H for down)
  int I;                   // gate_up: offset of the up rows
  AlphaSpec al;            // per expert input scale, per row scale_2 (stride Nw)
  // kGateUp outputs
  uint16_t *inter, *inter_lo;
  // kDown outputs
  void *y;
  int y_dtype;
  const int32_t *dst_row;
  int y_ld;
};

template <int MODE>
__global__ void __launch_bounds__(kMtThreads, 1)
    moe_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                  const __grid_constant__ CUtensorMap tmB0, const __grid_constant__ CUtensorMap tmB1,
                  MoeTcArgs a) {
  using C = MtCfg<MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + C::offBar;
  const uint32_t bar_dec = bar_full + 8 * C::S;
  const uint32_t bar_empty = bar_dec + 8 * C::S;
  const uint32_t bar_tfull = bar_empty + 8 * C::S;
  const uint32_t bar_tempty = bar_tfull + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::offTmem);
  uint32_t *lut = reinterpret_cast<uint32_t *>(smem + C::offLut);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.K / kMtBK;
  const int n_tiles = (*a.n_work) * a.n_tiles_n;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::S; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_dec + 8 * s, kMtDecWarps);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < C::NBUF; ++b) {
      mbar_init(bar_tfull + 8 * b, 1);
      mbar_init(bar_tempty + 8 * b, kMtEpiWarps);
    }
    mbar_fence_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
    prefetch_tmap(&tmB0);
    if (C::NB > 1) prefetch_tmap(&tmB1);
  }
  if (threadIdx.x >= 128 && threadIdx.x < 384) lut[threadIdx.x - 128] = scale_to_bf16x2_2p119(threadIdx.x - 128);
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::tmem_cols);
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
        const SkinnyWork wk = a.work[t / a.n_tiles_n];
        const int n0 = (t % a.n_tiles_n) * kMtBM;
        const int wrow0 = wk.group * a.Nw + n0;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % C::S, u = g / C::S;
          if (u > 0 && !mbar_wait(bar_empty + 8 * s, (u - 1) & 1, &g_moe_tc_status,
                                  kDevTimeoutEmpty, abort)) {
            ok = false;
            break;
          }
          const bool with_scales = (kb & 3) == 0;
          mbar_arrive_expect_tx(bar_full + 8 * s,
                                C::NB * C::kB + C::NA * C::kR + (with_scales ? C::NA * C::kS : 0));
          tma_load_2d(sbase + C::offB + (s * C::NB) * C::kB, &tmB0, kb * kMtBK, wk.slot0,
                      bar_full + 8 * s);
          if (C::NB > 1)
            tma_load_2d(sbase + C::offB + (s * C::NB + 1) * C::kB, &tmB1, kb * kMtBK, wk.slot0,
                        bar_full + 8 * s);
#pragma unroll
          for (int i = 0; i < C::NA; ++i) {
            const int row = wrow0 + i * a.I;  // kGateUp: up rows follow the gate rows by I
            tma_load_2d(sbase + C::offR + (s * C::NA + i) * C::kR, &tmW, kb * (kMtBK / 2), row,
                        bar_full + 8 * s);
            // Scale buffers alternate on the global chunk count (K % 256 == 0:
            // chunks never straddle tiles); the one reused here last served
            // chunk g/4 - 2, released before bar_empty of stage g - S (S <= 5).
            if (with_scales)
              tma_load_2d(sbase + C::offS + (((g >> 2) & 1) * C::NA + i) * C::kS, &tmS,
                          (kb >> 2) * 16, row, bar_full + 8 * s);
          }
          issued = g + 1;
        }
      }
      for (int q = issued - C::S > 0 ? issued - C::S : 0; q < issued; ++q) {
        volatile int no_abort = 0;
        mbar_wait(bar_full + 8 * (q % C::S), (q / C::S) & 1, &g_moe_tc_status, kDevTimeoutFull,
                  &no_abort);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kMtBM, kMtBN);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++i) {
        const int b = i % C::NBUF, ub = i / C::NBUF;
        if (ub > 0 && !mbar_wait(bar_tempty + 8 * b, (ub - 1) & 1, &g_moe_tc_status,
                                 kDevTimeoutAcc, abort))
          break;
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % C::S, u = g / C::S;
          if (!mbar_wait(bar_full + 8 * s, u & 1, &g_moe_tc_status, kDevTimeoutFull, abort) ||
              !mbar_wait(bar_dec + 8 * s, u & 1, &g_moe_tc_status, kDevTimeoutDec, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int ia = 0; ia < C::NA; ++ia) {
            const uint32_t d = tmem + (b * C::NA + ia) * kMtBN;
            const uint32_t sa = sbase + C::offA + (s * C::NA + ia) * C::kA;
#pragma unroll
            for (int ib = 0; ib < C::NB; ++ib) {
              const uint32_t sb = sbase + C::offB + (s * C::NB + ib) * C::kB;
#pragma unroll
              for (int k = 0; k < kMtBK / 16; ++k)
                tc_mma_f16(d, sw128_kmajor_desc(sa + 32 * k), sw128_kmajor_desc(sb + 32 * k),
                           idesc, (kb | k | ib) != 0);
            }
          }
          tc_commit(bar_empty + 8 * s);
        }
        tc_commit(bar_tfull + 8 * b);
      }
    }
  } else if (warp >= 4 && warp < 4 + kMtDecWarps) {
    // ---------------- decoders ----------------
    const int dt = threadIdx.x - 128;
    const int wi = 2 * (dt & 3);
    const int rbase = dt >> 2;
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++g) {
        const int s = g % C::S, u = g / C::S;
        bool w_ok = u == 0 || mbar_wait(bar_empty + 8 * s, (u - 1) & 1, &g_moe_tc_status,
                                        kDevTimeoutEmpty, abort);
        w_ok = w_ok && mbar_wait(bar_full + 8 * s, u & 1, &g_moe_tc_status, kDevTimeoutFull, abort);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        const int scol = (kb & 3) * 4 + (wi >> 1);
#pragma unroll
        for (int ia = 0; ia < C::NA; ++ia) {
          const uint8_t *R = smem + C::offR + (s * C::NA + ia) * C::kR;
          const uint8_t *Sc = smem + C::offS + (((g >> 2) & 1) * C::NA + ia) * C::kS;
          uint8_t *A = smem + C::offA + (s * C::NA + ia) * C::kA;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int row = rbase + 64 * j;
            const uint2 w2 = *reinterpret_cast<const uint2 *>(R + row * 32 + wi * 4);
            const uint32_t s2 = lut[Sc[row * 16 + scol]];
            uint32_t d0[4], d1[4];
            decode8_natural(w2.x, s2, d0);
            decode8_natural(w2.y, s2, d1);
            *reinterpret_cast<uint4 *>(A + row * 128 + ((wi ^ (row & 7)) << 4)) =
                make_uint4(d0[0], d0[1], d0[2], d0[3]);
            *reinterpret_cast<uint4 *>(A + row * 128 + (((wi + 1) ^ (row & 7)) << 4)) =
                make_uint4(d1[0], d1[1], d1[2], d1[3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_dec + 8 * s);
      }
    }
  } else if (warp >= 4 + kMtDecWarps) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int b = i % C::NBUF, ub = i / C::NBUF;
      const bool w_ok = mbar_wait(bar_tfull + 8 * b, ub & 1, &g_moe_tc_status, kDevTimeoutAcc, abort);
      if (!__all_sync(0xffffffffu, w_ok && !*abort)) break;
      tc_fence_after();
      const SkinnyWork wk = a.work[t / a.n_tiles_n];
      const int n = (t % a.n_tiles_n) * kMtBM + 32 * q + lane;  // row within the expert
      const int e = wk.group;
      const float ins = a.al.input_scales ? a.al.input_scales[e] : a.al.input_scale;
      const float *w2 = a.al.ws2_rows ? a.al.ws2_rows + (int64_t)e * a.Nw : nullptr;
      const float alpha0 = ins * (w2 ? w2[n] : a.al.ws2) * kDecodeUnscale;
      const float alpha1 = MODE == kGateUp ? ins * (w2 ? w2[a.I + n] : a.al.ws2) * kDecodeUnscale : 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < kMtBN; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * C::NA * kMtBN + c0, v);
        if (MODE == kGateUp) {
          uint32_t vu[32];
          tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + (b * C::NA + 1) * kMtBN + c0, vu);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j < wk.count) {
              const int64_t p = wk.slot0 + c0 + j;
              const float hg = __uint_as_float(v[j]) * alpha0;
              const float hu = __uint_as_float(vu[j]) * alpha1;
              const float o = silu_f32(hg) * hu;
              const uint16_t hb = f32_to_bf16_bits(o);
              a.inter[p * a.I + n] = hb;
              a.inter_lo[p * a.I + n] = f32_to_bf16_bits(o - __uint_as_float((uint32_t)hb << 16));
            }
          }
        } else {
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j < wk.count) {
              const int64_t dst = a.dst_row[wk.slot0 + c0 + j];
              const float o = __uint_as_float(v[j]) * alpha0;
              if (a.y_dtype == kF32)
                reinterpret_cast<float *>(a.y)[dst * a.y_ld + n] = o;
              else
                reinterpret_cast<uint16_t *>(a.y)[dst * a.y_ld + n] = f32_to_bf16_bits(o);
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
    tmem_dealloc(tmem, C::tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
bool make_tmap_2d(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base,
                  int64_t rows, int64_t cols, int64_t ld_elems, int box_cols, int box_rows,
                  CUtensorMapSwizzle sw);
int tc_sm_count();

template <int MODE>
static cudaError_t launch_moe_tc_mode(const MoeTcLaunch &L, cudaStream_t st) {
  using C = MtCfg<MODE>;
  CUtensorMap tmW, tmS, tmB0, tmB1;
  const int64_t wrows = (int64_t)L.E * L.Nw;
  if (!make_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.w, wrows, L.K / 2, L.K / 2,
                    kMtBK / 2, kMtBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tmap_2d(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.sf, wrows, L.K / 16, L.K / 16, 16,
                    kMtBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tmap_2d(&tmB0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, L.b0, L.R, L.K, L.K, kMtBK, kMtBN,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmB1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, L.b1 ? L.b1 : L.b0, L.R, L.K, L.K,
                    kMtBK, kMtBN, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(moe_tc_kernel<MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::alloc);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  MoeTcArgs a;
  a.work = L.work;
  a.n_work = L.n_work;
  a.n_tiles_n = (MODE == kGateUp ? L.Nw / 2 : L.Nw) / kMtBM;
  a.K = L.K;
  a.Nw = L.Nw;
  a.I = MODE == kGateUp ? L.Nw / 2 : 0;
  a.al = L.al;
  a.inter = L.inter;
  a.inter_lo = L.inter_lo;
  a.y = L.y;
  a.y_dtype = L.y_dtype;
  a.dst_row = L.dst_row;
  a.y_ld = L.y_ld;
  // Upper bound of the tile count: every item is at most kMtBN rows.
  const int64_t max_items = (L.R + kMtBN - 1) / kMtBN + L.E;
  const int64_t max_tiles = max_items * a.n_tiles_n;
  const int grid = (int)(max_tiles < tc_sm_count() ? max_tiles : tc_sm_count());
  moe_tc_kernel<MODE><<<grid, kMtThreads, C::alloc, st>>>(tmW, tmS, tmB0, tmB1, a);
  return cudaGetLastError();
}

cudaError_t launch_moe_tc(const MoeTcLaunch &L, bool gate_up, cudaStream_t st) {
  return gate_up ? launch_moe_tc_mode<kGateUp>(L, st) : launch_moe_tc_mode<kDown>(L, st);
}

bool moe_tc_supported(int H, int I) {
  // K % 256 (whole blockscale tiles) for both GEMMs; weight rows per tile 128.
  return (H % 256) == 0 && (I % 256) == 0 && (I % kMtBM) == 0 && (H % kMtBM) == 0;
}

int moe_tc_rows_per_item() { return kMtBN; }

int read_moe_tc_device_status() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_moe_tc_status, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_moe_tc_status, &zero, sizeof(int));
  return v;
}

}  // namespace nvfp4

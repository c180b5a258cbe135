// gemv_ts.cu -- decode GEMV for M <= 8 tokens on the tcgen05 tensor cores,
// with the decoded weights as the MMA's A operand in tensor memory.
//
//   y[t, n] = alpha[n] * sum_k x[t, k] * LUT[code(n, k)] * float(sf(n, k / 16))
//
// (nvfp4_matvec, nvfp4/deltanet.mojo:549-584, for M tokens; alpha applied
// after accumulation, nvfp4/config.mojo:93-95.)
//
// Why this shape.  At M <= 8 the GEMV is bound by HBM: 0.5625 bytes per
// weight, ~40 weights per SM per cycle at 6.5 TB/s.  Decoding into shared
// memory for an SS-form MMA would move ~3.5x the weight bytes through shared
// memory twice (decoded writes, MMA reads), beyond its bandwidth; the legacy
// mma.sync path spends ~15 issue cycles per 256 weights on the MMA alone.
// Here the tensor core reads A from TMEM (tcgen05.mma ... [a_tmem] form,
// kind::f16), so the CUDA cores only convert: per 16 weights eight hardware
// E2M1x2 -> f16x2 conversions, eight f16x2 multiplies by the block scale
// (E4M3 -> f16, exact) and one tcgen05.st.  E2M1 x E4M3 products have at
// most 6 significant bits and lie in [2^-10, 2688], so the f16 weights are
// exact; the bf16 activations are exact in f16 after a per-token power-of-two
// scale 2^e (elements more than 2^28 below the row's largest become f16
// subnormals), which the epilogue takes back out.  Products are exact and
// accumulate in fp32 in TMEM.
//
// CTA (320 threads): warp 0 = TMA producer (128 x 256-k code tile, 128-byte
// swizzle, + 128 x 16 scale bytes per stage, evict-first), warp 1 = TMEM
// allocator and the MMA issuer (one thread), warps 2-9 = decoders: warp
// (q, h) writes rows 32q..32q+31 (its TMEM lane quarter) of k-half h of each
// stage into a ring of three 64-column A buffers.  Before decoding, the
// decoders turn this CTA's K range of x into the B tile (f16, 128-byte
// swizzled K-major, [8 rows][K range]; the MMA's N = 16 rows alias rows 0-7
// through a zero 8-row-group stride, so the padding costs no shared memory).
// MMA: M = 128, N = 16, K = 16, fp32 accumulator in 16 TMEM columns.  K is
// split over a cluster of C CTAs when the tiles alone do not fill the GPU;
// the partial sums meet in the leader CTA's shared memory (DSMEM) and are
// added there in rank order, so results do not depend on timing.
//
// Programmatic dependent launch: the producer issues the first stages' weight
// loads before griddepcontrol.wait (weights are constant in inference and must
// not be written by the kernel launched just before this one); x is read only
// after the wait, with L2-coherent loads.
#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

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

static __device__ int g_gemv_ts_status;

constexpr int kTsBM = 128;                  // weight rows per tile (MMA M)
constexpr int kTsBK = 256;                  // k per TMA stage
constexpr int kTsTok = 8;                   // tokens per call
constexpr int kTsDec = 8;                   // decode warps
constexpr int kTsThreads = 32 * (2 + kTsDec);
constexpr int kTsABufs = 3;                 // A buffers (one per 128-k half stage)
constexpr int kTsACols = 64;                // TMEM columns per A buffer
constexpr int kTsDCol = kTsABufs * kTsACols;  // accumulator columns [192, 208)
constexpr int kTsTmemCols = 256;
constexpr int kTsStageBytes = kTsBM * kTsBK / 2 + kTsBM * kTsBK / 16;  // 16 KB + 2 KB
constexpr int kTsMaxStages = 6;
constexpr int kTsMaxC = 8;
static_assert(kTsDCol + 16 <= kTsTmemCols, "TMEM columns");
static_assert(kTsStageBytes % 1024 == 0, "stages stay 1024-byte aligned");

// Instruction descriptor, kind::f16: f16 A (TMEM) x f16 B (smem, K-major) -> f32.
constexpr uint32_t kTsIdesc = (1u << 4) | (static_cast<uint32_t>(16 >> 3) << 17) |
                              (static_cast<uint32_t>(kTsBM >> 4) << 24);

struct TsArgs {
  AlphaSpec al;
  const uint16_t *x;
  int64_t x_ld;
  void *y;
  int y_dtype;
  int64_t y_ld;
  int M, N, K;
  int C;       // CTAs per cluster (K split)
  int ks;      // K per CTA
  int stages;  // TMA ring depth
};

struct TsSmem {
  int stages, b_bytes, red_bytes;
  int off_b, off_red, off_bar, off_misc, total;
  __host__ __device__ TsSmem(int S, int ks, int C) {
    stages = S;
    b_bytes = (ks / 64) * 1024;        // 8 rows x 128 B per 64-k slab
    red_bytes = (C - 1) * kTsTok * kTsBM * 4;
    off_b = S * kTsStageBytes;
    off_red = off_b + b_bytes;
    off_bar = off_red + red_bytes;
    // full[S], empty[S], afull[3], aempty[3], dfull
    off_misc = off_bar + 8 * (2 * S + 2 * kTsABufs + 1);
    total = off_misc + 64;  // TMEM base slot + inverse activation scales
  }
};

__device__ __forceinline__ void mma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// K-major, 128-byte swizzled B operand; `sbo` = bytes between 8-row groups
// (0: rows 8-15 read rows 0-7 again).
__device__ __forceinline__ uint64_t ts_b_desc(uint32_t saddr, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>((sbo & 0x3FFFFu) >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
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

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// f16x2 of E2M1 code byte `I` of w: low half = low nibble (even k).
template <int I>
__device__ __forceinline__ uint32_t e2m1_byte_f16x2(uint32_t w) {
  uint32_t d;
  if constexpr (I == 0)
    asm("{.reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %1;\n cvt.rn.f16x2.e2m1x2 %0, b0;}"
        : "=r"(d) : "r"(w));
  else if constexpr (I == 1)
    asm("{.reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %1;\n cvt.rn.f16x2.e2m1x2 %0, b1;}"
        : "=r"(d) : "r"(w));
  else if constexpr (I == 2)
    asm("{.reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %1;\n cvt.rn.f16x2.e2m1x2 %0, b2;}"
        : "=r"(d) : "r"(w));
  else
    asm("{.reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %1;\n cvt.rn.f16x2.e2m1x2 %0, b3;}"
        : "=r"(d) : "r"(w));
  return d;
}

// f16x2 (s_lo, s_hi) of two E4M3 scale bytes (exact).
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t two) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)two));
  return r;
}

// a * (s.lo, s.lo) (hi = 0) or a * (s.hi, s.hi) (hi = 1).
__device__ __forceinline__ uint32_t hmul2_bc(uint32_t a, uint32_t s, int hi) {
  const __half2 av = *reinterpret_cast<const __half2 *>(&a);
  const __half2 sv = *reinterpret_cast<const __half2 *>(&s);
  const __half2 r = __hmul2(av, hi ? __high2half2(sv) : __low2half2(sv));
  return *reinterpret_cast<const uint32_t *>(&r);
}

// Sixteen E2M1 codes (two words, low nibble first) times a block scale
// (half `hi` of the f16x2 scale pair sp) -> eight f16x2 A columns.
__device__ __forceinline__ void decode_block(uint32_t w0, uint32_t w1, uint32_t sp, int hi,
                                             uint32_t *o) {
  o[0] = hmul2_bc(e2m1_byte_f16x2<0>(w0), sp, hi);
  o[1] = hmul2_bc(e2m1_byte_f16x2<1>(w0), sp, hi);
  o[2] = hmul2_bc(e2m1_byte_f16x2<2>(w0), sp, hi);
  o[3] = hmul2_bc(e2m1_byte_f16x2<3>(w0), sp, hi);
  o[4] = hmul2_bc(e2m1_byte_f16x2<0>(w1), sp, hi);
  o[5] = hmul2_bc(e2m1_byte_f16x2<1>(w1), sp, hi);
  o[6] = hmul2_bc(e2m1_byte_f16x2<2>(w1), sp, hi);
  o[7] = hmul2_bc(e2m1_byte_f16x2<3>(w1), sp, hi);
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

// Stores v at the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ void st_cluster_f32(uint32_t local_addr, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__global__ void __launch_bounds__(kTsThreads, 1)
    gemv_ts_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                   TsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const TsSmem L(a.stages, a.ks, a.C);
  const int S = a.stages;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + L.off_bar;
  const uint32_t bar_empty = bar_full + 8 * S;
  const uint32_t bar_afull = bar_empty + 8 * S;
  const uint32_t bar_aempty = bar_afull + 8 * kTsABufs;
  const uint32_t bar_dfull = bar_aempty + 8 * kTsABufs;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.off_misc);
  float *s_inv = reinterpret_cast<float *>(smem + L.off_misc + 32);  // [8]
  __shared__ int abort_flag;
  volatile int *abort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int part = a.C > 1 ? (int)cluster_ctarank() : 0;
  const int tile = blockIdx.y;
  const int row0 = tile * kTsBM;
  const int k0 = part * a.ks;
  const int nck = a.ks / kTsBK;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, kTsDec);
    }
    for (int b = 0; b < kTsABufs; ++b) {
      mbar_init(bar_afull + 8 * b, kTsDec / 2);
      mbar_init(bar_aempty + 8 * b, 1);
    }
    mbar_init(bar_dfull, 1);
    mbar_fence_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTsTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      const int pre = nck < S ? nck : S;
      for (int g = 0; g < pre; ++g) {
        const uint32_t st = sbase + g * kTsStageBytes;
        const int kx = k0 + g * kTsBK;
        mbar_arrive_expect_tx(bar_full + 8 * g, kTsStageBytes);
        tma_load_2d_hint(st, &tmW, kx / 2, row0, bar_full + 8 * g, pol);
        tma_load_2d_hint(st + kTsBM * kTsBK / 2, &tmS, kx / kGroup, row0, bar_full + 8 * g, pol);
      }
      pdl_wait();
      pdl_trigger();
      int issued = pre;
      for (int g = pre; g < nck; ++g) {
        const int s = g % S;
        if (!mbar_wait(bar_empty + 8 * s, ((g / S) - 1) & 1, &g_gemv_ts_status, kDevTimeoutEmpty,
                       abort))
          break;
        const uint32_t st = sbase + s * kTsStageBytes;
        const int kx = k0 + g * kTsBK;
        mbar_arrive_expect_tx(bar_full + 8 * s, kTsStageBytes);
        tma_load_2d_hint(st, &tmW, kx / 2, row0, bar_full + 8 * s, pol);
        tma_load_2d_hint(st + kTsBM * kTsBK / 2, &tmS, kx / kGroup, row0, bar_full + 8 * s, pol);
        issued = g + 1;
      }
      // No load may still be in flight when the CTA exits.
      for (int g = issued - S > 0 ? issued - S : 0; g < issued; ++g) {
        volatile int no_abort = 0;
        mbar_wait(bar_full + 8 * (g % S), (g / S) & 1, &g_gemv_ts_status, kDevTimeoutFull,
                  &no_abort);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    pdl_wait();
    named_bar_sync(1, 32 * (kTsDec + 1));  // B tile written (decoders' prologue)
    if (lane == 0) {
      tc_fence_after();
      const uint32_t bbase = sbase + L.off_b;
      for (int i = 0; i < 2 * nck; ++i) {
        const int buf = i % kTsABufs;
        if (!mbar_wait(bar_afull + 8 * buf, (i / kTsABufs) & 1, &g_gemv_ts_status,
                       kDevTimeoutDec, abort))
          break;
        tc_fence_after();
        const uint32_t acol = tmem + buf * kTsACols;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int kl = (i >> 1) * kTsBK + (i & 1) * 128 + 16 * j;  // k within this CTA
          const uint32_t baddr = bbase + (kl >> 6) * 1024 + 2 * (kl & 63);
          mma_ts_f16(tmem + kTsDCol, acol + 8 * j, ts_b_desc(baddr, 0), kTsIdesc,
                     (i | j) != 0 ? 1u : 0u);
        }
        tc_commit(bar_aempty + 8 * buf);
      }
      tc_commit(bar_dfull);  // also after an abort: the epilogue waits for every MMA
    }
    __syncwarp();
  } else {
    // ---------------- decoders (+ prologue, epilogue) ----------------
    const int dw = warp - 2;  // 0..7
    const int q = warp & 3;   // TMEM lane quarter this warp may access
    const int h = dw >> 2;    // k half of each stage
    const int r = 32 * q + lane;
    pdl_wait();
    pdl_trigger();
    // Prologue: warp t converts token t's K range of x into B row t.
    if (dw < a.M) {
      const int t = dw;
      const uint16_t *xr = a.x + (int64_t)t * a.x_ld + k0;
      const int units = a.ks / 8;
      float m = 0.0f;
      for (int u = lane; u < units; u += 32) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(xr) + u);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          m = fmaxf(m, fmaxf(fabsf(bf16lo(w[j])), fabsf(bf16hi(w[j]))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      // 2^e with max|x| * 2^e in [2^14, 2^15); |e| <= 110 keeps 2^e and 2^-e normal.
      int e = 0;
      if (m > 0.0f && m <= 3.0e38f) {
        e = 14 - (int)((__float_as_uint(m) >> 23) & 0xFF) + 127;
        e = e < -110 ? -110 : (e > 110 ? 110 : e);
      }
      const float sc = __uint_as_float((uint32_t)(e + 127) << 23);
      if (lane == 0) s_inv[t] = __uint_as_float((uint32_t)(127 - e) << 23);
      uint8_t *brow = smem + L.off_b + t * 128;
      for (int u = lane; u < units; u += 32) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(xr) + u);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2 hv = __floats2half2_rn(bf16lo(w[j]) * sc, bf16hi(w[j]) * sc);
          o[j] = *reinterpret_cast<const uint32_t *>(&hv);
        }
        // slab u/8 (64 k), 16-byte unit u%8 of the row, 128-byte swizzle.
        *reinterpret_cast<uint4 *>(brow + (u >> 3) * 1024 + (((u & 7) ^ t) << 4)) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    fence_proxy_async_smem();  // generic-proxy B writes, read by the MMA
    named_bar_sync(1, 32 * (kTsDec + 1));

    // Main loop: stage g, half h -> A buffer (2g + h) % 3.
    for (int g = 0; g < nck; ++g) {
      const int s = g % S, i = 2 * g + h, buf = i % kTsABufs;
      const bool ok_full =
          mbar_wait(bar_full + 8 * s, (g / S) & 1, &g_gemv_ts_status, kDevTimeoutFull, abort);
      const bool ok_a = ok_full && (i < kTsABufs ||
                                    mbar_wait(bar_aempty + 8 * buf, ((i / kTsABufs) - 1) & 1,
                                              &g_gemv_ts_status, kDevTimeoutEmpty, abort));
      if (!__all_sync(0xffffffffu, ok_a)) break;
      tc_fence_after();
      const uint32_t st = sbase + s * kTsStageBytes;
      uint4 cw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        cw[u] = lds_v4(st + r * 128 + ((((4 * h + u) ^ (r & 7))) << 4));
      uint32_t sw0, sw1;
      asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                   : "=r"(sw0), "=r"(sw1)
                   : "r"(st + kTsBM * kTsBK / 2 + 16 * r + 8 * h));
      // The stage's bytes are in registers: release it to the producer
      // (cross-proxy: these generic reads before the next TMA write).
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
      const uint32_t sp[4] = {e4m3x2_f16x2(sw0), e4m3x2_f16x2(sw0 >> 16), e4m3x2_f16x2(sw1),
                              e4m3x2_f16x2(sw1 >> 16)};
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * kTsACols;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        // 16-byte unit u = blocks 2u (words x, y) and 2u+1 (z, w); their
        // scales are the two halves of pair sp[u]; columns 16u..16u+15.
        uint32_t o[16];
        decode_block(cw[u].x, cw[u].y, sp[u], 0, o);
        decode_block(cw[u].z, cw[u].w, sp[u], 1, o + 8);
        tmem_st_x16(taddr + 16 * u, o);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_afull + 8 * buf);
    }

    // Epilogue: warps of half 0 (one per lane quarter) read the accumulator.
    float acc[kTsTok];
#pragma unroll
    for (int t = 0; t < kTsTok; ++t) acc[t] = 0.0f;
    bool have = false;
    if (h == 0) {
      volatile int no_abort = 0;
      const bool ok = mbar_wait(bar_dfull, 0, &g_gemv_ts_status, kDevTimeoutAcc, &no_abort);
      if (__all_sync(0xffffffffu, ok) && !*abort) {
        tc_fence_after();
        uint32_t v[16];
        tmem_ld_x16(tmem + (static_cast<uint32_t>(32 * q) << 16) + kTsDCol, v);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < kTsTok; ++t) acc[t] = __uint_as_float(v[t]) * s_inv[t];
        have = true;
      }
      if (a.C > 1 && part != 0) {
        const uint32_t red = sbase + L.off_red + ((part - 1) * kTsTok * kTsBM + r) * 4;
#pragma unroll
        for (int t = 0; t < kTsTok; ++t)
          if (t < a.M) st_cluster_f32(red + t * kTsBM * 4, 0, have ? acc[t] : 0.0f);
      }
    }
    if (a.C > 1) cluster_sync_all();
    if (h == 0 && part == 0 && have) {
      const int n = row0 + r;
      if (n < a.N) {
        const float al = alpha_of(a.al, 0, n);
        const float *red = reinterpret_cast<const float *>(smem + L.off_red);
#pragma unroll
        for (int t = 0; t < kTsTok; ++t) {
          if (t >= a.M) break;
          float v = acc[t];
          for (int p = 1; p < a.C; ++p) v += red[((p - 1) * kTsTok + t) * kTsBM + r];
          v *= al;
          if (a.y_dtype == kBF16)
            reinterpret_cast<uint16_t *>(a.y)[(int64_t)t * a.y_ld + n] = f32_to_bf16_bits(v);
          else
            reinterpret_cast<float *>(a.y)[(int64_t)t * a.y_ld + n] = v;
        }
      }
    }
  }
  if (a.C > 1 && warp < 2) cluster_sync_all();

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTsTmemCols);
  }
}

std::mutex g_ts_mu;
size_t g_ts_attr[64] = {};  // dynamic shared memory the kernel is opted in for, per device

// Opts the kernel in for `bytes` of dynamic shared memory (its static shared
// memory comes on top, so the opt-in maximum itself would be refused).
cudaError_t ts_set_attr(size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_ts_mu);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (g_ts_attr[dev] < bytes) {
    cudaError_t e = cudaFuncSetAttribute(gemv_ts_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    g_ts_attr[dev] = bytes;
  }
  return cudaSuccess;
}

struct TsPlan {
  int C = 0, stages = 0, per_sm = 1;
  size_t smem = 0;
};

// K split C (a divisor of the stage count, at most 8) and ring depth.  Cost
// = the weight bytes of the busiest SM (CTAs per SM x bytes per CTA); ties go
// to the split that keeps more SMs streaming, then to the smaller C.
TsPlan ts_plan(int N, int K) {
  const int sms = tc_sm_count();
  const int tiles = (N + kTsBM - 1) / kTsBM;
  const int nck = K / kTsBK;
  TsPlan best;
  double best_cost = 0.0;
  int best_active = 0;
  for (int C = 1; C <= kTsMaxC; ++C) {
    if (nck % C) continue;
    const int ks = K / C;
    const int ctas = tiles * C;
    const int per_sm = (ctas + sms - 1) / sms;
    // Opt-in maximum 227 KB per CTA (a little kept for static shared memory).
    const size_t cap = per_sm <= 1 ? (size_t)226 * 1024 : (size_t)226 * 1024 / per_sm;
    int S = kTsMaxStages;
    while (S > 2 && (size_t)TsSmem(S, ks, C).total + 1024 > cap) --S;
    if ((size_t)TsSmem(S, ks, C).total + 1024 > cap) continue;
    if (S > ks / kTsBK) S = ks / kTsBK < 2 ? 2 : ks / kTsBK;
    const double cost = (double)per_sm * ks;
    const int active = ctas < sms ? ctas : sms;
    if (best.C == 0 || cost < best_cost * 0.999 ||
        (cost <= best_cost * 1.001 && active > best_active)) {
      best.C = C;
      best.stages = S;
      best.per_sm = per_sm;
      best.smem = (size_t)TsSmem(S, ks, C).total + 1024;
      best_cost = cost;
      best_active = active;
    }
  }
  return best;
}

}  // namespace

bool gemv_ts_supported(int M, int N, int K, const void *w, const void *sf, const void *x,
                       int64_t x_ld) {
  return M >= 1 && M <= kTsTok && N >= 1 && K % kTsBK == 0 && K > 0 &&
         ((uintptr_t)w & 15) == 0 && ((uintptr_t)sf & 15) == 0 && ((uintptr_t)x & 15) == 0 &&
         x_ld % 8 == 0 && (N + kTsBM - 1) / kTsBM <= 65535 && ts_plan(N, K).C > 0;
}

int read_gemv_ts_device_status() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_ts_status, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_gemv_ts_status, &zero, sizeof(int));
  return v;
}

cudaError_t launch_gemv_ts(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                           int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                           cudaStream_t st) {
  if (M == 0 || ws.N == 0) return cudaSuccess;
  const TsPlan p = ts_plan(ws.N, ws.K);
  if (p.C == 0) return cudaErrorInvalidValue;
  cudaError_t e = ts_set_attr(p.smem);
  if (e != cudaSuccess) return e;
  CUtensorMap tmW, tmS;
  if (!make_tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.w, ws.N, ws.K / 2, ws.K / 2,
                    kTsBK / 2, kTsBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws.sf, ws.N, ws.K / kGroup,
                    ws.K / kGroup, kTsBK / kGroup, kTsBM, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  TsArgs a;
  a.al = al;
  a.x = x;
  a.x_ld = x_ld;
  a.y = y;
  a.y_dtype = y_dtype;
  a.y_ld = y_ld;
  a.M = M;
  a.N = ws.N;
  a.K = ws.K;
  a.C = p.C;
  a.ks = ws.K / p.C;
  a.stages = p.stages;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.C, (ws.N + kTsBM - 1) / kTsBM, 1);
  cfg.blockDim = dim3(kTsThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemv_ts_kernel, tmW, tmS, a);
}

}  // namespace nvfp4

// gemv.cu -- decode GEMV for M <= 8 tokens: y[M, N] = alpha[n] * x[M, K] . W[N, K]^T
// with W in NVFP4 (the reference's nvfp4_matvec / nvfp4_linear_forward at
// batch_seq_len <= 8: nvfp4/deltanet.mojo:549-584, nvfp4/nvfp4_gemm_gpu.mojo:185-224).
//
// HBM-bound: every weight byte is read once, so the kernel is organised around
// keeping enough bytes in flight with few instructions per byte.  Two kernels
// share the decode and MMA code below: gemv_kernel (the plain linear, and the
// MoE experts' work items one cluster grid each where the persistent form
// does not fit) and gemv_grouped_kernel (the MoE expert GEMMs as a
// persistent grid, see its comment).  Notes on gemv_kernel:
//
//   * Two CTAs per SM.  A cluster of C CTAs (grid.x = C) splits K into C
//     slices and reduces the fp32 partial sums through distributed shared
//     memory; the clusters split the 16-row tiles as evenly as tile counts
//     allow.  CTA = one consumer warp per tile + 1 producer warp.
//   * The producer streams 256-k chunks of the CTA's tiles with TMA (codes in
//     a 128-byte-swizzled box, blockscales in a plain one) through an
//     S-stage mbarrier ring: per-thread loads through L1 cannot keep enough
//     bytes in flight to saturate HBM, the TMA engine can.  Lane quad c of
//     row g takes bytes [32c, 32c + 32) of each 128-byte row chunk.
//   * Launched with programmatic stream serialization: the set-up overlaps
//     the previous kernel's tail (griddepcontrol).
//   * Decode: the hardware E2M1x2 -> f16x2 conversion (exact), times the E4M3
//     blockscale converted E4M3x2 -> f16x2 (exact); the product LUT*scale has
//     at most 6 significant bits and lies in [2^-10, 2688], so it is exact in
//     f16.  mma.sync m16n8k16 f16 x f16 -> f32 does the multiply-adds.
//   * K permutation: the MMA's 16 k positions are taken as the lane quad's
//     4 codes at k = 64c + 4j .. 4j+3 of the chunk (MMA j = 0..15), so each
//     lane's A fragment comes from 2 bytes of its own loaded words, its
//     blockscale is byte j/4 of one 4-byte scale word per row and chunk, and
//     its B fragment is x[token g][64c + 4j .. +3]: 8 bytes of the token's row.
//   * Activations: each CTA converts its K slice of x (bf16) to f16 in shared
//     memory, scaled per token by a power of two 2^s chosen so that
//     max|x| * 2^s lies in [2^14, 2^15): bf16 values are then exact in f16
//     (apart from elements below max|x| * 2^-28, which become f16 subnormals),
//     and the partial sums are multiplied by 2^-s (exact) before the reduction.
//     Rows of x are stored with their 16-byte units permuted within each
//     chunk (lane quad c's unit p of the chunk at 4p + c) and a 64-byte pad:
//     the B-fragment loads (LDS.128) are bank-conflict free and a lane's 8
//     loads of a chunk sit at one base plus immediate offsets.  Lanes of
//     tokens >= M read a zeroed row instead.
#include <algorithm>
#include <cooperative_groups.h>
#include <map>
#include <mutex>
#include <tuple>
#include <cuda_fp16.h>

#include "../../include/nvfp4.h"
#include "kernels.h"
#include "nvfp4_common.cuh"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace nvfp4 {

bool make_tmap_2d(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base,
                  int64_t rows, int64_t cols, int64_t ld_elems, int box_cols, int box_rows,
                  CUtensorMapSwizzle sw);
int tc_sm_count();

namespace {

static __device__ int g_gemv_status;  // DeviceStatus of the last failing CTA

constexpr int kGvChunk = 256;  // k per row chunk (128 bytes of codes)
constexpr int kGvTok = 8;      // tokens per MMA (n = 8)

// Four f16x2 from the four bytes of w: d_i = (lo: low nibble, hi: high nibble of byte i).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&d)[4]) {
  asm("{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      "mov.b32 {b0, b1, b2, b3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n"
      "}"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(w));
}

// f16x2 of the blockscale pair in half `h` (0: bytes 0-1, 1: bytes 2-3) of sw.
__device__ __forceinline__ uint32_t scale_pair_f16x2(uint32_t sw, int h) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)(h ? sw >> 16 : sw)));
  return r;
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ float *cluster_map(float *p, int rank) {
  return cg::this_cluster().map_shared_rank(p, rank);
}

// Physical 16-byte unit of logical unit u = 32 ch + 8 c + p (c < 4, p < 8)
// in a token row of x: 32 ch + 4 p + c.
__device__ __forceinline__ int xs_unit(int u) {
  return (u & ~31) | ((u & 7) << 2) | ((u >> 3) & 3);
}

// Kernel modes: the plain linear, and the two grouped MoE expert GEMMs over
// work items (expert, up to 8 token slots) from the MoE permutation.
enum GemvMode : int {
  kGvPlain = 0,
  kGvGateUp = 1,  // W = [gate; up] rows of the expert, out = silu(gate) * up, bf16 hi + lo
  kGvDown = 2,    // x = bf16 hi + lo parts (two f16 B operands), out rows scattered
};

struct GemvArgs {
  const uint8_t *w;
  const uint8_t *sf;
  AlphaSpec al;
  const uint16_t *x;
  const uint16_t *x_lo;  // kGvDown: low parts of x
  int64_t x_ld;
  void *y;
  uint16_t *y_lo;        // kGvGateUp: low parts of the output
  int y_dtype;
  int64_t y_ld;
  int M, N, K;           // N: rows of one weight matrix (an expert's, in grouped modes)
  int ks;                // K per CTA (multiple of kGvChunk)
  int xstride;           // bytes per token row of the f16 x slice in shared memory
  int stages;            // TMA ring stages
  const SkinnyWork *work;  // grouped modes: items (expert, first slot, slots <= 8)
  const int *n_work;
  const int32_t *x_rows;   // kGvGateUp: slot -> activation row
  const int32_t *y_rows;   // kGvDown: slot -> output row
  int ggroups;             // gemv_grouped_kernel: row groups per item
  int max_items;           // gemv_grouped_kernel: items one CTA may meet
};

// Consumer view of one staged chunk: codes of rows g and g+8 of the warp's
// tile (bytes [32c, 32c + 32) of each 128-byte row) and their scale words.
struct GemvChunk {
  uint32_t wg[8], wh[8];
  uint32_t sg, sh;
};

// The lane's words of two staged rows (byte offsets rowA, rowB of
// 128-byte-swizzled rows: 16-byte unit u of a row whose box row index is R
// sits at u ^ (R & 7), swA / swB) and their scale words.
__device__ __forceinline__ void gemv_fetch_rows(GemvChunk &b, uint32_t rowA, uint32_t rowB,
                                                int swA, int swB, uint32_t scA, uint32_t scB,
                                                int c) {
  const uint4 a0 = lds_v4(rowA + 16u * ((2 * c) ^ swA)), a1 = lds_v4(rowA + 16u * ((2 * c + 1) ^ swA));
  const uint4 b0 = lds_v4(rowB + 16u * ((2 * c) ^ swB)), b1 = lds_v4(rowB + 16u * ((2 * c + 1) ^ swB));
  b.wg[0] = a0.x; b.wg[1] = a0.y; b.wg[2] = a0.z; b.wg[3] = a0.w;
  b.wg[4] = a1.x; b.wg[5] = a1.y; b.wg[6] = a1.z; b.wg[7] = a1.w;
  b.wh[0] = b0.x; b.wh[1] = b0.y; b.wh[2] = b0.z; b.wh[3] = b0.w;
  b.wh[4] = b1.x; b.wh[5] = b1.y; b.wh[6] = b1.z; b.wh[7] = b1.w;
  b.sg = lds_u32(scA);
  b.sh = lds_u32(scB);
}

// Rows rl and rl + 8 of a warp's 16-row tile (codes: the tile's first row).
__device__ __forceinline__ void gemv_fetch(GemvChunk &b, uint32_t codes, uint32_t scales, int rl,
                                           int c) {
  gemv_fetch_rows(b, codes + 128u * rl, codes + 128u * (rl + 8), rl & 7, rl & 7,
                  scales + 16u * rl + 4u * c, scales + 16u * (rl + 8) + 4u * c, c);
}

// f16 multiply of the pair a by a scale pair already broadcast.
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t s) {
  const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a),
                            *reinterpret_cast<const __half2 *>(&s));
  return *reinterpret_cast<const uint32_t *>(&r);
}

// (s.lo, s.lo) and (s.hi, s.hi) of an f16 pair.
__device__ __forceinline__ uint32_t bcast_lo(uint32_t s) { return __byte_perm(s, 0, 0x1010); }
__device__ __forceinline__ uint32_t bcast_hi(uint32_t s) { return __byte_perm(s, 0, 0x3232); }

// One 256-k chunk of a warp's tile; SPLIT adds the MMAs of the low parts.
// xb (xb_lo): this lane's x units of the chunk, logical 32 ch + 8 c + p at
// xb + 64 p (xs_unit), i.e. xrow + 16 (32 ch + c).
template <bool SPLIT>
__device__ __forceinline__ void gemv_compute(const GemvChunk &b, float (&acc)[4], uint32_t xb,
                                             uint32_t xb_lo) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {  // blockscales 2hh, 2hh+1 of the lane's 64 k
    const uint32_t s_g = scale_pair_f16x2(b.sg, hh), s_h = scale_pair_f16x2(b.sh, hh);
    const uint32_t sg[2] = {bcast_lo(s_g), bcast_hi(s_g)}, sh[2] = {bcast_lo(s_h), bcast_hi(s_h)};
#pragma unroll
    for (int p4 = 0; p4 < 4; ++p4) {  // code word p = 4hh + p4: MMAs j = 2p, 2p+1
      const int p = 4 * hh + p4, hi = p4 >> 1;  // blockscale q = p / 2 = 2hh + hi
      const uint4 xv = lds_v4(xb + 64u * p);
      uint32_t dg[4], dh[4];
      e2m1x8_to_f16x2(b.wg[p], dg);
      e2m1x8_to_f16x2(b.wh[p], dh);
      const uint32_t a0 = hmul2_u32(dg[0], sg[hi]), a1 = hmul2_u32(dh[0], sh[hi]);
      const uint32_t a2 = hmul2_u32(dg[1], sg[hi]), a3 = hmul2_u32(dh[1], sh[hi]);
      const uint32_t a4 = hmul2_u32(dg[2], sg[hi]), a5 = hmul2_u32(dh[2], sh[hi]);
      const uint32_t a6 = hmul2_u32(dg[3], sg[hi]), a7 = hmul2_u32(dh[3], sh[hi]);
      mma_f16_16816(acc, a0, a1, a2, a3, xv.x, xv.y);
      mma_f16_16816(acc, a4, a5, a6, a7, xv.z, xv.w);
      if constexpr (SPLIT) {
        const uint4 xl = lds_v4(xb_lo + 64u * p);
        mma_f16_16816(acc, a0, a1, a2, a3, xl.x, xl.y);
        mma_f16_16816(acc, a4, a5, a6, a7, xl.z, xl.w);
      }
    }
  }
}

// E2M1x2 -> f16x2 of byte i (0..3) of w (low nibble -> low half).
template <int I>
__device__ __forceinline__ uint32_t e2m1_byte_to_f16x2(uint32_t w) {
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

// The four blockscales of a scale word as fp32 (E4M3 -> f16 is exact, f16 -> f32 too).
__device__ __forceinline__ void scale_word_f32(uint32_t sw, float (&f)[4]) {
  const uint32_t lo = scale_pair_f16x2(sw, 0), hi = scale_pair_f16x2(sw, 1);
  const __half2 l = *reinterpret_cast<const __half2 *>(&lo);
  const __half2 h = *reinterpret_cast<const __half2 *>(&hi);
  f[0] = __low2float(l);
  f[1] = __high2float(l);
  f[2] = __low2float(h);
  f[3] = __high2float(h);
}

__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}

// One 256-k chunk for a single token (M = 1), with the blockscales applied
// after the MMAs instead of to every weight.  The MMA's 8 columns carry 8
// different 16-k blocks ("block-diagonal" B): in MMA j (0..15) lane quad c
// supplies byte j/2 of its block 4c + (j & 1) as k pair slot 0 (column 2c)
// and of its block 4c + 2 + (j & 1) as slot 1 (column 2c + 1); the B fragment
// of lane (g, c) is the token's x pair of that byte where g is the slot's
// column (g = 2c: slot 0, g = 2c + 1: slot 1) and zero elsewhere.  Each
// column then accumulates one block's products over the 8 MMAs of equal
// parity, and the lane's own D columns are exactly its own blocks, so the
// lane scales them with its own blockscales (8 FMAs per chunk).  Slot 0 of
// lane quad c reads logical x units 32 ch + 8 c + {0..3} (its blocks 4c,
// 4c + 1) at xb + 64 {0..3} (xb = xrow + 16 (32 ch + c), see xs_unit), slot 1
// units 32 ch + 8 c + {4..7} (blocks 4c + 2, 4c + 3) at xb + 64 {4..7}; lanes
// that own neither read the zero row.  The codes of rows rl and rl + 8 are
// read from the staged 128-byte-swizzled tile per parity (8 words at a
// time); `release` runs once all of the chunk's operands are in registers.
template <class Release>
__device__ __forceinline__ void gemv_compute_m1(uint32_t codes, uint32_t sgw, uint32_t shw,
                                                int rl, int c, float (&tot)[2],
                                                uint32_t xb, uint32_t zero, bool own_a,
                                                bool own_b, Release release) {
  const int sw = rl & 7;
  const uint32_t rg = codes + 128u * rl, rh = rg + 128u * 8;
  const uint32_t u0 = 16u * ((2 * c) ^ sw), u1 = 16u * ((2 * c + 1) ^ sw);
  float e[4] = {0.0f, 0.0f, 0.0f, 0.0f}, o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int par = 0; par < 2; ++par) {
    // Words 2q + hf of a row's 8 hold bytes 4 hf .. 4 hf + 3 of its block q:
    // block par is in the first 16-byte unit, block 2 + par in the second.
    const uint2 g01 = lds_v2(rg + u0 + 8u * par), g23 = lds_v2(rg + u1 + 8u * par);
    const uint2 h01 = lds_v2(rh + u0 + 8u * par), h23 = lds_v2(rh + u1 + 8u * par);
    if (par == 1) release();
    float(&d)[4] = par ? o : e;
    // Not unrolled: unrolling both halves lets the compiler hoist the
    // conversions of both, which needs ~25 more registers than the launch
    // bound leaves.
#pragma unroll 1
    for (int hf = 0; hf < 2; ++hf) {
      // Unit v = 2 par + hf of the lane's four: x pairs of bytes 4 hf .. 4 hf + 3
      // of its block par (slot 0) and 2 + par (slot 1).
      const int v = 2 * par + hf;
      const uint32_t za = zero + 16u * (uint32_t)v;
      const uint4 va = lds_v4(own_a ? xb + 64u * (uint32_t)v : za);
      const uint4 vb = lds_v4(own_b ? xb + 64u * (uint32_t)(4 + v) : za);
      const uint32_t g0 = hf ? g01.y : g01.x, g1 = hf ? g23.y : g23.x;
      const uint32_t h0 = hf ? h01.y : h01.x, h1 = hf ? h23.y : h23.x;
      mma_f16_16816(d, e2m1_byte_to_f16x2<0>(g0), e2m1_byte_to_f16x2<0>(h0),
                    e2m1_byte_to_f16x2<0>(g1), e2m1_byte_to_f16x2<0>(h1), va.x, vb.x);
      mma_f16_16816(d, e2m1_byte_to_f16x2<1>(g0), e2m1_byte_to_f16x2<1>(h0),
                    e2m1_byte_to_f16x2<1>(g1), e2m1_byte_to_f16x2<1>(h1), va.y, vb.y);
      mma_f16_16816(d, e2m1_byte_to_f16x2<2>(g0), e2m1_byte_to_f16x2<2>(h0),
                    e2m1_byte_to_f16x2<2>(g1), e2m1_byte_to_f16x2<2>(h1), va.z, vb.z);
      mma_f16_16816(d, e2m1_byte_to_f16x2<3>(g0), e2m1_byte_to_f16x2<3>(h0),
                    e2m1_byte_to_f16x2<3>(g1), e2m1_byte_to_f16x2<3>(h1), va.w, vb.w);
    }
  }
  float sg[4], sh[4];
  scale_word_f32(sgw, sg);
  scale_word_f32(shw, sh);
  tot[0] += sg[0] * e[0] + sg[2] * e[1] + sg[1] * o[0] + sg[3] * o[1];
  tot[1] += sh[0] * e[2] + sh[2] * e[3] + sh[1] * o[2] + sh[3] * o[3];
}

constexpr int kGvMaxWarps = 13;    // consumer warps: 2 CTAs of 14 warps per SM
constexpr int kGvTileCodes = 16 * (kGvChunk / 2);       // 2 KB: one 16-row tile
constexpr int kGvTileScales = 16 * (kGvChunk / kGroup);  // 256 B
constexpr int kGvMaxKs = 2048;     // K per CTA (f16 x slice in shared memory)
constexpr int kGvSmemCap = 110 * 1024;  // dynamic shared memory per CTA (two per SM)

// Shared memory of a CTA with `w` consumer warps, `stages` ring stages, `m`
// token rows of x (twice for hi + lo), a K split of `cs` and `parts` partial
// sums per owned row (2 for gate + up): the ring, the f16 x slice(s), a zero
// row of x (tokens >= M), the receive buffer of the cluster
// reduction ([cs][per][parts][8] fp32, per =
// ceil(16 w / parts / cs)), per-token scales and exponents, alpha of the rows
// this CTA finalises, the mbarriers.
struct GemvSmem {
  int stage, codes, ring, xs, xs_lo, zero, recv, inv, emax, alpha, bars, total;
  __host__ __device__ GemvSmem(int w, int stages, int xstride, int m, int cs, int parts,
                               bool split) {
    codes = w * kGvTileCodes;
    stage = (codes + w * kGvTileScales + 1023) & ~1023;
    ring = 0;
    xs = stages * stage;
    xs_lo = xs + m * xstride;
    zero = xs_lo + (split ? m * xstride : 0);
    recv = zero + xstride;
    const int per = (16 * w / parts + cs - 1) / cs;
    inv = recv + (int)sizeof(float) * cs * per * parts * kGvTok;
    emax = inv + (int)sizeof(float) * kGvTok;
    alpha = emax + (int)sizeof(int) * kGvTok;
    bars = (alpha + (int)sizeof(float) * parts * per + 7) & ~7;
    total = bars + 16 * stages;
  }
};

// Staging of an item's activations: M (<= 8) token rows of nunits 16-byte
// units (8 consecutive k each) -> f16 in shared memory (row tt at xs + tt *
// xstride, units XOR-swizzled), each token scaled by a power of two 2^s
// chosen from its largest exponent (warp max, then shared atomicMax into
// emax[], which must be zero on entry).  load(tt, u, v, vl) fetches unit u of
// token tt (vl: the low part, kGvDown's x = hi + lo, kept as f16 hi + f16 lo).
// Called by the nthr consumer threads (tid < nthr) together: they meet at
// named barrier 1 between the two passes.  With `regs`, up to 4 units per
// thread stay in registers (one read of the source); else the source is
// read twice.  nunits is a multiple of 32, so every warp-wide test below is
// uniform over the warp.
template <int MODE, class Load>
__device__ __forceinline__ void gv_stage_units(const Load &load, int M, int nunits, int xstride,
                                               uint8_t *xs, uint8_t *xs_lo, int *emax, int tid,
                                               int nthr, bool regs) {
  constexpr bool kSplit = MODE == kGvDown;
  const int total_units = M * nunits;
  auto load_units = [&](int base, uint4 (&v)[4], uint4 (&vl)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * nthr;
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      vl[j] = make_uint4(0u, 0u, 0u, 0u);
      if (i < total_units) {
        const int tt = i / nunits;
        load(tt, i - tt * nunits, v[j], vl[j]);
      }
    }
  };
  // fp32 values of a unit (x, or hi + lo).
  auto unit_f32 = [&](const uint4 &v, const uint4 &vl, float (&f)[8]) {
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    const uint32_t il[4] = {vl.x, vl.y, vl.z, vl.w};
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) {
      f[2 * q2] = bf16lo(in[q2]);
      f[2 * q2 + 1] = bf16hi(in[q2]);
      if constexpr (kSplit) {
        f[2 * q2] += bf16lo(il[q2]);
        f[2 * q2 + 1] += bf16hi(il[q2]);
      }
    }
  };
  auto max_units = [&](int base, const uint4 (&v)[4], const uint4 (&vl)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * nthr;
      if (i < total_units) {
        uint32_t m;
        if constexpr (kSplit) {
          float f[8];
          unit_f32(v[j], vl[j], f);
          float mx = 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(f[e]));
          m = (__float_as_uint(mx) >> 23) & 0xFFu;  // biased f32 exponent = bf16's
        } else {
          m = __vmaxu2(__vmaxu2(v[j].x & 0x7F807F80u, v[j].y & 0x7F807F80u),
                       __vmaxu2(v[j].z & 0x7F807F80u, v[j].w & 0x7F807F80u));
          m = max(m & 0xFFFFu, m >> 16) >> 7;
        }
        // The warp's 32 units belong to one token (nunits % 32 == 0).
        m = __reduce_max_sync(0xffffffffu, m);
        if ((tid & 31) == 0) atomicMax(&emax[i / nunits], (int)m);
      }
    }
  };
  auto convert_units = [&](int base, const uint4 (&v)[4], const uint4 (&vl)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * nthr;
      if (i < total_units) {
        const int tt = i / nunits, u = i - tt * nunits;
        const int e = max(emax[tt], 1);  // biased exponent of max|x|
        const int sc = min(max(141 - e, -126), 127);
        const float fs = __int_as_float((sc + 127) << 23);
        float f[8];
        unit_f32(v[j], vl[j], f);
        uint32_t o[4], ol[4];
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          const float x0 = f[2 * q2] * fs, x1 = f[2 * q2 + 1] * fs;
          const __half2 h2 = __floats2half2_rn(x0, x1);
          o[q2] = *reinterpret_cast<const uint32_t *>(&h2);
          if constexpr (kSplit) {
            const __half2 l2 = __floats2half2_rn(x0 - __low2float(h2), x1 - __high2float(h2));
            ol[q2] = *reinterpret_cast<const uint32_t *>(&l2);
          }
        }
        const int off = tt * xstride + 16 * xs_unit(u);
        *reinterpret_cast<uint4 *>(xs + off) = make_uint4(o[0], o[1], o[2], o[3]);
        if constexpr (kSplit)
          *reinterpret_cast<uint4 *>(xs_lo + off) = make_uint4(ol[0], ol[1], ol[2], ol[3]);
      }
    }
  };
  if (regs && total_units <= 4 * nthr) {
    uint4 v[4], vl[4];
    load_units(tid, v, vl);
    max_units(tid, v, vl);
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    convert_units(tid, v, vl);
  } else {
    for (int base = tid; base < total_units; base += 4 * nthr) {
      uint4 v[4], vl[4];
      load_units(base, v, vl);
      max_units(base, v, vl);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    for (int base = tid; base < total_units; base += 4 * nthr) {
      uint4 v[4], vl[4];
      load_units(base, v, vl);
      convert_units(base, v, vl);
    }
  }
}

// gv_stage_units over the x slice [k0, k0 + ks) in global memory: kGvGateUp
// reads token tt from row x_rows[slot0 + tt] (or slot0 + tt), kGvDown from
// row slot0 + tt of x (+ x_lo), plain mode from row tt.
template <int MODE>
__device__ __forceinline__ void gv_stage_x(const GemvArgs &a, int slot0, int M, int k0, int ks,
                                           int xstride, uint8_t *xs, uint8_t *xs_lo, int *emax,
                                           int tid, int nthr) {
  auto load = [&](int tt, int u, uint4 &v, uint4 &vl) {
    int64_t row = tt;
    if constexpr (MODE == kGvGateUp) row = a.x_rows ? __ldcg(a.x_rows + slot0 + tt) : slot0 + tt;
    if constexpr (MODE == kGvDown) row = slot0 + tt;
    const int64_t off = row * a.x_ld + k0 + 8 * u;
    v = __ldcg(reinterpret_cast<const uint4 *>(a.x + off));
    if constexpr (MODE == kGvDown) vl = __ldcg(reinterpret_cast<const uint4 *>(a.x_lo + off));
  };
  gv_stage_units<MODE>(load, M, ks / 8, xstride, xs, xs_lo, emax, tid, nthr, true);
}

// 1 / 2^s of token t's staging scale (0 for tokens >= M).
__device__ __forceinline__ float gv_inv_scale(const int *emax, int t, int M) {
  const int e = max(emax[t], 1);
  const int sc = min(max(141 - e, -126), 127);
  return t < M ? __frcp_rn(__int_as_float((sc + 127) << 23)) : 0.0f;
}

// Cluster q of a K split into gridDim.x slices owns row tiles
// [q * nt / nq, (q + 1) * nt / nq) (nq = gridDim.y clusters, nt = 16-row
// tiles; in kGvGateUp a "tile" is a pair: gate rows and the matching up
// rows): tile counts differ by at most one, so every SM gets the same weight
// bytes to within one tile.  CTA = one consumer warp per 16-row tile + a
// producer warp that streams the CTA's 256-k chunks of those tiles with TMA
// (per stage: a 128-byte-swizzled box of the tiles' rows x 128 B of codes and
// one of their rows x 16 B of blockscales, twice in kGvGateUp) through an
// S-stage ring.  Grouped modes: blockIdx.z = work item.
//
// Everything the previous kernel wrote (activations, work items) is read with
// L2-coherent loads after griddepcontrol.wait: under programmatic dependent
// launch the CTAs start before that kernel has finished, and the read-only
// (non-coherent) cache path could return lines cached before its writes.
template <int MODE>
__global__ void __launch_bounds__(32 * (kGvMaxWarps + 1), 2)
    gemv_kernel(const __grid_constant__ CUtensorMap tmW_hi, const __grid_constant__ CUtensorMap tmS_hi,
                const __grid_constant__ CUtensorMap tmW_lo, const __grid_constant__ CUtensorMap tmS_lo,
                GemvArgs a) {
  constexpr bool kSplit = MODE == kGvDown;
  constexpr int kParts = MODE == kGvGateUp ? 2 : 1;
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  uint8_t *gsm = reinterpret_cast<uint8_t *>(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
  __shared__ int abort_flag;

  const int W = (int)(blockDim.x >> 5) - 1;  // consumer warps
  const int S = a.stages;
  const GemvSmem L(W, S, a.xstride, a.M, gridDim.x, kParts, kSplit);
  uint8_t *ring = gsm + L.ring;
  uint8_t *xs = gsm + L.xs;
  uint8_t *xs_lo = gsm + L.xs_lo;
  uint32_t *zero_row = reinterpret_cast<uint32_t *>(gsm + L.zero);
  float *recv = reinterpret_cast<float *>(gsm + L.recv);
  float *inv_scale = reinterpret_cast<float *>(gsm + L.inv);
  int *emax = reinterpret_cast<int *>(gsm + L.emax);
  float *alpha_s = reinterpret_cast<float *>(gsm + L.alpha);
  uint64_t *bars = reinterpret_cast<uint64_t *>(gsm + L.bars);  // full[S], empty[S]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, c = lane & 3;
  const int Cn = gridDim.x, slice = blockIdx.x;
  // Tiles (pairs in kGvGateUp) of one weight matrix and this cluster's share.
  const int nt = (MODE == kGvGateUp ? a.N / 2 : a.N + 15) / 16;
  const int nq = gridDim.y, q = blockIdx.y;
  const int tile0 = (int)((int64_t)q * nt / nq), ntiles = (int)((int64_t)(q + 1) * nt / nq) - tile0;
  const int nwarps_used = kParts * ntiles;  // consumer warps with a tile
  const int k0 = slice * a.ks;
  const int nch = a.ks / kGvChunk;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  volatile int *abort = &abort_flag;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, nwarps_used);
    }
    abort_flag = 0;
    mbar_fence_init();
  }
  if (tid < kGvTok) emax[tid] = 0;
  for (int i = tid; i < a.xstride / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(zero_row)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  // Programmatic dependent launch: everything above overlapped the previous
  // kernel.  What that kernel may have written (activations, work items,
  // outputs it still reads) is touched only after griddepcontrol.wait.  In
  // plain mode the weights are not among it: the producer streams them
  // before waiting, so that a launch which follows another (it can start on
  // the SMs that kernel leaves free) has its first stages in flight while
  // the previous layer finishes.
  if constexpr (MODE != kGvPlain) asm volatile("griddepcontrol.wait;" ::: "memory");
  // Work item (grouped modes): expert g, token slots [slot0, slot0 + M).
  // The whole cluster shares blockIdx.z, so it leaves together.
  int g = 0, slot0 = 0, M = a.M;
  if constexpr (MODE != kGvPlain) {
    if ((int)blockIdx.z >= __ldcg(a.n_work)) return;
    const int *it = reinterpret_cast<const int *>(a.work + blockIdx.z);
    g = __ldcg(it);
    slot0 = __ldcg(it + 1);
    M = __ldcg(it + 2);
  }
  const int64_t grow0 = (int64_t)g * a.N;  // first row of the expert in the stacked matrix
  // Rows this CTA finalises: [lo, lo + nr) of the cluster's 16 * ntiles
  // (pair rows in kGvGateUp).
  const int rows = 16 * ntiles;
  const int per = (rows + Cn - 1) / Cn;
  const int lo = min(slice * per, rows), nr = min(lo + per, rows) - lo;
  for (int i = tid; i < kParts * nr; i += blockDim.x) {
    const int part = i / nr, r = i - part * nr;
    const int n = 16 * tile0 + lo + r + (part ? a.N / 2 : 0);  // row within the matrix
    alpha_s[i] = (MODE == kGvGateUp || n < a.N) ? alpha_of(a.al, g, n) : 0.0f;
  }

  if (warp == W) {
    // Producer: one thread issues the TMA loads, S stages ahead of use; one
    // box per stage (per part) for all of the CTA's tiles (maps with W and
    // W-1 tiles per part).
    if (lane == 0) {
      const bool full_count = kParts * ntiles == W;
      const CUtensorMap *tmW = full_count ? &tmW_hi : &tmW_lo;
      const CUtensorMap *tmS = full_count ? &tmS_hi : &tmS_lo;
      const uint64_t pol = l2_evict_first_policy();
      prefetch_tmap(tmW);
      prefetch_tmap(tmS);
      int issued = 0;
      for (int ch = 0; ch < nch; ++ch) {
        const int s = ch % S, u = ch / S;
        if (u > 0 && !mbar_wait(empty0 + 8 * s, (u - 1) & 1, &g_gemv_status, kDevTimeoutEmpty,
                                abort))
          break;
        const uint32_t st = smem_u32(ring + s * L.stage);
        mbar_arrive_expect_tx(full0 + 8 * s, kParts * ntiles * (kGvTileCodes + kGvTileScales));
        const int xc = (k0 + ch * kGvChunk) / 2, xsf = (k0 + ch * kGvChunk) / kGroup;
#pragma unroll
        for (int part = 0; part < kParts; ++part) {
          const int row = (int)(grow0 + 16 * tile0 + (part ? a.N / 2 : 0));
          tma_load_2d_hint(st + part * ntiles * kGvTileCodes, tmW, xc, row, full0 + 8 * s, pol);
          tma_load_2d_hint(st + L.codes + part * ntiles * kGvTileScales, tmS, xsf, row,
                           full0 + 8 * s, pol);
        }
        issued = ch + 1;
      }
      // After an abort, wait (bounded) for the copies still in flight before exit.
      volatile int no_abort = 0;
      for (int ch = max(issued - S, 0); ch < issued; ++ch)
        mbar_wait(full0 + 8 * (ch % S), (ch / S) & 1, &g_gemv_status, kDevTimeoutFull,
                  &no_abort);
    }
    __syncwarp();
    // Plain mode: the output stores below come after the previous kernel.
    if constexpr (MODE == kGvPlain) asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    if constexpr (MODE == kGvPlain) asm volatile("griddepcontrol.wait;" ::: "memory");
    // x slice -> f16 with a per-token power-of-two scale (gv_stage_x).
    gv_stage_x<MODE>(a, slot0, M, k0, a.ks, a.xstride, xs, xs_lo, emax, tid, 32 * W);
    if (tid < kGvTok) inv_scale[tid] = gv_inv_scale(emax, tid, M);
    asm volatile("bar.sync 1, %0;" ::"r"(32 * W) : "memory");  // consumer warps only
    // The next kernel in the stream may start its prologue now.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp < nwarps_used) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const bool has_x = gq < M;  // tokens >= M: the zero row (zero B fragments)
      const uint32_t xrow = has_x ? smem_u32(xs + gq * a.xstride) : smem_u32(zero_row);
      const uint32_t xrow_lo = has_x ? smem_u32(xs_lo + gq * a.xstride) : smem_u32(zero_row);
      if (MODE == kGvPlain && M == 1) {
        // One token: blockscales applied per block after the MMAs
        // (gemv_compute_m1); per lane, sums over its own blocks of rows g
        // and g + 8, added over the lane quad at the end.
        const uint32_t x0 = smem_u32(xs), zero = smem_u32(zero_row);
        const bool own_a = gq == 2 * c, own_b = gq == 2 * c + 1;
        float tot[2] = {0.0f, 0.0f};
        for (int ch = 0; ch < nch; ++ch) {
          const int s = ch % S, u = ch / S;
          const bool ok = mbar_wait(full0 + 8 * s, u & 1, &g_gemv_status, kDevTimeoutFull, abort);
          if (!__all_sync(0xffffffffu, ok)) break;
          const uint32_t st = smem_u32(ring + s * L.stage);
          const uint32_t scales = st + L.codes + warp * kGvTileScales;
          const uint32_t sgw = lds_u32(scales + 16u * gq + 4u * c);
          const uint32_t shw = lds_u32(scales + 16u * (gq + 8) + 4u * c);
          gemv_compute_m1(st + warp * kGvTileCodes, sgw, shw, gq, c, tot,
                          x0 + 16u * (uint32_t)(32 * ch + c), zero, own_a, own_b, [&] {
                            fence_proxy_async_smem();  // as in the general path below
                            __syncwarp();
                            if (lane == 0) mbar_arrive(empty0 + 8 * s);
                          });
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tot[h] += __shfl_xor_sync(0xffffffffu, tot[h], 1);
          tot[h] += __shfl_xor_sync(0xffffffffu, tot[h], 2);
        }
        acc[0] = tot[0];
        acc[2] = tot[1];
      } else {
        for (int ch = 0; ch < nch; ++ch) {
          const int s = ch % S, u = ch / S;
          const bool ok = mbar_wait(full0 + 8 * s, u & 1, &g_gemv_status, kDevTimeoutFull, abort);
          if (!__all_sync(0xffffffffu, ok)) break;
          const uint32_t st = smem_u32(ring + s * L.stage);
          GemvChunk b;
          gemv_fetch(b, st + warp * kGvTileCodes, st + L.codes + warp * kGvTileScales, gq, c);
          // The stage is refilled by TMA (async proxy) once released: order
          // these generic-proxy reads before that write.  Without the fence
          // the refill was seen to overtake the reads (rows of one tile
          // decoded from the next chunk's codes, a few calls in a hundred).
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(empty0 + 8 * s);  // operands are in registers
          // The MMA's fp32 accumulation is not IEEE round-to-nearest: chains are
          // kept to one chunk (16 or 32 MMAs) and chunk sums added with fp32 adds.
          float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          const uint32_t xo = 16u * (uint32_t)(32 * ch + c);
          gemv_compute<kSplit>(b, part, xrow + xo, xrow_lo + xo);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i] += part[i];
        }
      }
      // Partial sums (times 2^-s per token) go straight to the CTA of the
      // cluster that owns the row: slot [slice][row - owner's first row][part].
      const float is0 = inv_scale[2 * c], is1 = inv_scale[2 * c + 1];
      const int part = warp / ntiles;  // kGvGateUp: warps [0, ntiles) gate, then up
      const int wt = warp - part * ntiles;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = wt * 16 + gq + 8 * h;
        const int owner = r / per, local = r - owner * per;
        float *dst = recv + (((size_t)slice * per + local) * kParts + part) * kGvTok + 2 * c;
        if (Cn > 1) dst = cluster_map(dst, owner);
        if (2 * c < M) dst[0] = acc[2 * h] * is0;
        if (2 * c + 1 < M) dst[1] = acc[2 * h + 1] * is1;
      }
    }
  }

  // One cluster barrier (release / acquire) publishes the pushed partial
  // sums; each CTA then adds its rows' Cn slices in slice order and stores.
  if (Cn > 1) {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
  } else {
    __syncthreads();
  }
  for (int i = tid; i < nr * M; i += blockDim.x) {
    const int r = i % nr, tok = i / nr;
    float v[kParts];
#pragma unroll
    for (int part = 0; part < kParts; ++part) {
      float sum = 0.0f;
      for (int qq = 0; qq < Cn; ++qq)
        sum += recv[(((size_t)qq * per + r) * kParts + part) * kGvTok + tok];
      v[part] = sum * alpha_s[part * nr + r];
    }
    const int n = 16 * tile0 + lo + r;
    if constexpr (MODE == kGvGateUp) {
      // silu(gate) * up as bf16 hi + lo (the down projection's operand).
      const float o = silu_f32(v[0]) * v[1];
      const uint16_t h = f32_to_bf16_bits(o);
      const float hf = __uint_as_float((uint32_t)h << 16);
      const int64_t idx = (int64_t)(slot0 + tok) * a.y_ld + n;
      reinterpret_cast<uint16_t *>(a.y)[idx] = h;
      a.y_lo[idx] = f32_to_bf16_bits(o - hf);
    } else {
      if (n < a.N) {
        int64_t row = tok;
        if constexpr (MODE == kGvDown)
          row = a.y_rows ? __ldcg(a.y_rows + slot0 + tok) : slot0 + tok;
        if (a.y_dtype == kBF16)
          reinterpret_cast<uint16_t *>(a.y)[row * a.y_ld + n] = f32_to_bf16_bits(v[0]);
        else
          reinterpret_cast<float *>(a.y)[row * a.y_ld + n] = v[0];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Persistent grouped GEMV of the MoE experts (kGvGateUp / kGvDown).
//
// The work of one call is n_work items (expert, up to 8 token slots) x G row
// groups of the expert's matrix; a "unit" is one (item, row group) over the
// whole K.  The grid is one CTA per SM; CTA b takes the contiguous unit range
// [b U / P, (b + 1) U / P) of the U = n_work * G units (item-major, so a CTA
// meets few item changes and the items of one expert run side by side, their
// weights shared through L2).  Row group q of an expert owns tiles
// [q nt / G, (q + 1) nt / G): the groups differ by at most one tile, which
// the two tensor maps (W and W - 1 tiles) cover.  A tile is the 16 rows of
// one MMA: kGvDown, 16 consecutive down rows; kGvGateUp, 8 gate rows and the
// same 8 rows of up (MMA rows 0-7 and 8-15), so that every lane holds the
// gate and the up sums of its output rows and applies silu(gate) * up in
// registers (no exchange between warps, no barrier per unit).
//
// Nothing on the consumer warps' path reads global memory, whose latency
// under the kernel's own TMA stream is several microseconds:
//   * at the start, all threads load the CTA's items into a shared table
//     (expert, slots, input_scale, the slots' activation or output rows);
//   * the producer warp streams the 256-k chunks of unit after unit through
//     one S-stage ring (so the TMA queue stays full across unit boundaries),
//     and with a unit's first chunk the unit's weight_scale_2 rows;
//   * for each item it copies the item's bf16 activation rows into shared
//     memory with bulk copies (one item ahead), which the consumers then
//     convert to scaled f16 in shared memory (gv_stage_units);
//   * the consumer warps (one per tile) accumulate over all of K in
//     registers (no K split, no cluster reduction) and write their rows at
//     the end of the unit.
// ---------------------------------------------------------------------------
constexpr int kGgSmemCap = 226 * 1024 - 64;  // dynamic smem: 227 KB less the static 1 KB
constexpr int kGgMaxStages = 8;
constexpr int kGgMaxItems = 64;  // items one CTA may meet (the shared table)

// One row of the item table: expert, first slot, slots, alpha's input_scale
// and, per slot, the activation row (kGvGateUp) or output row (kGvDown).
struct GgItem {
  int g, slot0, M;
  float ins;
  int rows[kGvTok];
};

// Shared memory of a grouped CTA with w consumer warps (tiles), `stages` ring
// stages (each: codes, blockscales and the weight_scale_2 rows of w tiles;
// kGvGateUp: the gate half of each at offset 0, the up half at half its
// size), K and at most `items` items: the ring, the f16 activations of one
// item (twice for hi + lo), a zero row (tokens >= M), the bf16 rows they are
// converted from (twice for hi + lo), the token scales, the item table, the
// mbarriers.
struct GgSmem {
  int stage, codes, ws2, xstride, xs, xs_lo, zero, raw, raw_lo, inv, emax, items, bars, total;
  __host__ __device__ GgSmem(int w, int stages, int K, bool split, int n_items) {
    codes = w * kGvTileCodes;
    ws2 = codes + w * kGvTileScales;
    stage = (ws2 + 64 * w + 1023) & ~1023;
    xstride = 2 * K + 64;
    xs = stages * stage;
    xs_lo = xs + kGvTok * xstride;
    zero = xs_lo + (split ? kGvTok * xstride : 0);
    raw = zero + xstride;
    raw_lo = raw + kGvTok * 2 * K;
    inv = raw_lo + (split ? kGvTok * 2 * K : 0);
    emax = inv + (int)sizeof(float) * kGvTok;
    items = emax + (int)sizeof(int) * kGvTok;
    bars = (items + (int)sizeof(GgItem) * n_items + 7) & ~7;
    total = bars + 16 * stages + 16;
  }
};

// Rows of the weight matrix per tile: 16 (kGvDown), 8 of gate and the same 8
// of up (kGvGateUp).
template <int MODE>
__host__ __device__ constexpr int gg_tile_rows() {
  return MODE == kGvGateUp ? 8 : 16;
}

template <int MODE>
__global__ void __launch_bounds__(32 * (kGvMaxWarps + 1), 1)
    gemv_grouped_kernel(const __grid_constant__ CUtensorMap tmW_hi,
                        const __grid_constant__ CUtensorMap tmS_hi,
                        const __grid_constant__ CUtensorMap tmW_lo,
                        const __grid_constant__ CUtensorMap tmS_lo, GemvArgs a) {
  static_assert(MODE == kGvGateUp || MODE == kGvDown, "grouped modes only");
  constexpr bool kSplit = MODE == kGvDown;
  constexpr bool kPair = MODE == kGvGateUp;
  constexpr int kTR = gg_tile_rows<MODE>();
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  uint8_t *gsm = reinterpret_cast<uint8_t *>(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
  __shared__ int abort_flag;

  const int W = (int)(blockDim.x >> 5) - 1;  // consumer warps = tiles of a full group
  const int S = a.stages;
  const GgSmem L(W, S, a.K, kSplit, a.max_items);
  uint8_t *ring = gsm;
  uint8_t *xs = gsm + L.xs;
  uint8_t *xs_lo = gsm + L.xs_lo;
  float *inv_scale = reinterpret_cast<float *>(gsm + L.inv);
  int *emax = reinterpret_cast<int *>(gsm + L.emax);
  GgItem *tab = reinterpret_cast<GgItem *>(gsm + L.items);
  uint64_t *bars = reinterpret_cast<uint64_t *>(gsm + L.bars);  // full[S], empty[S], x full, x empty

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, c = lane & 3;
  const int G = a.ggroups;
  const int nt = kPair ? a.N / 2 / kTR : (a.N + kTR - 1) / kTR;
  const int nch = a.K / kGvChunk;
  const int rowb = 2 * a.K;  // bytes of one bf16 activation row
  // kGvGateUp stage layout: the up half of codes, blockscales and
  // weight_scale_2 starts half a full group's size after the gate half.
  const uint32_t up_codes = 128u * kTR * W, up_scales = 16u * kTR * W, up_ws2 = 4u * kTR * W;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  const uint32_t xfull = smem_u32(bars + 2 * S), xempty = smem_u32(bars + 2 * S + 1);
  const bool ws2_copy = a.al.ws2_rows != nullptr;
  volatile int *abort = &abort_flag;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, W);  // every consumer warp releases every stage
    }
    mbar_init(xfull, 1);
    mbar_init(xempty, 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  if (tid < kGvTok) emax[tid] = 0;
  for (int i = tid; i < L.xstride / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(gsm + L.zero)[i] = make_uint4(0u, 0u, 0u, 0u);
  // The work items come from the previous kernel (griddepcontrol.wait), and
  // so do the activations.  The next kernel may launch now: its CTAs take
  // the SMs this grid's CTAs leave and wait for this grid's completion.
  pdl_wait();
  pdl_trigger();
  const int64_t U = (int64_t)__ldcg(a.n_work) * G;
  const int P = gridDim.x, b = blockIdx.x;
  const int u_begin = (int)(U * b / P), u_end = (int)(U * (b + 1) / P);
  if (u_begin >= u_end) return;
  const int i0 = u_begin / G, n_items = (u_end - 1) / G - i0 + 1;
  if (n_items > a.max_items) {  // the launch sized the table for fewer items
    if (tid == 0) atomicCAS(&g_gemv_status, 0, (int)kDevBadPlan);
    return;
  }
  for (int j = tid; j < n_items; j += blockDim.x) {
    const int *it = reinterpret_cast<const int *>(a.work + i0 + j);
    GgItem e;
    e.g = __ldcg(it);
    e.slot0 = __ldcg(it + 1);
    e.M = __ldcg(it + 2);
    e.ins = a.al.input_scales ? __ldg(a.al.input_scales + e.g) : a.al.input_scale;
    const int32_t *map = MODE == kGvGateUp ? a.x_rows : a.y_rows;
#pragma unroll
    for (int t = 0; t < kGvTok; ++t)
      e.rows[t] = t < e.M ? (map ? __ldcg(map + e.slot0 + t) : e.slot0 + t) : 0;
    tab[j] = e;
  }
  __syncthreads();
  auto tile_lo = [&](int q) { return (int)((int64_t)q * nt / G); };

  if (warp == W) {
    // Producer: one thread issues the bulk copies of every item's activation
    // rows and the TMA loads of every chunk of every unit, up to S chunks
    // ahead of the consumers.
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      prefetch_tmap(&tmW_hi);
      prefetch_tmap(&tmS_hi);
      prefetch_tmap(&tmW_lo);
      prefetch_tmap(&tmS_lo);
      int gc = 0, k = 0;
      bool alive = true;
      for (int u = u_begin; u < u_end && alive; ++u) {
        const int q = u % G;
        const GgItem &e = tab[u / G - i0];
        if (u == u_begin || q == 0) {
          // The item's activation rows, once the consumers have converted the
          // previous item's.
          if (k > 0 && !mbar_wait(xempty, (k - 1) & 1, &g_gemv_status, kDevTimeoutEmpty, abort)) {
            alive = false;
            break;
          }
          mbar_arrive_expect_tx(xfull, e.M * rowb * (kSplit ? 2 : 1));
          const uint32_t raw = smem_u32(gsm + L.raw), raw_lo = smem_u32(gsm + L.raw_lo);
          for (int t = 0; t < e.M; ++t) {
            const int64_t row = MODE == kGvGateUp ? e.rows[t] : e.slot0 + t;
            bulk_load(raw + t * rowb, a.x + row * a.x_ld, rowb, xfull);
            if constexpr (kSplit) bulk_load(raw_lo + t * rowb, a.x_lo + row * a.x_ld, rowb, xfull);
          }
          ++k;
        }
        const int tile0 = tile_lo(q), ntiles = tile_lo(q + 1) - tile0;
        const bool full_count = ntiles == W;
        const CUtensorMap *tmW = full_count ? &tmW_hi : &tmW_lo;
        const CUtensorMap *tmS = full_count ? &tmS_hi : &tmS_lo;
        const int64_t grow0 = (int64_t)e.g * a.N + kTR * tile0;
        const int box_rows = kTR * ntiles;  // rows per box (per half in kGvGateUp)
        constexpr int kHalves = kPair ? 2 : 1;
        for (int ch = 0; ch < nch; ++ch, ++gc) {
          const int s = gc % S, r = gc / S;
          if (r > 0 && !mbar_wait(empty0 + 8 * s, (r - 1) & 1, &g_gemv_status, kDevTimeoutEmpty,
                                  abort)) {
            alive = false;
            break;
          }
          const uint32_t st = smem_u32(ring + s * L.stage);
          const bool w2 = ch == 0 && ws2_copy;
          mbar_arrive_expect_tx(full0 + 8 * s,
                                kHalves * box_rows * (128 + 16 + (w2 ? 4 : 0)));
#pragma unroll
          for (int h = 0; h < kHalves; ++h) {
            const int row = (int)(grow0 + (h ? a.N / 2 : 0));
            tma_load_2d_hint(st + h * up_codes, tmW, ch * (kGvChunk / 2), row, full0 + 8 * s, pol);
            tma_load_2d_hint(st + L.codes + h * up_scales, tmS, ch * (kGvChunk / kGroup), row,
                             full0 + 8 * s, pol);
            if (w2)
              bulk_load(st + L.ws2 + h * up_ws2,
                        a.al.ws2_rows + (int64_t)e.g * a.al.ws2_group_stride + kTR * tile0 +
                            (h ? a.N / 2 : 0),
                        4 * box_rows, full0 + 8 * s);
          }
        }
      }
      // Wait (bounded) for the copies still in flight before the CTA exits.
      volatile int no_abort = 0;
      for (int i = max(gc - S, 0); i < gc; ++i)
        mbar_wait(full0 + 8 * (i % S), (i / S) & 1, &g_gemv_status, kDevTimeoutFull, &no_abort);
      if (k > 0) mbar_wait(xfull, (k - 1) & 1, &g_gemv_status, kDevTimeoutFull, &no_abort);
    }
    return;
  }

  // Consumers.  Every consumer warp takes every named barrier of every item
  // change (after a timeout they skip the waits and the math, not the
  // barriers).  Warp w's tile: MMA rows gq and gq + 8 of the lane are
  // kGvDown, rows 16 w + gq and 16 w + gq + 8 of the row group; kGvGateUp,
  // gate row 8 w + gq and up row 8 w + gq.
  const int nthr = 32 * W;
  const uint8_t *raw = gsm + L.raw, *raw_lo = gsm + L.raw_lo;
  auto load_raw = [&](int tt, int u, uint4 &v, uint4 &vl) {
    v = *reinterpret_cast<const uint4 *>(raw + tt * rowb + 16 * u);
    if constexpr (kSplit) vl = *reinterpret_cast<const uint4 *>(raw_lo + tt * rowb + 16 * u);
  };
  // This lane's two weight rows within a stage (row index in the box) and
  // their byte offsets.
  const int rA = kPair ? kTR * warp + gq : kTR * warp + gq;
  const int rB = kPair ? kTR * warp + gq : kTR * warp + gq + 8;
  const uint32_t offA = 128u * rA, offB = (kPair ? up_codes : 0u) + 128u * rB;
  const uint32_t sofA = 16u * rA + 4u * c, sofB = (kPair ? up_scales : 0u) + 16u * rB + 4u * c;
  const int swA = rA & 7, swB = rB & 7;
  int gc = 0, k = 0;
  bool ok_all = true;
  for (int u = u_begin; u < u_end; ++u) {
    const int q = u % G;
    const GgItem &e = tab[u / G - i0];
    const int M = e.M;
    if (u == u_begin || q == 0) {
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");  // xs of the last item is dead
      if (ok_all) {
        const bool ok = mbar_wait(xfull, k & 1, &g_gemv_status, kDevTimeoutFull, abort);
        ok_all = __all_sync(0xffffffffu, ok);
      }
      // Its barriers are taken by all; a warp that gave up converts garbage.
      gv_stage_units<MODE>(load_raw, M, a.K / 8, L.xstride, xs, xs_lo, emax, tid, nthr, false);
      fence_proxy_async_smem();  // the reads of raw before the next item's bulk copies
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");  // emax complete, raw read
      if (tid < kGvTok) {
        inv_scale[tid] = gv_inv_scale(emax, tid, M);
        emax[tid] = 0;  // for the next item
      }
      if (tid == 0) mbar_arrive(xempty);
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
      ++k;
    }
    const int tile0 = tile_lo(q), ntiles = tile_lo(q + 1) - tile0;
    const bool has_tile = warp < ntiles;
    // weight_scale_2 of the lane's rows A and B, read from the unit's first
    // stage (the stage is refilled later).
    float w2a = a.al.ws2, w2b = a.al.ws2;
    const bool has_x = gq < M;  // tokens >= M: the zero row (zero B fragments)
    const uint32_t xrow = smem_u32(has_x ? xs + gq * L.xstride : gsm + L.zero);
    const uint32_t xrow_lo = smem_u32(has_x ? xs_lo + gq * L.xstride : gsm + L.zero);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int ch = 0; ch < nch; ++ch, ++gc) {
      const int s = gc % S, r = gc / S;
      if (!ok_all) continue;
      const bool ok = mbar_wait(full0 + 8 * s, r & 1, &g_gemv_status, kDevTimeoutFull, abort);
      ok_all = __all_sync(0xffffffffu, ok);
      if (!ok_all) continue;
      const uint32_t st = smem_u32(ring + s * L.stage);
      if (ch == 0 && ws2_copy && has_tile) {
        const float *w2s = reinterpret_cast<const float *>(ring + s * L.stage + L.ws2);
        w2a = w2s[rA];
        w2b = w2s[(kPair ? up_ws2 / 4 : 0) + rB];
      }
      GemvChunk bch;
      if (has_tile)
        gemv_fetch_rows(bch, st + offA, st + offB, swA, swB, st + L.codes + sofA,
                        st + L.codes + sofB, c);
      fence_proxy_async_smem();  // generic reads before the TMA refill (see gemv_kernel)
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
      if (has_tile) {
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t xo = 16u * (uint32_t)(32 * ch + c);
        gemv_compute<kSplit>(bch, part, xrow + xo, xrow_lo + xo);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += part[i];
      }
    }
    if (!has_tile) continue;
    const float is0 = inv_scale[2 * c], is1 = inv_scale[2 * c + 1];
    const float ins = e.ins;
    if constexpr (MODE == kGvDown) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = kTR * (tile0 + warp) + gq + 8 * h;
        if (n >= a.N) continue;
        const float al = ins * (h ? w2b : w2a);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int tok = 2 * c + t;
          if (tok >= M) continue;
          const float v = acc[2 * h + t] * (t ? is1 : is0) * al;
          const int64_t row = e.rows[tok];
          if (a.y_dtype == kBF16)
            reinterpret_cast<uint16_t *>(a.y)[row * a.y_ld + n] = f32_to_bf16_bits(v);
          else
            reinterpret_cast<float *>(a.y)[row * a.y_ld + n] = v;
        }
      }
    } else {
      // The lane's gate (acc[0..1]) and up (acc[2..3]) sums of output row n
      // for tokens 2c, 2c + 1: silu(gate) * up as bf16 hi + lo (the down
      // projection's operand).
      const int n = kTR * (tile0 + warp) + gq;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int tok = 2 * c + t;
        if (tok >= M) continue;
        const float is = t ? is1 : is0;
        const float vg = acc[t] * is * (ins * w2a);
        const float vu = acc[2 + t] * is * (ins * w2b);
        const float o = silu_f32(vg) * vu;
        const uint16_t hb = f32_to_bf16_bits(o);
        const float hf = __uint_as_float((uint32_t)hb << 16);
        const int64_t idx = (int64_t)(e.slot0 + tok) * a.y_ld + n;
        reinterpret_cast<uint16_t *>(a.y)[idx] = hb;
        a.y_lo[idx] = f32_to_bf16_bits(o - hf);
      }
    }
  }
}

// Ring stages that fit in the per-CTA budget (two CTAs per SM).
int gemv_stages(int w, int xstride, int m, int cs, int parts, bool split) {
  int s = 4;
  while (s > 2 && GemvSmem(w, s, xstride, m, cs, parts, split).total + 1024 > kGvSmemCap) --s;
  return GemvSmem(w, s, xstride, m, cs, parts, split).total + 1024 <= kGvSmemCap ? s : 0;
}

// Clusters of C CTAs (w consumer warps, smem bytes) the GPU holds at once.
template <int MODE>
int gemv_cluster_capacity(int C, int w, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, C, w, smem);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, 1, 1);
  cfg.blockDim = dim3(32 * (w + 1), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemv_kernel<MODE>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

template <int MODE>
cudaError_t set_smem_attr() {
  static std::mutex mu;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kGvSmemCap + 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return cudaSuccess;
}

// Plans (K split C, clusters, warps, stages) and launches a GEMV of `items`
// weight matrices of N rows (grid.z = items; 1 in plain mode).
//
// Two CTAs per SM.  K split C (cluster size): a divisor of the chunk count,
// at most 8, with K / C <= kGvMaxKs.  Clusters per matrix: two CTAs per SM /
// (C * items), or fewer when the GPU cannot hold that many clusters of C at
// once (a cluster must fit in one GPC); consumer warps W = the largest tile
// count of a cluster (at most kGvMaxWarps).  The C taken minimises the work of
// the busiest CTA times the waves of clusters, ks * (W + 0.16 M) * waves: W
// tiles of decode + MMA plus the conversion of M activation rows (about 0.16
// of a tile's instructions per row of x).
template <int MODE>
cudaError_t launch_mode(GemvArgs a, int items, int64_t total_rows, cudaStream_t st) {
  constexpr int kParts = MODE == kGvGateUp ? 2 : 1;
  constexpr bool kSplit = MODE == kGvDown;
  cudaError_t e = set_smem_attr<MODE>();
  if (e != cudaSuccess) return e;
  const int M = a.M;
  const int nck = a.K / kGvChunk;
  const int nt = (MODE == kGvGateUp ? a.N / 2 : a.N + 15) / 16;
  const int max_tiles = kGvMaxWarps / kParts;
  // Plain linear: one CTA per SM (a CTA takes at most half of an SM's shared
  // memory), so that the CTAs of the next launch in the stream fit beside
  // this one's and start streaming their weights before it ends.  Grouped
  // modes read their work items before any load and gain nothing from that:
  // two CTAs per SM.
  const int ctas_target = (MODE == kGvPlain ? 1 : 2) * tc_sm_count();
  int bestC = 0, bestW = 0, bestNq = 0, bestS = 0;
  double best_cost = 0.0;
  for (int C = 1; C <= 8; ++C) {
    if (nck % C || a.K / C > kGvMaxKs) continue;
    const int xstride = 2 * (a.K / C) + 64;
    int nq = ctas_target / (C * items);
    if (nq > nt) nq = nt;
    if (nq < 1) nq = 1;
    int tiles = 0, stages = 0, waves = 1;
    for (int it = 0; it < 2; ++it) {
      tiles = (nt + nq - 1) / nq;
      if (tiles > max_tiles) {
        tiles = max_tiles;
        nq = (nt + tiles - 1) / tiles;
        tiles = (nt + nq - 1) / nq;
      }
      stages = gemv_stages(kParts * tiles, xstride, M, C, kParts, kSplit);
      const int cap = gemv_cluster_capacity<MODE>(
          C, kParts * tiles,
          1024 + GemvSmem(kParts * tiles, stages, xstride, M, C, kParts, kSplit).total);
      if (cap <= 0) break;
      waves = (nq * items + cap - 1) / cap;
      if (waves == 1 || it == 1 || items > 1) break;
      nq = cap;  // one wave of the clusters that fit, with more tiles each
    }
    if (tiles <= 0 || stages <= 0) continue;
    const double cost =
        (double)(a.K / C) * (kParts * tiles + 0.16 * M) * waves * (1.0 + 0.01 * (waves - 1));
    if (bestC == 0 || cost < best_cost) {
      bestC = C;
      bestW = kParts * tiles;
      bestNq = nq;
      bestS = stages;
      best_cost = cost;
    }
  }
  if (bestC == 0) return cudaErrorInvalidValue;
  if (MODE == kGvPlain) {
    // Leave room on each SM for one CTA of the next launch (which then
    // streams its weights beside this one's tail): fewer ring stages, down
    // to two, until (CTAs per SM + 1) CTAs fit.  K=4096, N=14336 (clusters
    // of 4, 276 CTAs): three stages -> two took M = 1 from 12.8 to 11.8 us.
    const int sms = tc_sm_count();
    const int per_sm = (bestC * bestNq + sms - 1) / sms;
    const int xstride = 2 * (a.K / bestC) + 64;
    while (bestS > 2 &&
           (size_t)(per_sm + 1) *
                   (1024 + GemvSmem(bestW, bestS, xstride, M, bestC, kParts, kSplit).total) >
               (size_t)227 * 1024)
      --bestS;
  }
  a.ks = a.K / bestC;
  a.xstride = 2 * a.ks + 64;
  a.stages = bestS;
  // Boxes of W and W-1 tiles per part (clusters own one or the other count).
  CUtensorMap tm[4];
  for (int i = 0; i < 2; ++i) {
    const int t = bestW / kParts - i;
    const int rows = 16 * (t > 0 ? t : 1);
    if (!make_tmap_2d(&tm[2 * i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, total_rows, a.K / 2,
                      a.K / 2, kGvChunk / 2, rows, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tm[2 * i + 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.sf, total_rows,
                      a.K / kGroup, a.K / kGroup, kGvChunk / kGroup, rows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  }
  const size_t smem =
      1024 + (size_t)GemvSmem(bestW, a.stages, a.xstride, M, bestC, kParts, kSplit).total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bestC, bestNq, items);
  cfg.blockDim = dim3(32 * (bestW + 1), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = bestC;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<MODE>, tm[0], tm[1], tm[2], tm[3], a);
}

// Plan of the persistent grouped kernel: row groups G per item, consumer
// warps W, ring stages S (as many as fit beside one item's activations, at
// most kGgMaxStages), grid P and the item-table size.  False when the shapes
// or alignments do not suit it (then one cluster grid per item runs).
struct GgPlan {
  int G, W, S, P, max_items;
};

template <int MODE>
bool grouped_plan(const GemvArgs &a, int items, GgPlan &p) {
  constexpr bool kSplit = MODE == kGvDown;
  constexpr int kTR = gg_tile_rows<MODE>();
  const int N = a.N, K = a.K;
  const int nt = MODE == kGvGateUp ? N / 2 / kTR : (N + kTR - 1) / kTR;
  auto al16 = [](const void *q) { return ((uintptr_t)q & 15) == 0; };
  // Bulk copies: 16-byte aligned activation rows; weight_scale_2 rows in
  // whole tiles (32 or 64 bytes), the up half at a multiple of 16 rows.
  if (nt <= 0 || K % kGvChunk || N % 32 || !al16(a.x) || (a.x_ld * 2) % 16 ||
      (kSplit && !al16(a.x_lo)) ||
      (a.al.ws2_rows && (!al16(a.al.ws2_rows) || a.al.ws2_group_stride % 16)))
    return false;
  p.G = (nt + kGvMaxWarps - 1) / kGvMaxWarps;
  p.W = (nt + p.G - 1) / p.G;
  const int64_t units = (int64_t)items * p.G;
  p.P = (int)std::min<int64_t>(tc_sm_count(), units);
  if (p.P <= 0) return false;
  // A CTA's units span at most ceil(units / P) / G + 2 items.
  p.max_items = (int)(((units + p.P - 1) / p.P + p.G - 1) / p.G + 2);
  if (p.max_items > kGgMaxItems) return false;
  p.S = kGgMaxStages;
  while (p.S >= 2 && 1024 + GgSmem(p.W, p.S, K, kSplit, p.max_items).total > kGgSmemCap) --p.S;
  return p.S >= 2;
}

template <int MODE>
cudaError_t launch_grouped(GemvArgs a, const GgPlan &p, int64_t total_rows, cudaStream_t st) {
  constexpr bool kSplit = MODE == kGvDown;
  constexpr int kTR = gg_tile_rows<MODE>();
  {
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gemv_grouped_kernel<MODE>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kGgSmemCap);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  a.ks = a.K;
  a.stages = p.S;
  a.ggroups = p.G;
  a.max_items = p.max_items;
  // Boxes of W tiles and of one tile fewer (row groups differ by at most one
  // tile); kTR rows per tile (per half in kGvGateUp).
  CUtensorMap tm[4];
  for (int i = 0; i < 2; ++i) {
    const int t = p.W - i;
    const int rows = kTR * (t > 0 ? t : 1);
    if (!make_tmap_2d(&tm[2 * i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, total_rows, a.K / 2,
                      a.K / 2, kGvChunk / 2, rows, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tm[2 * i + 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.sf, total_rows,
                      a.K / kGroup, a.K / kGroup, kGvChunk / kGroup, rows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.P, 1, 1);
  cfg.blockDim = dim3(32 * (p.W + 1), 1, 1);
  cfg.dynamicSmemBytes = 1024 + (size_t)GgSmem(p.W, p.S, a.K, kSplit, p.max_items).total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_grouped_kernel<MODE>, tm[0], tm[1], tm[2], tm[3], a);
}

}  // namespace

bool gemv_supported(int M, int K, const void *w, const void *sf, const void *x, int64_t x_ld) {
  return M >= 1 && M <= kGvTok && K % kGvChunk == 0 && K <= 8 * kGvMaxKs &&
         ((uintptr_t)w & 15) == 0 && ((uintptr_t)sf & 15) == 0 && ((uintptr_t)x & 15) == 0 &&
         x_ld % 8 == 0 && tc_gemm_supported(K, w, x, x_ld);
}

int read_gemv_device_status() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_status, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(int));
  return v;
}

cudaError_t launch_gemv(const WeightSpec &ws, const AlphaSpec &al, const uint16_t *x,
                        int64_t x_ld, void *y, int y_dtype, int64_t y_ld, int M,
                        cudaStream_t st) {
  if (M == 0 || ws.N == 0) return cudaSuccess;
  GemvArgs a = {};
  a.w = ws.w;
  a.sf = ws.sf;
  a.al = al;
  a.x = x;
  a.x_ld = x_ld;
  a.y = y;
  a.y_dtype = y_dtype;
  a.y_ld = y_ld;
  a.M = M;
  a.N = ws.N;
  a.K = ws.K;
  return launch_mode<kGvPlain>(a, 1, ws.N, st);
}

bool moe_gemv_supported(int H, int I, const void *gate_up, const void *gate_up_sf,
                        const void *down, const void *down_sf) {
  auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  // K % 256 for both GEMMs (whole chunks), 16-row tiles of gate and up rows,
  // 16-byte aligned TMA bases; tc_gemm_supported also confirms the TMA
  // descriptor encoder is available.
  return H % kGvChunk == 0 && I % kGvChunk == 0 && H <= 8 * kGvMaxKs && I <= 8 * kGvMaxKs &&
         al16(gate_up) && al16(gate_up_sf) && al16(down) && al16(down_sf) &&
         tc_gemm_supported(H, gate_up, down, H);
}

cudaError_t launch_moe_gemv(const MoeGemvLaunch &m, cudaStream_t st) {
  if (m.items == 0) return cudaSuccess;
  GemvArgs a = {};
  a.w = m.w;
  a.sf = m.sf;
  a.al = m.al;
  a.x = m.x;
  a.x_lo = m.x_lo;
  a.x_ld = m.x_ld;
  a.y = m.y;
  a.y_lo = m.y_lo;
  a.y_dtype = m.y_dtype;
  a.y_ld = m.y_ld;
  a.M = kGvTok;  // items hold up to 8 slots; shared memory is sized for 8
  a.N = m.N;
  a.K = m.K;
  a.work = m.work;
  a.n_work = m.n_work;
  a.x_rows = m.x_rows;
  a.y_rows = m.y_rows;
  const int64_t total_rows = (int64_t)m.groups * m.N;
  // The persistent kernel when one item's activations fit beside a ring of
  // two or more stages; else one cluster grid per item (K split over CTAs).
  GgPlan p;
  if (m.gate_up && grouped_plan<kGvGateUp>(a, m.items, p))
    return launch_grouped<kGvGateUp>(a, p, total_rows, st);
  if (!m.gate_up && grouped_plan<kGvDown>(a, m.items, p))
    return launch_grouped<kGvDown>(a, p, total_rows, st);
  return m.gate_up ? launch_mode<kGvGateUp>(a, m.items, total_rows, st)
                   : launch_mode<kGvDown>(a, m.items, total_rows, st);
}

}  // namespace nvfp4

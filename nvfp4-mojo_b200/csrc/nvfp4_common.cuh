// nvfp4_common.cuh -- device helpers shared by the NVFP4 kernels (sm_100a).
//
// Format (nvfp4/config.mojo:13-35, :106-121):
//   * weights: uint8 [rows, K/2]; low nibble = even k, high nibble = odd k;
//     each nibble an E2M1 code, LUT {0,.5,1,1.5,2,3,4,6, -0,-.5,...,-6}.
//   * blockscales: float8_e4m3fn [rows, K/16], one per 16 consecutive k.
//   * value = LUT[code] * float(scale); weight_scale_2 and input_scale are
//     applied after accumulation as alpha (nvfp4/config.mojo:93-95,
//     nvfp4/deltanet.mojo:584).
//
// Decoding to bf16 on the tensor-core paths.  For code c = s.e1e0.m, the bf16
// bit pattern (s << 15) | ((c & 7) << 6) is exactly LUT[c] * 2^-126 (for
// e = 0 it is the bf16 subnormal m * 2^-127).  One bf16x2 multiply by
// float(scale) * 2^119 (at most 448 * 2^119 < bf16 max, and never a
// subnormal product since LUT*scale >= 2^-10) gives LUT*scale*2^-7 exactly:
// E2M1 x E4M3 products have at most 6 significant bits.  The 2^7 is folded
// into the epilogue's alpha, so GEMM results equal those of an exact decode.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4 {

constexpr int kGroup = 16;  // NVFP4_GROUP_SIZE
constexpr int kPack = 2;    // NVFP4_PACK_FACTOR
// Decoded tensor-core operands carry LUT*scale*2^-7; epilogues multiply by 2^7.
constexpr float kDecodeUnscale = 128.0f;

// float8_e4m3fn -> float32, exact (OCP FP8; 0x7F/0xFF are NaN, no Inf).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t s = (b >> 7) & 1u, e = (b >> 3) & 15u, m = b & 7u;
  float v;
  if (e == 0) {
    v = __uint2float_rn(m) * 0.001953125f;  // m * 2^-9, exact
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  }
  if (e == 15u && m == 7u) v = __uint_as_float(0x7fc00000u);
  return s ? -v : v;
}

// bf16x2 holding float(scale) * 2^119 in both halves (exact: <= 4 sig. bits).
__device__ __forceinline__ uint32_t scale_to_bf16x2_2p119(uint32_t b) {
  float f = e4m3_to_f32(b) * 6.6461399789245794e35f;  // * 2^119, exact (NaN stays NaN)
  uint32_t h = __float_as_uint(f) >> 16;               // exact truncation
  return h | (h << 16);
}

// Two e4m3 blockscales (low byte = first group) -> bf16x2 of float(s)*2^119
// broadcast to both halves, for each.  Fast path: the hardware e4m3x2 -> f16x2
// conversion is exact and every finite non-zero e4m3 is an f16 normal, so the
// bf16 pattern is ((|h| >> 3) + (231 << 7)) | sign.  Zero and NaN scales (the
// only inputs that leave that range) take the exact scalar path.
__device__ __forceinline__ void scale_pair_to_bf16x2(uint32_t u16, uint32_t &s0, uint32_t &s1) {
  // Zero (|b| == 0) and NaN (|b| == 0x7F) scales are the only codes outside
  // the fast path: (|b| - 1) >= 0x7E as unsigned catches both.
  const uint32_t b0 = u16 & 0x7Fu, b1 = (u16 >> 8) & 0x7Fu;
  if (__builtin_expect(((b0 - 1u) >= 0x7Eu) | ((b1 - 1u) >= 0x7Eu), 0)) {
    s0 = scale_to_bf16x2_2p119(u16 & 0xffu);
    s1 = scale_to_bf16x2_2p119((u16 >> 8) & 0xffu);
    return;
  }
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((unsigned short)u16));
  const uint32_t r = (((h & 0x7FFF7FFFu) >> 3) + 0x73807380u) | (h & 0x80008000u);
  asm("prmt.b32 %0, %1, %1, 0x1010;" : "=r"(s0) : "r"(r));
  asm("prmt.b32 %0, %1, %1, 0x3232;" : "=r"(s1) : "r"(r));
}

// Four bf16x2 words of LUT*2^-126 from one 32-bit word of 8 packed codes
// e0..e7 (e_j = nibble j = k offset j).  out[i] = (lo: e_i, hi: e_{i+4}).
__device__ __forceinline__ void decode8_raw_pairs(uint32_t w, uint32_t out[4]) {
  const uint32_t M = 0x81C081C0u;
  uint32_t w8 = w >> 8;
  out[0] = ((w & 0x000F000Fu) * 0x1040u) & M;
  out[1] = ((w & 0x00F000F0u) * 0x0104u) & M;
  out[2] = ((w8 & 0x000F000Fu) * 0x1040u) & M;
  out[3] = ((w8 & 0x00F000F0u) * 0x0104u) & M;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Byte permute: result byte i = selector nibble i picks from {b:a}.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Eight decoded bf16 values (LUT*scale*2^-7) in natural k order:
// out[j] = (lo: e_{2j}, hi: e_{2j+1}).
__device__ __forceinline__ void decode8_natural(uint32_t w, uint32_t s2, uint32_t out[4]) {
  uint32_t r[4];
  decode8_raw_pairs(w, r);
  // r[i] = (e_i, e_{i+4}) -> natural pairs (e0,e1), (e2,e3), (e4,e5), (e6,e7).
  uint32_t p0 = prmt(r[0], r[1], 0x5410u), p1 = prmt(r[2], r[3], 0x5410u);
  uint32_t p2 = prmt(r[0], r[1], 0x7632u), p3 = prmt(r[2], r[3], 0x7632u);
  out[0] = bf16x2_mul(p0, s2);
  out[1] = bf16x2_mul(p1, s2);
  out[2] = bf16x2_mul(p2, s2);
  out[3] = bf16x2_mul(p3, s2);
}

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t *>(&b);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// LUT[c] in fp32 via the same bit pattern (f32 subnormal for e = 0) * 2^126.
__device__ __forceinline__ float e2m1_to_f32(uint32_t c) {
  float raw = __uint_as_float(((c & 7u) << 22) | ((c & 8u) << 28));
  return raw * 8.5070591730234616e37f;  // 2^126, exact (denormals kept)
}

// mma.sync m16n8k16, bf16 inputs, fp32 accumulate (in place).
__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---- cp.async (sm_80+ LDGSTS) and shared-memory loads -------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the previous kernel in the stream is still running: it must execute
// pdl_wait() before touching anything that kernel wrote (and read that data
// with L2-coherent loads), and every such kernel waits, so that a chain of
// them stays ordered transitively.  pdl_trigger() lets the next kernel's CTAs
// launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ float silu_f32(float x) {
  // nvfp4/deltanet.mojo:66-80: sign-split logistic, then x * sigmoid(x).
  float s;
  if (x >= 0.0f) {
    float e = expf(-x);
    s = 1.0f / (1.0f + e);
  } else {
    float e = expf(x);
    s = e / (1.0f + e);
  }
  return x * s;
}

}  // namespace nvfp4

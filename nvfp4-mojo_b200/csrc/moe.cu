// moe.cu -- NVFP4 MoE expert path: router + softmax top-k, permutation of
// token slots by expert, grouped gate_up GEMM with fused SiLU(gate) * up,
// grouped down GEMM, weighted combine (+ optional residual).
//
// The reference has no MoE compute; it defines the per-expert NVFP4 weight
// layout (nvfp4/weight_loader.mojo:767-793, :873-887: gate/up/down linears
// per expert, router `mlp.gate.weight`) and the SiLU it uses
// (nvfp4/deltanet.mojo:66-80).  Semantics here: logits = x @ router (fp32),
// softmax over experts, top-k by probability with ties to the lower expert
// index, optional renormalisation of the k weights, then per selected expert
// h = gate_up(x) [2I], a = silu(h[:I]) * h[I:], y_e = down(a), and
// y = sum_j w_j * y_e_j.
#include <cfloat>

#include "../../include/nvfp4.h"
#include "abi_util.h"
#include "kernels.h"
#include "moe.h"
#include "nvfp4_common.cuh"
#include "router_topk.cuh"

namespace nvfp4 {

// ---------------------------------------------------------------------------
// Router: logits[t, e] = sum_h x[t, h] * router[h, e].
//
// Few tokens (decode): CUDA-core fp32 FMA, split over H so that enough CTAs
// run: CTA (32 experts, 8 tokens, H slice z) writes partial sums
// part[z][t][e]; lane = expert (router rows are expert-contiguous: 128
// coalesced bytes per h per warp), warps split the slice, their sums are added
// in a fixed order.  The top-k kernel adds the slices in z order.
// Many tokens (prefill): tensor cores, TF32 with the router split into
// hi + lo TF32 parts (x is bf16, exact in TF32), two MMAs per k step, so the
// logits carry fp32-level accuracy (~2^-21 relative residue of the split);
// also split over H when the token tiles alone do not cover the GPU.
// ---------------------------------------------------------------------------
constexpr int kRouterTok = 8;
constexpr int kRouterWarps = 8;
constexpr int kRouterTcMinTokens = 256;

__global__ void __launch_bounds__(32 * kRouterWarps)
    router_logits_kernel(const uint16_t *__restrict__ x, const float *__restrict__ router,
                         float *__restrict__ part, int T, int H, int E, int hslice) {
  extern __shared__ float4 rsm[];  // xs [hslice][8] fp32, then red [warps][8][32]
  float *xs = reinterpret_cast<float *>(rsm);
  float *red = xs + (size_t)hslice * kRouterTok;
  const int e0 = blockIdx.x * 32, t0 = blockIdx.y * kRouterTok, h0 = blockIdx.z * hslice;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();  // x may come from the previous kernel
  pdl_trigger();
  if (hslice % 8 == 0 && H % 8 == 0 && ((uintptr_t)x & 15) == 0) {
    // 8 bf16 at a time: thread i takes token i % 8 and rows 8 (i / 8) .. + 7.
    for (int i = threadIdx.x; i < hslice; i += blockDim.x) {
      const int tt = i % kRouterTok, h = 8 * (i / kRouterTok), t = t0 + tt;
      const uint4 v = t < T ? __ldcg(reinterpret_cast<const uint4 *>(x + (int64_t)t * H + h0 + h))
                            : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xs[(h + 2 * j) * kRouterTok + tt] = __uint_as_float(q[j] << 16);
        xs[(h + 2 * j + 1) * kRouterTok + tt] = __uint_as_float(q[j] & 0xFFFF0000u);
      }
    }
  } else {
    for (int i = threadIdx.x; i < hslice * kRouterTok; i += blockDim.x) {
      const int h = i / kRouterTok, tt = i % kRouterTok;
      const int t = t0 + tt;
      xs[i] = t < T ? __uint_as_float((uint32_t)__ldcg(x + (int64_t)t * H + h0 + h) << 16) : 0.0f;
    }
  }
  __syncthreads();
  const int e = min(e0 + lane, E - 1);
  const int hs = hslice / kRouterWarps, hb = warp * hs;
  float acc[kRouterTok];
#pragma unroll
  for (int i = 0; i < kRouterTok; ++i) acc[i] = 0.0f;
  const float *rp = router + (int64_t)(h0 + hb) * E + e;
  // 32 router rows per batch: all 32 loads in flight before their FMAs (the
  // warp's rows are one latency-bound stream otherwise).
  for (int hc = 0; hc < hs; hc += 32) {
    float r[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = hc + j < hs ? __ldg(rp + (int64_t)(hc + j) * E) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (hc + j >= hs) break;
      const float4 xa = *reinterpret_cast<const float4 *>(xs + (hb + hc + j) * kRouterTok);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + (hb + hc + j) * kRouterTok + 4);
      acc[0] = fmaf(xa.x, r[j], acc[0]);
      acc[1] = fmaf(xa.y, r[j], acc[1]);
      acc[2] = fmaf(xa.z, r[j], acc[2]);
      acc[3] = fmaf(xa.w, r[j], acc[3]);
      acc[4] = fmaf(xb.x, r[j], acc[4]);
      acc[5] = fmaf(xb.y, r[j], acc[5]);
      acc[6] = fmaf(xb.z, r[j], acc[6]);
      acc[7] = fmaf(xb.w, r[j], acc[7]);
    }
  }
#pragma unroll
  for (int i = 0; i < kRouterTok; ++i) red[(warp * kRouterTok + i) * 32 + lane] = acc[i];
  __syncthreads();
  if (threadIdx.x < kRouterTok * 32) {
    const int tt = threadIdx.x >> 5, l = threadIdx.x & 31;
    float v = 0.0f;
    for (int w = 0; w < kRouterWarps; ++w) v += red[(w * kRouterTok + tt) * 32 + l];
    const int t = t0 + tt, ee = e0 + l;
    if (t < T && ee < E) part[((int64_t)blockIdx.z * T + t) * E + ee] = v;
  }
}

__device__ __forceinline__ uint32_t tf32_rna(float f) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(f));
  return r;
}

__device__ __forceinline__ void mma_tf32_1688(float c[4], const uint32_t a[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// CTA: 64 tokens x 64 experts x one H slice (blockIdx.z), 4 warps of 16
// tokens x 64 experts, the slice in chunks of 32.  Each chunk is fetched with
// 16-byte loads into registers one chunk ahead (2 x loads + 4 router loads
// per thread in flight while the previous chunk is multiplied), then stored to
// shared memory: x as TF32 [token][h] (row stride 36 words), the router as
// TF32 hi and lo parts [h][expert] (row stride 72 words), strides at which the
// fragment reads are bank-conflict free.  The tensor cores' fp32 accumulation
// is not IEEE round-to-nearest, so each chunk's 8 MMAs accumulate into a fresh
// partial that is then added to the running sum with an ordinary fp32 add
// (chains of 8 MMAs instead of 2 H / 8), which keeps the logits within ~1e-6
// of an fp32 dot product.  Requires E % 4 == 0, H % (32 * slices) == 0 and
// 16-byte aligned x and router.
constexpr int kRtcTok = 64, kRtcExp = 64, kRtcK = 32, kRtcXLd = 36, kRtcRLd = 72;

__global__ void __launch_bounds__(128) router_logits_tc_kernel(const uint16_t *__restrict__ x,
                                                               const float *__restrict__ router,
                                                               float *__restrict__ part, int T,
                                                               int H, int E, int hslice) {
  __shared__ __align__(16) uint32_t xs[kRtcTok][kRtcXLd];  // tf32 x
  __shared__ __align__(16) uint32_t rh[kRtcK][kRtcRLd];    // tf32 hi of router
  __shared__ __align__(16) uint32_t rl[kRtcK][kRtcRLd];    // tf32 lo of router
  const int t0 = blockIdx.y * kRtcTok, e0 = blockIdx.x * kRtcExp;
  const int hbeg = blockIdx.z * hslice, hend = hbeg + hslice;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;

  // Fetch assignment: x chunk = 64 tokens x 32 h bf16 = 256 uint4 (2 per
  // thread); router chunk = 32 h x 64 experts fp32 = 512 float4 (4 per thread).
  int xt[2], xk[2], rk[4], re[4];
  bool xv[2], rv[4];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int i = tid + 128 * u;
    xt[u] = i >> 2;
    xk[u] = (i & 3) * 8;
    xv[u] = t0 + xt[u] < T;
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = tid + 128 * u;
    rk[u] = i >> 4;
    re[u] = (i & 15) * 4;
    rv[u] = e0 + re[u] < E;
  }
  uint4 xr[2];
  float4 rr[4];
  auto fetch = [&](int h0) {
#pragma unroll
    for (int u = 0; u < 2; ++u)
      xr[u] = xv[u] ? __ldcg(reinterpret_cast<const uint4 *>(x + (int64_t)(t0 + xt[u]) * H + h0 +
                                                             xk[u]))
                    : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      rr[u] = rv[u] ? __ldg(reinterpret_cast<const float4 *>(router + (int64_t)(h0 + rk[u]) * E +
                                                             e0 + re[u]))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
  };

  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.0f;
  pdl_wait();  // x may come from the previous kernel
  pdl_trigger();
  fetch(hbeg);
  for (int h0 = hbeg; h0 < hend; h0 += kRtcK) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t w[4] = {xr[u].x, xr[u].y, xr[u].z, xr[u].w};
      uint4 q0, q1;  // h = xk..xk+3 and xk+4..xk+7
      q0.x = w[0] << 16;
      q0.y = w[0] & 0xFFFF0000u;
      q0.z = w[1] << 16;
      q0.w = w[1] & 0xFFFF0000u;
      q1.x = w[2] << 16;
      q1.y = w[2] & 0xFFFF0000u;
      q1.z = w[3] << 16;
      q1.w = w[3] & 0xFFFF0000u;
      *reinterpret_cast<uint4 *>(&xs[xt[u]][xk[u]]) = q0;
      *reinterpret_cast<uint4 *>(&xs[xt[u]][xk[u] + 4]) = q1;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float v[4] = {rr[u].x, rr[u].y, rr[u].z, rr[u].w};
      uint32_t hv[4], lv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        hv[q] = tf32_rna(v[q]);
        lv[q] = tf32_rna(v[q] - __uint_as_float(hv[q]));
      }
      *reinterpret_cast<uint4 *>(&rh[rk[u]][re[u]]) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      *reinterpret_cast<uint4 *>(&rl[rk[u]][re[u]]) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
    __syncthreads();
    if (h0 + kRtcK < hend) fetch(h0 + kRtcK);
    float pa[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) pa[j][i] = 0.0f;
#pragma unroll
    for (int k8 = 0; k8 < kRtcK; k8 += 8) {
      const int tr = 16 * warp + g;
      const uint32_t a[4] = {xs[tr][k8 + c], xs[tr + 8][k8 + c], xs[tr][k8 + c + 4],
                             xs[tr + 8][k8 + c + 4]};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int en = 8 * j + g;
        mma_tf32_1688(pa[j], a, rl[k8 + c][en], rl[k8 + c + 4][en]);
        mma_tf32_1688(pa[j], a, rh[k8 + c][en], rh[k8 + c + 4][en]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[j][i] += pa[j][i];
    __syncthreads();
  }
  float *out = part + (int64_t)blockIdx.z * T * E;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = e0 + 8 * j + 2 * c;
    const int t = t0 + 16 * warp + g;
    if (e < E) {  // E % 4 == 0: e + 1 < E as well
      if (t < T)
        *reinterpret_cast<float2 *>(out + (int64_t)t * E + e) = make_float2(acc[j][0], acc[j][1]);
      if (t + 8 < T)
        *reinterpret_cast<float2 *>(out + (int64_t)(t + 8) * E + e) =
            make_float2(acc[j][2], acc[j][3]);
    }
  }
}

// One warp per token: the slices' partial logits added in z order, then the
// softmax top-k (router_topk.cuh).
__global__ void router_topk_kernel(const float *__restrict__ part, int nslices,
                                   float *__restrict__ logits_out, int T, int E, int k,
                                   int renormalize, int32_t *__restrict__ topk_ids,
                                   float *__restrict__ topk_w) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  if (warp >= T) return;
  float p[8];
  router_sum_slices(part, nslices, T, warp, E, lane, p, logits_out);
  int id_sel;
  float w_sel;
  router_softmax_topk(p, lane, E, k, renormalize, id_sel, w_sel);
  if (lane < k) {
    topk_ids[(int64_t)warp * k + lane] = id_sel;
    topk_w[(int64_t)warp * k + lane] = w_sel;
  }
}

static bool router_tc_ok(int T, int H, int E) {
  return T >= kRouterTcMinTokens && E % 4 == 0 && H % kRtcK == 0;
}

// H slices of the router for T tokens: enough CTAs to cover the GPU.  The
// logits workspace holds this many [T, E] partial sums.
int router_slices(int T, int H, int E) {
  int ctas, unit;
  if (router_tc_ok(T, H, E)) {
    ctas = ((E + kRtcExp - 1) / kRtcExp) * ((T + kRtcTok - 1) / kRtcTok);
    unit = kRtcK;
  } else {
    ctas = ((E + 31) / 32) * ((T + kRouterTok - 1) / kRouterTok);
    unit = kRouterWarps;
  }
  int hs = 1;
  while (hs < 16 && ctas * hs < 148 && H % (2 * hs * unit) == 0 && H / (2 * hs) >= 128) hs *= 2;
  return hs;
}

cudaError_t launch_router_logits(const uint16_t *x, const float *router, float *part,
                                 int nslices, int T, int H, int E, cudaStream_t st, int *used) {
  if (nslices < 1) nslices = 1;
  *used = nslices;
  if (T == 0) return cudaSuccess;
  const bool aligned16 = (((uintptr_t)x | (uintptr_t)router) & 15) == 0;
  if (router_tc_ok(T, H, E) && aligned16 && H % (nslices * kRtcK) == 0) {
    dim3 grid((E + kRtcExp - 1) / kRtcExp, (T + kRtcTok - 1) / kRtcTok, nslices);
    return launch_pdl(router_logits_tc_kernel, grid, dim3(128), 0, st, x, router, part, T, H, E,
                      H / nslices);
  }
  while (nslices > 1 && H % (nslices * kRouterWarps) != 0) nslices >>= 1;
  *used = nslices;
  const int hslice = H / nslices;
  const size_t smem = sizeof(float) * ((size_t)hslice * kRouterTok + kRouterWarps * kRouterTok * 32);
  static size_t configured = 48 * 1024;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(router_logits_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  dim3 grid((E + 31) / 32, (T + kRouterTok - 1) / kRouterTok, nslices);
  return launch_pdl(router_logits_kernel, grid, dim3(32 * kRouterWarps), smem, st, x, router,
                    part, T, H, E, hslice);
}

cudaError_t launch_router(const uint16_t *x, const float *router, float *part, int nslices,
                          float *logits_out, int T, int H, int E, int k, int renormalize,
                          int32_t *ids, float *w, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  int used = 0;
  cudaError_t e = launch_router_logits(x, router, part, nslices, T, H, E, st, &used);
  if (e != cudaSuccess) return e;
  return launch_pdl(router_topk_kernel, dim3((T * 32 + 255) / 256), dim3(256), 0, st, part, used,
                    logits_out, T, E, k, renormalize, ids, w);
}

// ---------------------------------------------------------------------------
// Permutation: rows (one expert each) sorted by expert into contiguous
// groups; work items of at most `tpi` rows for the grouped GEMMs.  A single
// CTA of 1024 threads (R is at most a few tens of thousands of rows).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) moe_permute_kernel(const int32_t *__restrict__ row_expert,
                                                          const int32_t *__restrict__ x_row_index,
                                                          int row_div, int R, int E, int tpi,
                                                          MoePlan plan) {
  __shared__ int cnt[1024], off[1025], cur[1024], items[1025];
  const int tid = threadIdx.x;
  pdl_wait();  // the routing ids come from the previous kernels
  pdl_trigger();
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  // The first 4 x 1024 routing ids stay in registers for the scatter below.
  int my_e[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tid + i * 1024;
    my_e[i] = r < R ? __ldcg(row_expert + r) : -1;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (my_e[i] >= 0 && my_e[i] < E) atomicAdd(&cnt[my_e[i]], 1);
  for (int r = tid + 4 * 1024; r < R; r += blockDim.x) {
    const int e = __ldcg(row_expert + r);
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // Exclusive scans of the counts and of the items per expert (E <= 256):
  // one warp, 8 experts per lane.
  if (tid < 32) {
    int c[8], n[8], sc = 0, sn = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = tid * 8 + j;
      c[j] = e < E ? cnt[e] : 0;
      n[j] = (c[j] + tpi - 1) / tpi;
      sc += c[j];
      sn += n[j];
    }
    int ic = sc, in = sn;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int uc = __shfl_up_sync(0xffffffffu, ic, o), un = __shfl_up_sync(0xffffffffu, in, o);
      if (tid >= o) {
        ic += uc;
        in += un;
      }
    }
    int ac = ic - sc, an = in - sn;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = tid * 8 + j;
      if (e < E) {
        off[e] = ac;
        items[e] = an;
      }
      ac += c[j];
      an += n[j];
    }
    if (tid == 31) {
      off[E] = ic;
      items[E] = in;
      *plan.n_work = in;
      *plan.n_rows = ic;
    }
  }
  __syncthreads();
  for (int e = tid; e <= E; e += blockDim.x) plan.offsets[e] = off[e];
  for (int e = tid; e < E; e += blockDim.x) {
    cur[e] = off[e];
    int i0 = items[e];
    for (int s = 0; s < cnt[e]; s += tpi, ++i0) {
      SkinnyWork w;
      w.group = e;
      w.slot0 = off[e] + s;
      w.count = min(tpi, cnt[e] - s);
      plan.work[i0] = w;
    }
  }
  __syncthreads();
  for (int r = tid; r < R; r += blockDim.x) {
    const int i = (r - tid) / 1024;
    const int e = i < 4 ? my_e[i] : __ldcg(row_expert + r);
    if (e >= 0 && e < E) {
      const int p = atomicAdd(&cur[e], 1);
      plan.src_row[p] = x_row_index ? __ldcg(x_row_index + r) : r / row_div;
      plan.dst_row[p] = r;
    }
  }
  // Positions past the valid rows (ids outside [0, E)) stay in bounds for a
  // whole-array gather and belong to no work item.
  for (int p = off[E] + tid; p < R; p += blockDim.x) {
    plan.src_row[p] = 0;
    plan.dst_row[p] = -1;
  }
}

cudaError_t launch_moe_permute(const int32_t *row_expert, const int32_t *x_row_index,
                               int row_div, int R, int E, int tpi, const MoePlan &plan,
                               cudaStream_t st) {
  if (E <= 0 || E > 256) return cudaErrorInvalidValue;  // the one-warp scan covers 256 experts
  if (row_div < 1) return cudaErrorInvalidValue;
  return launch_pdl(moe_permute_kernel, dim3(1), dim3(1024), 0, st, row_expert, x_row_index,
                    row_div, R, E, tpi, plan);
}

// Slot -> token index for the single-GPU forward: row r = t * k + j reads x[t].
// ---------------------------------------------------------------------------
// Expert-parallel dispatch plan.  Slot r (= token r / k, choice r % k) goes to
// rank dst = id / experts_per_rank as local expert id % experts_per_rank.
// Output: per-rank counts, the send order (slots grouped by destination rank,
// in slot order within a rank: a stable counting sort) as token index and
// local expert id per send position, and slot_pos[r] = send position of slot r
// (so the returned expert outputs can be combined in slot order).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t *__restrict__ ids, int R,
                                                      int k, int epr, int world,
                                                      int32_t *__restrict__ counts,
                                                      int32_t *__restrict__ send_token,
                                                      int32_t *__restrict__ send_expert,
                                                      int32_t *__restrict__ slot_pos) {
  __shared__ int cnt[64], off[64];
  __shared__ int chunk_cnt[32][64];  // per-warp counts of the current chunk
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 64) cnt[tid] = 0;
  __syncthreads();
  for (int r = tid; r < R; r += blockDim.x) {
    const int d = ids[r] / epr;
    if (d >= 0 && d < world) atomicAdd(&cnt[d], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int d = 0; d < world; ++d) {
      off[d] = acc;
      counts[d] = cnt[d];
      acc += cnt[d];
    }
  }
  __syncthreads();
  // Stable placement, one 1024-slot chunk at a time: rank of the slot among
  // same-destination slots = (earlier warps' counts) + (earlier lanes' count).
  for (int base = 0; base < R; base += blockDim.x) {
    const int r = base + tid;
    const int id = r < R ? ids[r] : -1;
    const int d = (id >= 0) ? id / epr : -1;
    const bool ok = d >= 0 && d < world;
    int mine = 0, before = 0;
    for (int dd = 0; dd < world; ++dd) {
      const unsigned m = __ballot_sync(0xffffffffu, ok && d == dd);
      if (lane == 0) chunk_cnt[warp][dd] = __popc(m);
      if (ok && d == dd) before = __popc(m & ((1u << lane) - 1u));
    }
    __syncthreads();
    if (ok) {
      mine = 0;
      for (int w = 0; w < warp; ++w) mine += chunk_cnt[w][d];
      const int p = off[d] + mine + before;
      send_token[p] = r / k;
      send_expert[p] = id % epr;
      slot_pos[r] = p;
    } else if (r < R) {
      slot_pos[r] = -1;  // expert id outside [0, world * epr): not dispatched
    }
    __syncthreads();
    if (tid < world) {
      int tot = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += chunk_cnt[w][tid];
      off[tid] += tot;
    }
    __syncthreads();
  }
}

cudaError_t launch_ep_plan(const int32_t *ids, int R, int k, int epr, int world, int32_t *counts,
                           int32_t *send_token, int32_t *send_expert, int32_t *slot_pos,
                           cudaStream_t st) {
  ep_plan_kernel<<<1, 1024, 0, st>>>(ids, R, k, epr, world, counts, send_token, send_expert,
                                     slot_pos);
  return cudaGetLastError();
}

// dst[i, :] = src[idx[i], :] for rows of `bytes` bytes (16-byte vectors).
__global__ void gather_rows_kernel(const uint4 *__restrict__ src, const int32_t *__restrict__ idx,
                                   int64_t n, int vec, uint4 *__restrict__ dst) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n * vec) return;
  const int64_t row = i / vec, v = i % vec;
  dst[i] = src[(int64_t)idx[row] * vec + v];
}

cudaError_t launch_gather_rows(const void *src, const int32_t *idx, int64_t n, int64_t row_bytes,
                               void *dst, cudaStream_t st) {
  const int vec = (int)(row_bytes / 16);
  const int64_t total = n * vec;
  if (total == 0) return cudaSuccess;
  gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
      static_cast<const uint4 *>(src), idx, n, vec, static_cast<uint4 *>(dst));
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Fixed-capacity dispatch: the plan's send order re-laid into `world` blocks
// of `cap` rows (block r = the rows for rank r, padded with zero rows and
// expert id -1), so that the exchange has the same sizes on every layer and
// needs no host-side count (the step can be captured in a CUDA graph).
// One warp per padded row; slot_pad[s] = padded position of slot s (or -1).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ep_offset(const int32_t *counts, int r) {
  int o = 0;
  for (int q = 0; q < r; ++q) o += counts[q];
  return o;
}

__global__ void ep_pad_rows_kernel(const int32_t *__restrict__ counts,
                                   const int32_t *__restrict__ send_token,
                                   const int32_t *__restrict__ send_expert, int world, int cap,
                                   const uint4 *__restrict__ x, int vec, uint4 *__restrict__ out,
                                   int32_t *__restrict__ out_expert) {
  const int q = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= world * cap) return;
  const int r = q / cap, p = q - r * cap;
  const int n = min(counts[r], cap);
  uint4 *dst = out + (int64_t)q * vec;
  if (p < n) {
    const int i = ep_offset(counts, r) + p;
    const uint4 *src = x + (int64_t)send_token[i] * vec;
    for (int v = lane; v < vec; v += 32) dst[v] = src[v];
    if (lane == 0) out_expert[q] = send_expert[i];
  } else {
    for (int v = lane; v < vec; v += 32) dst[v] = make_uint4(0u, 0u, 0u, 0u);
    if (lane == 0) out_expert[q] = -1;
  }
}

__global__ void ep_slot_pad_kernel(const int32_t *__restrict__ counts,
                                   const int32_t *__restrict__ slot_pos, int R, int world, int cap,
                                   int32_t *__restrict__ slot_pad) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= R) return;
  const int i = slot_pos[s];
  int pad = -1;
  if (i >= 0) {
    int o = 0;
    for (int r = 0; r < world; ++r) {
      const int c = counts[r];
      if (i < o + c) {
        if (i - o < cap) pad = r * cap + (i - o);
        break;
      }
      o += c;
    }
  }
  slot_pad[s] = pad;
}

cudaError_t launch_ep_pad(const int32_t *counts, const int32_t *send_token,
                          const int32_t *send_expert, const int32_t *slot_pos, int R, int world,
                          int cap, const void *x, int64_t row_bytes, void *out, int32_t *out_expert,
                          int32_t *slot_pad, cudaStream_t st) {
  const int vec = (int)(row_bytes / 16);
  const int64_t rows = (int64_t)world * cap;
  if (rows > 0) {
    ep_pad_rows_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(
        counts, send_token, send_expert, world, cap, static_cast<const uint4 *>(x), vec,
        static_cast<uint4 *>(out), out_expert);
  }
  if (R > 0)
    ep_slot_pad_kernel<<<(R + 255) / 256, 256, 0, st>>>(counts, slot_pos, R, world, cap, slot_pad);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Combine: y[t, :] = sum_j w[t, j] * ys[t*k + j, :] (+ residual[t, :]), fp32
// sums in j order, residual added last, one bf16 rounding at the end.  Slot
// outputs are fp32 (or bf16).  8 features per thread.
// ---------------------------------------------------------------------------
// L2-coherent loads: the data comes from the kernels before (programmatic
// dependent launch).
template <typename SlotT>
__device__ __forceinline__ void load8(const SlotT *p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float *p, float (&v)[8]) {
  const float4 a = __ldcg(reinterpret_cast<const float4 *>(p));
  const float4 b = __ldcg(reinterpret_cast<const float4 *>(p + 4));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<uint16_t>(const uint16_t *p, float (&v)[8]) {
  const uint4 r = __ldcg(reinterpret_cast<const uint4 *>(p));
  const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[2 * q] = bf16lo(rr[q]);
    v[2 * q + 1] = bf16hi(rr[q]);
  }
}

template <typename SlotT, typename OutT>
__global__ void moe_combine_kernel(const SlotT *__restrict__ ys, const float *__restrict__ w,
                                   const uint16_t *__restrict__ residual,
                                   const int32_t *__restrict__ slot_pos,
                                   const float *__restrict__ extra, OutT *__restrict__ y,
                                   int T, int k, int H) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // vector index
  const int hv = H / 8;
  pdl_wait();
  pdl_trigger();
  if (i >= (int64_t)T * hv) return;
  const int t = (int)(i / hv), h8 = (int)(i % hv);
  float s[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) s[q] = 0.0f;
  // Slots in groups of 8: the group's loads first, then the sums in slot order.
  for (int j0 = 0; j0 < k; j0 += 8) {
    float wv[8], v[8][8];
    int64_t rows[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int j = j0 + jj;
      rows[jj] = -1;
      if (j < k) {
        wv[jj] = __ldcg(w + (int64_t)t * k + j);
        rows[jj] = slot_pos ? __ldcg(slot_pos + (int64_t)t * k + j) : (int64_t)t * k + j;
      }
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
      if (rows[jj] >= 0) load8<SlotT>(ys + rows[jj] * H + 8 * h8, v[jj]);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      if (rows[jj] < 0) continue;  // slot that was not dispatched contributes nothing
#pragma unroll
      for (int q = 0; q < 8; ++q) s[q] = fmaf(wv[jj], v[jj][q], s[q]);
    }
  }
  if (extra) {  // fp32 rows added after the routed sum (the shared expert)
    float e[8];
    load8<float>(extra + (int64_t)t * H + 8 * h8, e);
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] += e[q];
  }
  if (residual) {
    float r[8];
    load8<uint16_t>(residual + (int64_t)t * H + 8 * h8, r);
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] += r[q];
  }
  if constexpr (sizeof(OutT) == 4) {
    float *yo = reinterpret_cast<float *>(y) + (int64_t)t * H + 8 * h8;
    *reinterpret_cast<float4 *>(yo) = make_float4(s[0], s[1], s[2], s[3]);
    *reinterpret_cast<float4 *>(yo + 4) = make_float4(s[4], s[5], s[6], s[7]);
  } else {
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = pack_bf16x2(s[2 * q], s[2 * q + 1]);
    *reinterpret_cast<uint4 *>(y + (int64_t)t * H + 8 * h8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t launch_moe_combine(const void *ys, int ys_dtype, const float *w,
                               const uint16_t *residual, const int32_t *slot_pos,
                               const float *extra, void *y, int y_dtype, int T, int k, int H,
                               cudaStream_t st) {
  const int64_t n = (int64_t)T * (H / 8);
  if (n == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  const float *yf = static_cast<const float *>(ys);
  const uint16_t *yb = static_cast<const uint16_t *>(ys);
  if (ys_dtype == kF32 && y_dtype == kF32)
    return launch_pdl(moe_combine_kernel<float, float>, dim3(blocks), dim3(256), 0, st, yf, w,
                      residual, slot_pos, extra, static_cast<float *>(y), T, k, H);
  else if (ys_dtype == kF32)
    return launch_pdl(moe_combine_kernel<float, uint16_t>, dim3(blocks), dim3(256), 0, st, yf, w,
                      residual, slot_pos, extra, static_cast<uint16_t *>(y), T, k, H);
  else if (y_dtype == kF32)
    return launch_pdl(moe_combine_kernel<uint16_t, float>, dim3(blocks), dim3(256), 0, st, yb, w,
                      residual, slot_pos, extra, static_cast<float *>(y), T, k, H);
  else
    return launch_pdl(moe_combine_kernel<uint16_t, uint16_t>, dim3(blocks), dim3(256), 0, st, yb,
                      w, residual, slot_pos, extra, static_cast<uint16_t *>(y), T, k, H);
}

}  // namespace nvfp4

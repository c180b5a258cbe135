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

namespace nvfp4 {

// ---------------------------------------------------------------------------
// Router: logits[t, e] = sum_h x[t, h] * router[h, e] (fp32), then per token
// softmax, top-k and renormalisation.  A CTA owns 16 tokens and all experts
// (E <= 256); router rows are staged through shared memory in chunks of 32.
// ---------------------------------------------------------------------------
constexpr int kRouterTok = 16;
constexpr int kRouterChunk = 32;

__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t *__restrict__ x,
                                                            const float *__restrict__ router,
                                                            float *__restrict__ logits, int T,
                                                            int H, int E) {
  __shared__ float rs[kRouterChunk][256];
  __shared__ float xs[kRouterTok][kRouterChunk];
  const int t0 = blockIdx.x * kRouterTok;
  const int tid = threadIdx.x;
  // Thread computes experts e = tid % 64 + 64 * c (c < 4) for tokens
  // tid / 64 + 4 * i (i < 4).
  const int e_lane = tid & 63, t_lane = tid >> 6;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[i][c] = 0.0f;
  for (int h0 = 0; h0 < H; h0 += kRouterChunk) {
    for (int idx = tid; idx < kRouterChunk * E; idx += 256) {
      const int hh = idx / E, e = idx % E;
      rs[hh][e] = (h0 + hh < H) ? router[(int64_t)(h0 + hh) * E + e] : 0.0f;
    }
    for (int idx = tid; idx < kRouterTok * kRouterChunk; idx += 256) {
      const int tt = idx / kRouterChunk, hh = idx % kRouterChunk;
      const int t = t0 + tt;
      xs[tt][hh] = (t < T && h0 + hh < H)
                       ? __uint_as_float((uint32_t)x[(int64_t)t * H + h0 + hh] << 16)
                       : 0.0f;
    }
    __syncthreads();
#pragma unroll 4
    for (int hh = 0; hh < kRouterChunk; ++hh) {
      float r[4], xv[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = rs[hh][e_lane + 64 * c];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = xs[t_lane + 4 * i][hh];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][c] = fmaf(xv[i], r[c], acc[i][c]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + t_lane + 4 * i;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int e = e_lane + 64 * c;
      if (t < T && e < E) logits[(int64_t)t * E + e] = acc[i][c];
    }
  }
}

// One warp per token: softmax over E (E <= 256: 8 logits per lane), top-k by
// repeated warp arg-max (ties to the lower index), optional renormalisation.
__global__ void router_topk_kernel(const float *__restrict__ logits, int T, int E, int k,
                                   int renormalize, int32_t *__restrict__ topk_ids,
                                   float *__restrict__ topk_w) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float *lg = logits + (int64_t)warp * E;
  float p[8];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? lg[e] : -FLT_MAX;
    mx = fmaxf(mx, p[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? expf(p[i] - mx) : 0.0f;
    sum += p[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = p[i] / sum;

  float wsum = 0.0f, wsel = 0.0f;
  int id_sel = 0;
  for (int j = 0; j < k; ++j) {
    // Best of this lane (lowest expert index among equals), then across lanes.
    float bv = -1.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (p[i] > bv)) {
        bv = p[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + 32 * i == bi) p[i] = -2.0f;  // taken
    }
    wsum += bv;
    if (lane == j) {
      wsel = bv;
      id_sel = bi;
    }
  }
  if (lane < k) {
    topk_ids[(int64_t)warp * k + lane] = id_sel;
    topk_w[(int64_t)warp * k + lane] = renormalize ? wsel / wsum : wsel;
  }
}

cudaError_t launch_router(const uint16_t *x, const float *router, float *logits, int T, int H,
                          int E, int k, int renormalize, int32_t *ids, float *w,
                          cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  router_logits_kernel<<<(T + kRouterTok - 1) / kRouterTok, 256, 0, st>>>(x, router, logits, T,
                                                                          H, E);
  router_topk_kernel<<<(T * 32 + 255) / 256, 256, 0, st>>>(logits, T, E, k, renormalize, ids, w);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Permutation: rows (one expert each) sorted by expert into contiguous
// groups; work items of at most `tpi` rows for the grouped GEMMs.  A single
// CTA of 1024 threads (R is at most a few tens of thousands of rows).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) moe_permute_kernel(const int32_t *__restrict__ row_expert,
                                                          const int32_t *__restrict__ x_row_index,
                                                          int R, int E, int tpi, MoePlan plan) {
  __shared__ int cnt[1024], off[1025], cur[1024], items[1025];
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int r = tid; r < R; r += blockDim.x) {
    const int e = row_expert[r];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0, it = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = acc;
      items[e] = it;
      acc += cnt[e];
      it += (cnt[e] + tpi - 1) / tpi;
    }
    off[E] = acc;
    items[E] = it;
    *plan.n_work = it;
    *plan.n_rows = acc;
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
    const int e = row_expert[r];
    if (e >= 0 && e < E) {
      const int p = atomicAdd(&cur[e], 1);
      plan.src_row[p] = x_row_index ? x_row_index[r] : r;
      plan.dst_row[p] = r;
    }
  }
}

cudaError_t launch_moe_permute(const int32_t *row_expert, const int32_t *x_row_index, int R,
                               int E, int tpi, const MoePlan &plan, cudaStream_t st) {
  moe_permute_kernel<<<1, 1024, 0, st>>>(row_expert, x_row_index, R, E, tpi, plan);
  return cudaGetLastError();
}

// Slot -> token index for the single-GPU forward: row r = t * k + j reads x[t].
__global__ void slot_token_kernel(int32_t *__restrict__ idx, int R, int k) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < R) idx[r] = r / k;
}

cudaError_t launch_slot_token(int32_t *idx, int R, int k, cudaStream_t st) {
  if (R == 0) return cudaSuccess;
  slot_token_kernel<<<(R + 255) / 256, 256, 0, st>>>(idx, R, k);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Combine: y[t, :] = sum_j w[t, j] * ys[t*k + j, :] (+ residual[t, :]), fp32
// sums in j order, residual added last, one bf16 rounding at the end.  Slot
// outputs are fp32 (or bf16).  8 features per thread.
// ---------------------------------------------------------------------------
template <typename SlotT>
__device__ __forceinline__ void load8(const SlotT *p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float *p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4 *>(p);
  const float4 b = *reinterpret_cast<const float4 *>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<uint16_t>(const uint16_t *p, float (&v)[8]) {
  const uint4 r = *reinterpret_cast<const uint4 *>(p);
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
                                   OutT *__restrict__ y, int T, int k, int H) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // vector index
  const int hv = H / 8;
  if (i >= (int64_t)T * hv) return;
  const int t = (int)(i / hv), h8 = (int)(i % hv);
  float s[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) s[q] = 0.0f;
  for (int j = 0; j < k; ++j) {
    const float wj = w[(int64_t)t * k + j];
    float v[8];
    load8<SlotT>(ys + ((int64_t)t * k + j) * H + 8 * h8, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] = fmaf(wj, v[q], s[q]);
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
                               const uint16_t *residual, void *y, int y_dtype, int T, int k, int H,
                               cudaStream_t st) {
  const int64_t n = (int64_t)T * (H / 8);
  if (n == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  const float *yf = static_cast<const float *>(ys);
  const uint16_t *yb = static_cast<const uint16_t *>(ys);
  if (ys_dtype == kF32 && y_dtype == kF32)
    moe_combine_kernel<float, float><<<blocks, 256, 0, st>>>(yf, w, residual, static_cast<float *>(y), T, k, H);
  else if (ys_dtype == kF32)
    moe_combine_kernel<float, uint16_t><<<blocks, 256, 0, st>>>(yf, w, residual, static_cast<uint16_t *>(y), T, k, H);
  else if (y_dtype == kF32)
    moe_combine_kernel<uint16_t, float><<<blocks, 256, 0, st>>>(yb, w, residual, static_cast<float *>(y), T, k, H);
  else
    moe_combine_kernel<uint16_t, uint16_t><<<blocks, 256, 0, st>>>(yb, w, residual, static_cast<uint16_t *>(y), T, k, H);
  return cudaGetLastError();
}

}  // namespace nvfp4

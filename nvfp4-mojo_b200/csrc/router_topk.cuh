// router_topk.cuh -- the router's softmax top-k for one token per warp,
// shared by the single-GPU router (moe.cu) and the expert-parallel fused
// top-k + dispatch (ep_p2p.cu), so both produce the same ids and weights.
#pragma once

#include <cfloat>
#include <cstdint>

namespace nvfp4 {

#ifdef __CUDACC__
// Logits of token t for the lane's experts lane + 32 i (-FLT_MAX beyond E):
// the router's nslices partial sums part[z][T][E], added in slice order
// (each expert's sum starts at 0 and adds slices 0, 1, 2, ...).  Loads go
// out 4 slices x 8 experts at a time, so a token costs ceil(nslices / 4) L2
// round trips instead of one per expert.  Written to logits_out [T, E] when
// it is not null.
__device__ __forceinline__ void router_sum_slices(const float *__restrict__ part, int nslices,
                                                  int T, int t, int E, int lane, float (&p)[8],
                                                  float *__restrict__ logits_out) {
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  for (int z0 = 0; z0 < nslices; z0 += 4) {
    float q[4][8];
#pragma unroll
    for (int zz = 0; zz < 4; ++zz)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int z = z0 + zz, e = lane + 32 * i;
        q[zz][i] = (z < nslices && e < E) ? __ldcg(part + ((int64_t)z * T + t) * E + e) : 0.0f;
      }
#pragma unroll
    for (int zz = 0; zz < 4; ++zz)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (z0 + zz < nslices) v[i] += q[zz][i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    if (e < E && logits_out) logits_out[(int64_t)t * E + e] = v[i];
    p[i] = e < E ? v[i] : -FLT_MAX;
  }
}

// Softmax over E logits (lane holds experts lane + 32 i, -FLT_MAX beyond E)
// and top-k by repeated warp arg-max (ties to the lower index).  Lane j < k
// returns the j-th expert and its weight (renormalised over the k if asked).
// NaN probabilities rank below every number and are still selectable, so k
// valid ids are always produced.
__device__ __forceinline__ void router_softmax_topk(float (&p)[8], int lane, int E, int k,
                                                    int renormalize, int &id_sel, float &w_sel) {
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) mx = fmaxf(mx, p[i]);
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
  // Taken experts are marked -inf.
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (p[i] != p[i]) p[i] = -1.0e30f;
  float wsum = 0.0f, wsel = 0.0f;
  int isel = 0;
  for (int j = 0; j < k; ++j) {
    // Best of this lane (lowest expert index among equals), then across lanes.
    float bv = -INFINITY;
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
        if (lane + 32 * i == bi) p[i] = -INFINITY;  // taken
    }
    const float wv = bv < -1.0e29f ? __int_as_float(0x7fc00000) : bv;  // NaN stays NaN
    wsum += wv;
    if (lane == j) {
      wsel = wv;
      isel = bi;
    }
  }
  id_sel = isel;
  w_sel = renormalize ? wsel / wsum : wsel;
}
#endif

}  // namespace nvfp4

// moe.h -- device-side plan of the grouped expert GEMMs (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/nvfp4_ep.h"

#include "kernels.h"

namespace nvfp4 {

// Rows sorted by expert: sorted position p holds row dst_row[p], whose
// activations are row src_row[p] of the input; expert e owns positions
// [offsets[e], offsets[e+1]).  work[0..n_work) are the grouped-GEMM items.
struct MoePlan {
  int32_t *offsets;  // [E + 1]
  int32_t *n_work;   // [1]
  int32_t *n_rows;   // [1] rows with a valid expert id
  SkinnyWork *work;  // [capacity]
  int32_t *src_row;  // [R]
  int32_t *dst_row;  // [R]
};

// Grouped tensor-core expert GEMM (moe_tc.cu).
struct MoeTcLaunch {
  const uint8_t *w = nullptr;   // stacked expert codes [E * Nw, K/2]
  const uint8_t *sf = nullptr;  // [E * Nw, K/16]
  int E = 0, Nw = 0, K = 0;
  const uint16_t *b0 = nullptr;  // activations in sorted-row order [R, K] (bf16)
  const uint16_t *b1 = nullptr;  // low parts (down projection) or null
  int64_t R = 0;
  const SkinnyWork *work = nullptr;
  const int *n_work = nullptr;
  AlphaSpec al;                 // ws2_rows with stride Nw per expert
  uint16_t *inter = nullptr, *inter_lo = nullptr;  // gate_up outputs [R, Nw/2]
  void *y = nullptr;            // down output rows (scattered by dst_row)
  int y_dtype = kF32;
  const int32_t *dst_row = nullptr;
  int y_ld = 0;
};
cudaError_t launch_moe_tc(const MoeTcLaunch &L, bool gate_up, cudaStream_t st);
bool moe_tc_supported(int H, int I);
int moe_tc_rows_per_item();

// Router: partial logits in `part` ([nslices][T][E]; nslices from
// router_slices), summed in slice order by the top-k kernel, which also
// writes the logits to logits_out (nullable).
int router_slices(int T, int H, int E);
// The partial-logits kernel of launch_router alone (its top-k left to the
// caller); returns the slice count it used (<= nslices) in *used.
cudaError_t launch_router_logits(const uint16_t *x, const float *router, float *part,
                                 int nslices, int T, int H, int E, cudaStream_t st, int *used);
cudaError_t launch_router(const uint16_t *x, const float *router, float *part, int nslices,
                          float *logits_out, int T, int H, int E, int k, int renormalize,
                          int32_t *ids, float *w, cudaStream_t st);
// Slot r's activation row: x_row_index[r], or r / row_div when it is null
// (row_div = top_k: slot r of the layer is token r / k).
cudaError_t launch_moe_permute(const int32_t *row_expert, const int32_t *x_row_index, int row_div,
                               int R, int E,
                               int tpi, const MoePlan &plan, cudaStream_t st);
// extra (nullable): fp32 rows [T, H] added after the routed sum, before the
// residual (the shared expert's output).
cudaError_t launch_moe_combine(const void *ys, int ys_dtype, const float *w,
                               const uint16_t *residual, const int32_t *slot_pos,
                               const float *extra, void *y, int y_dtype, int T, int k, int H,
                               cudaStream_t st);
// Expert-parallel top-k + dispatch in one launch (ep_p2p.cu), after the
// router's partial logits (launch_router_logits): one block per token runs
// the token's softmax top-k (router_topk.cuh) and dispatches its slots into
// the peers' windows.  Writes ids / weights [T, k] for the combine.  With
// wait_all the launch also waits for every rank's dispatch (the step of
// nvfp4_ep_p2p_wait_dispatch); without copy_rows (world 1 only) it stores the
// slots' expert ids but not their rows, which the expert pass then reads from
// x (slot s is token s / k).
int ep_p2p_topk_dispatch(const nvfp4_ep_peers *p, const uint16_t *x, const float *part,
                         int nslices, int64_t T, int k, int renormalize, int epr, int32_t *ids,
                         float *w, bool wait_all, bool copy_rows, cudaStream_t st);
cudaError_t launch_ep_plan(const int32_t *ids, int R, int k, int epr, int world, int32_t *counts,
                           int32_t *send_token, int32_t *send_expert, int32_t *slot_pos,
                           cudaStream_t st);
cudaError_t launch_gather_rows(const void *src, const int32_t *idx, int64_t n, int64_t row_bytes,
                               void *dst, cudaStream_t st);
cudaError_t launch_ep_pad(const int32_t *counts, const int32_t *send_token,
                          const int32_t *send_expert, const int32_t *slot_pos, int R, int world,
                          int cap, const void *x, int64_t row_bytes, void *out, int32_t *out_expert,
                          int32_t *slot_pad, cudaStream_t st);

}  // namespace nvfp4

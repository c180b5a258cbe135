/*
 * nvfp4_ep.h -- device-initiated expert-parallel exchange of libnvfp4.so:
 * the MoE layer's dispatch and combine move token rows through peer memory
 * (NVLink / NVSwitch loads and stores issued by the kernels themselves)
 * instead of host-driven NCCL all-to-alls.
 *
 * Replaces, for small batches, the exchange steps of the expert-parallel
 * layer (counts all-to-all, row all-to-all, reverse all-to-all); the routing,
 * expert and combine arithmetic is that of nvfp4_moe_forward
 * (include/nvfp4.h), so a rank's output equals the single-GPU layer's bit
 * for bit.  The reference has no multi-GPU MoE; its one-process entry points
 * are nvfp4_linear_forward (nvfp4/nvfp4_gemm_gpu.mojo:185-224) and the
 * per-expert linears of Qwen35LayerWeights (nvfp4/weight_loader.mojo:
 * 776-825), which this layer runs expert-parallel.
 *
 * Windows.  Every rank owns one window of device memory (created here,
 * cudaMalloc'd and zeroed) and maps the other ranks' windows through CUDA
 * IPC handles exchanged by the host (any transport: torch.distributed, a
 * file).  A window holds control words (one dispatch and one done flag per
 * source rank, an epoch, an error word, the row count of each source rank's
 * last dispatch), then room for world * max_rows received rows and expert ids
 * and as many fp32 expert-output rows.  In a step of T tokens the rows of
 * source rank p sit at p*T*k .. (p+1)*T*k - 1, so every rank must step with
 * the same T: the wait (step 3) checks it and sets NVFP4_EP_ERR_SHAPE when a
 * peer's row count differs (that step's results are then meaningless).
 *
 * One layer step on rank r (all ranks run the same steps with the same T):
 *   1. route its T tokens (softmax top-k over all E experts);
 *   2. dispatch: slot s = t*k + j with expert e goes to rank e / (E/world):
 *      the kernel stores x[t] and e % (E/world) at row r*T*k + s of that
 *      rank's window (expert id -1 in every other window), then, when all
 *      its blocks are done, raises its dispatch flag in every window;
 *   3. wait until every rank's dispatch flag for this step is up;
 *   4. run the local experts on the world*T*k received rows into this
 *      window's fp32 output rows (rows with id -1 are skipped);
 *   5. raise this rank's done flag in every window;
 *   6. combine: wait for every done flag, then
 *      y[t] = sum_j w[t,j] * out_{e_j / (E/world)}[r*T*k + t*k + j] (+ residual)
 *      with fp32 sums in j order, loading the rows from the peers' windows.
 *      Each block of the combine waits on its own: when the error word has
 *      NVFP4_EP_ERR_DONE_TIMEOUT, y is undefined (blocks that gave up leave
 *      their part untouched, blocks that saw a late flag write theirs).
 * Flags carry a step counter kept in each window, so nothing is reset
 * between steps and a step can be captured in a CUDA graph.
 *
 * Every wait is bounded (timeout_ms, 0 = 2000 ms): on expiry the kernel sets
 * a bit in its window's error word and returns without touching the data;
 * nvfp4_ep_p2p_error reads (and clears) it.  After an error the windows'
 * step counters disagree: recreate the windows.
 *
 * Conventions as in nvfp4.h: device pointers owned by the caller, 0 or a
 * negative nvfp4_status, work enqueued on `stream`.
 */
#ifndef NVFP4_EP_H
#define NVFP4_EP_H

#include <stddef.h>
#include <stdint.h>

#include "nvfp4.h"

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4_EP_MAX_WORLD 8
#define NVFP4_EP_HANDLE_BYTES 64

/* Error word bits (nvfp4_ep_p2p_error). */
#define NVFP4_EP_ERR_DISPATCH_TIMEOUT 0x1u /* a dispatch flag did not arrive */
#define NVFP4_EP_ERR_DONE_TIMEOUT 0x2u     /* a done flag did not arrive */
#define NVFP4_EP_ERR_SHAPE 0x4u            /* a peer dispatched a different T * k */
/* bit 8 + p set: rank p's flag was missing, or its row count differed
 * (bits 8..15, one per rank) */

typedef struct nvfp4_ep_peers {
  int32_t rank;
  int32_t world;      /* 1 .. NVFP4_EP_MAX_WORLD */
  int64_t max_rows;   /* rows per source rank the windows hold: the largest T * k */
  int32_t hidden;     /* H, a multiple of 128 */
  int32_t timeout_ms; /* bound of every wait; 0 = 2000 */
  void *windows[NVFP4_EP_MAX_WORLD]; /* rank p's window as mapped in this process */
} nvfp4_ep_peers;

/* Bytes of one window for `world` ranks, max_rows rows per rank, hidden H. */
size_t nvfp4_ep_window_size(int32_t world, int64_t max_rows, int32_t hidden);

/* Allocates and zeroes a window on the current device and returns its IPC
 * handle (NVFP4_EP_HANDLE_BYTES bytes) for the other ranks. */
int nvfp4_ep_window_create(size_t bytes, void **window, uint8_t *handle);
/* Maps another rank's window (a handle from nvfp4_ep_window_create in
 * another process) into this process. */
int nvfp4_ep_window_open(const uint8_t *handle, void **window);
/* Unmaps a window opened with nvfp4_ep_window_open. */
int nvfp4_ep_window_close(void *window);
/* Frees a window made by nvfp4_ep_window_create (synchronises the device). */
int nvfp4_ep_window_destroy(void *window);

/* This rank's received rows for a step of T tokens: bf16 rows [world*T*k, H],
 * local expert ids [world*T*k] and fp32 output rows [world*T*k, H], the
 * arguments of nvfp4_moe_experts in step 4. */
int nvfp4_ep_p2p_rows(const nvfp4_ep_peers *peers, int64_t T, int32_t k, void **recv_x,
                      int32_t **recv_expert, float **out_rows);

/* Step 2: topk_ids [T, k] (global expert ids), x bf16 [T, H]. */
int nvfp4_ep_p2p_dispatch(const nvfp4_ep_peers *peers, const int32_t *topk_ids, const void *x,
                          int64_t T, int32_t k, int32_t experts_per_rank, void *stream);
/* Step 3. */
int nvfp4_ep_p2p_wait_dispatch(const nvfp4_ep_peers *peers, void *stream);
/* Step 5. */
int nvfp4_ep_p2p_signal_done(const nvfp4_ep_peers *peers, void *stream);
/* Step 6: topk_w [T, k] fp32, residual bf16 [T, H] or NULL, y [T, H]
 * (y_dtype fp32 or bf16). */
int nvfp4_ep_p2p_combine(const nvfp4_ep_peers *peers, const int32_t *topk_ids,
                         const float *topk_w, int64_t T, int32_t k, int32_t experts_per_rank,
                         const void *residual, void *y, int y_dtype, void *stream);
/* Reads this rank's error word (synchronises `stream`); clears it when
 * `clear` is non-zero. */
int nvfp4_ep_p2p_error(const nvfp4_ep_peers *peers, uint32_t *error, int32_t clear,
                       void *stream);

/* The whole step (1-6) in one call: desc over all E experts (E divisible by
 * world), `local` = the router [H, E] and this rank's E/world experts
 * (nvfp4_moe_weights layout), x bf16 [T, H], residual bf16 or NULL, y [T, H]. */
size_t nvfp4_ep_p2p_workspace_size(const nvfp4_moe_desc *desc, const nvfp4_ep_peers *peers,
                                   int64_t T);
int nvfp4_ep_p2p_forward(const nvfp4_moe_desc *desc, const nvfp4_moe_weights *local,
                         const nvfp4_ep_peers *peers, const void *x, const void *residual,
                         void *y, int y_dtype, int64_t T, void *workspace,
                         size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_EP_H */

// ep_p2p.cu -- device-initiated expert-parallel exchange (include/nvfp4_ep.h):
// dispatch and combine kernels that store and load token rows directly in
// the other ranks' windows (peer memory over NVLink / NVSwitch), the
// cross-GPU flags that order the steps, and the windows' IPC plumbing.
//
// Memory ordering.  A rank writes into a peer's window only with plain
// stores ordered by a system-scope release (a fence, or a release
// read-modify-write that the publishing thread acquires), and publishes them
// with one st.release.sys of a flag in that window; the owner polls its own flags
// with ld.acquire.sys (local memory, bounded by time) and every later read
// of the published rows follows that acquire in the same stream.  With one
// rank every window is this GPU's own memory and the same releases and
// acquires are taken at GPU scope.  All waits
// are on this GPU's memory, all signals are remote stores, so no kernel ever
// waits on another kernel of its own GPU.  Every kernel here is launched with
// programmatic dependent launch and executes griddepcontrol.wait before it
// reads anything an earlier kernel of the stream wrote (ids, rows, the step
// counter), so it is resident when its predecessor ends instead of being
// launched then.
#include <string.h>

#include <algorithm>

#include "../../include/nvfp4.h"
#include "../../include/nvfp4_ep.h"
#include "abi_util.h"
#include "moe.h"
#include "nvfp4_common.cuh"
#include "router_topk.cuh"

namespace nvfp4 {
namespace {

constexpr int kMaxWorld = NVFP4_EP_MAX_WORLD;
constexpr size_t kWinAlign = 256;
constexpr uint64_t kDefaultTimeoutNs = 2000ull * 1000 * 1000;

size_t wup(size_t v) { return (v + kWinAlign - 1) & ~(kWinAlign - 1); }

// Control words at offset 0 of every window.
struct EpCtrl {
  uint32_t flag_dispatch[kMaxWorld];  // [source rank]: last step whose rows it stored here
  uint32_t flag_done[kMaxWorld];      // [source rank]: last step whose expert rows it finished
  uint32_t epoch;                     // steps this rank has entered (advanced by the wait)
  uint32_t error;                     // NVFP4_EP_ERR_* | missing-rank mask << 8
  uint32_t blocks_done;               // dispatch: blocks finished (last block resets it)
  uint32_t rows_from[kMaxWorld];      // [source rank]: T*k of its last dispatch here
};

struct WinLayout {
  size_t recv_expert, recv_x, out, total;
};

WinLayout win_layout(int world, int64_t max_rows, int H) {
  WinLayout L;
  size_t o = wup(sizeof(EpCtrl));
  const size_t rows = (size_t)world * (size_t)max_rows;
  L.recv_expert = o;
  o = wup(o + sizeof(int32_t) * rows);
  L.recv_x = o;
  o = wup(o + sizeof(uint16_t) * rows * H);
  L.out = o;
  o = wup(o + sizeof(float) * rows * H);
  L.total = o;
  return L;
}

// Kernel-side view of the peers: window bases and the offsets in them.
struct PeerTable {
  char *win[kMaxWorld];
  int rank, world, H;
  size_t off_expert, off_x, off_out;
  uint64_t timeout_ns;
};

// The control words are ordered at system scope when the windows span GPUs
// (`sys`: world > 1, peers over NVLink) and at GPU scope when every window is
// this GPU's own memory (world 1), where that order is all a reader needs.
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p, bool sys) {
  uint32_t v;
  if (sys)
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release(uint32_t *p, uint32_t v, bool sys) {
  if (sys)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
  else
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Eight fp32 from another rank's window: system-scope (volatile) loads, so
// no cache of this GPU can answer with a previous step's row.
__device__ __forceinline__ void ld_sys_f32x8(const float *p, float (&v)[8]) {
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
               : "l"(p));
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p + 4));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Polls `flag` until it reaches `step` (wrap-safe).  Bounded twice: by the
// global timer and, should that timer not advance, by an iteration count
// (each iteration sleeps >= 64 ns).  Returns false when it gave up.
__device__ bool wait_flag(const uint32_t *flag, uint32_t step, uint64_t timeout_ns, bool sys) {
  const uint64_t t0 = global_ns();
  const uint64_t max_iter = timeout_ns / 64 + 1024;
  for (uint64_t it = 0;; ++it) {
    if ((int32_t)(ld_acquire(flag, sys) - step) >= 0) return true;
    if (global_ns() - t0 > timeout_ns || it >= max_iter) return false;
    __nanosleep(64);
  }
}

__device__ __forceinline__ EpCtrl *ctrl_of(char *win) { return reinterpret_cast<EpCtrl *>(win); }

// P.win[r] for a run-time r, by selects (no local-memory copy of the table).
__device__ __forceinline__ char *win_at(const PeerTable &P, int r) {
  char *w = P.win[0];
#pragma unroll
  for (int q = 1; q < kMaxWorld; ++q)
    if (q == r) w = P.win[q];
  return w;
}

// One warp: slot s (expert e) of this rank.  The row of x[s / k] goes to row
// rank*R + s of the destination's window, the expert id to the same row of
// every window (-1 where the slot does not go).  Without `rows` only the ids
// are stored (one rank: the expert pass reads x[s / k] itself).
__device__ __forceinline__ void dispatch_slot(const PeerTable &P, char *const *s_win, int s, int e,
                                              int R, int k, int epr, const uint4 *__restrict__ x,
                                              int lane, bool rows) {
  const int E = epr * P.world, row_v = P.H / 8;  // uint4 per bf16 row
  const int d = (e >= 0 && e < E) ? e / epr : -1;
  const int64_t row = (int64_t)P.rank * R + s;
  if (lane < P.world)
    reinterpret_cast<int32_t *>(s_win[lane] + P.off_expert)[row] = lane == d ? e - d * epr : -1;
  if (d < 0 || !rows) return;
  const uint4 *src = x + (int64_t)(s / k) * row_v;
  uint4 *dst = reinterpret_cast<uint4 *>(s_win[d] + P.off_x) + row * row_v;
  // All of this lane's loads before any store: the store pointer may alias
  // the loads as far as the compiler can tell, which would otherwise
  // serialise one L2 round trip per 16 bytes.
  for (int i0 = 0; i0 < row_v; i0 += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + lane + 32 * j;
      v[j] = i < row_v ? __ldcg(src + i) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + lane + 32 * j;
      if (i < row_v) dst[i] = v[j];
    }
  }
}

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t *p, uint32_t v, bool sys) {
  uint32_t old;
  if (sys)
    asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], %2;"
                 : "=r"(old) : "l"(p), "r"(v) : "memory");
  else
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                 : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Step 3 in the lanes of one warp: lane p waits for rank p's dispatch flag
// and checks that rank p stored as many rows as this rank did (the fixed row
// layout needs the same T on every rank), then lane 0 advances the step
// counter (also after a timeout or a shape mismatch, which the error word
// records).
__device__ __forceinline__ void wait_dispatch_warp(const PeerTable &P, EpCtrl *own, uint32_t step,
                                                   int lane) {
  const bool sys = P.world > 1;
  if (lane < P.world) {
    if (!wait_flag(&own->flag_dispatch[lane], step, P.timeout_ns, sys))
      atomicOr(&own->error, NVFP4_EP_ERR_DISPATCH_TIMEOUT | (1u << (8 + lane)));
    else if (ld_acquire(&own->rows_from[lane], sys) != ld_acquire(&own->rows_from[P.rank], sys))
      atomicOr(&own->error, NVFP4_EP_ERR_SHAPE | (1u << (8 + lane)));
  }
  __syncwarp();
  if (lane == 0) own->epoch = step;
}

// Publication of a dispatch.  After the block barrier, thread 0 counts the
// block with a release (acq_rel, system scope) add on the rank's own block
// counter: the release is cumulative over the block's peer stores, which the
// barrier ordered before it (one such release per block; a system fence in
// each of the 256 threads cost ~6 us, a fence.sc.sys per block ~1.6 us more
// than this).  The block whose add completes the count acquires every other
// block's release through the counter, and its thread 0 then raises this
// rank's dispatch flag in every window with st.release.sys, after the row
// count R (so that every owner can check that all ranks step with the same
// T); each release is cumulative over all it acquired.
// With `wait_all`, the completing block's first warp then runs step 3
// (wait_dispatch_warp): the launch ends once every rank has dispatched, and
// the separate wait launch is not needed.  The other blocks are done by then,
// so the wait holds one block; it waits only on flags that other GPUs' kernels
// raise (or, for this rank's own flag, its thread 0 just did).
__device__ __forceinline__ void dispatch_publish(const PeerTable &P, char *const *s_win,
                                                 EpCtrl *own, uint32_t step, int R,
                                                 bool wait_all) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool sys = P.world > 1;
    const bool last = atom_add_acq_rel(&own->blocks_done, 1u, sys) == gridDim.x - 1;
    if (last) {
      own->blocks_done = 0;  // the next step's launch starts after this one
      for (int r = 0; r < P.world; ++r) ctrl_of(s_win[r])->rows_from[P.rank] = (uint32_t)R;
      for (int r = 0; r < P.world; ++r)
        st_release(&ctrl_of(s_win[r])->flag_dispatch[P.rank], step, sys);
    }
    s_last = last;
  }
  if (!wait_all) return;
  __syncthreads();
  if (s_last && threadIdx.x < 32) wait_dispatch_warp(P, own, step, threadIdx.x);
}

// Step 2: one warp per slot s = t*k + j of this rank (dispatch_slot); the
// last block to finish raises this rank's dispatch flag in every window
// (dispatch_publish).
__global__ void __launch_bounds__(256) ep_dispatch_kernel(PeerTable P, const int32_t *__restrict__ ids,
                                                          const uint4 *__restrict__ x, int T, int k,
                                                          int epr) {
  __shared__ char *s_win[kMaxWorld];
  pdl_wait();  // ids, x and the step counter come from earlier kernels
  pdl_trigger();
  if (threadIdx.x < kMaxWorld) s_win[threadIdx.x] = win_at(P, threadIdx.x < P.world ? threadIdx.x : 0);
  __syncthreads();
  EpCtrl *own = ctrl_of(s_win[P.rank]);
  const uint32_t step = __ldcg(&own->epoch) + 1;
  const int R = T * k;
  const int lane = threadIdx.x & 31;
  for (int s = blockIdx.x * 8 + (threadIdx.x >> 5); s < R; s += gridDim.x * 8)
    dispatch_slot(P, s_win, s, __ldcg(ids + s), R, k, epr, x, lane, true);
  dispatch_publish(P, s_win, own, step, R, false);
}

// Top-k + step 2 in one launch, one block per token t: warp 0 runs the
// token's softmax top-k from the router's partial logits (the arithmetic of
// the router's own top-k kernel, router_topk.cuh) into the ids / weights of
// the combine and the block's shared memory, then the block's warps dispatch
// its k slots (dispatch_slot) and the flag goes up as in ep_dispatch_kernel.
// With `wait_all` the completing block also runs step 3 (dispatch_publish);
// without `copy_rows` (one rank) the slots carry only their expert ids.
// Two kernel boundaries less than top-k, dispatch, wait.
__global__ void __launch_bounds__(256) ep_topk_dispatch_kernel(PeerTable P, const float *__restrict__ part,
                                                               int nslices,
                                                               const uint4 *__restrict__ x, int T,
                                                               int k, int renormalize, int epr,
                                                               int32_t *__restrict__ ids,
                                                               float *__restrict__ w,
                                                               int wait_all, int copy_rows) {
  __shared__ char *s_win[kMaxWorld];
  __shared__ int32_t s_ids[32];
  pdl_wait();  // the partial logits, x and the step counter come from earlier kernels
  pdl_trigger();
  if (threadIdx.x < kMaxWorld) s_win[threadIdx.x] = win_at(P, threadIdx.x < P.world ? threadIdx.x : 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x, E = epr * P.world;
  // The step counter's load goes out before the top-k (it is used after).
  const uint32_t step = __ldcg(&ctrl_of(win_at(P, P.rank))->epoch) + 1;
  if (warp == 0 && t < T) {
    float p[8];
    router_sum_slices(part, nslices, T, t, E, lane, p, nullptr);
    int id_sel;
    float w_sel;
    router_softmax_topk(p, lane, E, k, renormalize, id_sel, w_sel);
    if (lane < k) {
      ids[(int64_t)t * k + lane] = id_sel;
      w[(int64_t)t * k + lane] = w_sel;
      s_ids[lane] = id_sel;
    }
  }
  __syncthreads();
  EpCtrl *own = ctrl_of(s_win[P.rank]);
  const int R = T * k;
  if (t < T)
    for (int j = warp; j < k; j += blockDim.x >> 5)
      dispatch_slot(P, s_win, t * k + j, s_ids[j], R, k, epr, x, lane, copy_rows != 0);
  dispatch_publish(P, s_win, own, step, R, wait_all);
}

// Step 3 as its own launch (for callers that dispatch with
// ep_dispatch_kernel): one warp, wait_dispatch_warp.
__global__ void ep_wait_dispatch_kernel(PeerTable P) {
  pdl_wait();
  pdl_trigger();
  EpCtrl *own = ctrl_of(win_at(P, P.rank));
  wait_dispatch_warp(P, own, __ldcg(&own->epoch) + 1, threadIdx.x);
}

// Step 5: the expert rows of this step (written by the kernels before this
// one) are complete; tell every rank.
__global__ void ep_signal_done_kernel(PeerTable P) {
  pdl_wait();  // the expert rows are complete once the kernels before have finished
  pdl_trigger();
  EpCtrl *own = ctrl_of(win_at(P, P.rank));
  const uint32_t step = __ldcg(&own->epoch);
  const bool sys = P.world > 1;
  if (sys)
    __threadfence_system();
  else
    __threadfence();
  if (threadIdx.x < P.world)
    st_release(&ctrl_of(win_at(P, threadIdx.x))->flag_done[P.rank], step, sys);
}

// Step 6: every block first waits for all done flags (threads 0..world-1),
// then thread (t, 8-column group) sums its slots in j order, loading each
// slot's fp32 row from the window of the rank that computed it: the
// arithmetic of the single-GPU combine, bit for bit.  (Step 5 stays a launch
// of its own: raised by every combine block before its wait, the done signal
// took the combine from 5.6 to 19 us on the critical path, against 3.3 us for
// the separate signal kernel.)
template <typename OutT>
__global__ void __launch_bounds__(256) ep_combine_kernel(PeerTable P, const int32_t *__restrict__ ids,
                                                         const float *__restrict__ w,
                                                         const uint16_t *__restrict__ residual,
                                                         OutT *__restrict__ y, int T, int k, int epr) {
  __shared__ const float *s_out[kMaxWorld];
  __shared__ int s_ok;
  pdl_wait();
  pdl_trigger();
  EpCtrl *own = ctrl_of(win_at(P, P.rank));
  const uint32_t step = __ldcg(&own->epoch);
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < kMaxWorld) {
    const int p = threadIdx.x < P.world ? threadIdx.x : 0;
    s_out[threadIdx.x] = reinterpret_cast<const float *>(win_at(P, p) + P.off_out);
    if (threadIdx.x < P.world && !wait_flag(&own->flag_done[p], step, P.timeout_ns, P.world > 1)) {
      atomicOr(&own->error, NVFP4_EP_ERR_DONE_TIMEOUT | (1u << (8 + p)));
      s_ok = 0;
    }
  }
  __syncthreads();
  if (!s_ok) return;  // a peer's rows never arrived: leave y untouched
  const int H = P.H, hv = H / 8, R = T * k, E = epr * P.world;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * hv) return;
  const int t = (int)(i / hv), h8 = (int)(i % hv);
  const int64_t base = (int64_t)P.rank * R + (int64_t)t * k;  // this rank's rows in every window
  float s[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) s[q] = 0.0f;
  for (int j0 = 0; j0 < k; j0 += 8) {
    float wv[8], v[8][8];
    int dst[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int j = j0 + jj;
      dst[jj] = -1;
      if (j < k) {
        const int e = __ldcg(ids + (int64_t)t * k + j);
        wv[jj] = __ldcg(w + (int64_t)t * k + j);
        dst[jj] = (e >= 0 && e < E) ? e / epr : -1;
      }
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      if (dst[jj] < 0) continue;
      ld_sys_f32x8(s_out[dst[jj]] + (base + j0 + jj) * H + 8 * h8, v[jj]);
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      if (dst[jj] < 0) continue;  // a slot without a valid expert contributes nothing
#pragma unroll
      for (int q = 0; q < 8; ++q) s[q] = fmaf(wv[jj], v[jj][q], s[q]);
    }
  }
  if (residual) {
    const uint4 r = __ldcg(reinterpret_cast<const uint4 *>(residual + (int64_t)t * H + 8 * h8));
    const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      s[2 * q] += bf16lo(rr[q]);
      s[2 * q + 1] += bf16hi(rr[q]);
    }
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

int check_peers(const nvfp4_ep_peers *p) {
  if (!p) return fail(NVFP4_ERR_INVALID_ARG, "null peer table");
  if (p->world < 1 || p->world > kMaxWorld || p->rank < 0 || p->rank >= p->world)
    return fail(NVFP4_ERR_INVALID_ARG, "rank %d of world %d outside [0, world), world in [1, %d]",
                p->rank, p->world, kMaxWorld);
  if (p->max_rows < 1 || p->max_rows > (1 << 24) / p->world)
    return fail(NVFP4_ERR_INVALID_ARG, "max_rows must be in [1, 2^24 / world]");
  if (p->hidden <= 0 || p->hidden % 128)
    return fail(NVFP4_ERR_INVALID_ARG, "hidden must be a positive multiple of 128");
  if (p->timeout_ms < 0) return fail(NVFP4_ERR_INVALID_ARG, "negative timeout");
  for (int r = 0; r < p->world; ++r)
    if (!p->windows[r] || !aligned(p->windows[r], kWinAlign))
      return fail(NVFP4_ERR_INVALID_ARG, "window of rank %d null or not 256-byte aligned", r);
  return NVFP4_OK;
}

PeerTable make_table(const nvfp4_ep_peers &p) {
  PeerTable P = {};
  for (int r = 0; r < kMaxWorld; ++r) P.win[r] = static_cast<char *>(p.windows[r < p.world ? r : 0]);
  P.rank = p.rank;
  P.world = p.world;
  P.H = p.hidden;
  const WinLayout L = win_layout(p.world, p.max_rows, p.hidden);
  P.off_expert = L.recv_expert;
  P.off_x = L.recv_x;
  P.off_out = L.out;
  P.timeout_ns = p.timeout_ms ? (uint64_t)p.timeout_ms * 1000 * 1000 : kDefaultTimeoutNs;
  return P;
}

int check_step(const nvfp4_ep_peers *p, int64_t T, int32_t k, int32_t epr) {
  int rc = check_peers(p);
  if (rc) return rc;
  if (T < 0 || k < 1 || k > 32 || epr < 1 || (int64_t)epr * p->world > 65536)
    return fail(NVFP4_ERR_INVALID_ARG, "bad token count, top_k or experts per rank");
  if (T > p->max_rows / k)
    return fail(NVFP4_ERR_INVALID_ARG, "%lld tokens x top-%d exceed the windows' %lld rows per rank",
                (long long)T, (int)k, (long long)p->max_rows);
  return NVFP4_OK;
}

}  // namespace

int ep_p2p_topk_dispatch(const nvfp4_ep_peers *p, const uint16_t *x, const float *part,
                         int nslices, int64_t T, int k, int renormalize, int epr, int32_t *ids,
                         float *w, bool wait_all, bool copy_rows, cudaStream_t st) {
  int rc = check_step(p, T, k, epr);
  if (rc) return rc;
  if (T > 0 && (!x || !part || !ids || !w))
    return fail(NVFP4_ERR_INVALID_ARG, "null activations, logits, ids or weights");
  if (!aligned(x, 16)) return fail(NVFP4_ERR_INVALID_ARG, "x must be 16-byte aligned");
  if (!copy_rows && p->world != 1)
    return fail(NVFP4_ERR_INVALID_ARG, "a dispatch without its rows needs world 1");
  if (epr * p->world > 256 || nslices < 1)
    return fail(NVFP4_ERR_INVALID_ARG, "the fused top-k takes at most 256 experts");
  // At least one block, so the flags go up even for an empty step.
  const unsigned blocks = (unsigned)std::max<int64_t>(1, T);
  return check_launch(launch_pdl(ep_topk_dispatch_kernel, dim3(blocks), dim3(256), 0, st,
                                 make_table(*p), part, nslices, reinterpret_cast<const uint4 *>(x),
                                 (int)T, k, renormalize, epr, ids, w, (int)wait_all,
                                 (int)copy_rows),
                      wait_all ? "top-k + dispatch + wait launch" : "top-k + dispatch launch");
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" size_t nvfp4_ep_window_size(int32_t world, int64_t max_rows, int32_t hidden) {
  if (world < 1 || world > kMaxWorld || max_rows < 1 || max_rows > (1 << 24) / world ||
      hidden <= 0 || hidden % 128)
    return 0;
  return win_layout(world, max_rows, hidden).total;
}

extern "C" int nvfp4_ep_window_create(size_t bytes, void **window, uint8_t *handle) {
  if (!window || !handle || bytes < sizeof(EpCtrl))
    return fail(NVFP4_ERR_INVALID_ARG, "null window or handle pointer, or window too small");
  static_assert(sizeof(cudaIpcMemHandle_t) == NVFP4_EP_HANDLE_BYTES, "IPC handle size");
  void *p = nullptr;
  int rc = check_launch(cudaMalloc(&p, bytes), "window allocation");
  if (rc) return rc;
  // Zeroed (flags, step counter, error word) before any peer can see it.
  rc = check_launch(cudaMemset(p, 0, bytes), "window zeroing");
  if (!rc) rc = check_launch(cudaDeviceSynchronize(), "window zeroing");
  cudaIpcMemHandle_t h;
  if (!rc) rc = check_launch(cudaIpcGetMemHandle(&h, p), "window IPC handle");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  memcpy(handle, &h, sizeof(h));
  *window = p;
  return NVFP4_OK;
}

extern "C" int nvfp4_ep_window_open(const uint8_t *handle, void **window) {
  if (!handle || !window) return fail(NVFP4_ERR_INVALID_ARG, "null handle or window pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_launch(cudaIpcOpenMemHandle(window, h, cudaIpcMemLazyEnablePeerAccess),
                      "opening a peer window");
}

extern "C" int nvfp4_ep_window_close(void *window) {
  if (!window) return fail(NVFP4_ERR_INVALID_ARG, "null window");
  return check_launch(cudaIpcCloseMemHandle(window), "closing a peer window");
}

extern "C" int nvfp4_ep_window_destroy(void *window) {
  if (!window) return fail(NVFP4_ERR_INVALID_ARG, "null window");
  int rc = check_launch(cudaDeviceSynchronize(), "window release");
  const int rc2 = check_launch(cudaFree(window), "window release");
  return rc ? rc : rc2;
}

extern "C" int nvfp4_ep_p2p_rows(const nvfp4_ep_peers *p, int64_t T, int32_t k, void **recv_x,
                                 int32_t **recv_expert, float **out_rows) {
  int rc = check_step(p, T, k, 1);
  if (rc) return rc;
  const WinLayout L = win_layout(p->world, p->max_rows, p->hidden);
  char *own = static_cast<char *>(p->windows[p->rank]);
  if (recv_x) *recv_x = own + L.recv_x;
  if (recv_expert) *recv_expert = reinterpret_cast<int32_t *>(own + L.recv_expert);
  if (out_rows) *out_rows = reinterpret_cast<float *>(own + L.out);
  return NVFP4_OK;
}

extern "C" int nvfp4_ep_p2p_dispatch(const nvfp4_ep_peers *p, const int32_t *ids, const void *x,
                                     int64_t T, int32_t k, int32_t epr, void *stream) {
  int rc = check_step(p, T, k, epr);
  if (rc) return rc;
  if (T > 0 && (!ids || !x)) return fail(NVFP4_ERR_INVALID_ARG, "null expert ids or activations");
  if (!aligned(x, 16)) return fail(NVFP4_ERR_INVALID_ARG, "x must be 16-byte aligned");
  const int64_t R = T * k;
  // At least one block, so the flags go up even for an empty step.
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((R + 7) / 8, 148 * 8));
  return check_launch(launch_pdl(ep_dispatch_kernel, dim3(blocks), dim3(256), 0,
                                  static_cast<cudaStream_t>(stream), make_table(*p), ids,
                                  static_cast<const uint4 *>(x), (int)T, k, epr),
                      "dispatch launch");
}

extern "C" int nvfp4_ep_p2p_wait_dispatch(const nvfp4_ep_peers *p, void *stream) {
  int rc = check_peers(p);
  if (rc) return rc;
  return check_launch(launch_pdl(ep_wait_dispatch_kernel, dim3(1), dim3(32), 0,
                                  static_cast<cudaStream_t>(stream), make_table(*p)),
                      "dispatch wait launch");
}

extern "C" int nvfp4_ep_p2p_signal_done(const nvfp4_ep_peers *p, void *stream) {
  int rc = check_peers(p);
  if (rc) return rc;
  return check_launch(launch_pdl(ep_signal_done_kernel, dim3(1), dim3(32), 0,
                                  static_cast<cudaStream_t>(stream), make_table(*p)),
                      "done signal launch");
}

extern "C" int nvfp4_ep_p2p_combine(const nvfp4_ep_peers *p, const int32_t *ids, const float *w,
                                    int64_t T, int32_t k, int32_t epr, const void *residual,
                                    void *y, int y_dtype, void *stream) {
  int rc = check_step(p, T, k, epr);
  if (rc) return rc;
  if (y_dtype != NVFP4_DTYPE_F32 && y_dtype != NVFP4_DTYPE_BF16)
    return fail(NVFP4_ERR_INVALID_ARG, "bad output dtype");
  if (T > 0 && (!ids || !w || !y)) return fail(NVFP4_ERR_INVALID_ARG, "null combine pointer");
  if (!aligned(y, 16) || (residual && !aligned(residual, 16)))
    return fail(NVFP4_ERR_INVALID_ARG, "y and residual must be 16-byte aligned");
  // At least one block: the wait on the done flags runs even for T = 0.
  const int64_t n = T * (p->hidden / 8);
  const unsigned blocks = (unsigned)std::max<int64_t>(1, (n + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint16_t *res = static_cast<const uint16_t *>(residual);
  const PeerTable P = make_table(*p);
  cudaError_t e;
  if (y_dtype == NVFP4_DTYPE_F32)
    e = launch_pdl(ep_combine_kernel<float>, dim3(blocks), dim3(256), 0, st, P, ids, w, res,
                   static_cast<float *>(y), (int)T, k, epr);
  else
    e = launch_pdl(ep_combine_kernel<uint16_t>, dim3(blocks), dim3(256), 0, st, P, ids, w, res,
                   static_cast<uint16_t *>(y), (int)T, k, epr);
  return check_launch(e, "combine launch");
}

extern "C" int nvfp4_ep_p2p_error(const nvfp4_ep_peers *p, uint32_t *error, int32_t clear,
                                  void *stream) {
  int rc = check_peers(p);
  if (rc) return rc;
  if (!error) return fail(NVFP4_ERR_INVALID_ARG, "null error pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  EpCtrl *own = static_cast<EpCtrl *>(p->windows[p->rank]);
  rc = check_launch(cudaMemcpyAsync(error, &own->error, sizeof(uint32_t), cudaMemcpyDeviceToHost, st),
                    "error word read");
  if (!rc && clear)
    rc = check_launch(cudaMemsetAsync(&own->error, 0, sizeof(uint32_t), st), "error word clear");
  if (!rc) rc = check_launch(cudaStreamSynchronize(st), "error word read");
  return rc;
}

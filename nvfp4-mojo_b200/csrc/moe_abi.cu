// moe_abi.cu -- extern "C" MoE entry points (include/nvfp4.h): validation,
// workspace layout and the launch sequence of one MoE layer.
#include <algorithm>
#include "../../include/nvfp4.h"
#include "../../include/nvfp4_ep.h"
#include "abi_util.h"
#include "kernels.h"
#include "moe.h"

namespace nvfp4 {
namespace {

constexpr size_t kAlign = 256;

size_t up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

// Grouped-GEMM path: tcgen05 tiles when experts get many rows on average
// (prefill); the TMA-fed decode GEMV kernel (work items of <= 8 slots) when
// they get few; the register-decode skinny kernel in between, or when the
// shapes or alignments do not suit the GEMV kernel.
enum class ExpertPath { kTc, kGemv, kSkinny };

bool use_tc(const nvfp4_moe_desc &d, int64_t R) {
  return R >= 64LL * d.num_experts && moe_tc_supported(d.hidden, d.intermediate);
}

// GEMV path by shape: at most 32 rows per expert on average (items of 8
// slots re-read an expert's weights once per item).
bool gemv_shape_ok(const nvfp4_moe_desc &d, int64_t R) {
  return !use_tc(d, R) && R <= 32LL * d.num_experts && d.hidden % 256 == 0 &&
         d.intermediate % 256 == 0;
}

ExpertPath choose_path(const nvfp4_moe_desc &d, const nvfp4_moe_weights &w, int64_t R) {
  if (use_tc(d, R)) return ExpertPath::kTc;
  if (gemv_shape_ok(d, R) &&
      moe_gemv_supported(d.hidden, d.intermediate, w.gate_up, w.gate_up_scale, w.down,
                         w.down_scale))
    return ExpertPath::kGemv;
  return ExpertPath::kSkinny;
}

// Rows per grouped-GEMM work item.
int path_tpi(const nvfp4_moe_desc &d, int64_t R, ExpertPath p) {
  if (p == ExpertPath::kTc) return moe_tc_rows_per_item();
  if (p == ExpertPath::kGemv) return 8;
  const int64_t avg = (R + d.num_experts - 1) / d.num_experts;
  return avg <= 8 ? 8 : (avg <= 16 ? 16 : 32);
}

// Workspace sizing knows the shapes only: it takes the largest item count
// any path could need (items of 8 slots unless the tensor-core path runs).
int choose_tpi(const nvfp4_moe_desc &d, int64_t R) {
  if (use_tc(d, R)) return moe_tc_rows_per_item();
  return gemv_shape_ok(d, R) ? 8 : path_tpi(d, R, ExpertPath::kSkinny);
}

// Upper bound of the permutation's work items: every expert with slots adds
// at most one partial item, and at most min(E, R) experts have slots.
int64_t work_capacity(int64_t R, int E, int tpi) {
  return (R + tpi - 1) / tpi + std::min<int64_t>(E, R);
}

struct ExpertsLayout {
  size_t offsets, n_work, n_rows, work, src_row, dst_row, inter, inter_lo, x_perm, total;
};

ExpertsLayout experts_layout(const nvfp4_moe_desc &d, int64_t R) {
  ExpertsLayout L;
  const int tpi = choose_tpi(d, R);
  size_t o = 0;
  L.offsets = o;
  o = up(o + sizeof(int32_t) * (d.num_experts + 1));
  L.n_work = o;
  o = up(o + sizeof(int32_t));
  L.n_rows = o;
  o = up(o + sizeof(int32_t));
  L.work = o;
  o = up(o + sizeof(SkinnyWork) * work_capacity(R, d.num_experts, tpi));
  L.src_row = o;
  o = up(o + sizeof(int32_t) * R);
  L.dst_row = o;
  o = up(o + sizeof(int32_t) * R);
  L.inter = o;
  o = up(o + sizeof(uint16_t) * R * d.intermediate);
  L.inter_lo = o;
  o = up(o + sizeof(uint16_t) * R * d.intermediate);
  L.x_perm = o;  // tensor-core path: activation rows gathered in sorted order
  if (use_tc(d, R)) o = up(o + sizeof(uint16_t) * R * d.hidden);
  L.total = o;
  return L;
}

struct ForwardLayout {
  size_t ids, w, logits, y_slot, experts, total;
};

ForwardLayout forward_layout(const nvfp4_moe_desc &d, int64_t T) {
  ForwardLayout L;
  const int64_t R = T * d.top_k;
  size_t o = 0;
  L.ids = o;
  o = up(o + sizeof(int32_t) * R);
  L.w = o;
  o = up(o + sizeof(float) * R);
  L.logits = o;  // router partial sums, one [T, E] slice per H slice
  o = up(o + sizeof(float) * T * d.num_experts * router_slices((int)T, d.hidden, d.num_experts));
  L.y_slot = o;
  o = up(o + sizeof(float) * R * d.hidden);
  L.experts = o;
  o = up(o + experts_layout(d, R).total);
  L.total = o;
  return L;
}

int check_desc(const nvfp4_moe_desc *d) {
  if (!d) return fail(NVFP4_ERR_INVALID_ARG, "null MoE descriptor");
  if (d->num_experts <= 0 || d->num_experts > 256)
    return fail(NVFP4_ERR_INVALID_ARG, "num_experts must be in [1, 256]");
  if (d->top_k <= 0 || d->top_k > 32 || d->top_k > d->num_experts)
    return fail(NVFP4_ERR_INVALID_ARG, "top_k must be in [1, min(32, num_experts)]");
  if (d->hidden <= 0 || d->hidden % 128 || d->intermediate <= 0 || d->intermediate % 128)
    return fail(NVFP4_ERR_INVALID_ARG, "hidden and intermediate must be positive multiples of 128");
  if (d->hidden > 6144)
    return fail(NVFP4_ERR_INVALID_ARG, "hidden > 6144 exceeds the router's shared-memory tile");
  return NVFP4_OK;
}

int check_weights(const nvfp4_moe_weights *w) {
  if (!w || !w->gate_up || !w->gate_up_scale || !w->down || !w->down_scale)
    return fail(NVFP4_ERR_INVALID_ARG, "null expert weight pointer");
  if (!aligned(w->gate_up, 16) || !aligned(w->down, 16) || !aligned(w->gate_up_scale, 4) ||
      !aligned(w->down_scale, 4))
    return fail(NVFP4_ERR_INVALID_ARG, "expert weights must be 16-byte (scales 4-byte) aligned");
  return NVFP4_OK;
}

// Slot r's activation row is x_row_index[r], or r / row_div when x_row_index
// is null.
int run_experts(const nvfp4_moe_desc &d, const nvfp4_moe_weights &w, const uint16_t *x,
                const int32_t *x_row_index, int row_div, const int32_t *row_expert, int64_t R,
                void *y_rows, int y_dtype, uint8_t *ws, cudaStream_t st) {
  if (R == 0) return NVFP4_OK;
  const ExpertsLayout L = experts_layout(d, R);
  const int E = d.num_experts, H = d.hidden, I = d.intermediate;
  const ExpertPath path = choose_path(d, w, R);
  const int tpi = path_tpi(d, R, path);
  MoePlan plan;
  plan.offsets = reinterpret_cast<int32_t *>(ws + L.offsets);
  plan.n_work = reinterpret_cast<int32_t *>(ws + L.n_work);
  plan.n_rows = reinterpret_cast<int32_t *>(ws + L.n_rows);
  plan.work = reinterpret_cast<SkinnyWork *>(ws + L.work);
  plan.src_row = reinterpret_cast<int32_t *>(ws + L.src_row);
  plan.dst_row = reinterpret_cast<int32_t *>(ws + L.dst_row);
  // The SiLU*up activations are kept as bf16 hi + lo parts so the down
  // projection sees them to ~2^-16 (one bf16 rounding would cost up to 2^-9
  // relative per element on the MMA operand).
  uint16_t *inter = reinterpret_cast<uint16_t *>(ws + L.inter);
  uint16_t *inter_lo = reinterpret_cast<uint16_t *>(ws + L.inter_lo);
  int rc = check_launch(launch_moe_permute(row_expert, x_row_index, row_div, (int)R, E, tpi, plan,
                                           st),
                        "MoE permutation launch");
  if (rc) return rc;

  if (path == ExpertPath::kGemv) {
    MoeGemvLaunch gu;
    gu.w = w.gate_up;
    gu.sf = w.gate_up_scale;
    gu.al.input_scales = w.gate_up_input_scale;
    gu.al.ws2_rows = w.gate_up_scale_2;
    gu.al.ws2_group_stride = 2 * I;
    gu.x = x;
    gu.x_ld = H;
    gu.x_rows = plan.src_row;
    gu.y = inter;
    gu.y_lo = inter_lo;
    gu.y_ld = I;
    gu.N = 2 * I;
    gu.K = H;
    gu.groups = E;
    gu.items = (int)work_capacity(R, E, tpi);
    gu.work = plan.work;
    gu.n_work = plan.n_work;
    gu.gate_up = true;
    rc = check_launch(launch_moe_gemv(gu, st), "MoE gate_up (GEMV) launch");
    if (rc) return rc;
    MoeGemvLaunch dn = gu;
    dn.w = w.down;
    dn.sf = w.down_scale;
    dn.al = AlphaSpec();
    dn.al.input_scales = w.down_input_scale;
    dn.al.ws2_rows = w.down_scale_2;
    dn.al.ws2_group_stride = H;
    dn.x = inter;
    dn.x_lo = inter_lo;
    dn.x_ld = I;
    dn.x_rows = nullptr;
    dn.y = y_rows;
    dn.y_lo = nullptr;
    dn.y_dtype = y_dtype;
    dn.y_ld = H;
    dn.y_rows = plan.dst_row;
    dn.N = H;
    dn.K = I;
    dn.gate_up = false;
    return check_launch(launch_moe_gemv(dn, st), "MoE down (GEMV) launch");
  }

  if (path == ExpertPath::kTc) {
    uint16_t *x_perm = reinterpret_cast<uint16_t *>(ws + L.x_perm);
    rc = check_launch(launch_gather_rows(x, plan.src_row, R, (int64_t)H * 2, x_perm, st),
                      "MoE activation gather launch");
    if (rc) return rc;
    MoeTcLaunch g;
    g.w = w.gate_up;
    g.sf = w.gate_up_scale;
    g.E = E;
    g.Nw = 2 * I;
    g.K = H;
    g.b0 = x_perm;
    g.R = R;
    g.work = plan.work;
    g.n_work = plan.n_work;
    g.al.input_scales = w.gate_up_input_scale;
    g.al.ws2_rows = w.gate_up_scale_2;
    g.inter = inter;
    g.inter_lo = inter_lo;
    rc = check_launch(launch_moe_tc(g, true, st), "MoE gate_up (tensor core) launch");
    if (rc) return rc;
    MoeTcLaunch dn;
    dn.w = w.down;
    dn.sf = w.down_scale;
    dn.E = E;
    dn.Nw = H;
    dn.K = I;
    dn.b0 = inter;
    dn.b1 = inter_lo;
    dn.R = R;
    dn.work = plan.work;
    dn.n_work = plan.n_work;
    dn.al.input_scales = w.down_input_scale;
    dn.al.ws2_rows = w.down_scale_2;
    dn.y = y_rows;
    dn.y_dtype = y_dtype;
    dn.dst_row = plan.dst_row;
    dn.y_ld = H;
    return check_launch(launch_moe_tc(dn, false, st), "MoE down (tensor core) launch");
  }

  SkinnyArgs gu;
  gu.ws.w = w.gate_up;
  gu.ws.sf = w.gate_up_scale;
  gu.ws.w_group_stride = (int64_t)2 * I * (H / 2);
  gu.ws.sf_group_stride = (int64_t)2 * I * (H / 16);
  gu.ws.N = 2 * I;
  gu.ws.K = H;
  gu.al.input_scales = w.gate_up_input_scale;
  gu.al.ws2_rows = w.gate_up_scale_2;
  gu.al.ws2_group_stride = 2 * I;
  gu.x = x;
  gu.x_ld = H;
  gu.x_rows = plan.src_row;
  gu.y = inter;
  gu.y_lo = inter_lo;
  gu.y_dtype = kBF16;
  gu.y_ld = I;
  gu.work = plan.work;
  gu.n_work = plan.n_work;
  gu.work_capacity = (int)work_capacity(R, E, tpi);
  gu.silu_gate = true;
  gu.tokens_per_item = tpi;
  rc = check_launch(launch_skinny(gu, st), "MoE gate_up launch");
  if (rc) return rc;

  SkinnyArgs dn = gu;
  dn.ws.w = w.down;
  dn.ws.sf = w.down_scale;
  dn.ws.w_group_stride = (int64_t)H * (I / 2);
  dn.ws.sf_group_stride = (int64_t)H * (I / 16);
  dn.ws.N = H;
  dn.ws.K = I;
  dn.al = AlphaSpec();
  dn.al.input_scales = w.down_input_scale;
  dn.al.ws2_rows = w.down_scale_2;
  dn.al.ws2_group_stride = H;
  dn.x = inter;
  dn.x_lo = inter_lo;
  dn.y_lo = nullptr;
  dn.x_ld = I;
  dn.x_rows = nullptr;
  dn.y = y_rows;
  dn.y_dtype = y_dtype;
  dn.y_ld = H;
  dn.y_rows = plan.dst_row;
  dn.silu_gate = false;
  return check_launch(launch_skinny(dn, st), "MoE down launch");
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

// Token counts are bounded by T * top_k <= 2^24 slots, tested as a division so
// that no product of a caller's count can wrap.
bool tokens_ok(const nvfp4_moe_desc &d, int64_t T) { return T >= 0 && T <= (1 << 24) / d.top_k; }

extern "C" size_t nvfp4_moe_workspace_size(const nvfp4_moe_desc *d, int64_t T) {
  if (check_desc(d) || !tokens_ok(*d, T)) return 0;
  return forward_layout(*d, T).total;
}

extern "C" size_t nvfp4_moe_experts_workspace_size(const nvfp4_moe_desc *d, int64_t R) {
  if (check_desc(d) || R < 0 || R > (1 << 24)) return 0;
  return experts_layout(*d, R).total;
}

extern "C" int nvfp4_moe_route(const nvfp4_moe_desc *d, const float *router, const void *x,
                               int64_t T, int32_t *ids, float *w, float *logits, void *stream) {
  NVFP4_ABI_RANGE();
  int rc = check_desc(d);
  if (rc) return rc;
  if (T < 0 || T > (1 << 24)) return fail(NVFP4_ERR_INVALID_ARG, "bad token count");
  if (T == 0) return NVFP4_OK;
  if (!router || !x || !ids || !w || !logits)
    return fail(NVFP4_ERR_INVALID_ARG, "null router, activation or output pointer");
  // Same H slicing (hence the same logits, bit for bit) as nvfp4_moe_forward:
  // the per-slice partial sums go to stream-ordered scratch.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nslices = router_slices((int)T, d->hidden, d->num_experts);
  if (nslices == 1)
    return check_launch(launch_router(static_cast<const uint16_t *>(x), router, logits, 1, nullptr,
                                      (int)T, d->hidden, d->num_experts, d->top_k,
                                      d->renormalize, ids, w, st),
                        "router launch");
  void *part = nullptr;
  cudaError_t e = cudaMallocAsync(&part, sizeof(float) * nslices * T * d->num_experts, st);
  if (e != cudaSuccess) return check_launch(e, "router scratch (cudaMallocAsync)");
  rc = check_launch(launch_router(static_cast<const uint16_t *>(x), router,
                                  static_cast<float *>(part), nslices, logits, (int)T, d->hidden,
                                  d->num_experts, d->top_k, d->renormalize, ids, w, st),
                    "router launch");
  e = cudaFreeAsync(part, st);
  if (rc == NVFP4_OK && e != cudaSuccess) return check_launch(e, "router scratch release");
  return rc;
}

extern "C" int nvfp4_moe_experts(const nvfp4_moe_desc *d, const nvfp4_moe_weights *w,
                                 const void *x, const int32_t *x_row_index,
                                 const int32_t *row_expert, int64_t R, void *y_rows, int y_dtype,
                                 void *ws, size_t ws_bytes, void *stream) {
  NVFP4_ABI_RANGE();
  int rc = check_desc(d);
  if (rc) return rc;
  if ((rc = check_weights(w))) return rc;
  if (R < 0 || R > (1 << 24)) return fail(NVFP4_ERR_INVALID_ARG, "bad row count");
  if (R == 0) return NVFP4_OK;
  if (!x || !row_expert || !y_rows || !ws)
    return fail(NVFP4_ERR_INVALID_ARG, "null activation, expert id, output or workspace pointer");
  if (y_dtype != NVFP4_DTYPE_F32 && y_dtype != NVFP4_DTYPE_BF16)
    return fail(NVFP4_ERR_INVALID_ARG, "bad output dtype");
  if (!aligned(x, 16) || !aligned(ws, kAlign))
    return fail(NVFP4_ERR_INVALID_ARG, "x must be 16-byte and workspace 256-byte aligned");
  if (ws_bytes < experts_layout(*d, R).total)
    return fail(NVFP4_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", ws_bytes,
                experts_layout(*d, R).total);
  return run_experts(*d, *w, static_cast<const uint16_t *>(x), x_row_index, 1, row_expert, R,
                     y_rows,
                     y_dtype, static_cast<uint8_t *>(ws), static_cast<cudaStream_t>(stream));
}

extern "C" int nvfp4_moe_combine(const void *y_slots, int slot_dtype, const float *topk_w,
                                 const int32_t *slot_pos, const void *residual, void *y,
                                 int y_dtype, int64_t T, int32_t k, int32_t H, void *stream) {
  NVFP4_ABI_RANGE();
  if (T < 0 || k <= 0 || H <= 0 || H % 8) return fail(NVFP4_ERR_INVALID_ARG, "bad combine shape");
  if ((slot_dtype != NVFP4_DTYPE_F32 && slot_dtype != NVFP4_DTYPE_BF16) ||
      (y_dtype != NVFP4_DTYPE_F32 && y_dtype != NVFP4_DTYPE_BF16))
    return fail(NVFP4_ERR_INVALID_ARG, "bad slot or output dtype");
  if (T == 0) return NVFP4_OK;
  if (!y_slots || !topk_w || !y) return fail(NVFP4_ERR_INVALID_ARG, "null combine pointer");
  if (!aligned(y_slots, 16) || !aligned(y, 16) || (residual && !aligned(residual, 16)))
    return fail(NVFP4_ERR_INVALID_ARG, "combine buffers must be 16-byte aligned");
  return check_launch(launch_moe_combine(y_slots, slot_dtype, topk_w,
                                         static_cast<const uint16_t *>(residual), slot_pos,
                                         nullptr, y, y_dtype, (int)T, k, H,
                                         static_cast<cudaStream_t>(stream)),
                      "combine launch");
}

extern "C" int nvfp4_ep_dispatch_plan(const int32_t *topk_ids, int64_t T, int32_t k,
                                      int32_t experts_per_rank, int32_t world,
                                      int32_t *send_counts, int32_t *send_token,
                                      int32_t *send_expert, int32_t *slot_pos, void *stream) {
  if (T < 0 || k <= 0 || k > 32 || experts_per_rank <= 0 || world <= 0 || world > 64 ||
      T > (1 << 24) / k)
    return fail(NVFP4_ERR_INVALID_ARG, "bad dispatch-plan shape");
  if (!topk_ids || !send_counts || !send_token || !send_expert || !slot_pos)
    return fail(NVFP4_ERR_INVALID_ARG, "null dispatch-plan pointer");
  return check_launch(launch_ep_plan(topk_ids, (int)(T * k), k, experts_per_rank, world,
                                     send_counts, send_token, send_expert, slot_pos,
                                     static_cast<cudaStream_t>(stream)),
                      "dispatch plan launch");
}

extern "C" int nvfp4_gather_rows(const void *src, const int32_t *row_index, int64_t n,
                                 int64_t row_bytes, void *dst, void *stream) {
  if (n < 0 || row_bytes <= 0 || row_bytes % 16) return fail(NVFP4_ERR_INVALID_ARG, "bad gather shape");
  if (n == 0) return NVFP4_OK;
  if (!src || !row_index || !dst) return fail(NVFP4_ERR_INVALID_ARG, "null gather pointer");
  if (!aligned(src, 16) || !aligned(dst, 16))
    return fail(NVFP4_ERR_INVALID_ARG, "gather buffers must be 16-byte aligned");
  return check_launch(launch_gather_rows(src, row_index, n, row_bytes, dst,
                                         static_cast<cudaStream_t>(stream)),
                      "gather launch");
}

extern "C" int nvfp4_ep_dispatch_padded(const int32_t *send_counts, const int32_t *send_token,
                                        const int32_t *send_expert, const int32_t *slot_pos,
                                        int64_t T, int32_t k, int32_t world, int64_t cap,
                                        const void *x, int64_t row_bytes, void *send_rows,
                                        int32_t *send_expert_padded, int32_t *slot_padded,
                                        void *stream) {
  if (T < 0 || k <= 0 || k > 32 || world <= 0 || world > 64 || cap < 0 || T > (1 << 24) / k ||
      cap > (1 << 24) / world || row_bytes <= 0 || row_bytes % 16)
    return fail(NVFP4_ERR_INVALID_ARG, "bad padded-dispatch shape");
  if (cap < T * k)
    return fail(NVFP4_ERR_INVALID_ARG, "capacity %lld below the %lld slots of this rank",
                (long long)cap, (long long)(T * k));
  if (!send_counts || !send_token || !send_expert || !slot_pos || !send_rows ||
      !send_expert_padded || !slot_padded || (T > 0 && !x))
    return fail(NVFP4_ERR_INVALID_ARG, "null padded-dispatch pointer");
  if (!aligned(x, 16) || !aligned(send_rows, 16))
    return fail(NVFP4_ERR_INVALID_ARG, "row buffers must be 16-byte aligned");
  return check_launch(launch_ep_pad(send_counts, send_token, send_expert, slot_pos, (int)(T * k),
                                    world, (int)cap, x, row_bytes, send_rows, send_expert_padded,
                                    slot_padded, static_cast<cudaStream_t>(stream)),
                      "padded dispatch launch");
}

namespace nvfp4 {
namespace {

// The shared expert's part of the workspace: its fp32 output rows [T, H], the
// expert id (0) and the x row (t) of each of its T slots, and its own expert
// workspace.
struct SharedLayout {
  size_t y_shared, ids0, experts, total;
};

nvfp4_moe_desc shared_desc(const nvfp4_moe_desc &d, int32_t shared_intermediate) {
  nvfp4_moe_desc s = d;
  s.num_experts = 1;
  s.top_k = 1;
  s.intermediate = shared_intermediate;
  s.renormalize = 0;
  return s;
}

SharedLayout shared_layout(const nvfp4_moe_desc &ds, int64_t T) {
  SharedLayout L;
  size_t o = 0;
  L.y_shared = o;
  o = up(o + sizeof(float) * T * ds.hidden);
  L.ids0 = o;
  o = up(o + sizeof(int32_t) * T);
  L.experts = o;
  o = up(o + experts_layout(ds, T).total);
  L.total = o;
  return L;
}

// One MoE layer; with `shared` (nullable) the shared expert's output (every
// token, weight 1) is added after the routed sum, before the residual.
int moe_forward_impl(const nvfp4_moe_desc *d, const nvfp4_moe_weights *w,
                     const nvfp4_moe_weights *shared, int32_t shared_intermediate, const void *x,
                     const void *residual, void *y, int y_dtype, int64_t T, int32_t *topk_ids,
                     float *topk_w, void *ws, size_t ws_bytes, void *stream) {
  int rc = check_desc(d);
  if (rc) return rc;
  if ((rc = check_weights(w))) return rc;
  if (!w->router) return fail(NVFP4_ERR_INVALID_ARG, "null router pointer");
  nvfp4_moe_desc ds = {};
  if (shared) {
    ds = shared_desc(*d, shared_intermediate);
    if ((rc = check_desc(&ds))) return rc;
    if ((rc = check_weights(shared))) return rc;
  }
  if (!tokens_ok(*d, T)) return fail(NVFP4_ERR_INVALID_ARG, "bad token count");
  if (T == 0) return NVFP4_OK;
  if (!x || !y || !ws) return fail(NVFP4_ERR_INVALID_ARG, "null activation, output or workspace");
  if (y_dtype != NVFP4_DTYPE_F32 && y_dtype != NVFP4_DTYPE_BF16)
    return fail(NVFP4_ERR_INVALID_ARG, "bad output dtype");
  if (!aligned(x, 16) || !aligned(y, 16) || (residual && !aligned(residual, 16)) ||
      !aligned(ws, kAlign))
    return fail(NVFP4_ERR_INVALID_ARG, "x/y/residual must be 16-byte and workspace 256-byte aligned");
  const ForwardLayout L = forward_layout(*d, T);
  const size_t need = L.total + (shared ? shared_layout(ds, T).total : 0);
  if (ws_bytes < need)
    return fail(NVFP4_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", ws_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *base = static_cast<uint8_t *>(ws);
  int32_t *ids = topk_ids ? topk_ids : reinterpret_cast<int32_t *>(base + L.ids);
  float *tw = topk_w ? topk_w : reinterpret_cast<float *>(base + L.w);
  float *logits = reinterpret_cast<float *>(base + L.logits);
  float *y_slot = reinterpret_cast<float *>(base + L.y_slot);
  const int64_t R = T * d->top_k;
  rc = check_launch(launch_router(static_cast<const uint16_t *>(x), w->router, logits,
                                  router_slices((int)T, d->hidden, d->num_experts), nullptr,
                                  (int)T, d->hidden, d->num_experts, d->top_k, d->renormalize,
                                  ids, tw, st),
                    "router launch");
  if (rc) return rc;
  // Slot r = t * k + j reads token r / k (the permutation computes it).
  rc = run_experts(*d, *w, static_cast<const uint16_t *>(x), nullptr, d->top_k, ids, R, y_slot, kF32,
                   base + L.experts, st);
  if (rc) return rc;
  float *y_shared = nullptr;
  if (shared) {
    // Every token is one slot of expert 0 of the one-expert "layer".
    uint8_t *sb = base + L.total;
    const SharedLayout SL = shared_layout(ds, T);
    y_shared = reinterpret_cast<float *>(sb + SL.y_shared);
    int32_t *ids0 = reinterpret_cast<int32_t *>(sb + SL.ids0);
    rc = check_launch(cudaMemsetAsync(ids0, 0, sizeof(int32_t) * T, st), "shared expert ids");
    if (rc) return rc;
    rc = run_experts(ds, *shared, static_cast<const uint16_t *>(x), nullptr, 1, ids0, T, y_shared,
                     kF32,
                     sb + SL.experts, st);
    if (rc) return rc;
  }
  return check_launch(launch_moe_combine(y_slot, kF32, tw, static_cast<const uint16_t *>(residual),
                                         nullptr, y_shared, y, y_dtype, (int)T, d->top_k,
                                         d->hidden, st),
                      "combine launch");
}

}  // namespace
}  // namespace nvfp4

extern "C" int nvfp4_moe_forward(const nvfp4_moe_desc *d, const nvfp4_moe_weights *w,
                                 const void *x, const void *residual, void *y, int y_dtype,
                                 int64_t T, int32_t *topk_ids, float *topk_w, void *ws,
                                 size_t ws_bytes, void *stream) {
  NVFP4_ABI_RANGE();
  return moe_forward_impl(d, w, nullptr, 0, x, residual, y, y_dtype, T, topk_ids, topk_w, ws,
                          ws_bytes, stream);
}

extern "C" size_t nvfp4_moe_shared_workspace_size(const nvfp4_moe_desc *d,
                                                  int32_t shared_intermediate, int64_t T) {
  if (check_desc(d) || !tokens_ok(*d, T)) return 0;
  const nvfp4_moe_desc ds = shared_desc(*d, shared_intermediate);
  if (check_desc(&ds)) return 0;
  return forward_layout(*d, T).total + shared_layout(ds, T).total;
}

extern "C" int nvfp4_moe_forward_shared(const nvfp4_moe_desc *d, const nvfp4_moe_weights *w,
                                        const nvfp4_moe_weights *shared,
                                        int32_t shared_intermediate, const void *x,
                                        const void *residual, void *y, int y_dtype, int64_t T,
                                        int32_t *topk_ids, float *topk_w, void *ws,
                                        size_t ws_bytes, void *stream) {
  NVFP4_ABI_RANGE();
  if (!shared) return fail(NVFP4_ERR_INVALID_ARG, "null shared-expert weights");
  return moe_forward_impl(d, w, shared, shared_intermediate, x, residual, y, y_dtype, T,
                          topk_ids, topk_w, ws, ws_bytes, stream);
}

extern "C" int nvfp4_stack_rows(const void *const *srcs, const int64_t *rows, int32_t n,
                                int64_t row_bytes, void *dst, void *stream) {
  if (n < 0 || row_bytes <= 0) return fail(NVFP4_ERR_INVALID_ARG, "bad stack shape");
  if (n == 0) return NVFP4_OK;
  if (!srcs || !rows || !dst) return fail(NVFP4_ERR_INVALID_ARG, "null stack pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *o = static_cast<uint8_t *>(dst);
  for (int32_t i = 0; i < n; ++i) {
    if (rows[i] < 0) return fail(NVFP4_ERR_INVALID_ARG, "negative row count at %d", (int)i);
    if (rows[i] == 0) continue;
    if (!srcs[i]) return fail(NVFP4_ERR_INVALID_ARG, "null source %d", (int)i);
    const size_t bytes = (size_t)rows[i] * (size_t)row_bytes;
    const cudaError_t e = cudaMemcpyAsync(o, srcs[i], bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) return check_launch(e, "row stack copy");
    o += bytes;
  }
  return NVFP4_OK;
}
namespace nvfp4 {
namespace {

// Workspace of the expert-parallel step through peer memory: the routing of
// this rank's T tokens and the expert workspace for the world*T*k received rows.
struct EpP2pLayout {
  size_t ids, w, part, experts, total;
};

nvfp4_moe_desc ep_local_desc(const nvfp4_moe_desc &d, int world) {
  nvfp4_moe_desc l = d;
  l.num_experts = d.num_experts / world;
  l.top_k = 1;  // the expert pass takes one expert id per row
  return l;
}

EpP2pLayout ep_p2p_layout(const nvfp4_moe_desc &d, int world, int64_t T) {
  EpP2pLayout L;
  const int64_t R = T * d.top_k;
  size_t o = 0;
  L.ids = o;
  o = up(o + sizeof(int32_t) * R);
  L.w = o;
  o = up(o + sizeof(float) * R);
  L.part = o;
  o = up(o + sizeof(float) * T * d.num_experts * router_slices((int)T, d.hidden, d.num_experts));
  L.experts = o;
  o = up(o + experts_layout(ep_local_desc(d, world), (int64_t)world * R).total);
  L.total = o;
  return L;
}

int check_ep_desc(const nvfp4_moe_desc *d, const nvfp4_ep_peers *p) {
  int rc = check_desc(d);
  if (rc) return rc;
  if (!p || p->world < 1 || p->world > NVFP4_EP_MAX_WORLD)
    return fail(NVFP4_ERR_INVALID_ARG, "null peer table or bad world size");
  if (d->num_experts % p->world)
    return fail(NVFP4_ERR_INVALID_ARG, "num_experts %d not divisible by world %d", d->num_experts,
                p->world);
  if (p->hidden != d->hidden)
    return fail(NVFP4_ERR_INVALID_ARG, "peer windows sized for hidden %d, layer has %d",
                p->hidden, d->hidden);
  return NVFP4_OK;
}

}  // namespace
}  // namespace nvfp4

extern "C" size_t nvfp4_ep_p2p_workspace_size(const nvfp4_moe_desc *d, const nvfp4_ep_peers *p,
                                              int64_t T) {
  if (check_ep_desc(d, p) || T < 0 || T > p->max_rows / d->top_k) return 0;
  return ep_p2p_layout(*d, p->world, T).total;
}

extern "C" int nvfp4_ep_p2p_forward(const nvfp4_moe_desc *d, const nvfp4_moe_weights *local,
                                    const nvfp4_ep_peers *p, const void *x, const void *residual,
                                    void *y, int y_dtype, int64_t T, void *ws, size_t ws_bytes,
                                    void *stream) {
  NVFP4_ABI_RANGE();
  int rc = check_ep_desc(d, p);
  if (rc) return rc;
  if ((rc = check_weights(local))) return rc;
  if (!local->router) return fail(NVFP4_ERR_INVALID_ARG, "null router pointer");
  if (T < 0 || T > p->max_rows / d->top_k)
    return fail(NVFP4_ERR_INVALID_ARG, "bad token count for the windows' capacity");
  if ((T > 0 && (!x || !y)) || !ws)
    return fail(NVFP4_ERR_INVALID_ARG, "null activation, output or workspace");
  if (!aligned(x, 16) || !aligned(y, 16) || (residual && !aligned(residual, 16)) ||
      !aligned(ws, kAlign))
    return fail(NVFP4_ERR_INVALID_ARG, "x/y/residual must be 16-byte and workspace 256-byte aligned");
  const EpP2pLayout L = ep_p2p_layout(*d, p->world, T);
  if (ws_bytes < L.total)
    return fail(NVFP4_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", ws_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *base = static_cast<uint8_t *>(ws);
  int32_t *ids = reinterpret_cast<int32_t *>(base + L.ids);
  float *tw = reinterpret_cast<float *>(base + L.w);
  const int epr = d->num_experts / p->world, k = d->top_k;
  // Every rank takes every step, also with no tokens: the peers wait on its
  // flags.  Seven launches: router logits; top-k + dispatch + the wait for
  // every rank's dispatch; the expert pass (permutation, gate_up, down); the
  // done signal; the combine.
  float *part = reinterpret_cast<float *>(base + L.part);
  int nslices = 1;
  if (T > 0) {
    rc = check_launch(launch_router_logits(static_cast<const uint16_t *>(x), local->router, part,
                                           router_slices((int)T, d->hidden, d->num_experts),
                                           (int)T, d->hidden, d->num_experts, st, &nslices),
                      "router launch");
    if (rc) return rc;
  }
  // One rank: the expert pass reads the token rows from x (slot s = token
  // s / k) and the dispatch stores only the slots' expert ids.
  const bool one_rank = p->world == 1;
  if ((rc = ep_p2p_topk_dispatch(p, static_cast<const uint16_t *>(x), part, nslices, T, k,
                                 d->renormalize, epr, ids, tw, true, !one_rank, st)))
    return rc;
  void *recv_x = nullptr;
  int32_t *recv_e = nullptr;
  float *out = nullptr;
  if ((rc = nvfp4_ep_p2p_rows(p, T, k, &recv_x, &recv_e, &out))) return rc;
  rc = run_experts(ep_local_desc(*d, p->world), *local,
                   static_cast<const uint16_t *>(one_rank ? x : recv_x), nullptr, one_rank ? k : 1,
                   recv_e, (int64_t)p->world * T * k, out, kF32, base + L.experts, st);
  if (rc) return rc;
  if ((rc = nvfp4_ep_p2p_signal_done(p, stream))) return rc;
  return nvfp4_ep_p2p_combine(p, ids, tw, T, k, epr, residual, y, y_dtype, stream);
}

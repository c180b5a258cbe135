// deltanet.cu -- gated DeltaNet decode step with NVFP4 projections
// (include/nvfp4_deltanet.h; the reference's deltanet_forward,
// nvfp4/deltanet.mojo:335-546).
//
//   projections  qkv, z, beta, alpha: nvfp4_linear_forward (M = B sequences)
//   dn_conv      causal conv1d (:287-328) + SiLU (:471-479) per channel,
//                one thread per (sequence, channel); shifts the window
//   dn_recur     one CTA per (value head, sequence): beta, decay (:481-494),
//                S^T k, delta rule, state update, S^T q (:509-532), RMS norm
//                and SiLU gate (:534-541); the head's kd x vd state slice
//                stays in registers between the two passes over it
//   projection   out: nvfp4_linear_forward
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include <cooperative_groups.h>

#include "../../include/nvfp4.h"
#include "../../include/nvfp4_deltanet.h"
#include "abi_util.h"

namespace nvfp4 {
namespace {

constexpr size_t kDnAlign = 256;
size_t dn_up(size_t v) { return (v + kDnAlign - 1) & ~(kDnAlign - 1); }

// The reference's scalar functions (nvfp4/deltanet.mojo:55-80), fp32.
__device__ __forceinline__ float dn_sigmoid(float x) {
  if (x >= 0.0f) {
    const float e = expf(-x);
    return 1.0f / (1.0f + e);
  }
  const float e = expf(x);
  return e / (1.0f + e);
}
__device__ __forceinline__ float dn_silu(float x) { return x * dn_sigmoid(x); }
__device__ __forceinline__ float dn_softplus(float x) {
  if (x > 20.0f) return x;
  if (x < -20.0f) return 0.0f;
  return logf(1.0f + expf(x));
}

struct DnDims {
  int d, nkh, nvh, kd, vd, ck, vg, q_dim, k_dim, v_dim, qkv_dim, z_dim;
};

DnDims dims_of(const nvfp4_deltanet_desc &s) {
  DnDims d;
  d.d = s.d_model;
  d.nkh = s.num_key_heads;
  d.nvh = s.num_value_heads;
  d.kd = s.key_dim;
  d.vd = s.value_dim;
  d.ck = s.conv_kernel;
  d.vg = s.num_value_heads / s.num_key_heads;
  d.q_dim = d.nkh * d.kd;
  d.k_dim = d.nkh * d.kd;
  d.v_dim = d.nvh * d.vd;
  d.qkv_dim = d.q_dim + d.k_dim + d.v_dim;
  d.z_dim = d.nvh * d.vd;
  return d;
}

struct DnLayout {
  size_t hx, qkv, z, braw, araw, post, og, total;
};

DnLayout dn_layout(const DnDims &d, int64_t B) {
  DnLayout L;
  size_t o = 0;
  L.hx = o;
  o = dn_up(o + 4 * (size_t)B * d.d);
  // qkv .. araw also hold the fused projection's [B, qkv + z + 2 nvh] output.
  L.qkv = o;
  o = dn_up(o + 4 * (size_t)B * d.qkv_dim);
  L.z = o;
  o = dn_up(o + 4 * (size_t)B * d.z_dim);
  L.braw = o;
  o = dn_up(o + 4 * (size_t)B * d.nvh);
  L.araw = o;
  o = dn_up(o + 4 * (size_t)B * d.nvh);
  o = std::max(o, dn_up(L.qkv + 4 * (size_t)B * (d.qkv_dim + d.z_dim + 2 * d.nvh)));
  L.post = o;
  o = dn_up(o + 4 * (size_t)B * d.qkv_dim);
  L.og = o;
  o = dn_up(o + 4 * (size_t)B * d.z_dim);
  L.total = o;
  return L;
}

__global__ void dn_convert_kernel(const void *in, int in_dt, void *out, int out_dt, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = in_dt == NVFP4_DTYPE_F32
                      ? static_cast<const float *>(in)[i]
                      : __bfloat162float(static_cast<const __nv_bfloat16 *>(in)[i]);
  if (out_dt == NVFP4_DTYPE_F32)
    static_cast<float *>(out)[i] = v;
  else
    static_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(v);
}

struct ConvArgs {
  const float *qkv;  // [B, qkv_ld] projection output (qkv_dim columns used)
  int64_t qkv_ld;
  float *post;       // [B, qkv_dim] conv + SiLU
  float *buf[3];     // windows of q, k, v: [B, dim, ck - 1]
  const float *w[3], *bias[3];
  int dim[3], qkv_dim, ck;
  int64_t n;  // B * qkv_dim
};

// conv1d_step (nvfp4/deltanet.mojo:287-328) then SiLU, one thread per
// (sequence, channel): the window of that channel is read, then shifted.
// Launched with programmatic dependent launch after the input projection:
// the window (last written by this layer's previous step, which completed
// before that projection could start) and the weights are read before
// griddepcontrol.wait, the projection's output after it (L2-coherent).
__global__ void dn_conv_kernel(ConvArgs a) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < a.n;
  const int64_t b = live ? i / a.qkv_dim : 0;
  int ch = live ? (int)(i - b * a.qkv_dim) : 0, seg = 0;
  if (ch >= a.dim[0]) {
    ch -= a.dim[0];
    seg = 1;
    if (ch >= a.dim[1]) {
      ch -= a.dim[1];
      seg = 2;
    }
  }
  // Selects, not indexing: a runtime index into the parameter arrays would
  // copy them to local memory.
  const int dim = seg == 0 ? a.dim[0] : seg == 1 ? a.dim[1] : a.dim[2];
  float *const sbuf = seg == 0 ? a.buf[0] : seg == 1 ? a.buf[1] : a.buf[2];
  const float *const sw = seg == 0 ? a.w[0] : seg == 1 ? a.w[1] : a.w[2];
  const float *const sbias = seg == 0 ? a.bias[0] : seg == 1 ? a.bias[1] : a.bias[2];
  const int hist = a.ck - 1;
  float *buf = sbuf + (b * dim + ch) * hist;
  const float *w = sw + (int64_t)ch * a.ck;
  float acc = 0.0f, wl = 0.0f, hb[8];  // conv_kernel <= 8: hist <= 7
  if (live) {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (t < hist) {
        hb[t] = __ldcg(buf + t);
        acc = __fadd_rn(acc, __fmul_rn(hb[t], w[t]));
      }
    }
    wl = w[hist];
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!live) return;
  const float x = __ldcg(a.qkv + b * a.qkv_ld + (i - b * a.qkv_dim));
  acc = __fadd_rn(acc, __fmul_rn(x, wl));
  if (sbias) acc = __fadd_rn(acc, sbias[ch]);
  a.post[i] = dn_silu(acc);
#pragma unroll
  for (int t = 0; t < 7; ++t)
    if (t + 1 < hist) buf[t] = hb[t + 1];
  if (hist > 0) buf[hist - 1] = x;
}

struct RecurArgs {
  const float *post;  // [B, qkv_dim]: q | k | v after conv + SiLU
  const float *z;     // [B, z_ld] (z_dim columns used)
  const float *braw, *araw;  // [B, ba_ld] (nvh columns used)
  int64_t z_ld, ba_ld;
  int nsplit;         // CTAs (a cluster) per value head, each vd / nsplit columns
  const float *a_log, *dt_bias;
  float *s;           // [B, nvh, kd, vd]
  void *og;           // [B, z_dim] gated output (og_dt)
  int og_dt;
  int nvh, kd, vd, vg, q_dim, k_dim, qkv_dim, z_dim, rg;
  float eps;
};

// A cluster of NS CTAs per (value head h, sequence b), CTA `part` owning
// the vl = vd / NS columns [part vl, (part + 1) vl) of the head's state
// S[kd][vd]: the delta rule and both passes over S are per column, only the
// head's RMS norm needs all columns (partial sums of squares, added in rank
// order through distributed shared memory).  Thread (group g, column cl) of
// the CTA's vl x RG threads holds rows r = g, g + RG, ... of its column in
// registers (kd = vd = 128: NS = 4, RG = 16, 8 rows per thread).
// STRIDE: RG * vd when known at compile time (row offsets become
// immediates), else 0.
template <int RPT, int STRIDE>
__global__ void __launch_bounds__(512) dn_recur_kernel(RecurArgs a) {
  namespace cg = cooperative_groups;
  __shared__ float sq[256], sk[256], red[512], vec[256];
  __shared__ float scal[3];  // beta, decay, this CTA's sum of squares
  const int NS = a.nsplit;
  const int part = blockIdx.x % NS, h = blockIdx.x / NS, b = blockIdx.y;
  const int vd = a.vd, vl = vd / NS, kd = a.kd, RG = a.rg;
  const int cl = threadIdx.x % vl, g = threadIdx.x / vl, c = part * vl + cl;
  const int kh = h / a.vg;
  // Launched with programmatic dependent launch after the conv kernel: the
  // state (last written by this layer's previous step, complete before the
  // conv kernel could start) is loaded before griddepcontrol.wait, the
  // outputs of the conv kernel and of the input projection after it.
  // Row r = g + i RG of column c sits at S + r vd + c: one pointer, one stride.
  float *const Sg = a.s + ((int64_t)b * a.nvh + h) * kd * vd + (int64_t)g * vd + c;
  const int stride = STRIDE ? STRIDE : RG * vd;
  float s[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) s[i] = g + i * RG < kd ? __ldcg(Sg + i * stride) : 0.0f;
  const float a_log = a.a_log[h], dt_bias = a.dt_bias[h];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const float *row = a.post + (int64_t)b * a.qkv_dim;
  for (int r = threadIdx.x; r < kd; r += blockDim.x) {
    sq[r] = __ldcg(row + kh * kd + r);
    sk[r] = __ldcg(row + a.q_dim + kh * kd + r);
  }
  if (threadIdx.x == 0) {
    const float braw = __ldcg(a.braw + (int64_t)b * a.ba_ld + h);
    const float araw = __ldcg(a.araw + (int64_t)b * a.ba_ld + h);
    scal[0] = dn_sigmoid(braw);  // beta (:484-487)
    const float a_val = dn_softplus(a_log);
    const float dt_val = dn_softplus(__fadd_rn(araw, dt_bias));
    scal[1] = expf(-__fmul_rn(a_val, dt_val));  // decay (:489-494)
  }
  __syncthreads();
  // S^T k (:512), partial over this thread's rows, then over the groups.
  float p = 0.0f;
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = g + i * RG;
    if (r < kd) p = __fadd_rn(p, __fmul_rn(s[i], sk[r]));
  }
  red[threadIdx.x] = p;
  __syncthreads();
  if (g == 0) {
    float stk = 0.0f;
    for (int q = 0; q < RG; ++q) stk = __fadd_rn(stk, red[q * vl + cl]);
    const float v = __ldcg(row + a.q_dim + a.k_dim + h * vd + c);
    vec[cl] = __fadd_rn(v, -stk);  // v - S^T k (:515-516)
  }
  __syncthreads();
  // S = decay * S + beta * k outer (v - S^T k) (:519-526), then S^T q (:529).
  const float beta = scal[0], decay = scal[1], vcc = vec[cl];
  p = 0.0f;
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = g + i * RG;
    if (r < kd) {
      const float nv = __fadd_rn(__fmul_rn(decay, s[i]), __fmul_rn(__fmul_rn(beta, sk[r]), vcc));
      Sg[i * stride] = nv;
      p = __fadd_rn(p, __fmul_rn(nv, sq[r]));
    }
  }
  __syncthreads();  // red and vec are reused
  red[threadIdx.x] = p;
  __syncthreads();
  float o = 0.0f;
  if (g == 0) {
    for (int q = 0; q < RG; ++q) o = __fadd_rn(o, red[q * vl + cl]);
    vec[cl] = __fmul_rn(o, o);
  }
  __syncthreads();
  // rms_norm_inplace (:270-284) over the head's vd outputs, then the gate (:537-541).
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int q = 0; q < vl; ++q) ss = __fadd_rn(ss, vec[q]);
    scal[2] = ss;
  }
  float total;
  if (NS > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every part's sum of squares is in place
    total = 0.0f;
    for (int q = 0; q < NS; ++q) total = __fadd_rn(total, *cluster.map_shared_rank(&scal[2], q));
    cluster.sync();  // no part leaves while another may still read its sum
  } else {
    __syncthreads();
    total = scal[2];
  }
  const float scale = 1.0f / sqrtf(__fadd_rn(total / (float)vd, a.eps));
  if (g == 0) {
    const float zc = __ldcg(a.z + (int64_t)b * a.z_ld + h * vd + c);
    const float out = __fmul_rn(dn_silu(zc), __fmul_rn(o, scale));
    const int64_t idx = (int64_t)b * a.z_dim + h * vd + c;
    if (a.og_dt == NVFP4_DTYPE_F32)
      static_cast<float *>(a.og)[idx] = out;
    else
      static_cast<__nv_bfloat16 *>(a.og)[idx] = __float2bfloat16_rn(out);
  }
}

int run_proj(const nvfp4_deltanet_proj &p, int64_t in_f, int64_t out_f, const void *x, int x_dt,
             void *y, int y_dt, int64_t B, cudaStream_t st) {
  nvfp4_linear_desc L;
  L.in_features = in_f;
  L.out_features = out_f;
  L.input_scale = p.input_scale;
  L.weight_scale_2 = p.weight_scale_2;
  L.weight_scale_2_rows = p.weight_scale_2_rows;
  return nvfp4_linear_forward(&L, p.packed_weights, p.blockscales, x, x_dt, y, y_dt, B, 0u, st);
}

int check_dn_desc(const nvfp4_deltanet_desc *s) {
  if (!s) return fail(NVFP4_ERR_INVALID_ARG, "null DeltaNet descriptor");
  const bool pow2 = s->value_dim >= 4 && s->value_dim <= 256 && (s->value_dim & (s->value_dim - 1)) == 0;
  if (s->d_model <= 0 || s->d_model % 16 || s->num_key_heads <= 0 ||
      s->num_value_heads <= 0 || s->num_value_heads % s->num_key_heads || s->key_dim <= 0 ||
      s->key_dim > 256 || !pow2 || s->conv_kernel < 1 || s->conv_kernel > 8 ||
      (s->num_value_heads * s->value_dim) % 16 || !(s->rms_eps >= 0.0f))
    return fail(NVFP4_ERR_INVALID_ARG,
                "bad DeltaNet shape (d_model % 16, value heads a multiple of key heads, "
                "key_dim <= 256, value_dim a power of two in [4, 256], conv kernel 1..8)");
  return NVFP4_OK;
}

template <int RPT, int STRIDE>
cudaError_t launch_recur_cfg(const RecurArgs &a, int B, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nvh * a.nsplit, B, 1);
  cfg.blockDim = dim3((a.vd / a.nsplit) * a.rg, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.nsplit;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.nsplit > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, dn_recur_kernel<RPT, STRIDE>, a);
}

template <int RPT>
cudaError_t launch_recur(const RecurArgs &a, int B, cudaStream_t st) {
  if constexpr (RPT == 8) {
    if (a.kd == 128 && a.vd == 128 && a.nsplit == 4 && a.rg == 16)
      return launch_recur_cfg<8, 16 * 128>(a, B, st);
  }
  return launch_recur_cfg<RPT, 0>(a, B, st);
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" size_t nvfp4_deltanet_workspace_size(const nvfp4_deltanet_desc *desc, int64_t B) {
  if (check_dn_desc(desc) || B < 0) return 0;
  return dn_layout(dims_of(*desc), B).total;
}

extern "C" int nvfp4_deltanet_forward(const nvfp4_deltanet_desc *desc,
                                      const nvfp4_deltanet_weights *w, const void *hidden,
                                      int hidden_dt, void *output, int out_dt, int64_t B,
                                      const nvfp4_deltanet_state *state, int proj_dt, void *ws,
                                      size_t ws_bytes, void *stream) {
  NVFP4_ABI_RANGE();
  int rc = check_dn_desc(desc);
  if (rc) return rc;
  if (!w || !state) return fail(NVFP4_ERR_INVALID_ARG, "null weights or state");
  if (B < 0 || B > (1 << 16)) return fail(NVFP4_ERR_INVALID_ARG, "bad sequence count");
  if (B == 0) return NVFP4_OK;
  auto dt_ok = [](int t) { return t == NVFP4_DTYPE_F32 || t == NVFP4_DTYPE_BF16; };
  if (!dt_ok(hidden_dt) || !dt_ok(out_dt) || !dt_ok(proj_dt))
    return fail(NVFP4_ERR_INVALID_ARG, "bad dtype");
  if (!hidden || !output || !ws || !aligned(ws, kDnAlign))
    return fail(NVFP4_ERR_INVALID_ARG, "null buffers or workspace not 256-byte aligned");
  if (!w->a_log || !w->dt_bias || !w->conv_q || !w->conv_k || !w->conv_v || !state->s ||
      (desc->conv_kernel > 1 && (!state->conv_q || !state->conv_k || !state->conv_v)))
    return fail(NVFP4_ERR_INVALID_ARG, "null DeltaNet weight or state pointer");
  const bool any_bias = w->conv_bias_q || w->conv_bias_k || w->conv_bias_v;
  if (any_bias && !(w->conv_bias_q && w->conv_bias_k && w->conv_bias_v))
    return fail(NVFP4_ERR_INVALID_ARG, "conv biases: all three or none (:378)");
  const DnDims d = dims_of(*desc);
  const DnLayout L = dn_layout(d, B);
  if (ws_bytes < L.total)
    return fail(NVFP4_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", ws_bytes, L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *base = static_cast<uint8_t *>(ws);
  float *qkv = reinterpret_cast<float *>(base + L.qkv);
  float *z = reinterpret_cast<float *>(base + L.z);
  float *braw = reinterpret_cast<float *>(base + L.braw);
  float *araw = reinterpret_cast<float *>(base + L.araw);
  float *post = reinterpret_cast<float *>(base + L.post);
  void *og = base + L.og;

  // Step 1 (:404-426): projections of the hidden state in the projection dtype.
  const void *hx = hidden;
  if (hidden_dt != proj_dt) {
    const int64_t n = B * d.d;
    dn_convert_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(hidden, hidden_dt,
                                                                   base + L.hx, proj_dt, n);
    if ((rc = check_launch(cudaGetLastError(), "DeltaNet input conversion"))) return rc;
    hx = base + L.hx;
  }
  // One GEMV over the fused rows [qkv; z; b; a] when given, else four.
  int64_t qkv_ld = d.qkv_dim, z_ld = d.z_dim, ba_ld = d.nvh;
  if (w->in_proj.packed_weights) {
    const int64_t rows = (int64_t)d.qkv_dim + d.z_dim + 2 * d.nvh;
    float *all = qkv;  // [B, rows] in the (contiguous) qkv .. araw regions
    if ((rc = run_proj(w->in_proj, d.d, rows, hx, proj_dt, all, NVFP4_DTYPE_F32, B, st))) return rc;
    qkv_ld = z_ld = ba_ld = rows;
    z = all + d.qkv_dim;
    braw = all + d.qkv_dim + d.z_dim;
    araw = braw + d.nvh;
  } else {
    if ((rc = run_proj(w->qkv, d.d, d.qkv_dim, hx, proj_dt, qkv, NVFP4_DTYPE_F32, B, st))) return rc;
    if ((rc = run_proj(w->z, d.d, d.z_dim, hx, proj_dt, z, NVFP4_DTYPE_F32, B, st))) return rc;
    if ((rc = run_proj(w->b, d.d, d.nvh, hx, proj_dt, braw, NVFP4_DTYPE_F32, B, st))) return rc;
    if ((rc = run_proj(w->a, d.d, d.nvh, hx, proj_dt, araw, NVFP4_DTYPE_F32, B, st))) return rc;
  }

  // Steps 2-3 (:431-479): causal conv1d + SiLU, windows shifted.
  ConvArgs ca;
  ca.qkv = qkv;
  ca.qkv_ld = qkv_ld;
  ca.post = post;
  ca.buf[0] = state->conv_q;
  ca.buf[1] = state->conv_k;
  ca.buf[2] = state->conv_v;
  ca.w[0] = w->conv_q;
  ca.w[1] = w->conv_k;
  ca.w[2] = w->conv_v;
  ca.bias[0] = w->conv_bias_q;
  ca.bias[1] = w->conv_bias_k;
  ca.bias[2] = w->conv_bias_v;
  ca.dim[0] = d.q_dim;
  ca.dim[1] = d.k_dim;
  ca.dim[2] = d.v_dim;
  ca.qkv_dim = d.qkv_dim;
  ca.ck = d.ck;
  ca.n = B * d.qkv_dim;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((ca.n + 255) / 256), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if ((rc = check_launch(cudaLaunchKernelEx(&cfg, dn_conv_kernel, ca), "DeltaNet conv launch")))
      return rc;
  }

  // Steps 4-5 (:481-541): the recurrence per (value head, sequence).
  RecurArgs ra;
  ra.post = post;
  ra.z = z;
  ra.braw = braw;
  ra.araw = araw;
  ra.z_ld = z_ld;
  ra.ba_ld = ba_ld;
  ra.a_log = w->a_log;
  ra.dt_bias = w->dt_bias;
  ra.s = state->s;
  ra.og = og;
  ra.og_dt = proj_dt;
  ra.nvh = d.nvh;
  ra.kd = d.kd;
  ra.vd = d.vd;
  ra.vg = d.vg;
  ra.q_dim = d.q_dim;
  ra.k_dim = d.k_dim;
  ra.qkv_dim = d.qkv_dim;
  ra.z_dim = d.z_dim;
  ra.eps = desc->rms_eps;
  // vd >= 64: clusters of vd / 32 CTAs of 32 columns each (at most 8).
  ra.nsplit = d.vd >= 64 ? std::min(8, d.vd / 32) : 1;
  const int vl = d.vd / ra.nsplit;
  ra.rg = std::min(d.kd, 512 / vl);  // vl x rg threads, up to 512
  const int rpt = (d.kd + ra.rg - 1) / ra.rg;
  cudaError_t e;
  if (rpt <= 1) e = launch_recur<1>(ra, (int)B, st);
  else if (rpt <= 2) e = launch_recur<2>(ra, (int)B, st);
  else if (rpt <= 4) e = launch_recur<4>(ra, (int)B, st);
  else if (rpt <= 8) e = launch_recur<8>(ra, (int)B, st);
  else if (rpt <= 16) e = launch_recur<16>(ra, (int)B, st);
  else if (rpt <= 32) e = launch_recur<32>(ra, (int)B, st);
  else if (rpt <= 64) e = launch_recur<64>(ra, (int)B, st);
  else e = launch_recur<128>(ra, (int)B, st);  // kd <= 256 and rg >= 2: rpt <= 128
  if ((rc = check_launch(e, "DeltaNet recurrence launch"))) return rc;

  // Step 6 (:543-546): output projection.
  return run_proj(w->out, d.z_dim, d.d, og, proj_dt, output, out_dt, B, st);
}

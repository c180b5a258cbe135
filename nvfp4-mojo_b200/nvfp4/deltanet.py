"""Mirror of nvfp4/deltanet.mojo: the activation helpers, the NVFP4 matvec
and the gated DeltaNet decode step with NVFP4 projections
(include/nvfp4_deltanet.h): `DeltaNetConfig`, a device `DeltaNetState` for B
sequences, `DeltaNetWeights` and `deltanet_forward`.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .config import NvFp4Linear
from .nvfp4_gemm_gpu import _dev, _stream, _u8, make_desc


def sigmoid(x: float) -> float:
    """nvfp4/deltanet.mojo:66-74 (sign-split form)."""
    if x >= 0.0:
        e = math.exp(-x)
        return 1.0 / (1.0 + e)
    e = math.exp(x)
    return e / (1.0 + e)


def silu(x: float) -> float:
    """nvfp4/deltanet.mojo:77-80."""
    return x * sigmoid(x)


def nvfp4_matvec(linear: NvFp4Linear, packed_weights: torch.Tensor, blockscales: torch.Tensor,
                 input_vec: torch.Tensor, result: torch.Tensor, stream=None) -> None:
    """nvfp4/deltanet.mojo:549-584: result = alpha * dequant(W) @ input_vec.

    fp32 input [in_features], fp32 result [out_features], on the GPU.
    """
    L = _lib.load()
    if input_vec.dtype != torch.float32 or result.dtype != torch.float32:
        raise TypeError("nvfp4_matvec takes fp32 input and result")
    if input_vec.numel() != linear.in_features or result.numel() != linear.out_features:
        raise ValueError("vector sizes do not match the linear's shape")
    desc = make_desc(linear)
    rc = L.nvfp4_matvec(ctypes.byref(desc), _dev(_u8(packed_weights), "packed_weights"),
                        _dev(_u8(blockscales), "blockscales"), _dev(input_vec, "input_vec"),
                        _dev(result, "result"), _stream(stream))
    _lib.check(rc)


def softplus(x: float) -> float:
    """nvfp4/deltanet.mojo:55-63."""
    if x > 20.0:
        return x
    if x < -20.0:
        return 0.0
    return math.log(1.0 + math.exp(x))


@dataclass
class DeltaNetConfig:
    """struct DeltaNetConfig (nvfp4/deltanet.mojo:87-178); the defaults are
    the reference's (Qwen3.5-35B-A3B DeltaNet layers, :42-48)."""

    d_model: int = 2048
    num_key_heads: int = 16
    num_value_heads: int = 32
    key_dim: int = 128
    value_dim: int = 128
    conv_kernel: int = 4
    rms_eps: float = 1e-6

    def v_groups(self) -> int:
        return self.num_value_heads // self.num_key_heads

    def state_size_per_head(self) -> int:
        return self.key_dim * self.value_dim

    def total_state_floats(self) -> int:
        return self.num_value_heads * self.key_dim * self.value_dim

    def total_qkv_dim(self) -> int:
        return 2 * self.num_key_heads * self.key_dim + self.num_value_heads * self.value_dim

    def q_dim(self) -> int:
        return self.num_key_heads * self.key_dim

    def k_dim(self) -> int:
        return self.num_key_heads * self.key_dim

    def v_dim(self) -> int:
        return self.num_value_heads * self.value_dim

    def z_dim(self) -> int:
        return self.num_value_heads * self.value_dim

    def desc(self) -> "_lib.DeltaNetDesc":
        return _lib.DeltaNetDesc(self.d_model, self.num_key_heads, self.num_value_heads,
                                 self.key_dim, self.value_dim, self.conv_kernel, self.rms_eps)


class DeltaNetState:
    """struct DeltaNetState (nvfp4/deltanet.mojo:181-218) for `batch`
    sequences, fp32 on the device, zero-initialised: s [B, nvh, kd, vd] and
    the conv windows [B, dim, conv_kernel - 1] (oldest first)."""

    def __init__(self, config: DeltaNetConfig, batch: int = 1, device="cuda"):
        c = config
        hist = c.conv_kernel - 1
        z = lambda *shape: torch.zeros(shape, dtype=torch.float32, device=device)
        self.config, self.batch = c, batch
        self.s_matrix = z(batch, c.num_value_heads, c.key_dim, c.value_dim)
        self.conv_buf_q = z(batch, c.q_dim(), hist)
        self.conv_buf_k = z(batch, c.k_dim(), hist)
        self.conv_buf_v = z(batch, c.v_dim(), hist)

    def ptrs(self) -> "_lib.DeltaNetStatePtrs":
        return _lib.DeltaNetStatePtrs(self.s_matrix.data_ptr(), self.conv_buf_q.data_ptr(),
                                      self.conv_buf_k.data_ptr(), self.conv_buf_v.data_ptr())


def _proj(lin: NvFp4Linear, w: torch.Tensor, sf: torch.Tensor) -> "_lib.DeltaNetProj":
    rows = lin.weight_scale_2_rows
    return _lib.DeltaNetProj(_dev(_u8(w), "packed_weights"), _dev(_u8(sf), "blockscales"),
                             float(lin.input_scale), float(lin.weight_scale_2),
                             None if rows is None else _dev(rows, "weight_scale_2_rows"))


@dataclass
class DeltaNetWeights:
    """The weights of deltanet_forward (nvfp4/deltanet.mojo:335-352) with the
    five projections in NVFP4: each a (NvFp4Linear, packed weights,
    blockscales) triple; the small fp32 tensors on the device."""

    qkv: tuple
    z: tuple
    b: tuple
    a: tuple
    out: tuple
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    conv_q: torch.Tensor
    conv_k: torch.Tensor
    conv_v: torch.Tensor
    conv_bias_q: Optional[torch.Tensor] = None
    conv_bias_k: Optional[torch.Tensor] = None
    conv_bias_v: Optional[torch.Tensor] = None
    in_proj: Optional[tuple] = None  # rows [qkv; z; b; a] fused (fuse_in_proj)

    def ptrs(self) -> "_lib.DeltaNetWeightPtrs":
        f = lambda t, n: None if t is None else _dev(t, n)
        return _lib.DeltaNetWeightPtrs(
            _proj(*self.qkv), _proj(*self.z), _proj(*self.b), _proj(*self.a), _proj(*self.out),
            _proj(*self.in_proj) if self.in_proj is not None else _lib.DeltaNetProj(),
            f(self.a_log, "a_log"), f(self.dt_bias, "dt_bias"), f(self.conv_q, "conv_q"),
            f(self.conv_k, "conv_k"), f(self.conv_v, "conv_v"),
            f(self.conv_bias_q, "conv_bias_q"), f(self.conv_bias_k, "conv_bias_k"),
            f(self.conv_bias_v, "conv_bias_v"))


def fuse_in_proj(weights: DeltaNetWeights, stream=None) -> DeltaNetWeights:
    """The same weights with the qkv, z, b and a projections row-stacked into
    one NVFP4 matrix (nvfp4_stack_rows), so a step takes one input
    projection launch instead of four.  The four must share input_scale;
    their per-row weight_scale_2 are stacked (scalar ones broadcast)."""
    from .moe import stack_rows

    parts = [weights.qkv, weights.z, weights.b, weights.a]
    ins = {float(p[0].input_scale) for p in parts}
    if len(ins) != 1:
        raise ValueError("the fused projection needs one input_scale")
    K = parts[0][0].in_features
    rows = []
    for lin, _, _ in parts:
        r = lin.weight_scale_2_rows
        rows.append(r if r is not None else
                    torch.full((lin.out_features,), float(lin.weight_scale_2),
                               dtype=torch.float32, device=parts[0][1].device))
    w = stack_rows([p[1] for p in parts], stream=stream)
    sf = stack_rows([_u8(p[2]) for p in parts], stream=stream)
    ws2 = stack_rows(rows, stream=stream)
    lin = NvFp4Linear(K, w.shape[0], input_scale=ins.pop(), weight_scale_2_rows=ws2)
    from dataclasses import replace

    return replace(weights, in_proj=(lin, w, sf))


_DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def deltanet_forward(hidden: torch.Tensor, output: torch.Tensor, weights: DeltaNetWeights,
                     state: DeltaNetState, config: DeltaNetConfig,
                     proj_dtype=torch.bfloat16, workspace: Optional[torch.Tensor] = None,
                     stream=None) -> torch.Tensor:
    """deltanet_forward (nvfp4/deltanet.mojo:335-546) for B sequences at once:
    hidden [B, d_model] -> output [B, d_model] (bf16 or fp32), state updated
    in place.  proj_dtype: the activations of the NVFP4 projections
    (torch.float32: the reference's fp32 arithmetic; torch.bfloat16: the
    decode GEMV)."""
    L = _lib.load()
    B = hidden.shape[0] if hidden.dim() == 2 else 1
    if hidden.numel() != B * config.d_model or output.numel() != B * config.d_model:
        raise ValueError("hidden and output must hold [B, d_model] values")
    if B != state.batch:
        raise ValueError("hidden and state hold different numbers of sequences")
    desc = config.desc()
    need = L.nvfp4_deltanet_workspace_size(ctypes.byref(desc), B)
    if need == 0:
        raise ValueError("unsupported DeltaNet configuration")
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(need, dtype=torch.uint8, device=hidden.device)
    w, st = weights.ptrs(), state.ptrs()
    rc = L.nvfp4_deltanet_forward(ctypes.byref(desc), ctypes.byref(w),
                                  _dev(hidden, "hidden"), _DT[hidden.dtype],
                                  _dev(output, "output"), _DT[output.dtype], B,
                                  ctypes.byref(st), _DT[proj_dtype], _dev(ws, "workspace"),
                                  ws.numel(), _stream(stream))
    _lib.check(rc)
    return output

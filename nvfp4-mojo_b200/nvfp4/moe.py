"""NVFP4 MoE expert path over libnvfp4 (no counterpart in the reference,
which defines only the per-expert NVFP4 weight layout,
nvfp4/weight_loader.mojo:767-793 and :873-887, and SiLU,
nvfp4/deltanet.mojo:66-80).

`MoEWeights` holds the stacked expert tensors on the GPU; `moe_forward` runs
one layer (router -> top-k -> grouped gate_up with fused SiLU*up -> grouped
down -> weighted combine) entirely in CUDA kernels.  `moe_route`,
`moe_experts` and `moe_combine` are the building blocks the expert-parallel
layer (nvfp4.ep) composes around its NCCL exchange.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .nvfp4_gemm_gpu import _stream


MoEDesc = _lib.MoEDesc
MoEWeightPtrs = _lib.MoEWeightPtrs


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("MoE tensors must be contiguous CUDA tensors")
    return t.data_ptr()


@dataclass
class MoEWeights:
    """Stacked expert weights (device tensors).

    router [H, E] fp32; gate_up [E, 2I, H/2] u8 (gate rows then up rows);
    gate_up_scale [E, 2I, H/16] e4m3 bytes; gate_up_scale_2 [E, 2I] fp32;
    down [E, H, I/2] u8; down_scale [E, H, I/16]; down_scale_2 [E, H];
    optional per-expert input scales [E].
    """

    router: torch.Tensor
    gate_up: torch.Tensor
    gate_up_scale: torch.Tensor
    gate_up_scale_2: Optional[torch.Tensor]
    down: torch.Tensor
    down_scale: torch.Tensor
    down_scale_2: Optional[torch.Tensor]
    gate_up_input_scale: Optional[torch.Tensor] = None
    down_input_scale: Optional[torch.Tensor] = None

    @property
    def num_experts(self) -> int:
        return self.gate_up.shape[0]

    @property
    def hidden(self) -> int:
        return self.down.shape[1]

    @property
    def intermediate(self) -> int:
        return self.gate_up.shape[1] // 2

    def ptrs(self) -> MoEWeightPtrs:
        u8 = lambda t: None if t is None else (t.view(torch.uint8) if t.dtype != torch.uint8 else t)
        return MoEWeightPtrs(_ptr(self.router), _ptr(self.gate_up), _ptr(u8(self.gate_up_scale)),
                             _ptr(self.gate_up_scale_2), _ptr(self.gate_up_input_scale),
                             _ptr(self.down), _ptr(u8(self.down_scale)), _ptr(self.down_scale_2),
                             _ptr(self.down_input_scale))

    @classmethod
    def from_dict(cls, d, device="cuda"):
        """From the synthetic / loader dictionary (numpy or torch values)."""
        def t(v):
            if v is None:
                return None
            return (torch.as_tensor(v) if not isinstance(v, torch.Tensor) else v).to(device).contiguous()
        return cls(router=t(d["router"]), gate_up=t(d["gu_w"]), gate_up_scale=t(d["gu_sf"]),
                   gate_up_scale_2=t(d.get("gu_ws2")), down=t(d["dn_w"]),
                   down_scale=t(d["dn_sf"]), down_scale_2=t(d.get("dn_ws2")),
                   gate_up_input_scale=t(d.get("gu_in")), down_input_scale=t(d.get("dn_in")))


def make_desc(w: MoEWeights, top_k: int, renormalize: bool = True) -> MoEDesc:
    return MoEDesc(w.num_experts, top_k, w.hidden, w.intermediate, int(renormalize))


def _sig():
    return _lib.load()


def workspace_size(w: MoEWeights, top_k: int, T: int) -> int:
    L = _sig()
    return L.nvfp4_moe_workspace_size(ctypes.byref(make_desc(w, top_k)), T)


def experts_workspace_size(w: MoEWeights, top_k: int, R: int) -> int:
    L = _sig()
    return L.nvfp4_moe_experts_workspace_size(ctypes.byref(make_desc(w, top_k)), R)


class MoELayer:
    """One NVFP4 MoE FFN layer with its own reusable workspace."""

    def __init__(self, weights: MoEWeights, top_k: int = 8, renormalize: bool = True):
        self.w = weights
        self.top_k = top_k
        self.desc = make_desc(weights, top_k, renormalize)
        self.ptrs = weights.ptrs()
        self._ws = None

    def workspace(self, T: int, device) -> torch.Tensor:
        need = _sig().nvfp4_moe_workspace_size(ctypes.byref(self.desc), T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        return self._ws

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None, topk_ids: Optional[torch.Tensor] = None,
                topk_w: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.w.hidden:
            raise ValueError("x must be bf16 [T, hidden]")
        T = x.shape[0]
        y = out if out is not None else torch.empty_like(x)
        ydt = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}[y.dtype]
        ws = self.workspace(T, x.device)
        rc = _sig().nvfp4_moe_forward(ctypes.byref(self.desc), ctypes.byref(self.ptrs), _ptr(x),
                                      _ptr(residual), _ptr(y), ydt, T, _ptr(topk_ids),
                                      _ptr(topk_w), _ptr(ws), ws.numel(), _stream(stream))
        _lib.check(rc)
        return y

    __call__ = forward


def moe_forward(weights: MoEWeights, x: torch.Tensor, top_k: int = 8, renormalize: bool = True,
                residual: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    return MoELayer(weights, top_k, renormalize).forward(x, residual, stream=stream)


def moe_route(weights: MoEWeights, x: torch.Tensor, top_k: int = 8, renormalize: bool = True,
              stream=None):
    """(topk_ids int32 [T, k], topk_w fp32 [T, k], logits fp32 [T, E])."""
    T = x.shape[0]
    desc = make_desc(weights, top_k, renormalize)
    ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    tw = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    logits = torch.empty((T, weights.num_experts), dtype=torch.float32, device=x.device)
    rc = _sig().nvfp4_moe_route(ctypes.byref(desc), _ptr(weights.router), _ptr(x), T, _ptr(ids),
                                _ptr(tw), _ptr(logits), _stream(stream))
    _lib.check(rc)
    return ids, tw, logits


def moe_experts(weights: MoEWeights, x: torch.Tensor, row_expert: torch.Tensor,
                x_row_index: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                top_k: int = 8, workspace: Optional[torch.Tensor] = None,
                out_dtype=torch.float32, stream=None):
    """y_rows[r] = expert_{row_expert[r]}(x[x_row_index[r] or r]) ([R, H], fp32 or bf16)."""
    R = row_expert.numel()
    desc = make_desc(weights, top_k)
    y = out if out is not None else torch.empty((R, weights.hidden), dtype=out_dtype,
                                                device=x.device)
    ydt = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}[y.dtype]
    need = _sig().nvfp4_moe_experts_workspace_size(ctypes.byref(desc), R)
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
    ptrs = weights.ptrs()
    rc = _sig().nvfp4_moe_experts(ctypes.byref(desc), ctypes.byref(ptrs), _ptr(x),
                                  _ptr(x_row_index), _ptr(row_expert), R, _ptr(y), ydt,
                                  _ptr(ws), ws.numel(), _stream(stream))
    _lib.check(rc)
    return y


def moe_combine(y_slots: torch.Tensor, topk_w: torch.Tensor, residual=None, out=None,
                slot_pos: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    T, k = topk_w.shape
    H = y_slots.shape[-1]
    y = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16,
                                                device=y_slots.device)
    dts = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}
    rc = _sig().nvfp4_moe_combine(_ptr(y_slots), dts[y_slots.dtype], _ptr(topk_w),
                                  _ptr(slot_pos), _ptr(residual), _ptr(y), dts[y.dtype], T, k, H,
                                  _stream(stream))
    _lib.check(rc)
    return y

"""NVFP4 MoE expert path over libnvfp4 (no counterpart in the reference,
which defines only the per-expert NVFP4 weight layout,
nvfp4/weight_loader.mojo:767-793 and :873-887, and SiLU,
nvfp4/deltanet.mojo:66-80).

`MoEWeights` holds the stacked expert tensors on the GPU; `moe_forward` runs
one layer (router -> top-k -> grouped gate_up with fused SiLU*up -> grouped
down -> weighted combine) entirely in CUDA kernels; with a shared expert
(`MoELayer(shared=...)`, the reference's `mlp.shared_expert.*` linears,
nvfp4/weight_loader.mojo:881-884) its output is added to every token.
`stack_gate_up` turns separate per-expert gate_proj / up_proj linears
(nvfp4/weight_loader.mojo:876-877) into the stacked gate_up layout.  `moe_route`,
`moe_experts` and `moe_combine` are the building blocks the expert-parallel
layer (nvfp4.ep) composes around its NCCL exchange.
"""
from __future__ import annotations

import ctypes
import math
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

    router: Optional[torch.Tensor]
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
        return cls(router=t(d.get("router")), gate_up=t(d["gu_w"]), gate_up_scale=t(d["gu_sf"]),
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
    """One NVFP4 MoE FFN layer with its own reusable workspace.

    `shared` (optional): a one-expert MoEWeights (router unused) whose output
    is added, with weight 1, to every token after the routed sum.
    """

    def __init__(self, weights: MoEWeights, top_k: int = 8, renormalize: bool = True,
                 shared: Optional[MoEWeights] = None):
        self.w = weights
        self.top_k = top_k
        self.desc = make_desc(weights, top_k, renormalize)
        self.ptrs = weights.ptrs()
        self.shared = shared
        if shared is not None:
            if shared.num_experts != 1 or shared.hidden != weights.hidden:
                raise ValueError("shared expert must be one expert of the layer's hidden size")
            self.shared_ptrs = shared.ptrs()
        self._ws = None

    def workspace_bytes(self, T: int) -> int:
        if self.shared is None:
            return _sig().nvfp4_moe_workspace_size(ctypes.byref(self.desc), T)
        return _sig().nvfp4_moe_shared_workspace_size(ctypes.byref(self.desc),
                                                      self.shared.intermediate, T)

    def workspace(self, T: int, device) -> torch.Tensor:
        need = self.workspace_bytes(T)
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
        if self.shared is None:
            rc = _sig().nvfp4_moe_forward(ctypes.byref(self.desc), ctypes.byref(self.ptrs),
                                          _ptr(x), _ptr(residual), _ptr(y), ydt, T,
                                          _ptr(topk_ids), _ptr(topk_w), _ptr(ws), ws.numel(),
                                          _stream(stream))
        else:
            rc = _sig().nvfp4_moe_forward_shared(
                ctypes.byref(self.desc), ctypes.byref(self.ptrs), ctypes.byref(self.shared_ptrs),
                self.shared.intermediate, _ptr(x), _ptr(residual), _ptr(y), ydt, T,
                _ptr(topk_ids), _ptr(topk_w), _ptr(ws), ws.numel(), _stream(stream))
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


def stack_rows(parts, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Row-concatenation of `parts` (same dtype and trailing shape; CUDA or
    host tensors) into one CUDA tensor, through nvfp4_stack_rows."""
    parts = [p.contiguous() for p in parts]
    if not parts:
        raise ValueError("nothing to stack")
    tail = parts[0].shape[1:]
    if any(p.shape[1:] != tail or p.dtype != parts[0].dtype for p in parts):
        raise ValueError("parts differ in dtype or trailing shape")
    rows = [p.shape[0] for p in parts]
    row_bytes = math.prod(tail) * parts[0].element_size()
    y = out if out is not None else torch.empty((sum(rows),) + tuple(tail), dtype=parts[0].dtype,
                                                device="cuda")
    if not y.is_cuda or not y.is_contiguous() or y.shape[0] != sum(rows):
        raise ValueError("out must be a contiguous CUDA tensor of the stacked shape")
    srcs = (ctypes.c_void_p * len(parts))(*[p.data_ptr() for p in parts])
    nrows = (ctypes.c_int64 * len(parts))(*rows)
    rc = _sig().nvfp4_stack_rows(srcs, nrows, len(parts), row_bytes, _ptr(y), _stream(stream))
    _lib.check(rc)
    return y


def _row_scales(ws2, rows: int, input_scale) -> torch.Tensor:
    """Per-row weight_scale_2 [rows] fp32 with the linear's input_scale folded
    in (the expert kernels use input_scale * weight_scale_2 as one product)."""
    v = torch.as_tensor(ws2, dtype=torch.float32).reshape(-1)
    v = v.expand(rows) if v.numel() == 1 else v
    if v.numel() != rows:
        raise ValueError("weight_scale_2 is neither a scalar nor one value per row")
    if input_scale is not None:
        v = v * torch.as_tensor(input_scale, dtype=torch.float32).reshape(())
    return v.contiguous()


def stack_gate_up(gates, ups, stream=None):
    """Stacked (gate_up, gate_up_scale, gate_up_scale_2) from per-expert
    separate linears.

    gates[e], ups[e]: dicts with "w" [I, H/2] u8 codes, "sf" [I, H/16] e4m3
    bytes, "ws2" (scalar or [I] fp32) and optional "in" (input_scale scalar),
    the reference's `experts.{e}.gate_proj` / `up_proj` weights.  Expert e's
    rows are its gate rows then its up rows.  The input scales are folded
    into the per-row weight_scale_2, so gate and up may carry different ones.
    """
    if len(gates) != len(ups) or not gates:
        raise ValueError("need one gate and one up linear per expert")
    I = gates[0]["w"].shape[0]
    pairs = [t for g, u in zip(gates, ups) for t in (g, u)]
    if any(t["w"].shape[0] != I for t in pairs):
        raise ValueError("every gate/up linear must have I rows")
    E = len(gates)
    as_u8 = lambda a: torch.as_tensor(a).view(torch.uint8) if torch.is_tensor(a) and \
        a.dtype != torch.uint8 else torch.as_tensor(a)
    w = stack_rows([as_u8(t["w"]) for t in pairs], stream=stream)
    sf = stack_rows([as_u8(t["sf"]) for t in pairs], stream=stream)
    ws2 = stack_rows([_row_scales(t["ws2"], I, t.get("in")).to(w.device) for t in pairs],
                     stream=stream)
    return (w.view(E, 2 * I, w.shape[1]), sf.view(E, 2 * I, sf.shape[1]), ws2.view(E, 2 * I))

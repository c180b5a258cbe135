"""Safetensors loading of NVFP4 checkpoints, mirroring nvfp4/weight_loader.mojo
(the safetensors part) over the C++ reader of libnvfp4.so
(include/nvfp4_loader.h): the same names and argument meanings, with tensors
landing in device memory (torch CUDA tensors) instead of host lists.

    sf = open_safetensors(path)                   # :366-410
    lw = load_linear_safetensors(sf, "model.layers.0.mlp.experts.3.up_proj")
    model = open_model_shards(model_dir)          # :948-954
    experts = load_moe_experts(model, layer=0)    # stacked, for nvfp4.moe
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib
from .config import NvFp4Linear
from .nvfp4_gemm_gpu import _stream


def _L():
    return _lib.load()


@dataclass
class TensorInfo:
    """struct TensorInfo (nvfp4/weight_loader.mojo:190-238)."""

    name: str
    dtype: str
    shape: List[int]
    data_offset: int
    data_size: int

    def num_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


class SafetensorsModel:
    """The opened shards of a model (open_model_shards, :948-954): a handle
    to the C shard set; `shards[i]` are SafetensorsFile views of it."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)
        n = _L().nvfp4_st_model_num_shards(self._h)
        self.shards = [SafetensorsFile(self, i) for i in range(n)]

    @classmethod
    def from_dir(cls, model_dir: str) -> "SafetensorsModel":
        h = ctypes.c_void_p()
        _lib.check(_L().nvfp4_st_open_model(str(model_dir).encode(), ctypes.byref(h)))
        return cls(h.value)

    @classmethod
    def from_files(cls, paths: List[str]) -> "SafetensorsModel":
        arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
        h = ctypes.c_void_p()
        _lib.check(_L().nvfp4_st_open_files(arr, len(paths), ctypes.byref(h)))
        return cls(h.value)

    @property
    def paths(self) -> List[str]:
        return [_L().nvfp4_st_model_shard_path(self._h, i).decode()
                for i in range(len(self.shards))]

    def find(self, name: str) -> Tuple[int, int]:
        """(shard, tensor index) of the first shard holding `name`."""
        s, i = ctypes.c_int32(), ctypes.c_int64()
        _lib.check(_L().nvfp4_st_model_find(self._h, name.encode(), ctypes.byref(s),
                                            ctypes.byref(i)))
        return s.value, i.value

    def close(self):
        if self._h is not None and self._h.value:
            _L().nvfp4_st_close_model(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # pragma: no cover - interpreter shutdown
            pass

    def __len__(self):
        return len(self.shards)

    def __getitem__(self, i):
        return self.shards[i]


class SafetensorsFile:
    """struct SafetensorsFile (nvfp4/weight_loader.mojo:241-289): one file of
    a SafetensorsModel."""

    def __init__(self, model: SafetensorsModel, shard: int):
        self.model = model
        self.shard = shard
        self._f = ctypes.c_void_p(_L().nvfp4_st_model_shard(model._h, shard))
        self.tensors: List[TensorInfo] = []
        info = _lib.StTensorInfo()
        for i in range(_L().nvfp4_st_num_tensors(self._f)):
            _lib.check(_L().nvfp4_st_get_tensor_info(self._f, i, ctypes.byref(info)))
            self.tensors.append(TensorInfo(_L().nvfp4_st_tensor_name(self._f, i).decode(),
                                           info.dtype.decode(), list(info.shape[:info.ndim]),
                                           info.data_offset, info.data_size))

    @property
    def path(self) -> str:
        return _L().nvfp4_st_model_shard_path(self.model._h, self.shard).decode()

    def find_tensor(self, name: str) -> int:
        return _L().nvfp4_st_find(self._f, name.encode())

    def has_tensor(self, name: str) -> bool:
        return self.find_tensor(name) >= 0

    def read_tensor_bytes(self, i: int) -> np.ndarray:
        """Host bytes of tensor i (read_tensor_bytes, :279-283)."""
        out = np.empty(self.tensors[i].data_size, dtype=np.uint8)
        n = _L().nvfp4_st_read_host(self._f, i, out.ctypes.data, out.size)
        if n < 0:
            _lib.check(int(n))
        return out

    def read_tensor_into(self, i: int, dst: torch.Tensor, stream=None) -> int:
        """read_tensor_into (:285-289): into a CUDA tensor (through pinned
        staging) or a host tensor; returns the bytes read."""
        nbytes = self.tensors[i].data_size
        if not dst.is_contiguous() or dst.numel() * dst.element_size() < nbytes:
            raise ValueError("destination must be contiguous and hold the tensor's bytes")
        if dst.is_cuda:
            _lib.check(_L().nvfp4_st_read_device(self._f, i, dst.data_ptr(), _stream(stream)))
            return nbytes
        n = _L().nvfp4_st_read_host(self._f, i, dst.data_ptr(), dst.numel() * dst.element_size())
        if n < 0:
            _lib.check(int(n))
        return int(n)

    def close(self):
        self.model.close()


def open_safetensors(path: str) -> SafetensorsFile:
    """open_safetensors (nvfp4/weight_loader.mojo:366-410)."""
    return SafetensorsModel.from_files([path]).shards[0]


def read_f32_from_bytes(buf) -> float:
    """_read_f32_from_bytes (:678-700) as the C loader applies it."""
    b = np.ascontiguousarray(np.frombuffer(bytes(buf), dtype=np.uint8))
    return float(_L().nvfp4_st_f32_from_bytes(b.ctypes.data if b.size else None, b.size))


def discover_safetensor_shards(model_dir: str) -> List[str]:
    """discover_safetensor_shards (:909-945): the shard files of a model
    directory (all of them; see include/nvfp4_loader.h for where the
    reference's probe loop stops earlier)."""
    m = SafetensorsModel.from_dir(model_dir)
    try:
        return m.paths
    finally:
        m.close()


def open_model_shards(model_dir: str) -> SafetensorsModel:
    """open_model_shards (:948-954)."""
    return SafetensorsModel.from_dir(model_dir)


@dataclass
class LoadedWeight:
    """struct LoadedWeight (nvfp4/weight_loader.mojo:614-675) on the device:
    packed_weights uint8 [out, in/2], blockscales uint8 (E4M3 bytes)
    [out, in/16], scalar weight_scale_2 / input_scale, and the per-row
    second-level scales when the checkpoint stores them."""

    packed_weights: torch.Tensor
    blockscales: torch.Tensor
    weight_scale_2: float
    input_scale: float
    out_features: int
    in_features: int
    weight_scale_2_rows: Optional[torch.Tensor] = None

    def to_linear(self) -> NvFp4Linear:
        return NvFp4Linear(self.in_features, self.out_features, input_scale=self.input_scale,
                           weight_scale_2=self.weight_scale_2,
                           weight_scale_2_rows=self.weight_scale_2_rows)

    def packed_weight_bytes(self) -> int:
        return self.out_features * (self.in_features // 2)

    def blockscale_bytes(self) -> int:
        return self.out_features * (self.in_features // 16)


def _model_of(sf) -> SafetensorsModel:
    if isinstance(sf, SafetensorsModel):
        return sf
    if isinstance(sf, SafetensorsFile):
        return sf.model
    raise TypeError("expected a SafetensorsFile or a SafetensorsModel")


def linear_info(sf, prefix: str) -> "_lib.StLinearInfo":
    info = _lib.StLinearInfo()
    _lib.check(_L().nvfp4_st_get_linear_info(_model_of(sf)._h, prefix.encode(),
                                             ctypes.byref(info)))
    return info


def load_linear_safetensors(sf, prefix: str, device="cuda", stream=None) -> LoadedWeight:
    """load_linear_safetensors (:703-760) from a file, or _find_load_linear
    (:828-836) from a shard set: `{prefix}.weight`, `.weight_scale` (both
    required), `.weight_scale_2`, `.input_scale` (optional, 1.0)."""
    model = _model_of(sf)
    info = linear_info(model, prefix)
    w = torch.empty((info.out_features, info.in_features // 2), dtype=torch.uint8, device=device)
    s = torch.empty((info.out_features, info.in_features // 16), dtype=torch.uint8, device=device)
    rows = torch.empty(info.out_features, dtype=torch.float32, device=device) \
        if info.weight_scale_2_rows else None
    _lib.check(_L().nvfp4_st_load_linear(model._h, prefix.encode(), w.data_ptr(), s.data_ptr(),
                                         None if rows is None else rows.data_ptr(), 0,
                                         _stream(stream)))
    return LoadedWeight(w, s, float(info.weight_scale_2), float(info.input_scale),
                        int(info.out_features), int(info.in_features), rows)


def _find_load_linear(shards, prefix: str) -> LoadedWeight:
    """_find_load_linear (:828-836)."""
    return load_linear_safetensors(_model_of(shards), prefix)


def _find_load_raw(shards, name: str) -> np.ndarray:
    """_find_load_raw (:839-847): host bytes from the first shard holding name."""
    model = _model_of(shards)
    s, i = model.find(name)
    return model.shards[s].read_tensor_bytes(i)


def load_moe_experts(model, layer, num_experts: Optional[int] = None, first: int = 0,
                     shared: bool = False, router: bool = True, device="cuda", stream=None):
    """Experts [first, first + num_experts) of a layer as stacked nvfp4.moe
    MoEWeights (gate_up = each expert's gate_proj rows then up_proj rows,
    input scales folded into the per-row weight_scale_2), read straight into
    device memory.  `layer` is an index (model.layers.{layer}) or a prefix.
    shared=True loads the layer's shared expert (one expert, no router).
    num_experts None: all experts the router has."""
    from .moe import MoEWeights

    model = _model_of(model)
    prefix = f"model.layers.{layer}" if isinstance(layer, int) else str(layer)
    L = _L()
    router_t = None
    if not shared:
        E, H = ctypes.c_int32(), ctypes.c_int32()
        _lib.check(L.nvfp4_st_load_router(model._h, prefix.encode(), None, ctypes.byref(E),
                                          ctypes.byref(H), _stream(stream)))
        if num_experts is None:
            num_experts = E.value - first
        if router:
            router_t = torch.empty((H.value, E.value), dtype=torch.float32, device=device)
            _lib.check(L.nvfp4_st_load_router(model._h, prefix.encode(), router_t.data_ptr(),
                                              None, None, _stream(stream)))
            if first != 0 or num_experts != E.value:
                router_t = router_t[:, first:first + num_experts].contiguous()
        base = f"{prefix}.mlp.experts.{first}"
    else:
        num_experts, first = 1, 0
        base = f"{prefix}.mlp.shared_expert"
    g = linear_info(model, base + ".gate_proj")
    I, H = int(g.out_features), int(g.in_features)
    E = int(num_experts)
    u8 = dict(dtype=torch.uint8, device=device)
    gu = torch.empty((E, 2 * I, H // 2), **u8)
    gus = torch.empty((E, 2 * I, H // 16), **u8)
    gu2 = torch.empty((E, 2 * I), dtype=torch.float32, device=device)
    dn = torch.empty((E, H, I // 2), **u8)
    dns = torch.empty((E, H, I // 16), **u8)
    dn2 = torch.empty((E, H), dtype=torch.float32, device=device)
    _lib.check(L.nvfp4_st_load_experts(model._h, prefix.encode(), first, E, int(shared),
                                       gu.data_ptr(), gus.data_ptr(), gu2.data_ptr(),
                                       dn.data_ptr(), dns.data_ptr(), dn2.data_ptr(),
                                       _stream(stream)))
    return MoEWeights(router=router_t, gate_up=gu, gate_up_scale=gus, gate_up_scale_2=gu2,
                      down=dn, down_scale=dns, down_scale_2=dn2)


@dataclass
class Qwen35LayerWeights:
    """struct Qwen35LayerWeights (nvfp4/weight_loader.mojo:776-825) on the
    device: attention projections as LoadedWeight, the routed experts and
    the shared expert as stacked MoEWeights, the router as fp32 [H, E] (in
    the routed MoEWeights), the layer norms as raw host bytes."""

    q_proj: LoadedWeight
    k_proj: LoadedWeight
    v_proj: LoadedWeight
    o_proj: LoadedWeight
    experts: object
    shared_expert: object
    input_layernorm: np.ndarray
    post_attn_layernorm: np.ndarray
    extra: Dict[str, object] = field(default_factory=dict)


def load_qwen35_layer(shards, layer_idx: int, num_experts: int) -> Qwen35LayerWeights:
    """load_qwen35_layer (nvfp4/weight_loader.mojo:850-893): the same tensor
    names, loaded into device memory (experts stacked for the MoE kernels)."""
    model = _model_of(shards)
    lp = f"model.layers.{layer_idx}"
    att = {p: _find_load_linear(model, f"{lp}.self_attn.{p}")
           for p in ("q_proj", "k_proj", "v_proj", "o_proj")}
    experts = load_moe_experts(model, lp, num_experts=num_experts)
    shared = load_moe_experts(model, lp, shared=True)
    return Qwen35LayerWeights(att["q_proj"], att["k_proj"], att["v_proj"], att["o_proj"],
                              experts, shared,
                              _find_load_raw(model, f"{lp}.input_layernorm.weight"),
                              _find_load_raw(model, f"{lp}.post_attention_layernorm.weight"))

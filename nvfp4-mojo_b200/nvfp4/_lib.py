"""Loader of libnvfp4.so (the C ABI of include/nvfp4.h) via ctypes.

The shared library is built in-tree (``make -C nvfp4-mojo_b200``) and loaded
from this folder.  There is no fallback: if the library is missing or does
not load, every compute call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("NVFP4_LIB", _HERE / "libnvfp4.so"))

NVFP4_OK = 0
NVFP4_ERR_INVALID_ARG = -1
NVFP4_ERR_UNSUPPORTED = -2
NVFP4_ERR_CUDA = -3
NVFP4_ERR_WORKSPACE = -4
NVFP4_ERR_TIMEOUT = -5

DTYPE_F32 = 0
DTYPE_BF16 = 1

FLAG_W4A4 = 0x1
FLAG_FORCE_SKINNY = 0x2
FLAG_FORCE_TC = 0x4
FLAG_FORCE_F32 = 0x8
FLAG_TS_GEMV = 0x10
FLAG_DIGIT_GEMV = 0x20

_STATUS_NAMES = {
    NVFP4_ERR_INVALID_ARG: "invalid argument",
    NVFP4_ERR_UNSUPPORTED: "unsupported",
    NVFP4_ERR_CUDA: "CUDA error",
    NVFP4_ERR_WORKSPACE: "workspace too small",
    NVFP4_ERR_TIMEOUT: "device wait timed out",
}


class Nvfp4Error(RuntimeError):
    """A libnvfp4 entry point returned a negative status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"libnvfp4: {_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class LinearDesc(ctypes.Structure):
    """struct nvfp4_linear_desc (mirrors NvFp4Linear, nvfp4/config.mojo:64-103)."""

    _fields_ = [
        ("in_features", ctypes.c_int64),
        ("out_features", ctypes.c_int64),
        ("input_scale", ctypes.c_float),
        ("weight_scale_2", ctypes.c_float),
        ("weight_scale_2_rows", ctypes.c_void_p),
    ]


class MoEDesc(ctypes.Structure):
    """struct nvfp4_moe_desc."""

    _fields_ = [("num_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("renormalize", ctypes.c_int32)]


class MoEWeightPtrs(ctypes.Structure):
    """struct nvfp4_moe_weights (device pointers)."""

    _fields_ = [("router", ctypes.c_void_p), ("gate_up", ctypes.c_void_p),
                ("gate_up_scale", ctypes.c_void_p), ("gate_up_scale_2", ctypes.c_void_p),
                ("gate_up_input_scale", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("down_scale", ctypes.c_void_p), ("down_scale_2", ctypes.c_void_p),
                ("down_input_scale", ctypes.c_void_p)]


class StTensorInfo(ctypes.Structure):
    """struct nvfp4_st_tensor_info (include/nvfp4_loader.h)."""

    _fields_ = [("dtype", ctypes.c_char * 16), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 8), ("data_offset", ctypes.c_int64),
                ("data_size", ctypes.c_int64)]


class StLinearInfo(ctypes.Structure):
    """struct nvfp4_st_linear_info (include/nvfp4_loader.h)."""

    _fields_ = [("out_features", ctypes.c_int64), ("in_features", ctypes.c_int64),
                ("weight_scale_2", ctypes.c_float), ("input_scale", ctypes.c_float),
                ("weight_scale_2_rows", ctypes.c_int32), ("shard", ctypes.c_int32)]


ST_FOLD_INPUT_SCALE = 0x1


class DeltaNetDesc(ctypes.Structure):
    """struct nvfp4_deltanet_desc (include/nvfp4_deltanet.h)."""

    _fields_ = [("d_model", ctypes.c_int32), ("num_key_heads", ctypes.c_int32),
                ("num_value_heads", ctypes.c_int32), ("key_dim", ctypes.c_int32),
                ("value_dim", ctypes.c_int32), ("conv_kernel", ctypes.c_int32),
                ("rms_eps", ctypes.c_float)]


class DeltaNetProj(ctypes.Structure):
    """struct nvfp4_deltanet_proj."""

    _fields_ = [("packed_weights", ctypes.c_void_p), ("blockscales", ctypes.c_void_p),
                ("input_scale", ctypes.c_float), ("weight_scale_2", ctypes.c_float),
                ("weight_scale_2_rows", ctypes.c_void_p)]


class DeltaNetWeightPtrs(ctypes.Structure):
    """struct nvfp4_deltanet_weights."""

    _fields_ = [("qkv", DeltaNetProj), ("z", DeltaNetProj), ("b", DeltaNetProj),
                ("a", DeltaNetProj), ("out", DeltaNetProj), ("in_proj", DeltaNetProj),
                ("a_log", ctypes.c_void_p),
                ("dt_bias", ctypes.c_void_p), ("conv_q", ctypes.c_void_p),
                ("conv_k", ctypes.c_void_p), ("conv_v", ctypes.c_void_p),
                ("conv_bias_q", ctypes.c_void_p), ("conv_bias_k", ctypes.c_void_p),
                ("conv_bias_v", ctypes.c_void_p)]


class DeltaNetStatePtrs(ctypes.Structure):
    """struct nvfp4_deltanet_state."""

    _fields_ = [("s", ctypes.c_void_p), ("conv_q", ctypes.c_void_p),
                ("conv_k", ctypes.c_void_p), ("conv_v", ctypes.c_void_p)]

EP_MAX_WORLD = 8
EP_HANDLE_BYTES = 64
EP_ERR_DISPATCH_TIMEOUT = 0x1
EP_ERR_DONE_TIMEOUT = 0x2
EP_ERR_SHAPE = 0x4


class EpPeers(ctypes.Structure):
    """struct nvfp4_ep_peers (include/nvfp4_ep.h)."""

    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("max_rows", ctypes.c_int64), ("hidden", ctypes.c_int32),
                ("timeout_ms", ctypes.c_int32), ("windows", ctypes.c_void_p * EP_MAX_WORLD)]


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u32 = ctypes.c_uint32
_f32 = ctypes.c_float

# name -> (restype, argtypes); every symbol include/nvfp4.h declares.
SIGNATURES = {
    "nvfp4_abi_version": (_int, []),
    "nvfp4_last_error_string": (ctypes.c_char_p, []),
    "nvfp4_linear_forward": (_int, [ctypes.POINTER(LinearDesc), _vp, _vp, _vp, _int, _vp, _int,
                                    _i64, _u32, _vp]),
    "nvfp4_gemm_kernel": (_int, [_i64, _i64, _i64, _vp, _vp, _vp, _int, _vp, _int, _f32, _vp]),
    "nvfp4_matvec": (_int, [ctypes.POINTER(LinearDesc), _vp, _vp, _vp, _vp, _vp]),
    "nvfp4_dequant_tile": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "nvfp4_dequant": (_int, [_vp, _vp, _i64, _i64, _vp, _int, _vp]),
    "nvfp4_device_status": (_int, []),
    "nvfp4_moe_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(MoEDesc), _i64]),
    "nvfp4_moe_experts_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(MoEDesc), _i64]),
    "nvfp4_moe_forward": (_int, [ctypes.POINTER(MoEDesc), ctypes.POINTER(MoEWeightPtrs), _vp, _vp,
                                 _vp, _int, _i64, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "nvfp4_moe_forward_noalloc": (_int, [ctypes.POINTER(MoEDesc), ctypes.POINTER(MoEWeightPtrs),
                                         _vp, _vp, _vp, _int, _i64, _vp, _vp, _vp]),
    "nvfp4_moe_shared_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(MoEDesc), ctypes.c_int32,
                                                          _i64]),
    "nvfp4_moe_forward_shared": (_int, [ctypes.POINTER(MoEDesc), ctypes.POINTER(MoEWeightPtrs),
                                        ctypes.POINTER(MoEWeightPtrs), ctypes.c_int32, _vp, _vp,
                                        _vp, _int, _i64, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "nvfp4_stack_rows": (_int, [_vp, _vp, ctypes.c_int32, _i64, _vp, _vp]),
    "nvfp4_moe_route": (_int, [ctypes.POINTER(MoEDesc), _vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "nvfp4_moe_experts": (_int, [ctypes.POINTER(MoEDesc), ctypes.POINTER(MoEWeightPtrs), _vp, _vp,
                                 _vp, _i64, _vp, _int, _vp, ctypes.c_size_t, _vp]),
    "nvfp4_moe_combine": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _int, _i64, ctypes.c_int32,
                                 ctypes.c_int32, _vp]),
    "nvfp4_ep_dispatch_plan": (_int, [_vp, _i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      _vp, _vp, _vp, _vp, _vp]),
    "nvfp4_gather_rows": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "nvfp4_ep_dispatch_padded": (_int, [_vp, _vp, _vp, _vp, _i64, ctypes.c_int32, ctypes.c_int32,
                                        _i64, _vp, _i64, _vp, _vp, _vp, _vp]),
    # include/nvfp4_ep.h
    "nvfp4_ep_window_size": (ctypes.c_size_t, [ctypes.c_int32, _i64, ctypes.c_int32]),
    "nvfp4_ep_window_create": (_int, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "nvfp4_ep_window_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "nvfp4_ep_window_close": (_int, [_vp]),
    "nvfp4_ep_window_destroy": (_int, [_vp]),
    "nvfp4_ep_p2p_rows": (_int, [ctypes.POINTER(EpPeers), _i64, ctypes.c_int32,
                                 ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "nvfp4_ep_p2p_dispatch": (_int, [ctypes.POINTER(EpPeers), _vp, _vp, _i64, ctypes.c_int32,
                                     ctypes.c_int32, _vp]),
    "nvfp4_ep_p2p_wait_dispatch": (_int, [ctypes.POINTER(EpPeers), _vp]),
    "nvfp4_ep_p2p_signal_done": (_int, [ctypes.POINTER(EpPeers), _vp]),
    "nvfp4_ep_p2p_combine": (_int, [ctypes.POINTER(EpPeers), _vp, _vp, _i64, ctypes.c_int32,
                                    ctypes.c_int32, _vp, _vp, _int, _vp]),
    "nvfp4_ep_p2p_error": (_int, [ctypes.POINTER(EpPeers), ctypes.POINTER(_u32), ctypes.c_int32,
                                  _vp]),
    "nvfp4_ep_p2p_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(MoEDesc),
                                                      ctypes.POINTER(EpPeers), _i64]),
    "nvfp4_ep_p2p_forward": (_int, [ctypes.POINTER(MoEDesc), ctypes.POINTER(MoEWeightPtrs),
                                    ctypes.POINTER(EpPeers), _vp, _vp, _vp, _int, _i64, _vp,
                                    ctypes.c_size_t, _vp]),
    # include/nvfp4_deltanet.h
    "nvfp4_deltanet_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(DeltaNetDesc), _i64]),
    "nvfp4_deltanet_forward": (_int, [ctypes.POINTER(DeltaNetDesc),
                                      ctypes.POINTER(DeltaNetWeightPtrs), _vp, _int, _vp, _int,
                                      _i64, ctypes.POINTER(DeltaNetStatePtrs), _int, _vp,
                                      ctypes.c_size_t, _vp]),
    # include/nvfp4_loader.h
    "nvfp4_st_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "nvfp4_st_close": (None, [_vp]),
    "nvfp4_st_num_tensors": (_i64, [_vp]),
    "nvfp4_st_tensor_name": (ctypes.c_char_p, [_vp, _i64]),
    "nvfp4_st_find": (_i64, [_vp, ctypes.c_char_p]),
    "nvfp4_st_get_tensor_info": (_int, [_vp, _i64, ctypes.POINTER(StTensorInfo)]),
    "nvfp4_st_read_host": (_i64, [_vp, _i64, _vp, _i64]),
    "nvfp4_st_read_device": (_int, [_vp, _i64, _vp, _vp]),
    "nvfp4_st_f32_from_bytes": (_f32, [_vp, _i64]),
    "nvfp4_st_open_model": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "nvfp4_st_open_files": (_int, [ctypes.POINTER(ctypes.c_char_p), ctypes.c_int32,
                                   ctypes.POINTER(_vp)]),
    "nvfp4_st_close_model": (None, [_vp]),
    "nvfp4_st_model_num_shards": (ctypes.c_int32, [_vp]),
    "nvfp4_st_model_shard_path": (ctypes.c_char_p, [_vp, ctypes.c_int32]),
    "nvfp4_st_model_shard": (_vp, [_vp, ctypes.c_int32]),
    "nvfp4_st_model_find": (_int, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32),
                                   ctypes.POINTER(_i64)]),
    "nvfp4_st_get_linear_info": (_int, [_vp, ctypes.c_char_p, ctypes.POINTER(StLinearInfo)]),
    "nvfp4_st_load_linear": (_int, [_vp, ctypes.c_char_p, _vp, _vp, _vp, _u32, _vp]),
    "nvfp4_st_load_experts": (_int, [_vp, ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_int32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "nvfp4_st_load_router": (_int, [_vp, ctypes.c_char_p, _vp, ctypes.POINTER(ctypes.c_int32),
                                    ctypes.POINTER(ctypes.c_int32), _vp]),
    "nvfp4_quantize_act": (_int, [_vp, _int, _i64, _i64, _i64, _f32, _vp, _vp, _vp]),
    "nvfp4_linear_w4a4": (_int, [ctypes.POINTER(LinearDesc), _vp, _vp, _vp, _vp, _vp, _int, _i64,
                                 _vp]),
}

_lib = None


def load():
    """Load libnvfp4.so once; raises if it is absent or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"libnvfp4.so not found at {LIB_PATH}: build it with "
            "`make -C nvfp4-mojo_b200` (there is no CPU fallback)")
    L = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != NVFP4_OK:
        msg = load().nvfp4_last_error_string().decode(errors="replace")
        raise Nvfp4Error(rc, msg)

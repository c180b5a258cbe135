"""NVFP4 matvec and the activation helpers -- mirror of the hot-path parts of
nvfp4/deltanet.mojo (the DeltaNet recurrence itself is not on the NVFP4 path).
"""
from __future__ import annotations

import ctypes
import math

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

"""GPU NVFP4 linear -- mirror of nvfp4/nvfp4_gemm_gpu.mojo over libnvfp4.

Same entry points as the reference module; each call enqueues CUDA kernels
(sm_100a) through the C ABI on the current torch stream.  Tensors must be on
the GPU; nothing is computed on the host.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .config import NVFP4_GROUP_SIZE, NVFP4_PACK_FACTOR, NvFp4Linear

# nvfp4/nvfp4_gemm_gpu.mojo:34-41 (the reference's tile constants; the B200
# kernels choose their own tiles, these keep the public names).
BM: int = 128
BN: int = 128
BK: int = 64
WM: int = 64
WN: int = 64
FP8_SCALE_DTYPE = torch.float8_e4m3fn

_DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _dev(t: torch.Tensor, name: str) -> int:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


def make_desc(linear: NvFp4Linear) -> _lib.LinearDesc:
    rows = linear.weight_scale_2_rows
    ptr = None
    if rows is not None:
        if rows.dtype != torch.float32 or rows.numel() != linear.out_features:
            raise ValueError("weight_scale_2_rows must be fp32 [out_features]")
        ptr = _dev(rows, "weight_scale_2_rows")
    return _lib.LinearDesc(linear.in_features, linear.out_features,
                           float(linear.input_scale), float(linear.weight_scale_2), ptr)


def nvfp4_linear_forward(linear: NvFp4Linear, packed_weights: torch.Tensor,
                         blockscales: torch.Tensor, activations: torch.Tensor,
                         output: torch.Tensor, batch_seq_len: int, ctx=None,
                         flags: int = 0) -> None:
    """nvfp4/nvfp4_gemm_gpu.mojo:185-224.

    packed_weights uint8 [out, in/2]; blockscales e4m3 (or its uint8 bytes)
    [out, in/16]; activations [batch_seq_len, in] bf16 or fp32; output
    [batch_seq_len, out] bf16 or fp32.  `ctx` is the stream (None = current).
    """
    L = _lib.load()
    desc = make_desc(linear)
    w, sf = _u8(packed_weights), _u8(blockscales)
    if w.numel() != linear.packed_weight_size() or sf.numel() != linear.scale_size():
        raise ValueError("weight / blockscale sizes do not match the linear's shape")
    if activations.dtype not in _DT or output.dtype not in _DT:
        raise TypeError("activations and output must be bf16 or fp32")
    if activations.numel() < batch_seq_len * linear.in_features or \
            output.numel() < batch_seq_len * linear.out_features:
        raise ValueError("activation / output buffers are too small")
    rc = L.nvfp4_linear_forward(ctypes.byref(desc), _dev(w, "packed_weights"),
                                _dev(sf, "blockscales"), _dev(activations, "activations"),
                                _DT[activations.dtype], _dev(output, "output"),
                                _DT[output.dtype], int(batch_seq_len), int(flags),
                                _stream(ctx))
    _lib.check(rc)


def nvfp4_linear(linear: NvFp4Linear, packed_weights: torch.Tensor, blockscales: torch.Tensor,
                 activations: torch.Tensor, out_dtype=torch.bfloat16, flags: int = 0,
                 stream=None) -> torch.Tensor:
    """Allocating convenience form: returns y [M, out_features]."""
    M = activations.shape[0]
    y = torch.empty((M, linear.out_features), dtype=out_dtype, device=activations.device)
    nvfp4_linear_forward(linear, packed_weights, blockscales, activations, y, M, stream, flags)
    return y


def nvfp4_gemm_kernel(packed_weights: torch.Tensor, blockscales: torch.Tensor,
                      activations: torch.Tensor, output: torch.Tensor, alpha: float,
                      stream=None) -> None:
    """nvfp4/nvfp4_gemm_gpu.mojo:99-182 in the reference kernel's layout:
    activations [K, N_tok], output [M_out, N_tok]."""
    L = _lib.load()
    w, sf = _u8(packed_weights), _u8(blockscales)
    M_out, Kh = w.shape
    K, N_tok = activations.shape
    if Kh * NVFP4_PACK_FACTOR != K or output.shape != (M_out, N_tok):
        raise ValueError("shape mismatch")
    rc = L.nvfp4_gemm_kernel(M_out, N_tok, K, _dev(w, "packed_weights"), _dev(sf, "blockscales"),
                             _dev(activations, "activations"), _DT[activations.dtype],
                             _dev(output, "output"), _DT[output.dtype], float(alpha),
                             _stream(stream))
    _lib.check(rc)


def load_and_dequant_fp4_tile(packed_weights: torch.Tensor, blockscales: torch.Tensor,
                              output: torch.Tensor, weight_stride: int, scale_stride: int,
                              start_row: int, start_col: int, tile_m: int, tile_k: int,
                              stream=None) -> None:
    """nvfp4/nvfp4_gemm_gpu.mojo:44-96: fp32 output [tile_m, tile_k]."""
    L = _lib.load()
    if output.dtype != torch.float32 or output.numel() < tile_m * tile_k:
        raise ValueError("output must be fp32 with tile_m * tile_k elements")
    rc = L.nvfp4_dequant_tile(_dev(_u8(packed_weights), "packed_weights"),
                              _dev(_u8(blockscales), "blockscales"), _dev(output, "output"),
                              weight_stride, scale_stride, start_row, start_col, tile_m,
                              tile_k, _stream(stream))
    _lib.check(rc)


def dequant(packed_weights: torch.Tensor, blockscales: torch.Tensor,
            out_dtype=torch.float32, stream=None, out: torch.Tensor = None) -> torch.Tensor:
    """dequant_fp4 over a whole [rows, K/2] matrix -> [rows, K] (into `out`
    when given: fp32 or bf16, rows * K elements)."""
    L = _lib.load()
    w = _u8(packed_weights)
    rows, Kh = w.shape
    K = Kh * NVFP4_PACK_FACTOR
    if out is None:
        out = torch.empty((rows, K), dtype=out_dtype, device=w.device)
    elif out.numel() != rows * K or out.dtype not in _DT:
        raise ValueError("out must hold rows * K fp32 or bf16 elements")
    out_dtype = out.dtype
    rc = L.nvfp4_dequant(_dev(w, "packed_weights"), _dev(_u8(blockscales), "blockscales"),
                         rows, K, _dev(out, "output"), _DT[out_dtype], _stream(stream))
    _lib.check(rc)
    return out


def quantize_act(activations: torch.Tensor, input_scale: float, stream=None):
    """W4A4 activation quantizer (nvfp4_quantize_act): x [M, K] bf16/fp32 ->
    (codes uint8 [M, K/2], blockscales uint8 (e4m3 bytes) [M, K/16])."""
    L = _lib.load()
    if activations.dtype not in _DT or activations.dim() != 2:
        raise TypeError("activations must be a 2-D bf16 or fp32 tensor")
    M, K = activations.shape
    codes = torch.empty((M, K // 2), dtype=torch.uint8, device=activations.device)
    scales = torch.empty((M, K // NVFP4_GROUP_SIZE), dtype=torch.uint8,
                         device=activations.device)
    rc = L.nvfp4_quantize_act(_dev(activations, "activations"), _DT[activations.dtype], M, K, K,
                              float(input_scale), _dev(codes, "codes"), _dev(scales, "scales"),
                              _stream(stream))
    _lib.check(rc)
    return codes, scales


def nvfp4_linear_w4a4(linear: NvFp4Linear, packed_weights: torch.Tensor,
                      blockscales: torch.Tensor, act_codes: torch.Tensor,
                      act_scales: torch.Tensor, output: torch.Tensor, stream=None) -> None:
    """W4A4 GEMM on the block-scaled FP4 tensor cores (nvfp4_linear_w4a4):
    output [M, out] = input_scale * ws2 * dequant(W) @ dequant(X)^T."""
    L = _lib.load()
    desc = make_desc(linear)
    M = act_codes.shape[0]
    if output.dtype not in _DT or output.numel() < M * linear.out_features:
        raise ValueError("output must be bf16/fp32 with M * out_features elements")
    rc = L.nvfp4_linear_w4a4(ctypes.byref(desc), _dev(_u8(packed_weights), "packed_weights"),
                             _dev(_u8(blockscales), "blockscales"), _dev(act_codes, "act_codes"),
                             _dev(act_scales, "act_scales"), _dev(output, "output"),
                             _DT[output.dtype], M, _stream(stream))
    _lib.check(rc)


__all__ = [
    "BM", "BN", "BK", "WM", "WN", "FP8_SCALE_DTYPE", "NVFP4_GROUP_SIZE",
    "nvfp4_linear_forward", "nvfp4_linear", "nvfp4_gemm_kernel",
    "load_and_dequant_fp4_tile", "dequant", "make_desc", "quantize_act", "nvfp4_linear_w4a4",
]

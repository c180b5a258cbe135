"""NVFP4 format constants and metadata -- mirror of nvfp4/config.mojo.

Same names, meanings and defaults as the reference module so that code
written against it reads the same.  These are host-side scalar helpers (the
reference marks them @always_inline for use inside kernels); the device-side
equivalents live in csrc/nvfp4_common.cuh.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence, Tuple

import torch

# nvfp4/config.mojo:13-14
NVFP4_GROUP_SIZE: int = 16
NVFP4_PACK_FACTOR: int = 2

# nvfp4/config.mojo:18-35 -- code 8 is -0.0.
FP4_E2M1_LUT: Tuple[float, ...] = (
    0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
    -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0,
)


@dataclass
class NvFp4Config:
    """nvfp4/config.mojo:38-61: u8 weights, e4m3fn scales, bf16 output."""

    group_size: int = NVFP4_GROUP_SIZE
    weight_dtype: torch.dtype = torch.uint8
    scale_dtype: torch.dtype = torch.float8_e4m3fn
    output_dtype: torch.dtype = torch.bfloat16


@dataclass
class NvFp4Linear:
    """nvfp4/config.mojo:64-103.  Weight pointers are passed separately.

    `weight_scale_2_rows` (optional, device fp32 [out_features]) extends the
    reference's scalar second-level scale to one per output row.
    """

    in_features: int
    out_features: int
    input_scale: float = 1.0
    weight_scale_2: float = 1.0
    weight_scale_2_rows: "torch.Tensor | None" = None

    def alpha(self) -> float:
        """nvfp4/config.mojo:93-95 (fp32 product)."""
        return float(torch.tensor(self.input_scale, dtype=torch.float32)
                     * torch.tensor(self.weight_scale_2, dtype=torch.float32))

    def packed_weight_size(self) -> int:
        return self.out_features * (self.in_features // NVFP4_PACK_FACTOR)

    def scale_size(self) -> int:
        return self.out_features * (self.in_features // NVFP4_GROUP_SIZE)


def unpack_fp4_pair(packed: int) -> Tuple[int, int]:
    """nvfp4/config.mojo:106-114 -> (lo, hi); lo is the even k."""
    return packed & 0x0F, (packed >> 4) & 0x0F


def dequant_fp4(fp4_val: int, scale: float) -> float:
    """nvfp4/config.mojo:117-121: LUT[v] * scale in fp32."""
    t = torch.tensor(FP4_E2M1_LUT[fp4_val & 15], dtype=torch.float32)
    return float(t * torch.tensor(scale, dtype=torch.float32))


def dequant_fp4_simd(fp4_vals: Sequence[int], scales: Sequence[float]) -> Tuple[float, ...]:
    """nvfp4/config.mojo:124-135: element-wise dequant_fp4."""
    return tuple(dequant_fp4(v, s) for v, s in zip(fp4_vals, scales))


def pack_fp4_pair(lo: int, hi: int) -> int:
    """nvfp4/config.mojo:138-140 (8-bit result, like the reference's UInt8)."""
    return ((hi << 4) | (lo & 0x0F)) & 0xFF


def compute_effective_scale(blockscale: float, weight_scale_2: float,
                            input_scale: float) -> float:
    """nvfp4/config.mojo:143-149: left-to-right fp32 products."""
    t = torch.tensor(blockscale, dtype=torch.float32) * torch.tensor(weight_scale_2,
                                                                      dtype=torch.float32)
    return float(t * torch.tensor(input_scale, dtype=torch.float32))

"""nvfp4 -- B200-native NVFP4 fused-dequant GEMM/GEMV and MoE expert path.

Python mirror of the reference package's public names (nvfp4/__init__.mojo:
1-59) over libnvfp4.so (include/nvfp4.h).  Compute entry points run CUDA
kernels for sm_100a; there is no CPU fallback.
"""
from .config import (
    FP4_E2M1_LUT,
    NVFP4_GROUP_SIZE,
    NVFP4_PACK_FACTOR,
    NvFp4Config,
    NvFp4Linear,
    compute_effective_scale,
    dequant_fp4,
    dequant_fp4_simd,
    pack_fp4_pair,
    unpack_fp4_pair,
)
from .deltanet import nvfp4_matvec, sigmoid, silu
from .nvfp4_gemm_gpu import (
    BK,
    BM,
    BN,
    FP8_SCALE_DTYPE,
    WM,
    WN,
    dequant,
    load_and_dequant_fp4_tile,
    nvfp4_gemm_kernel,
    nvfp4_linear,
    nvfp4_linear_forward,
    nvfp4_linear_w4a4,
    quantize_act,
)
from .weight_loader import (
    LoadedWeight,
    SafetensorsFile,
    TensorInfo,
    discover_safetensor_shards,
    load_linear_safetensors,
    load_moe_experts,
    load_qwen35_layer,
    open_model_shards,
    open_safetensors,
)
from ._lib import LIB_PATH, Nvfp4Error

__all__ = [
    "FP4_E2M1_LUT", "NVFP4_GROUP_SIZE", "NVFP4_PACK_FACTOR", "NvFp4Config", "NvFp4Linear",
    "compute_effective_scale", "dequant_fp4", "dequant_fp4_simd", "pack_fp4_pair",
    "unpack_fp4_pair", "nvfp4_matvec", "sigmoid", "silu", "BK", "BM", "BN", "WM", "WN",
    "FP8_SCALE_DTYPE", "dequant", "load_and_dequant_fp4_tile", "nvfp4_gemm_kernel",
    "nvfp4_linear", "nvfp4_linear_forward", "nvfp4_linear_w4a4", "quantize_act", "LIB_PATH",
    "Nvfp4Error", "LoadedWeight", "SafetensorsFile", "TensorInfo", "discover_safetensor_shards",
    "load_linear_safetensors", "load_moe_experts", "load_qwen35_layer", "open_model_shards",
    "open_safetensors",
]

"""Writers of small NVFP4 safetensors checkpoints for the loader tests, using
the `safetensors` package (the format's own writer) and the tensor names of
the reference's layout (nvfp4/weight_loader.mojo:703-760, :766-773)."""
from __future__ import annotations

import json
import struct
from typing import Dict, Optional

import numpy as np
import torch


def nvfp4_linear(tensors: Dict[str, torch.Tensor], prefix: str, w: np.ndarray, sf: np.ndarray,
                 ws2=None, ins=None):
    """{prefix}.weight U8 [out, in/2], .weight_scale F8_E4M3 [out, in/16],
    .weight_scale_2 F32 (scalar, or [out] per row), .input_scale F32 scalar."""
    tensors[prefix + ".weight"] = torch.from_numpy(np.ascontiguousarray(w, dtype=np.uint8))
    tensors[prefix + ".weight_scale"] = torch.from_numpy(
        np.ascontiguousarray(sf, dtype=np.uint8)).view(torch.float8_e4m3fn)
    if ws2 is not None:
        tensors[prefix + ".weight_scale_2"] = torch.tensor(np.asarray(ws2, np.float32))
    if ins is not None:
        tensors[prefix + ".input_scale"] = torch.tensor(np.float32(ins))


def save(path, tensors: Dict[str, torch.Tensor], metadata: Optional[Dict[str, str]] = None):
    from safetensors.torch import save_file

    save_file({k: v.contiguous() for k, v in tensors.items()}, str(path), metadata=metadata)


def raw_file(path, header: str, data: bytes = b"", header_size: Optional[int] = None):
    """A file with a hand-written JSON header (header_size overrides the
    8-byte length field)."""
    hb = header.encode()
    n = len(hb) if header_size is None else header_size
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", n))
        f.write(hb)
        f.write(data)


def header_json(entries) -> str:
    return json.dumps(entries)


def rand_linear(rng, out_f: int, in_f: int):
    w = rng.integers(0, 256, size=(out_f, in_f // 2), dtype=np.uint8)
    sf = torch.from_numpy(rng.uniform(0.25, 4.0, size=(out_f, in_f // 16)).astype(np.float32))
    sf = sf.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return w, sf

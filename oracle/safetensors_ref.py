"""Restatement of the reference's safetensors loader (nvfp4/weight_loader.mojo).

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the C++ loader
in libnvfp4.so (include/nvfp4_loader.h), never by the product path.

Each function follows the reference function it names, step for step,
including its quirks (a scanning "JSON" parser, the float32 decoding of
scalar scales by repeated multiplication, the shard probe loop).  The
reference ships no loader tests or fixtures, so parity is pinned two ways:
the header fields are checked against the `safetensors` package's own reader
(the format's canonical implementation) on files it writes, and the f32 rule
against IEEE-754 decoding by numpy on the values where the two must agree.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import List

import numpy as np

_WS = (9, 10, 32)  # tab, newline, space (nvfp4/weight_loader.mojo:37-40)


def json_find_string(js: bytes, key: str) -> str:
    """_json_find_string (nvfp4/weight_loader.mojo:124-143)."""
    needle = b'"' + key.encode() + b'"'
    pos = js.find(needle)
    if pos < 0:
        return ""
    pos += len(needle)
    n = len(js)
    while pos < n:
        b = js[pos]
        if b not in _WS and b != ord(":"):
            break
        pos += 1
    if pos >= n or js[pos] != ord('"'):
        return ""
    pos += 1
    end = pos
    while end < n and js[end] != ord('"'):
        end += 1
    return js[pos:end].decode("utf-8", "replace")


def json_find_int_array(js: bytes, key: str) -> List[int]:
    """_json_find_int_array (nvfp4/weight_loader.mojo:146-181)."""
    out: List[int] = []
    needle = b'"' + key.encode() + b'"'
    pos = js.find(needle)
    if pos < 0:
        return out
    pos += len(needle)
    n = len(js)
    while pos < n and js[pos] != ord("["):
        pos += 1
    if pos >= n:
        return out
    pos += 1
    while pos < n and js[pos] != ord("]"):
        b = js[pos]
        if b in _WS or b == ord(","):
            pos += 1
            continue
        start = pos
        while pos < n and ord("0") <= js[pos] <= ord("9"):
            pos += 1
        if pos > start:
            out.append(int(js[start:pos]))
        else:
            pos += 1  # (the reference spins here on a non-digit; never hit by valid headers)
    return out


@dataclass
class TensorInfo:
    """struct TensorInfo (nvfp4/weight_loader.mojo:190-238)."""

    name: str
    dtype: str
    shape: List[int]
    data_offset: int
    data_size: int


def parse_header(js: bytes) -> List[TensorInfo]:
    """_parse_safetensors_header (nvfp4/weight_loader.mojo:292-363)."""
    out: List[TensorInfo] = []
    pos, n = 0, len(js)
    while pos < n and js[pos] != ord("{"):
        pos += 1
    pos += 1
    while pos < n:
        while pos < n and js[pos] != ord('"'):
            if js[pos] == ord("}"):
                return out
            pos += 1
        if pos >= n:
            break
        pos += 1
        s = pos
        while pos < n and js[pos] != ord('"'):
            pos += 1
        name = js[s:pos].decode("utf-8", "replace")
        pos += 1
        while pos < n and js[pos] not in (ord("{"), ord("}")):
            pos += 1
        if pos >= n or js[pos] == ord("}"):
            break
        obj_start, depth = pos, 0
        while pos < n:
            b = js[pos]
            if b == ord("{"):
                depth += 1
            elif b == ord("}"):
                depth -= 1
                if depth == 0:
                    pos += 1
                    break
            pos += 1
        obj = js[obj_start:pos]
        if name == "__metadata__":
            continue
        offs = json_find_int_array(obj, "data_offsets")
        off, size = (offs[0], offs[1] - offs[0]) if len(offs) >= 2 else (0, 0)
        out.append(TensorInfo(name, json_find_string(obj, "dtype"),
                              json_find_int_array(obj, "shape"), off, size))
    return out


@dataclass
class SafetensorsFile:
    """struct SafetensorsFile (nvfp4/weight_loader.mojo:241-289), host-only."""

    path: str
    file_size: int
    header_size: int
    data_start: int
    tensors: List[TensorInfo] = field(default_factory=list)

    def find_tensor(self, name: str) -> int:
        for i, t in enumerate(self.tensors):
            if t.name == name:
                return i
        return -1

    def read_tensor_bytes(self, i: int) -> bytes:
        t = self.tensors[i]
        with open(self.path, "rb") as f:
            f.seek(self.data_start + t.data_offset)
            return f.read(t.data_size)


def open_safetensors(path: str) -> SafetensorsFile:
    """open_safetensors (nvfp4/weight_loader.mojo:366-410)."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 8:
        raise ValueError("Failed to read safetensors header size")
    hs = int.from_bytes(data[:8], "little")
    if hs <= 0 or hs > len(data) - 8:
        raise ValueError(f"Invalid safetensors header size: {hs}")
    return SafetensorsFile(path, len(data), hs, 8 + hs, parse_header(data[8:8 + hs]))


def read_f32_from_bytes(buf: bytes) -> np.float32:
    """_read_f32_from_bytes (nvfp4/weight_loader.mojo:678-700), including the
    2^exp by repeated float32 multiplication."""
    if len(buf) < 4:
        return np.float32(1.0)
    bits = buf[0] | (buf[1] << 8) | (buf[2] << 16) | (buf[3] << 24)
    sign = bits >> 31
    exp_bits = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp_bits == 0:
        return np.float32(-0.0) if sign else np.float32(0.0)
    if exp_bits == 255:
        return np.float32(1.0)
    result = np.float32(1.0) + np.float32(mant) / np.float32(1 << 23)
    e = exp_bits - 127
    two, half = np.float32(2.0), np.float32(0.5)
    for _ in range(abs(e)):
        result = np.float32(result * (two if e > 0 else half))
    return np.float32(-result) if sign else np.float32(result)


@dataclass
class LoadedWeight:
    """struct LoadedWeight (nvfp4/weight_loader.mojo:614-675), host bytes."""

    packed_weights: bytes
    blockscales: bytes
    weight_scale_2: np.float32
    input_scale: np.float32
    out_features: int
    in_features: int


def load_linear_safetensors(sf: SafetensorsFile, prefix: str) -> LoadedWeight:
    """load_linear_safetensors (nvfp4/weight_loader.mojo:703-760)."""
    wi = sf.find_tensor(prefix + ".weight")
    if wi < 0:
        raise ValueError("Tensor not found: " + prefix + ".weight")
    si = sf.find_tensor(prefix + ".weight_scale")
    if si < 0:
        raise ValueError("Tensor not found: " + prefix + ".weight_scale")
    w = sf.tensors[wi]
    if len(w.shape) < 2:
        raise ValueError("Weight tensor must be 2D: " + prefix + ".weight")
    out_f, in_f = w.shape[0], w.shape[1] * 2
    packed = sf.read_tensor_bytes(wi)
    if len(packed) != out_f * (in_f // 2):
        raise ValueError("Weight read size mismatch for " + prefix + ".weight")
    scales = sf.read_tensor_bytes(si)
    if len(scales) != out_f * (in_f // 16):
        raise ValueError("Scale read size mismatch for " + prefix + ".weight_scale")
    ws2 = ins = np.float32(1.0)
    i2 = sf.find_tensor(prefix + ".weight_scale_2")
    if i2 >= 0:
        ws2 = read_f32_from_bytes(sf.read_tensor_bytes(i2))
    ii = sf.find_tensor(prefix + ".input_scale")
    if ii >= 0:
        ins = read_f32_from_bytes(sf.read_tensor_bytes(ii))
    return LoadedWeight(packed, scales, ws2, ins, out_f, in_f)


def find_load_linear(shards: List[SafetensorsFile], prefix: str) -> LoadedWeight:
    """_find_load_linear (nvfp4/weight_loader.mojo:828-836)."""
    for s in shards:
        if s.find_tensor(prefix + ".weight") >= 0:
            return load_linear_safetensors(s, prefix)
    raise ValueError("No shard contains " + prefix + ".weight")


def discover_safetensor_shards(model_dir: str) -> List[str]:
    """discover_safetensor_shards (nvfp4/weight_loader.mojo:909-945), the probe
    loop as written (after the first hit it tries total = i only)."""
    single = model_dir + "/model.safetensors"
    if os.access(single, os.R_OK):
        return [single]
    paths: List[str] = []
    for i in range(1, 200):
        found = False
        for total in range(i, 200):
            p = f"{model_dir}/model-{i:05d}-of-{total:05d}.safetensors"
            if os.access(p, os.R_OK):
                paths.append(p)
                found = True
                break
            if paths:
                break
        if not found and paths:
            break
        if not found and i > 1:
            break
    if not paths:
        raise ValueError("No safetensors files found in " + model_dir)
    return paths

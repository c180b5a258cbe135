"""Seeded synthetic NVFP4 workloads in the shapes and value distributions of
the benchmark configurations (no public dataset is involved):

* linear weights: every nibble uniform over the 16 E2M1 codes (bytes uniform
  over 0..255); blockscales = e4m3(Uniform(0.25, 4)); weight_scale_2 per row
  = Uniform(1e-3, 1e-2);
* activations ~ N(0, 1);
* MoE: router fp32 [H, E] ~ N(0, 0.02); per expert fused gate_up [2I, H] and
  down [H, I] NVFP4 weights generated as above.

Host generation uses numpy's PCG64 (`default_rng(seed)`); large stacks are
generated on the GPU with a seeded torch generator.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch


def e4m3_bytes(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn (round-to-nearest-even) raw bytes."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def linear_weights(N: int, K: int, seed: int) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    sf = e4m3_bytes(rng.uniform(0.25, 4.0, size=(N, K // 16)).astype(np.float32))
    ws2 = rng.uniform(1e-3, 1e-2, size=(N,)).astype(np.float32)
    return {"w": w, "sf": sf, "ws2": ws2}


def activations(M: int, K: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (RNE) and back to fp32 -- the values a bf16 tensor holds."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def moe_weights(E: int, H: int, I: int, seed: int) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((H, E)) * 0.02).astype(np.float32)
    gu_w = rng.integers(0, 256, size=(E, 2 * I, H // 2), dtype=np.uint8)
    gu_sf = e4m3_bytes(rng.uniform(0.25, 4.0, size=(E, 2 * I, H // 16)).astype(np.float32))
    gu_ws2 = rng.uniform(1e-3, 1e-2, size=(E, 2 * I)).astype(np.float32)
    dn_w = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    dn_sf = e4m3_bytes(rng.uniform(0.25, 4.0, size=(E, H, I // 16)).astype(np.float32))
    dn_ws2 = rng.uniform(1e-3, 1e-2, size=(E, H)).astype(np.float32)
    return {"router": router, "gu_w": gu_w, "gu_sf": gu_sf, "gu_ws2": gu_ws2,
            "dn_w": dn_w, "dn_sf": dn_sf, "dn_ws2": dn_ws2}


def linear_weights_cuda(N: int, K: int, seed: int, device="cuda") -> Dict[str, torch.Tensor]:
    """Same distributions as linear_weights, generated on the GPU (large shapes)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randint(0, 256, (N, K // 2), generator=g, device=device, dtype=torch.int32)
    sf = torch.rand((N, K // 16), generator=g, device=device) * 3.75 + 0.25
    ws2 = torch.rand((N,), generator=g, device=device) * 9e-3 + 1e-3
    return {"w": w.to(torch.uint8), "sf": sf.to(torch.float8_e4m3fn).view(torch.uint8),
            "ws2": ws2.float()}


def moe_weights_cuda(E: int, H: int, I: int, seed: int, device="cuda") -> Dict[str, torch.Tensor]:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    router = torch.randn((H, E), generator=g, device=device) * 0.02

    def nv(rows, k):
        w = torch.randint(0, 256, (E, rows, k // 2), generator=g, device=device,
                          dtype=torch.int32).to(torch.uint8)
        sf = (torch.rand((E, rows, k // 16), generator=g, device=device) * 3.75 + 0.25)
        ws2 = torch.rand((E, rows), generator=g, device=device) * 9e-3 + 1e-3
        return w, sf.to(torch.float8_e4m3fn).view(torch.uint8), ws2.float()

    gu_w, gu_sf, gu_ws2 = nv(2 * I, H)
    dn_w, dn_sf, dn_ws2 = nv(H, I)
    return {"router": router.float(), "gu_w": gu_w, "gu_sf": gu_sf, "gu_ws2": gu_ws2,
            "dn_w": dn_w, "dn_sf": dn_sf, "dn_ws2": dn_ws2}

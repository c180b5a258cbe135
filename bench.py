"""Benchmark of the NVFP4 hot path on B200 -- one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default workload `ep` (one step = one pass of a 48-layer stack of the
128-expert, top-8 NVFP4 MoE layer, h = h + MoE(h), over a 64-token decode
batch, expert-parallel over the N ranks: 128/N experts and 64/N tokens per
GPU, device-initiated dispatch/combine through peer memory).  Beside it, at
N = 1, the same line carries the decode GEMV sweep and the W4A16 prefill sweep
(`secondary`), each with the roofline of its dominant launch, and the layer's
`parity` against the CPU oracle.  Other workloads: gemv, prefill,
prefill_w4a4, dequant, moe (one layer), deltanet.

`value` is device-timed (CUDA events, max over ranks) with weights resident
and the step replayed from a CUDA graph; `e2e` times the public Python API
(ctypes into libnvfp4.so) with the step's activations copied from pinned host
memory and its outputs copied back.  `--impl reference` times the
reference's CPU path (the oracle port, all host threads) on a bounded sample
of the same workload.  N > 1: one process per GPU (torchrun); workloads that
do not shard (gemv, prefill) run independent replicas.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "nvfp4-mojo_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "fused-dequant FP4 GEMM TFLOP/s & HBM GB/s vs peak; MoE layer tok/s at 1–8 GPU"


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic(key):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(key)


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# Workload: decode GEMV sweep.
# ---------------------------------------------------------------------------
GEMV_SHAPES = [(2048, 1536), (768, 2048), (4096, 14336)]
GEMV_MS = [1, 2, 4, 8]


def gemv_bytes(K, N):
    return N * K // 2 + N * K // 16 + 4 * N


class GemvSweep:
    name = "gemv"
    unit = "GB/s"
    workload = ("decode GEMV sweep: M in {1,2,4,8} x (K,N) in {(2048,1536),(768,2048),"
                "(4096,14336)}, bf16 activations ~N(0,1), NVFP4 weights (nibbles uniform, "
                "e4m3 scales U(0.25,4), per-row fp32 scale_2 U(1e-3,1e-2)); bf16 out")

    def __init__(self, device, seed=0, split=None, world=1, rank=0):
        import torch
        import nvfp4
        from nvfp4 import synthetic
        from nvfp4.column_split import shard_bounds

        self.torch, self.nvfp4 = torch, nvfp4
        self.dev = device
        # Column split: this GPU holds output rows [n0, n1) of every shape
        # (nvfp4.column_split's bounds) and computes that slice of y, no
        # collective; the job's work is the whole sweep (strong scaling).
        split = split if world > 1 else None
        self.scaling = "strong" if split else "weak"
        self.traffic_ok = not split
        self.sets = 2  # two weight sets alternate per step: reuse distance > L2
        self.calls = []  # per set: list of (lin, W, SF, X, Y, bytes, is_dominant)
        full_bytes = 0
        for s in range(self.sets):
            calls = []
            for (K, N) in GEMV_SHAPES:
                n0, n1 = shard_bounds(N, world, rank) if split else (0, N)
                n = n1 - n0
                for M in GEMV_MS:
                    wd = synthetic.linear_weights_cuda(n, K, seed=seed + 1000 * s + 7 * M + K + N,
                                                       device=device)
                    x = torch.randn((M, K), device=device).to(torch.bfloat16)
                    y = torch.empty((M, n), device=device, dtype=torch.bfloat16)
                    lin = nvfp4.NvFp4Linear(K, n, weight_scale_2_rows=wd["ws2"])
                    calls.append((lin, wd["w"], wd["sf"], x, y, gemv_bytes(K, n),
                                  (K, N) == (4096, 14336)))
                    if s == 0:
                        full_bytes += gemv_bytes(K, N)
            self.calls.append(calls)
        # Per-rank units: the harness multiplies by the world size, so a split
        # counts the whole sweep once (the slices differ by at most one tile).
        self.bytes_per_step = (full_bytes / world if split else
                               sum(c[5] for c in self.calls[0]))
        self.launches_per_step = len(self.calls[0])
        dn0, dn1 = shard_bounds(14336, world, rank) if split else (0, 14336)
        self.dominant_bytes = gemv_bytes(4096, dn1 - dn0)
        self.dominant_name = (f"gemv_kernel (decode GEMV, K=4096 N={dn1 - dn0}"
                              + (f", this GPU's column slice of N=14336)" if split else ")"))
        self.config = {"workload": self.workload, "shapes_KN": GEMV_SHAPES, "M": GEMV_MS,
                       "l2": "inputs larger than L2: two weight sets (2 x 143 MB) alternate per step"}
        if split:
            self.config["split"] = (f"columns: each of {world} GPUs holds N/{world} output rows "
                                    "of every shape (16-row tiles) and writes its slice of y, "
                                    "no collective")

    def run_step(self, i):
        for (lin, W, SF, X, Y, _b, _dom) in self.calls[i % self.sets]:
            self.nvfp4.nvfp4_linear_forward(lin, W, SF, X, Y, X.shape[0])

    def run_dominant(self, i):
        """The K=4096, N=14336 launches of one step (M = 1, 2, 4, 8)."""
        n = 0
        for (lin, W, SF, X, Y, _b, dom) in self.calls[i % self.sets]:
            if dom:
                self.nvfp4.nvfp4_linear_forward(lin, W, SF, X, Y, X.shape[0])
                n += 1
        return n

    def units(self, steps):
        return self.bytes_per_step * steps / 1e9  # GB

    # End to end through the public API: activations H2D from pinned host,
    # outputs D2H to pinned host, every step.
    def e2e_setup(self):
        torch = self.torch
        self.h_x = [torch.randn(c[3].shape).to(torch.bfloat16).pin_memory() for c in self.calls[0]]
        self.h_y = [torch.empty(c[4].shape, dtype=torch.bfloat16).pin_memory() for c in self.calls[0]]
        self.h2d = sum(t.numel() * 2 for t in self.h_x)
        self.d2h = sum(t.numel() * 2 for t in self.h_y)

    def e2e_step(self, i):
        calls = self.calls[i % self.sets]
        for j, (lin, W, SF, X, Y, _b, _d) in enumerate(calls):
            X.copy_(self.h_x[j], non_blocking=True)
            self.nvfp4.nvfp4_linear_forward(lin, W, SF, X, Y, X.shape[0])
            self.h_y[j].copy_(Y, non_blocking=True)

    # CPU baseline: the oracle (nvfp4_matvec restated) on a row sample.
    def cpu_sample(self, threads, rows_cap=256):
        from nvfp4 import synthetic
        from oracle import oracle as O

        work = []
        for (K, N) in GEMV_SHAPES:
            n = min(N, rows_cap)
            wd = synthetic.linear_weights(n, K, seed=5)
            for M in GEMV_MS:
                work.append((wd, synthetic.activations(M, K, seed=M), gemv_bytes(K, n)))

        def run():
            for wd, x, _b in work:
                O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"], n_threads=threads)

        nbytes = sum(b for *_x, b in work)
        desc = (f"all 12 sweep calls on the first {rows_cap} output rows of each shape "
                f"({nbytes / 1e6:.2f} MB of weights+scales per pass)")
        return run, nbytes / 1e9, desc


# ---------------------------------------------------------------------------
# Workload: prefill W4A16 GEMM sweep (tcgen05).
# ---------------------------------------------------------------------------
PREFILL_MS = [512, 2048, 8192]
PREFILL_K, PREFILL_N = 4096, 14336


class PrefillSweep:
    name = "prefill"
    unit = "TFLOP/s"
    flags = 0
    workload = ("prefill W4A16 GEMM sweep: bf16 x [M, 4096] ~N(0,1), M in {512, 2048, 8192} x "
                "NVFP4 W [14336, 4096] (u8 [14336, 2048], e4m3 [14336, 256], fp32 scale_2 "
                "[14336]); fp32 accumulate, bf16 out; 2*M*N*K flop per GEMM")

    def __init__(self, device, seed=0):
        import torch
        import nvfp4
        from nvfp4 import synthetic

        self.torch, self.nvfp4 = torch, nvfp4
        self.sets = 2
        K, N = PREFILL_K, PREFILL_N
        self.calls = []
        for s in range(self.sets):
            wd = synthetic.linear_weights_cuda(N, K, seed=seed + 31 * s, device=device)
            lin = nvfp4.NvFp4Linear(K, N, weight_scale_2_rows=wd["ws2"])
            calls = []
            for M in PREFILL_MS:
                x = torch.randn((M, K), device=device).to(torch.bfloat16)
                y = torch.empty((M, N), device=device, dtype=torch.bfloat16)
                calls.append((lin, wd["w"], wd["sf"], x, y, 2.0 * M * N * K, M == 8192))
            self.calls.append(calls)
        self.flop_per_step = sum(c[5] for c in self.calls[0])
        self.launches_per_step = len(self.calls[0])
        self.dominant_bytes = 2.0 * 8192 * N * K  # flop of the dominant launch
        self.dominant_name = "w4a16_tc_kernel (tcgen05, M=8192 K=4096 N=14336)"
        self.bound = "tensor"
        self.config = {"workload": self.workload, "M": PREFILL_MS, "K": K, "N": N,
                       "l2": "inputs larger than L2: two weight sets alternate per step "
                             "(2 x 33 MB weights + 88 MB activations per set)"}

    def run_step(self, i):
        for (lin, W, SF, X, Y, _f, _d) in self.calls[i % self.sets]:
            self.nvfp4.nvfp4_linear_forward(lin, W, SF, X, Y, X.shape[0], flags=self.flags)

    def run_dominant(self, i):
        n = 0
        for (lin, W, SF, X, Y, _f, dom) in self.calls[i % self.sets]:
            if dom:
                self.nvfp4.nvfp4_linear_forward(lin, W, SF, X, Y, X.shape[0], flags=self.flags)
                n += 1
        return n

    def units(self, steps):
        return self.flop_per_step * steps / 1e12  # TFLOP

    def e2e_setup(self):
        torch = self.torch
        self.h_x = [torch.randn(c[3].shape).to(torch.bfloat16).pin_memory() for c in self.calls[0]]
        self.h_y = [torch.empty(c[4].shape, dtype=torch.bfloat16).pin_memory() for c in self.calls[0]]
        self.h2d = sum(t.numel() * 2 for t in self.h_x)
        self.d2h = sum(t.numel() * 2 for t in self.h_y)

    def e2e_step(self, i):
        for j, (lin, W, SF, X, Y, _f, _d) in enumerate(self.calls[i % self.sets]):
            X.copy_(self.h_x[j], non_blocking=True)
            self.nvfp4.nvfp4_linear_forward(lin, W, SF, X, Y, X.shape[0], flags=self.flags)
            self.h_y[j].copy_(Y, non_blocking=True)

    def cpu_sample(self, threads, rows=8, cols=256):
        from nvfp4 import synthetic
        from oracle import oracle as O

        K, N = PREFILL_K, PREFILL_N
        wd = synthetic.linear_weights(cols, K, seed=5)
        x = synthetic.activations(rows, K, seed=6)

        def run():
            O.linear(wd["w"], wd["sf"], x, ws2_rows=wd["ws2"], n_threads=threads)

        flop = 2.0 * rows * cols * K
        desc = (f"{rows} tokens x {cols} output features of the K=4096 GEMM per pass "
                f"({flop / 1e6:.1f} MFLOP; the oracle's cost is linear in tokens x features)")
        return run, flop / 1e12, desc


class PrefillW4A4Sweep(PrefillSweep):
    """The prefill sweep in W4A4 mode: each call quantizes x to NVFP4 with
    input_scale = max|x| / (6 * 448) (nvfp4_quantize_act) and multiplies on the
    block-scaled FP4 tensor cores; the dominant launch is the GEMM alone, on
    activations quantized beforehand."""

    name = "prefill_w4a4"
    dtype = "fp4 e2m1 x e2m1, e4m3 block scales, fp32 accumulate"
    workload = ("prefill W4A4 GEMM sweep: bf16 x [M, 4096] ~N(0,1), M in {512, 2048, 8192}, "
                "quantized to NVFP4 each call with input_scale = max|x|/(6*448) x NVFP4 W "
                "[14336, 4096] (u8 [14336, 2048], e4m3 [14336, 256], fp32 scale_2 [14336]); "
                "block-scaled FP4 MMA, fp32 accumulate, bf16 out; 2*M*N*K flop per GEMM")

    def __init__(self, device, seed=0):
        import nvfp4

        super().__init__(device, seed)
        self.flags = nvfp4._lib.FLAG_W4A4
        self.config["workload"] = self.workload
        self.quant = []
        for calls in self.calls:
            q = []
            for (lin, W, SF, X, Y, _f, dom) in calls:
                lin.input_scale = float(X.float().abs().max().item() / (6 * 448))
                if dom:
                    q.append(nvfp4.quantize_act(X, lin.input_scale))
            self.quant.append(q)
        self.dominant_name = "w4a4_gemm_kernel (tcgen05 mxf4nvf4, M=8192 K=4096 N=14336)"
        self.peak_scale = 4.0  # dense FP4 = 4 x dense BF16

    def cpu_sample(self, threads, rows=8, cols=256):
        from nvfp4 import synthetic
        from oracle import oracle as O

        K = PREFILL_K
        wd = synthetic.linear_weights(cols, K, seed=5)
        x = synthetic.activations(rows, K, seed=6)
        ins = float(abs(x).max() / (6 * 448))

        def run():
            O.linear_w4a4(wd["w"], wd["sf"], x, ins, ws2_rows=wd["ws2"], n_threads=threads)

        flop = 2.0 * rows * cols * K
        desc = (f"{rows} tokens x {cols} output features of the K=4096 W4A4 GEMM per pass "
                f"(activation quantization included; {flop / 1e6:.1f} MFLOP)")
        return run, flop / 1e12, desc

    def run_dominant(self, i):
        n = 0
        for (lin, W, SF, X, Y, _f, dom) in self.calls[i % self.sets]:
            if dom:
                q, s = self.quant[i % self.sets][0]
                self.nvfp4.nvfp4_linear_w4a4(lin, W, SF, q, s, Y)
                n += 1
        return n


# ---------------------------------------------------------------------------
# Workload: dequant microbenchmark in the shape of the reference's
# bench_nvfp4.mojo (element counts 1024 .. 1048576, fp32 output), plus the
# [14336, 4096] prefill weight as the large, HBM-bound case.
# ---------------------------------------------------------------------------
DEQ_SIZES = [1024, 4096, 16384, 65536, 262144, 1048576]
DEQ_ROW = 1024  # elements per row for the small sizes


class DequantBench:
    name = "dequant"
    unit = "Gelem/s"
    workload = ("NVFP4 dequant to fp32 (LUT * e4m3 blockscale): element counts 1024, 4096, "
                "16384, 65536, 262144, 1048576 as in bench_nvfp4.mojo, plus the [14336, 4096] "
                "prefill weight; nibbles uniform, e4m3 scales U(0.25, 4)")

    def __init__(self, device, seed=0):
        import torch
        import nvfp4
        from nvfp4 import synthetic

        self.torch, self.nvfp4 = torch, nvfp4
        self.sets = 2
        self.calls = []
        shapes = [(n // DEQ_ROW, DEQ_ROW) for n in DEQ_SIZES] + [(PREFILL_N, PREFILL_K)]
        for s in range(self.sets):
            calls = []
            for (rows, K) in shapes:
                wd = synthetic.linear_weights_cuda(rows, K, seed=seed + 13 * s + rows, device=device)
                out = torch.empty((rows, K), dtype=torch.float32, device=device)
                calls.append((wd["w"], wd["sf"], out, rows * K, rows == PREFILL_N))
            self.calls.append(calls)
        self.elems_per_step = sum(c[3] for c in self.calls[0])
        self.launches_per_step = len(shapes)
        # HBM bytes per element: 0.5 packed + 1/16 e4m3 scale + 4 fp32 out.
        self.dominant_bytes = PREFILL_N * PREFILL_K * (0.5 + 1.0 / 16 + 4.0)
        self.dominant_name = "dequant_kernel (fp32 out, [14336, 4096])"
        self.config = {"workload": self.workload, "sizes": DEQ_SIZES,
                       "large": [PREFILL_N, PREFILL_K],
                       "l2": "inputs larger than L2: two sets alternate (2 x 268 MB in + out)"}

    def run_step(self, i):
        for (w, sf, out, _n, _d) in self.calls[i % self.sets]:
            self.nvfp4.dequant(w, sf, out=out)

    def run_dominant(self, i):
        n = 0
        for (w, sf, out, _n, dom) in self.calls[i % self.sets]:
            if dom:
                self.nvfp4.dequant(w, sf, out=out)
                n += 1
        return n

    def units(self, steps):
        return self.elems_per_step * steps / 1e9

    def e2e_setup(self):
        torch = self.torch
        self.h_w = [c[0].cpu().pin_memory() for c in self.calls[0]]
        self.h_out = [torch.empty(c[2].shape, dtype=torch.float32).pin_memory()
                      for c in self.calls[0]]
        self.h2d = sum(t.numel() for t in self.h_w)
        self.d2h = sum(t.numel() * 4 for t in self.h_out)

    def e2e_step(self, i):
        for j, (w, sf, out, _n, _d) in enumerate(self.calls[i % self.sets]):
            w.copy_(self.h_w[j], non_blocking=True)
            self.nvfp4.dequant(w, sf, out=out)
            self.h_out[j].copy_(out, non_blocking=True)

    def cpu_sample(self, threads):
        from nvfp4 import synthetic
        from oracle import oracle as O

        wd = synthetic.linear_weights(256, PREFILL_K, seed=5)

        def run():
            O.dequant(wd["w"], wd["sf"])

        n = 256 * PREFILL_K
        desc = (f"dequant of a [256, 4096] slice per pass ({n / 1e6:.2f} M elements; the "
                "oracle's cost is linear in elements; single thread)")
        return run, n / 1e9, desc, 1


# ---------------------------------------------------------------------------
# Workload: one MoE FFN layer (128 experts, top-8, H=2048, I=768).
# ---------------------------------------------------------------------------
MOE_E, MOE_K, MOE_H, MOE_I = 128, 8, 2048, 768


def moe_expert_bytes(H=MOE_H, I=MOE_I):
    # gate_up [2I, H] + down [H, I]: codes, scales, per-row fp32 scale_2
    return (2 * I * H // 2 + 2 * I * H // 16 + 4 * 2 * I) + (H * I // 2 + H * I // 16 + 4 * H)


class MoELayerBench:
    name = "moe"
    unit = "tokens/s"

    @staticmethod
    def describe(tokens, layers=None, world=1, exchange=None):
        return (f"one MoE FFN layer, 128 experts, top-8 (softmax, renormalised), hidden "
                f"2048, expert intermediate 768, NVFP4 gate_up [1536, 2048] and down "
                f"[2048, 768] per expert; T = {tokens} bf16 tokens ~N(0,1)")

    def __init__(self, device, seed=0, tokens=4096, layers=4):
        import torch
        from nvfp4 import synthetic
        from nvfp4.moe import MoELayer, MoEWeights

        self.torch = torch
        self.T = tokens
        self.workload = self.describe(tokens)
        # Distinct layers (weights 342 MB each) cycle so that inputs exceed L2.
        self.layers = []
        for l in range(layers):
            wd = synthetic.moe_weights_cuda(MOE_E, MOE_H, MOE_I, seed=seed + 97 * l, device=device)
            self.layers.append(MoELayer(MoEWeights.from_dict(wd, device), top_k=MOE_K))
        self.x = torch.randn((tokens, MOE_H), device=device).to(torch.bfloat16)
        self.y = torch.empty_like(self.x)
        for L in self.layers:
            L.workspace(tokens, device)
        self.sets = len(self.layers)
        # router x2, permute, gate_up, down, combine; the tensor-core expert
        # path (T * k >= 64 E) also gathers the rows into expert order.
        self.launches_per_step = 7 if tokens * MOE_K >= 64 * MOE_E else 6
        self.traffic_ok = tokens == 4096  # the captured layer
        # Distinct experts touched: expectation under uniform routing.
        touched = MOE_E * (1.0 - (1.0 - MOE_K / MOE_E) ** tokens)
        self.dominant_bytes = touched * moe_expert_bytes()
        self.dominant_name = f"MoE layer (T={tokens}): expert weight bytes of the experts touched"
        self.config = {"workload": self.workload, "T": tokens, "experts": MOE_E, "top_k": MOE_K,
                       "hidden": MOE_H, "intermediate": MOE_I,
                       "l2": f"inputs larger than L2: {layers} distinct layers (342 MB of expert "
                             f"weights each) cycle per step"}

    def run_step(self, i):
        self.layers[i % self.sets](self.x, out=self.y)

    def run_dominant(self, i):
        self.layers[i % self.sets](self.x, out=self.y)
        return 1

    def units(self, steps):
        return self.T * steps  # tokens

    def e2e_setup(self):
        torch = self.torch
        self.h_x = torch.randn(self.x.shape).to(torch.bfloat16).pin_memory()
        self.h_y = torch.empty(self.y.shape, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.h_x.numel() * 2
        self.d2h = self.h_y.numel() * 2

    def e2e_step(self, i):
        self.x.copy_(self.h_x, non_blocking=True)
        self.layers[i % self.sets](self.x, out=self.y)
        self.h_y.copy_(self.y, non_blocking=True)

    def cpu_sample(self, threads, n_tok=64):
        from nvfp4 import synthetic
        from oracle import oracle as O

        wd = synthetic.moe_weights(MOE_E, MOE_H, MOE_I, seed=5)
        x = synthetic.activations(n_tok, MOE_H, seed=6)

        def run():
            O.moe(x, wd, top_k=MOE_K, n_threads=threads)

        desc = f"{n_tok} tokens through one layer (oracle cost is linear in tokens)"
        return run, float(n_tok), desc


# ---------------------------------------------------------------------------
# Workload: gated DeltaNet decode step (the reference's default layer) with
# NVFP4 projections, B sequences.
# ---------------------------------------------------------------------------
def deltanet_weight_bytes():
    from nvfp4.deltanet import DeltaNetConfig

    c = DeltaNetConfig()
    rows = {"qkv": (c.total_qkv_dim(), c.d_model), "z": (c.z_dim(), c.d_model),
            "b": (c.num_value_heads, c.d_model), "a": (c.num_value_heads, c.d_model),
            "out": (c.d_model, c.z_dim())}
    return rows, sum(n * k // 2 + n * k // 16 + 4 * n for (n, k) in rows.values())


class DeltaNetBench:
    name = "deltanet"
    unit = "tokens/s"

    @staticmethod
    def describe(tokens, layers=None, world=1, exchange=None):
        return (f"one gated DeltaNet decode step of the reference's default layer (d_model "
                f"2048, 16 key / 32 value heads of 128 x 128, conv kernel 4) with NVFP4 "
                f"projections qkv [8192, 2048], z [4096, 2048], beta / alpha [32, 2048], out "
                f"[2048, 4096] (the four input projections row-stacked into one); {tokens} "
                f"sequences with their own fp32 state; bf16 activations on the decode GEMV")

    def __init__(self, device, seed=0, tokens=4, layers=8):
        import torch
        import nvfp4
        from nvfp4 import synthetic
        from nvfp4.deltanet import DeltaNetConfig, DeltaNetState, DeltaNetWeights, fuse_in_proj

        self.torch, self.B = torch, tokens
        self.cfg = DeltaNetConfig()
        self.workload = self.describe(tokens)
        rows, wbytes = deltanet_weight_bytes()
        c = self.cfg
        self.layers = []
        for l in range(layers):
            g = torch.Generator(device=device)
            g.manual_seed(seed + 31 * l)
            proj = {}
            for i, (name, (n, k)) in enumerate(rows.items()):
                wd = synthetic.linear_weights_cuda(n, k, seed=seed + 31 * l + i, device=device)
                proj[name] = (nvfp4.NvFp4Linear(k, n, weight_scale_2_rows=wd["ws2"]),
                              wd["w"], wd["sf"])
            r = lambda *shape: torch.randn(shape, generator=g, device=device) * 0.5
            w = DeltaNetWeights(**proj, a_log=r(c.num_value_heads), dt_bias=r(c.num_value_heads),
                                conv_q=r(c.q_dim(), c.conv_kernel), conv_k=r(c.k_dim(), c.conv_kernel),
                                conv_v=r(c.v_dim(), c.conv_kernel))
            self.layers.append((fuse_in_proj(w), DeltaNetState(c, batch=tokens, device=device)))
        self.x = torch.randn((tokens, c.d_model), device=device).to(torch.bfloat16)
        self.y = torch.empty_like(self.x)
        self.ws = torch.empty(64 << 20, dtype=torch.uint8, device=device)
        self.sets = layers
        self.launches_per_step = 4  # fused input projection, conv, recurrence, out projection
        state_bytes = 2 * 4 * tokens * (c.total_state_floats()
                                       + (c.q_dim() + c.k_dim() + c.v_dim()) * (c.conv_kernel - 1))
        self.dominant_bytes = wbytes + state_bytes
        self.dominant_name = (f"DeltaNet step (B={tokens}): NVFP4 projection weights "
                              f"{wbytes / 1e6:.1f} MB + fp32 state read and written")
        self.config = {"workload": self.workload, "B": tokens, "d_model": c.d_model,
                       "heads": [c.num_key_heads, c.num_value_heads],
                       "head_dims": [c.key_dim, c.value_dim],
                       "l2": f"inputs larger than L2: {layers} distinct layers "
                             f"({(wbytes + state_bytes / 2) / 1e6:.0f} MB each) cycle per step"}

    def _step(self, i):
        from nvfp4.deltanet import deltanet_forward

        w, st = self.layers[i % self.sets]
        deltanet_forward(self.x, self.y, w, st, self.cfg, proj_dtype=self.torch.bfloat16,
                         workspace=self.ws)

    def run_step(self, i):
        self._step(i)

    def run_dominant(self, i):
        self._step(i)
        return 1

    def units(self, steps):
        return self.B * steps  # tokens

    def e2e_setup(self):
        torch = self.torch
        self.h_x = torch.randn(self.x.shape).to(torch.bfloat16).pin_memory()
        self.h_y = torch.empty(self.y.shape, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.h_x.numel() * 2
        self.d2h = self.h_y.numel() * 2

    def e2e_step(self, i):
        self.x.copy_(self.h_x, non_blocking=True)
        self._step(i)
        self.h_y.copy_(self.y, non_blocking=True)

    def cpu_sample(self, threads):
        import numpy as np
        from nvfp4 import synthetic
        from nvfp4.deltanet import DeltaNetConfig
        from oracle import oracle as O

        c = DeltaNetConfig()
        rows, _ = deltanet_weight_bytes()
        rng = np.random.default_rng(5)
        w = {}
        for i, (name, (n, k)) in enumerate(rows.items()):
            wd = synthetic.linear_weights(n, k, seed=40 + i)
            w[name] = O.dequant(wd["w"], wd["sf"]) * wd["ws2"][:, None]
        f = lambda *sh: (rng.standard_normal(sh) * 0.5).astype(np.float32)
        w.update(a_log=f(c.num_value_heads), dt_bias=f(c.num_value_heads),
                 conv_q=f(c.q_dim(), c.conv_kernel), conv_k=f(c.k_dim(), c.conv_kernel),
                 conv_v=f(c.v_dim(), c.conv_kernel))
        cd = dict(d_model=c.d_model, num_key_heads=c.num_key_heads,
                  num_value_heads=c.num_value_heads, key_dim=c.key_dim, value_dim=c.value_dim,
                  conv_kernel=c.conv_kernel, rms_eps=c.rms_eps)
        st = O.deltanet_state(cd)
        x = rng.standard_normal(c.d_model).astype(np.float32)

        def run():
            O.deltanet_forward(cd, x, w, st)

        desc = ("one token through the layer: the reference's deltanet_forward restated "
                "(fp32, dequantized projection weights; single thread)")
        return run, 1.0, desc, 1


# ---------------------------------------------------------------------------
# Workload: 48-layer stack of the MoE layer, expert-parallel over the ranks.
# ---------------------------------------------------------------------------
class EPStackBench:
    """Config 4: a 48-layer stack of the config-3 MoE layer, h = h + MoE(h)
    (the residual add is fused in the combine kernel), expert-parallel over
    the ranks.  A step is one pass of the stack over the global token batch."""

    name = "ep"
    unit = "tokens/s"
    graphable = False  # set per batch: True with the fixed-capacity or peer exchange
    scaling = "strong"  # the global token batch is fixed; experts and tokens split over GPUs

    @staticmethod
    def describe(tokens, layers=48, world=1, exchange="p2p"):
        how = ("NCCL all-to-all dispatch/combine" if exchange == "nccl" else
               "device-initiated dispatch/combine through peer memory (NVLink stores and loads "
               "issued by the kernels, cross-GPU flags)")
        return (f"{layers}-layer stack of MoE FFN layers h = h + MoE(h) (128 experts, top-8, "
                f"hidden 2048, intermediate 768, NVFP4 experts; the residual add is fused in "
                f"the combine); expert-parallel over {world} GPU(s) ({MOE_E // world} experts "
                f"each) with {how}; {tokens} bf16 tokens ~N(0,1) per step "
                f"({tokens // world} per GPU)")

    def __init__(self, device, seed=0, tokens=64, layers=48, exchange="p2p"):
        import torch
        import torch.distributed as dist
        from nvfp4.ep import EPMoELayer
        from nvfp4.moe import MoEWeights

        self.torch = torch
        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        if tokens % world:
            raise ValueError("global token count must divide by the number of GPUs")
        self.world, self.rank = world, rank
        self.T = tokens
        self.T_local = tokens // world
        self.n_layers = layers
        self.epr = epr = MOE_E // world
        self.exchange_mode = exchange
        self.workload = self.describe(tokens, layers, world, exchange)
        self.layers, self.local_w = [], []
        # One set of peer windows for the whole stack: the layers run one
        # after another, so layer l+1 reuses layer l's receive rows (L2-resident).
        windows = None
        if exchange == "p2p":
            from nvfp4.ep import PeerWindows
            windows = PeerWindows.rendezvous(self.T_local * MOE_K, MOE_H, timeout_ms=10000)
        self.windows = windows
        for l in range(layers):
            g = torch.Generator(device=device)
            g.manual_seed(1000 + l)  # router identical on every rank
            router = torch.randn((MOE_H, MOE_E), generator=g, device=device) * 0.02
            wd = synthetic_local_experts(epr, seed=seed + 7919 * l + 104729 * rank, device=device)
            wd["router"] = router
            local = MoEWeights.from_dict(wd, device)
            self.local_w.append(local)
            self.layers.append(EPMoELayer(local, router, top_k=MOE_K, num_experts=MOE_E,
                                          exchange=exchange, max_tokens=self.T_local,
                                          windows=windows))
        g = torch.Generator(device=device)
        g.manual_seed(77 + rank)
        self.x = torch.randn((self.T_local, MOE_H), generator=g, device=device).to(torch.bfloat16)
        if exchange == "p2p":
            # router logits, top-k + dispatch + wait, permutation, 2 expert GEMVs,
            # done signal, combine
            self.graphable = True
            self.exchange = "peer memory, CUDA graph"
            self.launches_per_step = layers * 7
        else:
            # Fixed-capacity exchange (no host-side counts) for small batches:
            # the whole step, NCCL calls included, is replayed from a CUDA graph.
            self.graphable = self.layers[0].uses_static(self.T_local)
            self.exchange = "fixed capacity, CUDA graph" if self.graphable else "variable counts"
            self.launches_per_step = layers * 10
        self.sets = 1
        self.dominant_bytes = None
        # Expert weight bytes one GPU streams per layer: its experts that at
        # least one of the T tokens routes to (expectation under uniform routing).
        self.touched_per_gpu = epr * (1.0 - (1.0 - MOE_K / MOE_E) ** tokens)
        self.layer_bytes = self.touched_per_gpu * moe_expert_bytes()
        self.config = {"workload": self.workload, "layers": layers, "global_tokens": tokens,
                       "experts_per_gpu": epr, "parallelism": f"ep{world}",
                       "exchange": self.exchange,
                       "l2": f"inputs larger than L2: {layers} layers x {342 // world} MB of "
                             f"expert weights per GPU per step"}

    def run_step(self, i):
        h = self.x
        for L in self.layers:
            h = L(h, residual=h)
        self.out = h

    def units(self, steps):
        return self.T_local * steps  # per rank; the job total is this times the world size

    def roofline(self, ms_per_step, peaks):
        """Layer-level roofline: the expert weight bytes one GPU must stream
        per layer over the average layer time of the timed region."""
        layer_s = ms_per_step / 1e3 / self.n_layers
        achieved = self.layer_bytes / layer_s / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"],
                # The committed capture is of one layer at one GPU (its 7 launches).
                "traffic": load_traffic(self.name) if self.world == 1 and self.exchange.startswith(
                    "peer") else None,
                "kernel": (f"one expert-parallel MoE layer ({self.launches_per_step // self.n_layers}"
                           f" launches), per GPU"),
                "algorithmic_bytes_per_launch": self.layer_bytes,
                "algorithmic_bytes_note": (
                    f"{self.touched_per_gpu:.2f} of this GPU's {self.epr} experts touched by "
                    f"{self.T} tokens x top-{MOE_K} (expectation, uniform routing) x "
                    f"{moe_expert_bytes()} bytes per expert"),
                "avg_launch_us": layer_s * 1e6,
                "timing": "average layer time of the timed region (CUDA events)",
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, copy burst)"}

    def parity(self):
        """Layer 0 of the stack on this step's tokens, every rank's tokens,
        against the CPU oracle's MoE layer (the checker; outside every timed
        region).  Rank 0 gathers the tokens, the outputs and layer 0's experts
        from all ranks and evaluates the oracle on all tokens; router
        near-ties (a gap < 1e-5 among the k+1 largest probabilities) replay
        the GPU's expert choice."""
        import numpy as np
        import torch
        import torch.distributed as dist

        world, rank = self.world, self.rank
        L0 = self.layers[0]
        if self.exchange_mode == "p2p":
            y = L0.forward_p2p(self.x, out=torch.empty((self.T_local, MOE_H),
                                                       dtype=torch.float32, device=self.x.device))
            out_dtype = "f32"
        else:
            y = L0(self.x)
            out_dtype = "bf16"
        torch.cuda.synchronize()

        def gather(t):
            t = t.contiguous()
            if world == 1:
                return t
            out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype,
                              device=t.device)
            dist.all_gather_into_tensor(out, t)
            return out

        u8 = lambda t: t.view(torch.uint8) if t.dtype != torch.uint8 else t
        w = self.local_w[0]
        xs, ys = gather(self.x), gather(y)
        full = {"gu_w": gather(w.gate_up), "gu_sf": gather(u8(w.gate_up_scale)),
                "gu_ws2": gather(w.gate_up_scale_2), "dn_w": gather(w.down),
                "dn_sf": gather(u8(w.down_scale)), "dn_ws2": gather(w.down_scale_2)}
        ids_gpu = L0.backend.route(xs)[0] if rank == 0 else None
        torch.cuda.synchronize()
        if rank != 0:
            return None
        from oracle import oracle as O

        wd = {k: v.cpu().numpy() for k, v in full.items()}
        wd["router"] = w.router.float().cpu().numpy()
        x = xs.float().cpu().numpy()
        got = ys.float().cpu().numpy()
        ids_gpu = ids_gpu.cpu().numpy()
        cores = O.host_cores()
        _, probs = O.router(x, wd["router"])
        srt = -np.sort(-probs, axis=1)[:, : MOE_K + 1]
        ties = (srt[:, :-1] - srt[:, 1:]).min(axis=1) < 1e-5
        ref, ref_ids, _ = O.moe(x, wd, top_k=MOE_K, n_threads=cores)
        flips = [i for i in range(len(x)) if not np.array_equal(ref_ids[i], ids_gpu[i])]
        unexplained = [i for i in flips if not ties[i]]
        if flips:
            ref, _, _ = O.moe(x, wd, top_k=MOE_K, force_ids=ids_gpu, n_threads=cores)
        ref64 = ref.astype(np.float64)
        err = float(np.abs(got - ref64).max() / np.sqrt(np.mean(ref64 * ref64)))
        return {"max_err_over_rms": err, "tol": 2e-2, "ok": bool(err <= 2e-2 and not unexplained),
                "layer": 0, "tokens": int(len(x)), "out_dtype": out_dtype,
                "near_tie_tokens_replayed": len(flips), "routing_mismatches": len(unexplained),
                "oracle": "CPU oracle MoE layer (C), all tokens of every rank"}

    def e2e_setup(self):
        torch = self.torch
        self.h_x = torch.randn(self.x.shape).to(torch.bfloat16).pin_memory()
        self.h_y = torch.empty(self.x.shape, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.h_x.numel() * 2
        self.d2h = self.h_y.numel() * 2

    def e2e_step(self, i):
        self.x.copy_(self.h_x, non_blocking=True)
        self.run_step(i)
        self.h_y.copy_(self.out, non_blocking=True)

    def cpu_sample(self, threads, n_tok=8):
        from nvfp4 import synthetic
        from oracle import oracle as O

        wd = synthetic.moe_weights(MOE_E, MOE_H, MOE_I, seed=5)
        x = synthetic.activations(n_tok, MOE_H, seed=6)

        def run():
            O.moe(x, wd, top_k=MOE_K, n_threads=threads)

        n_layers = getattr(self, "n_layers", 48)
        desc = (f"{n_tok} tokens through one layer, reported per layer-token and divided by "
                f"the layer count {n_layers} (oracle cost is linear in tokens and layers)")
        return run, float(n_tok) / n_layers, desc


def synthetic_local_experts(epr, seed, device):
    """NVFP4 expert weights of `epr` experts (distributions of nvfp4.synthetic)."""
    from nvfp4 import synthetic

    d = synthetic.moe_weights_cuda(epr, MOE_H, MOE_I, seed=seed, device=device)
    d.pop("router")
    return d


WORKLOADS = {"gemv": GemvSweep, "prefill": PrefillSweep, "prefill_w4a4": PrefillW4A4Sweep,
             "dequant": DequantBench, "moe": MoELayerBench, "ep": EPStackBench,
             "deltanet": DeltaNetBench}


# ---------------------------------------------------------------------------
def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def time_cpu(run, units, reps_target_s=10.0, max_reps=50):
    run()  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el >= reps_target_s or n >= max_reps:
            break
    return units * n / el, n, el


def cpu_baselines(wl_cls, wl, target_s=10.0):
    """The oracle port of the reference's CPU loop on this host, timed twice:
    single-thread (the reference's own form, nvfp4/deltanet.mojo:569-584, one
    core) and with OpenMP over output rows on every host core.  The timing
    build is compiled for this host (-O3 -march=native, still without FMA
    contraction) when a compiler is present."""
    from oracle import oracle as O

    build = O.use_native_build()
    cores = O.host_cores()
    out = {}
    for label, threads in (("single_thread", 1), ("openmp", cores)):
        res = wl_cls.cpu_sample(wl, threads)
        run, units, desc = res[:3]
        used = res[3] if len(res) > 3 else threads
        v, n, el = time_cpu(run, units, reps_target_s=target_s)
        out[label] = {"value": v, "cores": used, "sample": f"{desc}; {n} passes in {el:.1f} s"}
        if used == 1 and label == "single_thread" and len(res) > 3:
            break  # the sample is single-threaded by construction
    best = out.get("openmp", out["single_thread"])
    return {"value": best["value"], "unit": wl_cls.unit, "cores": best["cores"], "kind": "port",
            "sample": best["sample"], "build": build, **out}


def run_reference(args, world, rank):
    """CPU reference arm: the oracle port of the reference's CPU path."""
    if rank != 0:
        return 0
    from oracle import oracle as O

    wl_cls = WORKLOADS[args.workload]
    build = O.use_native_build()
    cores = O.host_cores()
    # Build only what the CPU sample needs (no GPU use).
    wl = wl_cls.__new__(wl_cls)
    if args.workload == "ep":
        wl.n_layers = args.layers
    res = wl_cls.cpu_sample(wl, cores)
    run, units, desc = res[:3]
    cores = res[3] if len(res) > 3 else cores
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    el = time.perf_counter() - t0
    value = units * args.steps / el
    if hasattr(wl_cls, "describe"):
        wdesc = wl_cls.describe(args.tokens, args.layers, world, args.exchange)
    else:
        wdesc = wl_cls.workload
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": wl_cls.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
        "scaling": getattr(wl_cls, "scaling", "weak"),
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wdesc, "sample": desc},
        "cpu_baseline": {"value": value, "unit": wl_cls.unit, "cores": cores, "kind": "port",
                         "sample": desc, "build": build},
        "e2e": {"value": value, "unit": wl_cls.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def time_dominant(wl, stream, steps, warmup):
    """Average duration of one dominant launch: a CUDA graph holding only the
    dominant launches of each weight set, replayed back to back on the
    launching stream and timed with CUDA events (no host gaps)."""
    import torch

    dg = []
    n_dom = 1
    for s in range(getattr(wl, "sets", 1)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            n_dom = wl.run_dominant(s)
        dg.append(g)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(warmup):
            dg[i % len(dg)].replay()
        d0 = torch.cuda.Event(enable_timing=True)
        d1 = torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for i in range(steps):
            dg[i % len(dg)].replay()
        d1.record(stream)
    torch.cuda.synchronize()
    ms = d0.elapsed_time(d1) / (steps * n_dom)
    del dg
    return ms


def dominant_roofline(wl, dom_ms, peaks):
    # The committed captures are of the default shapes (a workload clears
    # traffic_ok when its dominant launch is another shape).
    traffic = load_traffic(wl.name) if getattr(wl, "traffic_ok", True) else None
    if getattr(wl, "bound", "hbm") == "tensor":
        achieved = wl.dominant_bytes / (dom_ms / 1e3) / 1e12
        scale = getattr(wl, "peak_scale", 1.0)
        peak = peaks["bf16_tflops"] * scale
        src = (f"{peaks['source']} (MEASURED_PEAKS.json bf16_tflops, cuBLAS bf16 burst)"
               if scale == 1.0 else
               f"{scale:g} x {peaks['source']} bf16_tflops (MEASURED_PEAKS.json, cuBLAS bf16 "
               f"burst): dense FP4 is {scale:g} x dense BF16 on B200; no FP4 peak is measured")
        return {"bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": traffic, "kernel": wl.dominant_name,
                "algorithmic_flop_per_launch": wl.dominant_bytes,
                "avg_launch_us": dom_ms * 1e3, "peak_source": src}
    achieved = wl.dominant_bytes / (dom_ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
            "kernel": wl.dominant_name, "algorithmic_bytes_per_launch": wl.dominant_bytes,
            "avg_launch_us": dom_ms * 1e3,
            "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, copy burst)"}


def capture_step_graphs(wl, stream):
    import torch

    graphs = []
    for s in range(getattr(wl, "sets", 1)):
        graphs.append(torch.cuda.CUDAGraph())
        with torch.cuda.graph(graphs[-1], stream=stream):
            wl.run_step(s)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):  # a first replay outside the timed region
        for g in graphs:
            g.replay()
    torch.cuda.synchronize()
    return graphs


def time_steps(wl, graphs, stream, steps, start=0):
    import torch

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(start, start + steps):
            if graphs:
                graphs[i % len(graphs)].replay()
            else:
                wl.run_step(i)
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def secondary_line(cls, device, peaks, steps, warmup):
    """A single-GPU workload measured beside the headline one (same process,
    same GPU): its sweep throughput and its dominant launch's roofline."""
    import torch

    wl = cls(device)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for i in range(warmup):
            wl.run_step(i)
    torch.cuda.synchronize()
    graphs = capture_step_graphs(wl, stream)
    t_ms = time_steps(wl, graphs, stream, steps)
    dom_ms = time_dominant(wl, stream, steps, warmup)
    out = {"workload": wl.workload, "value": wl.units(steps) / (t_ms / 1e3), "unit": wl.unit,
           "ms_per_step": t_ms / steps, "steps": steps,
           "roofline": dominant_roofline(wl, dom_ms, peaks), "l2": wl.config.get("l2")}
    del graphs, wl
    gc.collect()
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="ep", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the decode GEMV and prefill lines measured beside the EP stack")
    ap.add_argument("--tokens", type=int, default=None,
                    help="MoE: tokens per step (default 4096); EP stack: global tokens (default "
                         "64); DeltaNet: sequences per step (default 4)")
    ap.add_argument("--layers", type=int, default=48, help="EP stack: number of MoE layers")
    ap.add_argument("--split", default=None, choices=["columns"],
                    help="gemv at N > 1: split every linear by output rows over the GPUs "
                         "(default: independent replicas)")
    ap.add_argument("--exchange", default="p2p", choices=["nccl", "p2p"],
                    help="EP stack: device-initiated peer-memory exchange or NCCL all-to-all")
    ap.add_argument("--clock-window", type=float, default=0.6,
                    help="seconds of untimed step replays before the timed steps, inside the "
                         "clock-sampling window (so the sampler sees the GPU under this load)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.tokens is None:
        args.tokens = {"ep": 64, "deltanet": 4}.get(args.workload, 4096)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)

    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = load_peaks()
    kw = {"tokens": args.tokens} if args.workload in ("moe", "ep", "deltanet") else {}
    if args.workload == "gemv":
        kw.update(split=args.split, world=world, rank=rank)
    if args.workload == "ep":
        kw["layers"] = args.layers
        kw["exchange"] = args.exchange
    wl = WORKLOADS[args.workload](device, seed=17 * rank, **kw)
    stream = torch.cuda.Stream(device)

    # Warm-up (also loads the library and JITs nothing: all kernels are prebuilt).
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            wl.run_step(i)
    torch.cuda.synchronize()

    graphs = None
    if not args.no_graph and getattr(wl, "graphable", True):
        graphs = capture_step_graphs(wl, stream)

    dom_ms = None
    if hasattr(wl, "run_dominant"):
        dom_ms = time_dominant(wl, stream, args.steps, args.warmup)

    # Untimed replays fill the clock-sampling window before the timed steps;
    # every rank runs the same count (the peer exchange steps in lockstep).
    barrier(world)
    one = time_steps(wl, graphs, stream, 2) / 2
    n_pre = int(max_over_ranks(float(math.ceil(args.clock_window * 1e3 / max(one, 1e-3))), world))
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if n_pre:
        time_steps(wl, graphs, stream, n_pre)
    t_ms = time_steps(wl, graphs, stream, args.steps)
    clk = clocks.stop()
    clk["window"] = (f"{n_pre} untimed steps ({n_pre * one / 1e3:.2f} s) then the "
                     f"{args.steps} timed steps ({t_ms / 1e3:.3f} s)")
    barrier(world)
    t_ms = max_over_ranks(t_ms, world)
    ms_per_step = t_ms / args.steps
    value = wl.units(args.steps) * world / (t_ms / 1e3)

    # End to end through the public API with host buffers.
    wl.e2e_setup()
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            wl.e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            wl.e2e_step(i)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = wl.units(args.steps) * world / (e2e_ms / 1e3)

    roof = None
    if dom_ms and wl.dominant_bytes:
        roof = dominant_roofline(wl, dom_ms, peaks)
    elif hasattr(wl, "roofline"):
        roof = wl.roofline(ms_per_step, peaks)

    parity = None
    if hasattr(wl, "parity") and not args.no_parity:
        parity = wl.parity()

    used_graph = bool(graphs)
    secondary = None
    if args.workload == "ep" and world == 1 and not args.no_secondary:
        secondary = {}
        graphs = None
        for key, cls in (("gemv", GemvSweep), ("prefill", PrefillSweep)):
            secondary[key] = secondary_line(cls, device, peaks, max(args.steps, 20), args.warmup)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baselines(type(wl), wl)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": getattr(wl, "scaling", "weak"),
            "vs_baseline": None, "dtype": getattr(wl, "dtype", "bf16"),
            "data": "synthetic", "config": dict({"parallelism": (
                ("column split" if wl.config.get("split") else "replicas") if world > 1
                else "single GPU")}, **wl.config, graph=used_graph),
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d,
                    "d2h_bytes_per_step": wl.d2h},
            "clocks": clk, "gpu_launches": wl.launches_per_step * args.steps,
        }
        if parity is not None:
            line["parity"] = parity
        if secondary:
            line["secondary"] = secondary
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        # CUDA graphs that hold NCCL calls must be gone before the process
        # group is destroyed, or the exit waits for them forever.
        torch.cuda.synchronize()
        graphs = None
        if getattr(wl, "windows", None) is not None:
            wl.windows.close()  # collective: every rank unmaps, then each frees its own
        wl = None
        gc.collect()
        torch.cuda.synchronize()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

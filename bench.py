#!/usr/bin/env python
"""Benchmark of the packed-quadtree MTC GEMM on B200 (one JSON line on rank 0).

Metric: "dequant-GEMM TFLOP/s at M=4096; decode GEMV
packed-weight GB/s vs B200 peak".  ``--config`` picks one BASELINE.json
configuration; all inputs are seeded synthetic stand-ins with the
configuration's shapes and value distributions (no checkpoint or dataset is
available here).  Allocations are made on the GPU by tensorpack_b200.quant.

  llama_gate  (default; the headline) Llama-3-8B gate_proj 4096 x 14336,
              Student-t(4) * 0.02, MTC-QT-P at 4.25 b/w: prefill M = 4096,
              decode M = 1 and M = 16
  llama_layer the seven Llama-3-8B linears of one layer (q, k, v, o, gate,
              up, down) at 4.5 b/w: prefill M = 4096, decode M = 1 and 16
  llm_like    4096 x 4096 LLM-like layer at 4.25 b/w: prefill M = 512,
              decode M = 1 and 16
  cpu_ref     1024 x 1024 N(0, 1), unpermuted MTC-QT at 3.125 b/w: M = 256,
              decode M = 1
  qwen_stack  24 Qwen2.5-0.5B-shaped layers (q, k, v, o 896 / 128 wide,
              gate, up 896 x 4864, down 4864 x 896) at 3.125 b/w, 168
              distinct matrices: prefill M = 2048 and decode M = 1 over the
              whole stack
  stress      8192 x 8192 multi-scale matrix, unpermuted MTC-QT at 2.5 b/w,
              X bf16 values: prefill M = 8192, decode M = 1

Fields of the line:
  value     prefill TFLOP/s (2 M K N summed over the configuration's
            matrices / device time of gather + fused GEMM + column scatter),
            256 MB L2 flush before every step
  roofline  the prefill kernel alone (CUDA events on its stream) against the
            measured dense bf16 peak, and its committed ncu DRAM traffic
  decode    M = 1 (and decode_by_M for the other decode sizes): GB/s of
            accounted packed bytes (payload + scales + modes + split flags +
            permutation indices) per call, rotating over copies of the
            device layouts that total > 4x L2, launches captured in a CUDA
            graph; roofline against the measured HBM copy bandwidth
  e2e       the prefill metric through the public HostGemm with pinned host
            X and Y (copies in the timed region), with the achieved host-link
            GB/s
  parity    outside the timed region: the GPU dequant against the oracle
            rebuild (bit for bit) and the relative Frobenius error of the
            GEMM outputs against the fp64 product with that dequant
  cpu_baseline  the reference's packed Numba GEMM algorithm (oracle port,
            fixed 16x16 blocks at the same bits/weight, X packed as P16) on
            a bounded sample, on this host's cores

Multi-GPU (torchrun, one process per GPU, single-matrix configurations): the
layer is column-sharded across ranks (strong scaling), one NCCL all-gather
per GEMM; times are the max over ranks.  ``--impl reference`` times the
reference CPU implementation instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

METRIC = "dequant-GEMM TFLOP/s at M=4096; decode GEMV packed-weight GB/s vs B200 peak"
L2_BYTES = 126 * 1024 * 1024
TOL = 2e-3  # relative Frobenius error of the GEMM output


# ----------------------------------------------------------------------------- workloads

@dataclass
class Layer:
    name: str
    K: int
    N: int
    seed: int
    W: Optional[np.ndarray] = None
    h: Optional[np.ndarray] = None
    alloc: object = None
    mat: object = None


@dataclass
class Workload:
    name: str
    description: str
    model: str
    bits: float
    permuted: bool
    layers: List[Layer]
    prefill_M: int
    decode_Ms: List[int]
    x_kind: str = "llm"          # "llm" (1 % outlier channels x50), "normal", "bf16"
    parity_layers: int = 7       # how many layers the parity check rebuilds
    meta: Dict = field(default_factory=dict)

    @property
    def single(self) -> bool:
        return len(self.layers) == 1


def make_workload(name: str) -> Workload:
    if name == "llama_gate":
        return Workload(name, "llama3-8b gate_proj 4096x14336 MTC-QT-P @4.25 b/w (sizes 32..4), prefill M=4096 + "
                              "decode M=1, 16", "Llama-3-8B-shaped linear (random init, Student-t(4)*0.02)", 4.25, True,
                        [Layer("gate", 4096, 14336, 0)], 4096, [1, 16])
    if name == "llama_layer":
        shapes = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
                  ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]
        return Workload(name, "llama3-8b layer: q,o 4096x4096, k,v 4096x1024, gate,up 4096x14336, down 14336x4096, "
                              "MTC-QT-P @4.5 b/w, prefill M=4096 + decode M=1, 16",
                        "Llama-3-8B-shaped linears (random init, Student-t(4)*0.02)", 4.5, True,
                        [Layer(n, k, o, 100 + i) for i, (n, k, o) in enumerate(shapes)], 4096, [1, 16])
    if name == "llm_like":
        return Workload(name, "LLM-like layer 4096x4096 Student-t(4)*0.02, MTC-QT-P @4.25 b/w, prefill M=512 + decode "
                              "M=1, 16", "LLM-like single layer (synthetic)", 4.25, True,
                        [Layer("llm_like", 4096, 4096, 3)], 512, [1, 16])
    if name == "cpu_ref":
        return Workload(name, "CPU-ref config: W 1024x1024 N(0,1), MTC-QT @3.125 b/w (unpermuted), M=256 + decode M=1",
                        "CPU reference configuration (synthetic)", 3.125, False,
                        [Layer("cpu_ref", 1024, 1024, 0)], 256, [1], x_kind="normal")
    if name == "qwen_stack":
        shapes = [("q", 896, 896), ("k", 896, 128), ("v", 896, 128), ("o", 896, 896),
                  ("gate", 896, 4864), ("up", 896, 4864), ("down", 4864, 896)]
        layers = [Layer(f"l{li}.{n}", k, o, 1000 + 7 * li + i)
                  for li in range(24) for i, (n, k, o) in enumerate(shapes)]
        return Workload(name, "Qwen2.5-0.5B-shaped stack: 24 layers x (q,o 896x896, k,v 896x128, gate,up 896x4864, "
                              "down 4864x896), 168 distinct matrices, MTC-QT-P @3.125 b/w, prefill M=2048 + decode M=1",
                        "Qwen2.5-0.5B-shaped linear stack (random init, Student-t(4)*0.02)", 3.125, True, layers, 2048,
                        [1], parity_layers=7)
    if name == "stress":
        return Workload(name, "multi-scale stress 8192x8192 (32x32 blocks N(0,s2), s2 log-uniform 1e-3..1e2), MTC-QT "
                              "@2.5 b/w (unpermuted), X bf16 M=8192 + decode M=1",
                        "multi-scale stress matrix (synthetic)", 2.5, False, [Layer("stress", 8192, 8192, 2)], 8192,
                        [1], x_kind="bf16")
    raise ValueError(f"unknown config {name}")


CONFIGS = ("llama_gate", "llama_layer", "llm_like", "cpu_ref", "qwen_stack", "stress")


def layer_weights(wl: Workload, L: Layer):
    """Seeded weights and importance of one layer."""
    import inputs

    if wl.name == "cpu_ref":
        W, h, _ = inputs.cpu_ref_config()
        return W, h
    if wl.name == "stress":
        return inputs.multiscale(L.K, seed=L.seed), None
    return inputs.llm_like(L.K, L.N, seed=L.seed)


def activations(wl: Workload, M: int, K: int, seed: int) -> np.ndarray:
    import inputs

    if wl.x_kind == "normal":
        if wl.name == "cpu_ref" and M == 256 and K == 1024 and seed == 1:
            return inputs.cpu_ref_config()[2]
        return np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)
    if wl.x_kind == "bf16":
        X = np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)
        return (X.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)  # bf16 values (truncated)
    return inputs.llm_activations(M, K, seed=seed, outlier_seed=0)


def workload_config(wl: Workload, gpus: int) -> dict:
    cfg = {"workload": wl.description, "model": wl.model, "global_batch": wl.prefill_M, "seq_len": 1,
           "parallelism": f"column-shard x{gpus}" if gpus > 1 else "none", "bits_per_weight": wl.bits,
           "matrices": len(wl.layers),
           "l2_policy": "prefill: 256 MB L2 flush before each step; decode: device layouts rotated over copies "
                        "> 4x L2"}
    if wl.single:
        cfg["K"], cfg["N"] = wl.layers[0].K, wl.layers[0].N
    if wl.x_kind == "bf16":
        cfg["x_dtype"] = "bf16 values (passed as fp32)"
    return cfg


def allocate(wl: Workload, dev):
    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.quant import PermutedQuadtreeRD, QuadtreeRD

    for L in wl.layers:
        L.W, L.h = layer_weights(wl, L)
        rd = PermutedQuadtreeRD if wl.permuted else QuadtreeRD
        L.alloc = rd(L.W, L.h, (32, 16, 8, 4), device=dev).select(wl.bits)
        L.mat = MTCMatrix.from_qt_allocation(L.W, L.alloc)


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """NVML sampling of SM clock and throttle reasons during a timed region."""

    NAMES = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
             0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, index: int, period_s: float = 0.005):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self._t = threading.Thread(target=self._run, args=(period_s,), daemon=True)

    def _run(self, period):
        while not self._stop.is_set() and self._nv is not None:
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                mask = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.NAMES.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(period)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def committed_traffic(config: str, kernel: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/), if any."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 3 and not line.startswith("#") and parts[0] == config and parts[1] == kernel:
            return float(parts[2])
    return None


# ----------------------------------------------------------------------------- CPU leg (oracle as checker)

def cpu_reference_sample(wl: Workload, seed=0):
    """The reference's packed-GEMM algorithm (oracle port of mtc_gemm,
    mtc/kernels/gemm.py:124-210) on a bounded sample of the configuration:
    min(M, 256) tokens x K x min(N, 1024) output features of its largest
    matrix, fixed 16x16 blocks at the same bits/weight with bf16 scales (the
    reference cannot run quadtree leaves), X packed as P16."""
    import numba

    from oracle import mtc_oracle as O

    numba.set_num_threads(os.cpu_count() or 1)
    L = max(wl.layers, key=lambda l: l.K * l.N)
    W, h = (L.W, L.h) if L.W is not None else layer_weights(wl, L)
    n = min(L.N, 1024)
    rows = min(wl.prefill_M, 256)
    Ws = np.ascontiguousarray(W[:, :n])
    alloc = O.allocate_fixed(Ws, wl.bits, h, 16, scale_format="bf16")
    B = O.PackedFixed.from_allocation(Ws, alloc.modes, alloc.scales, 16)
    X = activations(wl, rows, L.K, seed + 7)
    A = O.p16_operand(X, 16)
    O.packed_gemm(A, B)  # JIT warm-up
    flops = 2.0 * rows * L.K * n
    sample = (f"{rows} tokens x {L.K} x {n} features of {L.name} (fixed 16x16 RD blocks @{wl.bits} b/w bf16 scales, "
              f"X as P16)")
    return (lambda: O.packed_gemm(A, B)), flops, numba.get_num_threads(), sample


def cpu_baseline(wl: Workload, seconds: float = 10.0):
    fn, cflops, cores, sample = cpu_reference_sample(wl)
    ts = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(ts) < 3:
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return {"value": cflops / statistics.median(ts) / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": sample + f", median of {len(ts)} calls"}


def parity_check(wl: Workload, dev, decode_outputs, prefill_outputs):
    """Checker outside the timed region: the GPU dequant of the first
    ``parity_layers`` matrices against the oracle rebuild (bit for bit) and
    the relative Frobenius error of the prefill and decode outputs against
    the fp64 product with that dequant (computed with torch on the device)."""
    import torch

    from oracle import mtc_oracle as O

    exact, pre_err, dec_err = True, 0.0, {}
    for i, L in enumerate(wl.layers[:wl.parity_layers]):
        a = L.alloc
        if wl.permuted:
            inner = a.inner
            ref = O.permuted_quadtree_dequant(L.W, a.row_perm, a.col_perm, inner.sizes, inner.leaf, inner.modes,
                                              inner.scales)
        else:
            ref = O.quadtree_dequant(L.W, a.sizes, a.leaf, a.modes, a.scales)
        gpu = L.mat.to_array()
        exact = exact and bool(np.array_equal(gpu, ref))
        R = torch.from_numpy(ref).to(dev, torch.float64)
        for (M, j), (X, Y) in list(prefill_outputs.items()) + list(decode_outputs.items()):
            if j != i:
                continue
            Yr = X.to(torch.float64) @ R
            e = float(torch.linalg.norm(Yr - Y.to(torch.float64)) / torch.linalg.norm(Yr))
            if (M, j) in prefill_outputs:
                pre_err = max(pre_err, e)
            else:
                dec_err[str(M)] = max(dec_err.get(str(M), 0.0), e)
        del R
    return {"dequant_bit_exact": exact, "matrices_checked": min(len(wl.layers), wl.parity_layers),
            "prefill_rel_err": pre_err, "decode_rel_err": dec_err, "tolerance": TOL,
            "pass": exact and pre_err < TOL and all(v < TOL for v in dec_err.values())}


def run_reference(args, rank):
    if rank != 0:
        return
    wl = make_workload(args.config)
    fn, flops, cores, sample = cpu_reference_sample(wl)
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    v = flops / t / 1e12
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": workload_config(wl, args.gpus),
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- GPU arm

def rotated_decoders(ds, M, copies, lib, stream_handle):
    """Per copy index, a function launching the decode of ``ds`` at M tokens
    on a private copy of the buffers the kernel streams (the strip stream
    for M <= 4, the sub-stage images for 4 < M <= 16)."""
    import ctypes

    import torch

    from tensorpack_b200 import _lib

    pr = None if ds.row_perm is None else ds.row_perm.data_ptr()
    pc = None if ds.col_perm is None else ds.col_perm.data_ptr()
    fns, keep = [], []
    if M <= 4 and ds.decode_kernel == "strip" and ds.strip_fits(M):
        sp = ds.strip()
        kernel, nbytes = "strip_kernel", sp.stream_bytes
        for _ in range(copies):
            bufs = [sp.stream.clone(), sp.batch_off.clone(), sp.strip_batch.clone()]
            keep.append(bufs)
            d = _lib.StripDesc.from_buffer_copy(sp.desc_for(M))
            d.stream, d.batch_off, d.strip_batch = [b.data_ptr() for b in bufs]
            keep.append(d)

            def f(X, Y, d=d):
                _lib.check(lib.mtc_strip_decode(ctypes.byref(d), X.data_ptr(), M, X.stride(0), pr, pc, Y.data_ptr(),
                                                Y.stride(0), ds.status.data_ptr(), None, stream_handle()),
                           "strip decode")
            fns.append(f)
    else:
        kernel, nbytes = "decode_kernel", ds.stage_images.numel()
        ws = torch.empty(max(int(lib.mtc_decode_workspace_bytes(ctypes.byref(ds.desc), M)), 256), dtype=torch.uint8,
                         device=ds.device)
        keep.append(ws)
        for _ in range(copies):
            bufs = [ds.stage_images.clone(), ds.stage_counts.clone(), ds.stage_offsets.clone(),
                    ds.stage_ranges.clone()]
            keep.append(bufs)
            d = _lib.StreamDesc.from_buffer_copy(ds.desc)
            d.stage_images, d.stage_counts, d.stage_offsets, d.stage_ranges = [b.data_ptr() for b in bufs]
            keep.append(d)

            def f(X, Y, d=d):
                _lib.check(lib.mtc_decode(ctypes.byref(d), X.data_ptr(), M, X.stride(0), pr, pc, Y.data_ptr(),
                                          Y.stride(0), ws.data_ptr(), ws.numel(), ds.decode_counters.data_ptr(),
                                          ds.status.data_ptr(), None, stream_handle()), "decode")
            fns.append(f)
    return fns, keep, kernel, nbytes


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="llama_gate", choices=CONFIGS)
    ap.add_argument("--decode-reps", type=int, default=8, help="passes over the rotated copies per decode timing")
    ap.add_argument("--decode-kernel", default="strip", choices=["tensor", "strip"],
                    help="M <= 4 decode through the strip kernel (default) or the tcgen05 decode")
    ap.add_argument("--only", default="all", choices=["all", "prefill", "decode"],
                    help="run one part only (small profiler captures); the JSON line then carries that part")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from tensorpack_b200 import build

    build.build()
    from tensorpack_b200 import _lib
    from tensorpack_b200.kernels.gemm import HostGemm
    from tensorpack_b200.sharding import ShardedMTCMatrix

    wl = make_workload(args.config)
    if world > 1 and not wl.single:
        raise SystemExit(f"--config {wl.name}: multi-GPU runs take a single-matrix configuration")
    allocate(wl, dev)
    accounted_bytes = sum(L.mat.accounted_bits for L in wl.layers) / 8.0
    Mp = wl.prefill_M
    Ks = sorted({L.K for L in wl.layers})
    X_host = {K: activations(wl, Mp, K, seed=1) for K in Ks}
    X = {K: torch.from_numpy(X_host[K]).to(dev) for K in Ks}

    if world > 1:
        sharded = ShardedMTCMatrix(wl.layers[0].mat, device=dev)
        streams = [sharded.stream]
        local_bytes = sharded.local.accounted_bits / 8.0
    else:
        sharded = None
        streams = [L.mat.device_stream(dev) for L in wl.layers]
        local_bytes = accounted_bytes
    for ds in streams:
        ds.decode_kernel = args.decode_kernel
    Y = [torch.empty(Mp, L.N, dtype=torch.float32, device=dev) for L in wl.layers]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def gemm_step():
        if sharded is not None:
            sharded.matmul(X[wl.layers[0].K], Y[0])
            return
        for L, ds, y in zip(wl.layers, streams, Y):
            ds.matmul(X[L.K], y)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    hbm_peak, tc_peak, peak_src = measured_peaks()
    flops = sum(2.0 * Mp * L.K * L.N for L in wl.layers)
    local_flops = sum(2.0 * Mp * L.K * ds.N for L, ds in zip(wl.layers, streams))
    per_step_launches = sum(3 if ds.col_perm is not None else 2 for ds in streams)

    # --- prefill (headline) ---
    do_prefill = args.only in ("all", "prefill")
    step_ms = kern_ms = value = achieved = None
    clocks = None
    if do_prefill:
        for _ in range(args.warmup):
            gemm_step()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        # clocks sampled every millisecond over both timed prefill loops
        # (the step and the kernel alone)
        clocks = ClockSampler(local_rank, period_s=0.001).__enter__()
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            gemm_step()
            ev[i][1].record(stream)
        barrier()
        step_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / args.steps)
        value = flops / (step_ms * 1e-3) / 1e12
        for ds in streams:
            ds.check_status()
        # the prefill kernel alone (gathers outside the events), for the roofline
        kev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in streams]
               for _ in range(args.steps)]
        for i in range(args.steps):
            flush.zero_()
            for j, (L, ds) in enumerate(zip(wl.layers, streams)):
                ds.prefill_gather(X[L.K])
                kev[i][j][0].record(stream)
                ds.prefill_gemm(Mp, Y[j])
                kev[i][j][1].record(stream)
        barrier()
        clocks.__exit__(None, None, None)
        kern_ms = max_over_ranks(sum(a.elapsed_time(b) for row in kev for a, b in row) / args.steps)
        achieved = local_flops / (kern_ms * 1e-3) / 1e12
        if args.only == "prefill":
            if rank == 0:
                print(json.dumps({"only": "prefill", "ms_per_step": step_ms, "kernel_ms": kern_ms,
                                  "kernel_tflops": achieved, "config": workload_config(wl, world)}), flush=True)
            if world > 1:
                barrier()
                dist.destroy_process_group()
            return

    # --- decode: rotating copies (> 4x L2), launches captured in a CUDA graph ---
    lib = _lib.load()
    decode_by_M = {}
    decode_outputs = {}
    cur = {"s": stream}
    for Md in wl.decode_Ms:
        copies = max(2, int(4 * L2_BYTES // max(1, sum(
            (ds.strip().stream_bytes if (Md <= 4 and args.decode_kernel == "strip") else ds.stage_images.numel())
            for ds in streams))) + 1)
        copies = min(copies, 64)
        xs = {K: X[K][:Md].contiguous() for K in Ks}
        ys = [torch.empty(Md, ds.N, dtype=torch.float32, device=dev) for ds in streams]
        per_layer, keeps, kernel_names, dev_bytes = [], [], set(), 0
        for ds in streams:
            fns, keep, kname, nb = rotated_decoders(ds, Md, copies, lib, lambda: cur["s"].cuda_stream)
            per_layer.append(fns)
            keeps.append(keep)
            kernel_names.add(kname)
            dev_bytes += nb

        def one_pass(ci):
            for L, fns, y in zip(wl.layers, per_layer, ys):
                fns[ci](xs[L.K], y)

        for ci in range(copies):  # warm-up (and the first-use set-up of every copy)
            one_pass(ci)
        barrier()
        side = torch.cuda.Stream(dev)
        graph = torch.cuda.CUDAGraph()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            cur["s"] = side
            with torch.cuda.graph(graph, stream=side):
                for ci in range(copies):
                    one_pass(ci)
        cur["s"] = stream
        stream.wait_stream(side)
        graph.replay()
        barrier()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for _ in range(args.decode_reps):
            graph.replay()
        d1.record(stream)
        barrier()
        dec_us = max_over_ranks(d0.elapsed_time(d1) * 1e3 / (args.decode_reps * copies))
        for ds in streams:
            ds.check_status()
        del graph
        gbs = accounted_bytes / (dec_us * 1e-6) / 1e9
        local_gbs = local_bytes / (dec_us * 1e-6) / 1e9
        kname = "+".join(sorted(kernel_names))
        decode_by_M[str(Md)] = {
            "value": gbs, "unit": "GB/s", "us_per_call": dec_us, "M": Md,
            "kernel": {"strip_kernel": "strip_kernel (mma.sync over the strip stream)",
                       "decode_kernel": "decode_kernel (tcgen05 over the sub-stage images)"}.get(kname, kname),
            "accounted_bytes": accounted_bytes, "device_bytes": dev_bytes, "launches_per_call": len(streams),
            "roofline": {"bound": "hbm", "achieved": local_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": local_gbs / hbm_peak, "traffic": committed_traffic(wl.name, kname),
                         "peak_source": peak_src},
            "copies_rotated": copies, "timing": "CUDA graph of the rotated calls, device events"}
        for j, y in enumerate(ys[:wl.parity_layers]):
            decode_outputs[(Md, j)] = (xs[wl.layers[j].K], y.clone())
        del keeps, per_layer
    if args.only == "decode":
        if rank == 0:
            print(json.dumps({"only": "decode", "decode_by_M": decode_by_M, "config": workload_config(wl, world)}),
                  flush=True)
        if world > 1:
            barrier()
            dist.destroy_process_group()
        return

    # --- end to end through the public API with pinned host buffers ---
    # One GPU: HostGemm per matrix (host X in, host Y out; copies in, GEMM
    # and copies out of row chunks overlapped).  Several: every rank copies X
    # in (each GPU needs all of it), runs the sharded GEMM, and rank 0 copies
    # the result out (it is the same on every rank; the host needs it once).
    Xh = {K: torch.from_numpy(X_host[K]).pin_memory() for K in Ks}
    Yh = [torch.empty(Mp, L.N, dtype=torch.float32).pin_memory() for L in wl.layers]
    if sharded is None:
        host_gemms = [HostGemm(L.mat, dev) for L in wl.layers]
    Xd = X[Ks[0]].clone() if sharded is not None else None

    def e2e_step():
        if sharded is None:
            for L, hg, yh in zip(wl.layers, host_gemms, Yh):
                hg(Xh[L.K], yh)
            return
        Xd.copy_(Xh[Ks[0]], non_blocking=True)
        sharded.matmul(Xd, Y[0])
        if rank == 0:
            Yh[0].copy_(Y[0], non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 4)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    h2d = sum(Mp * L.K * 4 for L in wl.layers)
    d2h = sum(Mp * L.N * 4 for L in wl.layers)

    # --- CPU leg (rank 0): parity check and CPU baseline, both with the oracle as checker ---
    parity = cpu = None
    if rank == 0:
        if not args.no_parity and sharded is None:
            prefill_outputs = {}
            for j, (L, ds) in enumerate(zip(wl.layers[:wl.parity_layers], streams)):
                ds.matmul(X[L.K], Y[j])
                prefill_outputs[(Mp, j)] = (X[L.K], Y[j])
            torch.cuda.synchronize(dev)
            parity = parity_check(wl, dev, decode_outputs, prefill_outputs)
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(wl, seconds=10.0 if world == 1 else 5.0)

    if rank == 0:
        dec1 = decode_by_M.get("1")
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 operands, fp32 accumulate", "data": "synthetic",
            "config": workload_config(wl, world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": achieved / tc_peak, "traffic": committed_traffic(wl.name, "prefill_kernel"),
                         "kernel": "prefill_kernel (fused dequant + tcgen05)", "peak_source": peak_src,
                         "kernel_ms": kern_ms},
            "decode": dec1,
            "decode_by_M": decode_by_M,
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h if sharded is None else Mp * wl.layers[0].N * 4,
                    "ms_per_step": e2e_ms,
                    "host_link_GBps": (h2d * (world if sharded is not None else 1)
                                       + (d2h if sharded is None else Mp * wl.layers[0].N * 4)) / (e2e_ms * 1e-3) / 1e9},
            "gpu_launches": per_step_launches * args.steps,
            "parity": parity,
            "cpu_baseline": cpu,
            "clocks": clocks.summary() if clocks is not None else None,
            "accounted_bits_per_weight": 8.0 * accounted_bytes / sum(L.K * L.N for L in wl.layers),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

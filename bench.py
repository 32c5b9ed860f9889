#!/usr/bin/env python
"""Benchmark of the packed-quadtree MTC GEMM on B200 (one JSON line on rank 0).

Workload (BASELINE.json metric "dequant-GEMM TFLOP/s at M=4096; decode GEMV
packed-weight GB/s vs B200 peak"): the Llama-3-8B gate_proj shape, W 4096 x
14336 with Student-t(4) * 0.02 entries, MTC-QT-P at 4.25 bits/weight with
sizes 32..4 and an importance vector from 512 synthetic calibration rows
whose 1 % outlier channels are scaled x50 (synthetic, seeded: no checkpoint
or dataset is available).  The allocation is produced on the GPU by
tensorpack_b200.quant.

  value     prefill: Y = X @ W at M = 4096 through the fused dequant +
            tcgen05 path (gather, GEMM, column scatter), TFLOP/s = 2 M K N / t,
            L2 flushed before every step (256 MB write)
  decode    M = 1 through the strip-stream decode kernel (mma.sync over
            precision-sorted steps; --decode-kernel tensor for the tcgen05
            decode), GB/s of accounted packed bytes (payload + scales + modes
            + split flags + permutation indices), rotating over copies of the
            stream totalling > 4x L2
  e2e       the prefill metric through the public API with pinned host X and
            Y: host->device copy, GEMM, device->host copy per step (one GPU:
            tensorpack_b200.kernels.gemm.HostGemm, which overlaps the copies
            and the GEMM of row chunks; several: the sharded GEMM between
            whole-matrix copies)
  roofline  the prefill kernel alone (CUDA events on its stream) against the
            measured dense bf16 peak; the decode kernel against measured HBM
  cpu_baseline  the reference's packed Numba GEMM algorithm (oracle port,
            fixed 16x16 blocks at the same bits/weight, X packed as P16) on a
            bounded sample, on this host's cores

Multi-GPU (torchrun, one process per GPU): the layer is column-sharded across
ranks (strong scaling), one NCCL all-gather per GEMM; times are the max over
ranks.  `--impl reference` times the reference CPU implementation instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

METRIC = "dequant-GEMM TFLOP/s at M=4096; decode GEMV packed-weight GB/s vs B200 peak"
K_IN, N_OUT, BITS = 4096, 14336, 4.25
M_PREFILL = 4096
L2_BYTES = 126 * 1024 * 1024


def workload_config(args):
    return {"workload": "llama3-8b gate_proj 4096x14336 MTC-QT-P @4.25 b/w (sizes 32..4), prefill M=4096 + decode M=1",
            "model": "Llama-3-8B-shaped linear (random init, Student-t(4)*0.02)", "global_batch": M_PREFILL,
            "seq_len": 1, "parallelism": f"column-shard x{args.gpus}" if args.gpus > 1 else "none",
            "K": K_IN, "N": N_OUT, "bits_per_weight": BITS,
            "l2_policy": "prefill: 256 MB L2 flush before each step; decode: weight copies > 4x L2 rotated"}


def make_weights():
    import inputs

    return inputs.llm_like(K_IN, N_OUT, seed=0)


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


def committed_traffic(kernel: str):
    """dram bytes per launch from the committed ncu summary (profiles/), if any."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel:
            return float(parts[1])
    return None


# ----------------------------------------------------------------------------- CPU reference

def cpu_reference_sample(W, h, seed=0):
    """The reference's packed-GEMM algorithm (oracle port of mtc_gemm, gemm.py:124-210)
    on a bounded sample: 256 tokens x K 4096 x 1024 output features, fixed
    16x16 blocks at the same bits/weight with bf16 scales (the reference
    cannot run quadtree leaves), X packed as P16."""
    import numba

    import inputs
    from oracle import mtc_oracle as O

    numba.set_num_threads(os.cpu_count() or 1)
    Ws = np.ascontiguousarray(W[:, :1024])
    alloc = O.allocate_fixed(Ws, BITS, h, 16, scale_format="bf16")
    B = O.PackedFixed.from_allocation(Ws, alloc.modes, alloc.scales, 16)
    X = inputs.llm_activations(256, K_IN, seed=seed + 7, outlier_seed=0)
    A = O.p16_operand(X, 16)
    O.packed_gemm(A, B)  # JIT warm-up
    flops = 2.0 * 256 * K_IN * 1024
    sample = "256 tokens x 4096 x 1024 features (fixed 16x16 RD blocks @4.25 b/w bf16 scales, X as P16)"
    return (lambda: O.packed_gemm(A, B)), flops, numba.get_num_threads(), sample


def run_reference(args, rank):
    if rank != 0:
        return
    W, h = make_weights()
    fn, flops, cores, sample = cpu_reference_sample(W, h)
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
        "config": workload_config(args),
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- GPU arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--decode-steps", type=int, default=300)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-kernel", default="strip", choices=["tensor", "strip", "strip-wide"],
                    help="decode M = 1 through the mma.sync kernel over the strip stream (strip, default), over "
                         "its wide form (strip-wide: 16-group steps, four MMAs per B fragment) or the tcgen05 "
                         "kernel over the sub-stage images (tensor)")
    ap.add_argument("--strip-batch-bytes", type=int, default=None,
                    help="batch record limit of the strip stream (default 4096; 2048..65536)")
    ap.add_argument("--strip-batch-steps", type=int, default=None, help="steps per strip batch record (default 64)")
    ap.add_argument("--strip-merge-modes", action="store_true",
                    help="strip stream with P2 items packed as P3 and P6 items as P8 (fewer step kinds)")
    ap.add_argument("--only", default="all", choices=["all", "prefill", "decode"],
                    help="run one part only (small profiler captures); the JSON line then carries that part")
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
    from tensorpack_b200.kernels.gemm import HostGemm, MTCMatrix
    from tensorpack_b200.quant import PermutedQuadtreeRD
    from tensorpack_b200.sharding import ShardedMTCMatrix

    import inputs

    W, h = make_weights()
    alloc = PermutedQuadtreeRD(W, h, (32, 16, 8, 4), device=dev).select(BITS)
    mat = MTCMatrix.from_qt_allocation(W, alloc)
    accounted_bytes = mat.accounted_bits / 8.0
    X_host = inputs.llm_activations(M_PREFILL, K_IN, seed=1, outlier_seed=0)
    X = torch.from_numpy(X_host).to(dev)

    if world > 1:
        sharded = ShardedMTCMatrix(mat, device=dev)
        ds = sharded.stream
        local_bytes = sharded.local.accounted_bits / 8.0

        def gemm(Xd, Yd):
            return sharded.matmul(Xd, Yd)
    else:
        sharded = None
        ds = mat.device_stream(dev)
        local_bytes = accounted_bytes

        def gemm(Xd, Yd):
            return ds.matmul(Xd, Yd)

    Y = torch.empty(M_PREFILL, N_OUT, dtype=torch.float32, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

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

    # --- prefill (headline) ---
    do_prefill = args.only in ("all", "prefill")
    for _ in range(args.warmup if do_prefill else 0):
        gemm(X, Y)
    hbm_peak, tc_peak, peak_src = measured_peaks()
    flops = 2.0 * M_PREFILL * K_IN * N_OUT
    step_ms = kern_ms = value = achieved = None
    clocks = None
    if do_prefill:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        with ClockSampler(local_rank) as clocks:
            for i in range(args.steps):
                flush.zero_()
                ev[i][0].record(stream)
                gemm(X, Y)
                ev[i][1].record(stream)
            barrier()
        step_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / args.steps)
        flops = 2.0 * M_PREFILL * K_IN * N_OUT
        value = flops / (step_ms * 1e-3) / 1e12
        ds.check_status()
        # prefill kernel alone (its own stream), for the roofline
        for i in range(args.steps):
            flush.zero_()
            ds.prefill_gather(X)
            kev[i][0].record(stream)
            ds.prefill_gemm(M_PREFILL, Y)
            kev[i][1].record(stream)
        barrier()
        kern_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / args.steps)
        local_flops = 2.0 * M_PREFILL * K_IN * ds.N
        achieved = local_flops / (kern_ms * 1e-3) / 1e12
        if args.only == "prefill":
            if rank == 0:
                print(json.dumps({"only": "prefill", "ms_per_step": step_ms, "kernel_ms": kern_ms,
                                  "kernel_tflops": achieved, "config": workload_config(args)}), flush=True)
            if world > 1:
                barrier()
                dist.destroy_process_group()
            return
    launches_per_step = 3

    # --- decode M = 1 over rotating copies of the stream (> 4x L2) ---
    # Every buffer the decode kernel streams is copied: the sub-stage images
    # and their metadata (tensor), or the batch records and their offsets (strip).
    lib = _lib.load()
    import ctypes

    x1 = X[:1].contiguous()
    y1 = torch.empty(1, ds.N, dtype=torch.float32, device=dev)
    descs, keep = [], []
    pr_ptr = None if ds.row_perm is None else ds.row_perm.data_ptr()
    pc_ptr = None if ds.col_perm is None else ds.col_perm.data_ptr()
    if args.decode_kernel.startswith("strip"):
        sp = ds.strip(wide=args.decode_kernel == "strip-wide", batch_bytes=args.strip_batch_bytes,
                      batch_steps=args.strip_batch_steps, merge_modes=args.strip_merge_modes)
        stream_bytes = sp.stream.numel()
        copies = max(2, int(4 * L2_BYTES // max(stream_bytes, 1)) + 1)
        for _ in range(copies):
            bufs = [sp.stream.clone(), sp.batch_off.clone(), sp.strip_batch.clone()]
            keep += bufs
            d = _lib.StripDesc.from_buffer_copy(sp.desc)
            d.stream, d.batch_off, d.strip_batch = [b.data_ptr() for b in bufs]
            descs.append(d)

        def decode(i):
            _lib.check(lib.mtc_strip_decode(ctypes.byref(descs[i % copies]), x1.data_ptr(), 1, x1.stride(0), pr_ptr,
                                            pc_ptr, y1.data_ptr(), y1.stride(0), ds.status.data_ptr(), None,
                                            stream.cuda_stream), "strip decode")
    else:
        stream_bytes = ds.stage_images.numel()
        copies = max(2, int(4 * L2_BYTES // max(stream_bytes, 1)) + 1)
        for _ in range(copies):
            bufs = [ds.stage_images.clone(), ds.stage_counts.clone(), ds.stage_offsets.clone(),
                    ds.stage_ranges.clone()]
            keep += bufs
            d = _lib.StreamDesc.from_buffer_copy(ds.desc)
            d.stage_images, d.stage_counts, d.stage_offsets, d.stage_ranges = [b.data_ptr() for b in bufs]
            descs.append(d)
        ws = torch.empty(max(int(lib.mtc_decode_workspace_bytes(ctypes.byref(ds.desc), 1)), 256), dtype=torch.uint8,
                         device=dev)

        def decode(i):
            _lib.check(lib.mtc_decode(ctypes.byref(descs[i % copies]), x1.data_ptr(), 1, x1.stride(0), pr_ptr, pc_ptr,
                                      y1.data_ptr(), y1.stride(0), ws.data_ptr(), ws.numel(),
                                      ds.decode_counters.data_ptr(), ds.status.data_ptr(), None, stream.cuda_stream),
                       "decode")

    for i in range(max(args.warmup, copies)):
        decode(i)
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for i in range(args.decode_steps):
        decode(i)
    d1.record(stream)
    barrier()
    dec_us = max_over_ranks(d0.elapsed_time(d1) * 1e3 / args.decode_steps)
    ds.check_status()
    dec_gbs = accounted_bytes / (dec_us * 1e-6) / 1e9          # whole layer bytes / slowest rank time
    dec_local_gbs = local_bytes / (dec_us * 1e-6) / 1e9
    if args.only == "decode":
        if rank == 0:
            print(json.dumps({"only": "decode", "kernel": args.decode_kernel, "us_per_call": dec_us,
                              "GB/s": dec_gbs, "stream_bytes": stream_bytes, "config": workload_config(args)}),
                  flush=True)
        if world > 1:
            barrier()
            dist.destroy_process_group()
        return

    # --- end to end through the public API with pinned host buffers ---
    # One GPU: HostGemm (host X in, host Y out; copies in, GEMM and copies out
    # of row chunks overlapped).  Several: every rank copies X in (each GPU
    # needs all of it), runs the sharded GEMM, and rank 0 copies the result
    # out (it is the same on every rank; the host needs it once).
    Xh = torch.from_numpy(X_host).pin_memory()
    Yh = torch.empty(M_PREFILL, N_OUT, dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(X)
    host_gemm = HostGemm(mat, dev) if sharded is None else None

    def e2e_step():
        if host_gemm is not None:
            host_gemm(Xh, Yh)
            return
        Xd.copy_(Xh, non_blocking=True)
        gemm(Xd, Y)
        if rank == 0:
            Yh.copy_(Y, non_blocking=True)

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

    # --- CPU baseline (rank 0, single GPU only) ---
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fn, cflops, cores, sample = cpu_reference_sample(W, h)
        ts = []
        t_end = time.perf_counter() + 10.0
        while time.perf_counter() < t_end or len(ts) < 3:
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        cpu = {"value": cflops / statistics.median(ts) / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": sample + f", median of {len(ts)} calls"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 operands, fp32 accumulate", "data": "synthetic",
            "config": workload_config(args),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": achieved / tc_peak, "traffic": committed_traffic("prefill_kernel"),
                         "kernel": "prefill_kernel (fused dequant + tcgen05)", "peak_source": peak_src,
                         "kernel_ms": kern_ms},
            "decode": {"value": dec_gbs, "unit": "GB/s", "us_per_call": dec_us, "M": 1,
                       "kernel": {"strip": "strip_kernel (mma.sync over the strip stream)",
                                  "strip-wide": "strip_kernel (mma.sync over the wide strip stream)",
                                  "tensor": "decode_kernel (tcgen05 over the sub-stage images)"}[args.decode_kernel],
                       "accounted_bytes": accounted_bytes, "device_bytes": stream_bytes,
                       "roofline": {"bound": "hbm", "achieved": dec_local_gbs, "peak": hbm_peak, "unit": "GB/s",
                                    "frac": dec_local_gbs / hbm_peak,
                                    "traffic": committed_traffic("strip_kernel" if args.decode_kernel == "strip"
                                                                 else "decode_kernel" if args.decode_kernel == "tensor"
                                                                 else None),
                                    "peak_source": peak_src},
                       "copies_rotated": copies},
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": M_PREFILL * K_IN * 4, "d2h_bytes_per_step": M_PREFILL * N_OUT * 4,
                    "ms_per_step": e2e_ms},
            "gpu_launches": launches_per_step * args.steps,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "accounted_bits_per_weight": mat.accounted_bits / (K_IN * N_OUT),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

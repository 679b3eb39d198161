#!/usr/bin/env python
"""Benchmark of the block-scaled quantised-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

N = 1 (default): the NVFP4 GEMM M = N = K = 8192 with a fused fp32 bias and bf16 output
(the configuration the headline metric is quoted on).  One step = one GEMM launch on operands
already quantised and resident in HBM; `e2e` times the public API from pinned host memory
(copy the bf16 activation in, amax + quantise it, GEMM against the resident quantised weight,
copy the bf16 result out).

N > 1 (launched by torch.distributed.run, one rank per GPU): the all-gather MXFP8 GEMM, total
A (32768, 8192) sharded by rows, weight (28672, 8192) sharded by output features; each rank
computes the full-M x N/world block while the NCCL all-gather of the activation shards
overlaps the tiles.  Strong scaling: the total work is fixed.

`--impl reference` times the CPU restatement of the reference's dequantise -> fp32 matmul path
(oracle/) on the host cores, on a bounded row slab of the same workload.

Prints ONE JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "blockscaled_gemm_tflops"
UNIT = "TFLOPS"


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm_gbs=p["hbm_gbs"], bf16=p["bf16_tflops"], bf16_sustained=p["bf16_tflops_sustained"], source="measured")
    return dict(hbm_gbs=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


class ClockSampler:
    """SM clock / power / throttle-reason samples (read-only NVML queries from a thread, every
    10 ms) while the timed region runs.  Falls back to an `nvidia-smi -lms` child without NVML."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        # rows: [sm MHz, max MHz, watts, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap] as strings
        self.index, self.rows, self.proc, self.thread, self.stop = index, [], None, None, threading.Event()
        self.nvml = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            p = torch.cuda.get_device_properties(self.index)
            bus_id = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus_id.encode())
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        return pynvml, handle

    def __enter__(self):
        try:
            self.nvml, self.handle = self._nvml_handle()
            self.max_mhz = self.nvml.nvmlDeviceGetMaxClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _poll(self):
        n = self.nvml
        bits = ((n.nvmlClocksEventReasonHwSlowdown if hasattr(n, "nvmlClocksEventReasonHwSlowdown") else 0x8),
                (n.nvmlClocksEventReasonHwThermalSlowdown if hasattr(n, "nvmlClocksEventReasonHwThermalSlowdown") else 0x40),
                (n.nvmlClocksEventReasonSwThermalSlowdown if hasattr(n, "nvmlClocksEventReasonSwThermalSlowdown") else 0x20),
                (n.nvmlClocksEventReasonSwPowerCap if hasattr(n, "nvmlClocksEventReasonSwPowerCap") else 0x4))
        get_reasons = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                watts = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                mask = get_reasons(self.handle)
                self.rows.append([str(mhz), str(self.max_mhz), f"{watts:.2f}"] +
                                 ["Active" if mask & b else "Not Active" for b in bits])
            except Exception:
                pass
            self.stop.wait(0.01)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                self.rows.append(parts)

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None and self.thread is not None:
            self.thread.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        clk = [num(r[0]) for r in self.rows if num(r[0]) is not None]
        # "under load": samples within 25 % of the maximum power seen
        pw = [num(r[2]) or 0.0 for r in self.rows]
        top = max(pw) if pw else 0.0
        loaded = [num(r[0]) for r, p in zip(self.rows, pw) if p >= 0.75 * top and num(r[0]) is not None] or clk
        reasons = []
        for name, col in (("hw_slowdown", 3), ("hw_thermal_slowdown", 4), ("sw_thermal_slowdown", 5), ("sw_power_cap", 6)):
            if any(r[col].lower().startswith("active") for r in self.rows):
                reasons.append(name)
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": num(self.rows[0][1]),
                "power_w_max": top, "reasons": reasons, "samples": len(self.rows),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ------------------------------------------------------------------------------------------
# CPU baseline: the oracle's dequantise -> fp32 matmul (+ bias) on a row slab
# ------------------------------------------------------------------------------------------

def cpu_gemm_sample(fmt: str, slab_m: int, n: int, k: int, repeats: int = 1, warmup: int = 0):
    """Seconds per pass of the reference path (dequantise both operands, fp32 matmul, tensor
    scales, bias, cast) on `slab_m` rows, operands quantised by the oracle beforehand (untimed);
    `warmup` untimed passes first."""
    from oracle import blockscaled_oracle as orc

    a = orc.make_activation(slab_m, k, 0)
    w = orc.make_weight(n, k, 1)
    bias = orc.make_bias(n)
    if fmt == "nvfp4":
        pa = orc.nvfp4_per_tensor_scale(a.float().abs().max().item())
        pb = orc.nvfp4_per_tensor_scale(w.float().abs().max().item())
        ac, asf = orc.to_nvfp4(a, pa)
        bc, bsf = orc.to_nvfp4(w, pb)
    else:
        pa = pb = None
        ac, asf = orc.to_mx_e4m3(a)
        bc, bsf = orc.to_mx_e4m3(w)
    times = []
    for it in range(warmup + repeats):
        t0 = time.perf_counter()
        if fmt == "nvfp4":
            adq, bdq = orc.dequant_nvfp4(ac, asf), orc.dequant_nvfp4(bc, bsf)
        else:
            adq, bdq = orc.dequant_mxfp8(ac, asf), orc.dequant_mxfp8(bc, bsf)
        out = orc.gemm_blockscaled_ref(adq, bdq, pts_a=pa, pts_b=pb, bias=bias)
        orc.to_bf16(out)
        if it >= warmup:
            times.append(time.perf_counter() - t0)
    return times


def run_reference(args):
    """--impl reference: the reference's CPU path, timed on the host cores (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    # the launcher of multi-process runs pins OMP_NUM_THREADS to 1; the other ranks have exited, so this rank
    # takes every host core it is allowed to use
    try:
        torch.set_num_threads(max(torch.get_num_threads(), len(os.sched_getaffinity(0))))
    except (AttributeError, RuntimeError):
        pass
    single = args.gpus == 1
    fmt, n, k = ("nvfp4", 8192, 8192) if single else ("mxfp8_e4m3", 28672 // args.gpus, 8192)
    # N = 1: the whole 8192^3 problem per step (about 6-10 s of host work); N > 1: a 1024-row slab of the rank's block
    slab = 8192 if single else 1024
    times = cpu_gemm_sample(fmt, slab, n, k, repeats=args.steps, warmup=max(args.warmup, 1))
    sec = max(times)
    tflops = 2.0 * slab * n * k / sec / 1e12
    cores = torch.get_num_threads()
    workload = ("nvfp4_gemm_8192x8192x8192_bias_bf16" if single else f"allgather_mxfp8_gemm_32768x28672x8192_tp{args.gpus}")
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak" if single else "strong",
        "vs_baseline": None, "dtype": "f32 (dequantised operands)", "data": "synthetic",
        "config": {"workload": workload, "sample": ("the whole problem per step" if single else f"{slab}-row slab of A against the rank's weight block")},
        "cpu_baseline": {"value": tflops, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": (f"oracle dequantise + fp32 matmul + bias on {slab} rows x {n} x {k} "
                                    f"({2.0 * slab * n * k / 1e9:.0f} GFLOP per step)")},
        "e2e": {"value": tflops, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
# N = 1: NVFP4 GEMM 8192^3 + bias
# ------------------------------------------------------------------------------------------

def run_single(args):
    from oracle import blockscaled_oracle as orc   # cpu_baseline leg and input generators only
    from quack_b200 import _lib, _ops
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    from quack_b200.gemm_interface import gemm

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    m = n = k = 8192
    fmt = "nvfp4"
    peaks = load_peaks()
    nsets = 3   # rotating operand sets: 3 x (A 32 MiB + W 32 MiB + scales 8 MiB) + D 128 MiB per step > 126 MB L2

    g = torch.Generator(device="cpu").manual_seed(0)
    a_host = orc.make_activation(m, k, 0).pin_memory()
    bias = orc.make_bias(n).to(dev)
    sets = []
    for s in range(nsets):
        a = orc.make_activation(m, k, 10 + s).to(dev) if s else a_host.to(dev)
        w = orc.make_weight(n, k, 20 + s).to(dev)
        A = BlockScaledOperand.quantize(a, fmt, per_tensor_scale=nvfp4_per_tensor_scale(a.abs().amax()))
        W = BlockScaledOperand.quantize(w, fmt, per_tensor_scale=nvfp4_per_tensor_scale(w.abs().amax()))
        sets.append((A, W))
        del a, w
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    d_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()

    def step(i):
        A, W = sets[i % nsets]
        gemm(A, W.mT, out=out, bias=bias)

    # warm-up: the W steps asked for (at least 3), then enough further launches (about 10 ms) for the SM clock
    # to come up from idle: the first launches after an idle period run ~20 % slower
    extra_warmup = 48
    for i in range(max(args.warmup, 3) + extra_warmup):
        step(i)
    torch.cuda.synchronize()
    _ops.check_status(dev)

    launches0 = _lib.launch_count()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(0) as clocks:
        torch.cuda.synchronize()
        ev[0].record()
        for i in range(args.steps):
            step(i)
            ev[i + 1].record()
        torch.cuda.synchronize()
        total_ms = ev[0].elapsed_time(ev[-1])
        launches = _lib.launch_count() - launches0
        # keep the GPU busy a little longer when the timed region is too short for a clock sample
        t_end = time.time() + max(0.0, 0.6 - total_ms / 1e3)
        i = 0
        while time.time() < t_end:
            step(i)
            i += 1
            if i % 64 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
    _ops.check_status(dev)
    ms_per_step = total_ms / args.steps
    flops = 2.0 * m * n * k
    value = flops / (ms_per_step * 1e-3) / 1e12
    per_launch_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    kernel_ms = statistics.mean(per_launch_ms)

    # ---- end to end through the public API from pinned host memory -----------------------
    # Every step copies its bf16 activations host -> device, quantises them, runs the GEMM and copies
    # the bf16 result device -> host.  The three phases of consecutive steps overlap the way a serving
    # loop would run them: copy-in, compute and copy-out streams with two buffers each (PCIe is full
    # duplex), so a step costs the slowest phase, not their sum.
    A0, W0 = sets[0]
    e2e_steps = max(4, min(args.steps, 32))
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    cur = torch.cuda.current_stream(dev)
    a_bufs = [torch.empty(m, k, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    o_bufs = [torch.empty(m, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    d_hosts = [d_host, torch.empty(m, n, dtype=torch.bfloat16).pin_memory()]
    ev_in = [torch.cuda.Event() for _ in range(2)]       # copy-in of the buffer finished
    ev_used = [torch.cuda.Event() for _ in range(2)]     # quantiser finished reading the input buffer
    ev_done = [torch.cuda.Event() for _ in range(2)]     # GEMM into the output buffer finished
    ev_out = [torch.cuda.Event() for _ in range(2)]      # copy-out of the buffer finished

    def e2e_run(steps):
        for i in range(steps):
            b = i & 1
            if i >= 2:
                s_in.wait_event(ev_used[b])
            with torch.cuda.stream(s_in):
                a_bufs[b].copy_(a_host, non_blocking=True)
                ev_in[b].record(s_in)
            cur.wait_event(ev_in[b])
            if i >= 2:
                cur.wait_event(ev_out[b])
            Aq = BlockScaledOperand.quantize(a_bufs[b], fmt, per_tensor_scale=nvfp4_per_tensor_scale(_ops.amax(a_bufs[b])))
            ev_used[b].record(cur)
            gemm(Aq, W0.mT, out=o_bufs[b], bias=bias)
            ev_done[b].record(cur)
            s_out.wait_event(ev_done[b])
            with torch.cuda.stream(s_out):
                d_hosts[b].copy_(o_bufs[b], non_blocking=True)
                ev_out[b].record(s_out)
        cur.wait_stream(s_out)

    e2e_run(2)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = _lib.launch_count()
    e0.record()
    e2e_run(e2e_steps)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    e2e_launches = (_lib.launch_count() - l0) // e2e_steps
    _ops.check_status(dev)
    assert torch.equal(d_hosts[0], d_hosts[1]), "the two end-to-end buffers must hold the same result"

    # ---- CPU baseline: the whole problem, once (about 10 s of host work) ------------------------
    slab = m if not args.skip_extras else 256
    cpu_t = cpu_gemm_sample(fmt, slab, n, k, repeats=1)
    cpu_tflops = 2.0 * slab * n * k / min(cpu_t) / 1e12

    extras = None if args.skip_extras else headline_extras(dev, peaks)

    # the GEMM is timed alone, launch by launch: the burst figure is its denominator (the fraction of the
    # seconds-long sustained figure is given beside it; under the 1000 W cap this kernel settles within milliseconds)
    peak = 4.0 * peaks["bf16"]
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp4_e2m1 x ue4m3 block scales, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "nvfp4_gemm_8192x8192x8192_bias_bf16", "m": m, "n": n, "k": k, "tile": "256x256x256, CTA pair",
                   "l2": f"rotating {nsets} operand sets (216 MiB of operands + 128 MiB output per step) > 126 MB L2",
                   "extra_warmup_launches": extra_warmup,
                   "pct_of_dense_fp4_peak_9000": 100.0 * value / 9000.0},
        "roofline": {"bound": "tensor", "achieved": flops / (kernel_ms * 1e-3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": flops / (kernel_ms * 1e-3) / 1e12 / peak,
                     "frac_of_sustained": flops / (kernel_ms * 1e-3) / 1e12 / (4.0 * peaks["bf16_sustained"]),
                     "peak_basis": f"4 x {peaks['bf16']} TFLOP/s burst bf16 ({peaks['source']}; sustained {peaks['bf16_sustained']}); "
                                   "NVFP4 dense rate is 4x bf16",
                     "traffic": measured_traffic("nvfp4_gemm_8192x8192x8192_bias_bf16")},
        "cpu_baseline": {"value": cpu_tflops, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"oracle dequantise + fp32 matmul + bias on {slab} rows x 8192 x 8192 of the same problem, one pass"},
        "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": a_host.numel() * 2,
                "d2h_bytes_per_step": d_host.numel() * 2, "ms_per_step": e2e_ms, "launches_per_step": e2e_launches,
                "path": "pinned bf16 A -> device, qk_amax, qk_quantize_blockscaled, qk_gemm_blockscaled(+bias), bf16 D -> pinned host; "
                        "copy-in / compute / copy-out of consecutive steps overlap on three streams (two buffers each)"},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "other_kernels": extras,
    }
    print(json.dumps(line), flush=True)


def headline_extras(dev, peaks):
    """Short measurements of the path's other kernels for the headline line (outside its timed region): the
    quantizer's bandwidth on the headline operand and on the all-gather activation (NVFP4 with its amax pass
    counted: 2 more bytes per element read), and the fused NVFP4 up-projection with SwiGLU and re-quantised
    output in both arithmetic modes of the activation."""
    from quack_b200 import _lib, _ops
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    from quack_b200.gemm_interface import gemm_act_quant

    out = {}
    for rows, k in ((8192, 8192), (32768, 8192)):
        nin = max(2, -(-(512 << 20) // (rows * k * 2)))     # rotating inputs of >= 512 MiB in total (> L2)
        xs = [torch.randn(rows, k, device=dev, dtype=torch.bfloat16) for _ in range(nin)]
        ms = _time_rotating([(lambda x=x: _ops.quantize_rows(x, _lib.FMT_MXFP8_E4M3)) for x in xs], 5 * nin)
        gbs = rows * k * (2 + 1 + 1 / 32) / ms / 1e6
        out[f"quantize_mxfp8_e4m3_{rows}x{k}"] = {"gbps": gbs, "ms": ms, "frac_of_measured_hbm": gbs / peaks["hbm_gbs"]}
        ms = _time_rotating([(lambda x=x: _ops.quantize_rows(x, _lib.FMT_NVFP4, _ops.amax(x) / 2688.0)) for x in xs], 5 * nin)
        gbs = rows * k * (2 + 2 + 0.5 + 1 / 16) / ms / 1e6
        out[f"amax_plus_quantize_nvfp4_{rows}x{k}"] = {"gbps": gbs, "ms": ms, "frac_of_measured_hbm": gbs / peaks["hbm_gbs"],
                                                       "bytes_per_element": 4.5625}
        del xs
    m, k, n = 16384, 4096, 28672
    g = torch.Generator(device=dev).manual_seed(3)
    a = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    A = BlockScaledOperand.quantize(a, "nvfp4", per_tensor_scale=nvfp4_per_tensor_scale(a.abs().amax()))
    W = BlockScaledOperand.quantize(w, "nvfp4", per_tensor_scale=nvfp4_per_tensor_scale(w.abs().amax()))
    del a, w
    bias = torch.randn(n, device=dev) * 0.1
    pts_out = torch.tensor([2e-3], device=dev)
    h = gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out)
    for exact in (True, False):
        torch.cuda.synchronize()
        time.sleep(0.3)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(3):
            gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out,
                           postact_out=h, exact_activation=exact)
        e0.record()
        for _ in range(10):
            gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out,
                           postact_out=h, exact_activation=exact)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 10
        tf = 2.0 * m * n * k / ms / 1e9
        out["nvfp4_up_proj_swiglu_nvfp4_out_16384x28672x4096_" + ("exact_silu" if exact else "fast_silu")] = {
            "tflops": tf, "ms": ms, "frac_of_4x_burst_bf16": tf / (4.0 * peaks["bf16"])}
    _ops.check_status(dev)
    return out


def measured_traffic(workload: str):
    """dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant kernel of `workload`, from
    the table of ncu captures kept with the profile summaries (None when there is no capture of it)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            entry = json.load(f).get(workload)
        return None if entry is None else float(entry["dram_bytes_read"]) + float(entry["dram_bytes_write"])
    except (OSError, ValueError, KeyError):
        return None


# ------------------------------------------------------------------------------------------
# extra workloads (not the headline line): --workload quantize | sweep
# ------------------------------------------------------------------------------------------

def _time_rotating(fns, iters):
    """CUDA-event time (ms) per call of the closures in `fns`, called round-robin, back to back, `iters` times.
    Each closure works on its own input tensor and together the inputs exceed L2, so no call finds its
    input cached; nothing is written between the calls (flushing L2 by rewriting a buffer leaves ~126 MB of
    dirty lines whose write-back then competes with the timed kernel for DRAM: +25 % on a 40 us quantizer)."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        fns[i % len(fns)]()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run_quantize(args):
    """Block-scale quantizer bandwidth on the operand of the headline GEMM (8192 x 8192 bf16)
    and on the all-gather GEMM's activation (32768 x 8192): algorithmic bytes / time."""
    from quack_b200 import _lib, _ops

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    peaks = load_peaks()
    for rows, k in ((8192, 8192), (32768, 8192)):
        nin = max(2, -(-(512 << 20) // (rows * k * 2)))     # inputs of >= 512 MiB in total: 4 x 128 MiB / 2 x 512 MiB
        xs = [torch.randn(rows, k, device=dev, dtype=torch.bfloat16) for _ in range(nin)]
        pts = (_ops.amax(xs[0]) / 2688.0)
        iters = max(args.steps, 3) * nin
        for name, fmt, bpe, p in (("mxfp8_e4m3", _lib.FMT_MXFP8_E4M3, 2 + 1 + 1 / 32, None),
                                  ("nvfp4", _lib.FMT_NVFP4, 2 + 0.5 + 1 / 16, pts)):
            l0 = _lib.launch_count()
            ms = _time_rotating([(lambda x=x: _ops.quantize_rows(x, fmt, p)) for x in xs], iters)
            gbs = rows * k * bpe / ms / 1e6
            print(json.dumps({
                "metric": "blockscale_quantize_gbps", "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": iters,
                "warmup": nin, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16 -> " + name, "data": "synthetic",
                "config": {"workload": f"quantize_{name}_{rows}x{k}", "bytes_per_element": bpe,
                           "l2": f"{nin} input tensors of {rows * k * 2 >> 20} MiB used in rotation (> 126 MB L2), launches back to back"},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": gbs / peaks["hbm_gbs"], "traffic": measured_traffic(f"quantize_{name}_{rows}x{k}")},
                "gpu_launches": (_lib.launch_count() - l0)}), flush=True)
        del xs


def _cublas_block_scaled_ms(A, W, iters):
    """CUDA-event time of cuBLAS's block-scaled GEMM (`torch._scaled_mm`) on the same operand bytes, the
    same-box comparator of the sweep: bf16 output, no tensor scales, launches back to back like the timing
    of this library's kernel.  None when this torch / cuBLAS build cannot run the case."""
    try:
        qa, qb = A.qdata, W.qdata
        sa, sb = A.scale.reshape(-1), W.scale.reshape(-1)
        fn = lambda: torch._scaled_mm(qa, qb.t(), sa, sb, out_dtype=torch.bfloat16)   # noqa: E731
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        if ms < 0.05:
            # host-paced: replay 20 launches from a CUDA graph, as for this library's kernel
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                fn()
                side.synchronize()
                with torch.cuda.graph(graph, stream=side):
                    for _ in range(20):
                        fn()
                graph.replay()
                side.synchronize()
                g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                g0.record(side)
                for _ in range(5):
                    graph.replay()
                g1.record(side)
                side.synchronize()
            ms = min(ms, g0.elapsed_time(g1) / 100)
        return ms
    except Exception:
        torch.cuda.synchronize()
        return None


def run_sweep(args):
    """GEMM throughput of the parity configurations (not bench lines): configuration 0, the
    Llama-3-8B linear shapes in MXFP8, the NVFP4 8192^3 GEMM and the fused NVFP4 up-projection
    (SwiGLU + re-quantised output).  One JSON line per case."""
    from quack_b200 import _ops
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    from quack_b200.gemm_interface import gemm, gemm_act_quant

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    peaks = load_peaks()

    def quant(rows, k, fmt, seed, scale=1.0):
        g = torch.Generator(device=dev).manual_seed(seed)
        x = (torch.randn(rows, k, generator=g, device=dev) * scale).to(torch.bfloat16)
        kw = dict(per_tensor_scale=nvfp4_per_tensor_scale(x.abs().amax())) if fmt == "nvfp4" else {}
        return BlockScaledOperand.quantize(x, fmt, **kw)

    cases = [("config0", "mxfp8_e4m3", 2048, 4096, 4096), ("config1", "nvfp4", 8192, 8192, 8192),
             ("mxfp8_8192", "mxfp8_e4m3", 8192, 8192, 8192)]
    for name, (n, k) in (("qkv", (6144, 4096)), ("o", (4096, 4096)), ("gate_up", (28672, 4096)), ("down", (4096, 14336))):
        for m in (1, 16, 128, 1024, 4096, 16384):
            cases.append((f"llama8b_{name}_m{m}", "mxfp8_e4m3", m, n, k))
    weights = {}
    if args.case:
        cases = [c for c in cases if args.case in c[0]]
    for name, fmt, m, n, k in cases:
        A = quant(m, k, fmt, 1)
        if (fmt, n, k) not in weights:
            weights = {(fmt, n, k): quant(n, k, fmt, 2, 0.02)}
        W = weights[(fmt, n, k)]
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        # every case starts from an idle GPU: after a power-capped case (1000 W) the SM clock stays low for a
        # while, which made the cases that followed it in the list 25-55 % slower than the same case run alone
        torch.cuda.synchronize()
        time.sleep(0.5)
        iters = max(5, min(args.steps, 30))
        # back-to-back launches (a GPU-side backlog): per-launch event pairs mis-time sub-10 us kernels
        for _ in range(3):
            gemm(A, W.mT, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            gemm(A, W.mT, out=out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        timing = "stream"
        if ms < 0.05:
            # a launch this short is paced by the host (~12-16 us of Python per call): replay the same 20
            # launches from a CUDA graph to time the device work
            try:
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.stream(side):
                    gemm(A, W.mT, out=out)      # first use of this stream: its split-K scratch is allocated outside the capture
                    side.synchronize()
                    with torch.cuda.graph(graph, stream=side):
                        for _ in range(20):
                            gemm(A, W.mT, out=out)
                    graph.replay()
                    side.synchronize()
                    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    g0.record(side)
                    for _ in range(5):
                        graph.replay()
                    g1.record(side)
                    side.synchronize()
                ms_graph = g0.elapsed_time(g1) / 100
                _ops.check_status(dev)
                if ms_graph < ms:
                    ms, timing = ms_graph, "cuda graph of 20 launches"
                del graph
            except Exception as e:   # capture not possible here: keep the stream timing
                timing = f"stream (graph capture failed: {type(e).__name__})"
                torch.cuda.synchronize()
        flops = 2.0 * m * n * k
        eb = 1.0 if fmt == "mxfp8_e4m3" else 0.5
        vec = 32 if fmt == "mxfp8_e4m3" else 16
        nbytes = (m + n) * k * eb + (m + n) * k / vec + 2.0 * m * n
        tf, gbs = flops / ms / 1e9, nbytes / ms / 1e6
        peak_tf = (2.0 if fmt == "mxfp8_e4m3" else 4.0) * peaks["bf16"]   # burst: every case starts from an idle GPU
        t_tensor, t_hbm = flops / (peak_tf * 1e12), nbytes / (peaks["hbm_gbs"] * 1e9)
        bound = "tensor" if t_tensor >= t_hbm else "hbm"
        # cuBLAS on the same bytes, from an idle GPU like the case above (without the tensor scales of NVFP4:
        # they are one multiplication in either epilogue)
        torch.cuda.synchronize()
        time.sleep(0.5)
        cublas_ms = _cublas_block_scaled_ms(A, W, iters) if not args.no_cublas else None
        print(json.dumps({"case": name, "format": fmt, "m": m, "n": n, "k": k, "ms": ms, "tflops": tf, "gbs": gbs,
                          "cublas_ms": cublas_ms, "speed_vs_cublas": None if cublas_ms is None else cublas_ms / ms,
                          "bound": bound, "frac_of_roof": max(t_tensor, t_hbm) / (ms * 1e-3), "timing": timing,
                          "frac_of_sustained_roof": max(t_tensor * peaks["bf16"] / peaks["bf16_sustained"], t_hbm) / (ms * 1e-3)}),
              flush=True)
    if args.case and args.case not in "config3_fused_up_proj_swiglu_nvfp4_out":
        return
    # fused up-projection: NVFP4 x NVFP4 -> SwiGLU -> NVFP4 (configuration 3)
    m, k, n = 16384, 4096, 28672
    A, W = quant(m, k, "nvfp4", 3), quant(n, k, "nvfp4", 4, 0.02)
    bias = torch.randn(n, device=dev) * 0.1
    pts_out = torch.tensor([1e-3], device=dev)
    h = gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out)
    iters = max(5, min(args.steps, 20))
    for exact in (True, False):
        torch.cuda.synchronize()
        time.sleep(0.5)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            gemm_act_quant(A, W.mT, bias=bias, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts_out,
                           postact_out=h, exact_activation=exact)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        print(json.dumps({"case": "config3_fused_up_proj_swiglu_nvfp4_out", "silu": "exact (expf, IEEE division)" if exact else "fast (ex2.approx)",
                          "format": "nvfp4", "m": m, "n": n, "k": k, "ms": ms,
                          "tflops": 2.0 * m * n * k / ms / 1e9, "bound": "tensor",
                          "frac_of_roof": 2.0 * m * n * k / (4.0 * peaks["bf16"] * 1e12) / (ms * 1e-3),
                          "frac_of_sustained_roof": 2.0 * m * n * k / (4.0 * peaks["bf16_sustained"] * 1e12) / (ms * 1e-3)}), flush=True)
    torch.cuda.synchronize()
    time.sleep(0.5)
    cublas_ms = _cublas_block_scaled_ms(A, W, iters) if not args.no_cublas else None
    print(json.dumps({"case": "config3_shape_plain_bf16_cublas", "m": m, "n": n, "k": k, "cublas_ms": cublas_ms,
                      "cublas_tflops": None if cublas_ms is None else 2.0 * m * n * k / cublas_ms / 1e9,
                      "note": "cuBLAS block-scaled GEMM of the same operands with a plain bf16 (16384 x 28672) output: no bias, "
                              "no SwiGLU, no re-quantisation"}), flush=True)
    _ops.check_status(dev)


def run_multi(args):
    from quack_b200.bench_allgather import run_allgather_bench   # N > 1 workload lives with the runner
    run_allgather_bench(args, METRIC, UNIT, load_peaks(), ClockSampler)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--case", default=None, help="with --workload sweep: run only the cases whose name contains this text")
    ap.add_argument("--no-cublas", action="store_true", help="with --workload sweep: skip the cuBLAS comparator")
    ap.add_argument("--skip-extras", action="store_true",
                    help="headline workload: skip the other-kernel measurements and shrink the CPU baseline to a 256-row slab "
                         "(for runs under a profiler)")
    ap.add_argument("--workload", default="headline", choices=["headline", "quantize", "sweep", "allgather"],
                    help="headline (default): the contract's single JSON line; quantize / sweep: extra measurements")
    args = ap.parse_args()
    if args.workload == "quantize":
        return run_quantize(args)
    if args.workload == "sweep":
        return run_sweep(args)
    if args.workload == "allgather":
        # the multi-GPU workload on whatever world this process is part of (a single process: world size 1,
        # the whole 32768 x 28672 x 8192 problem on one GPU with the local staging copy and no exchange)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29655")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        os.environ.setdefault("LOCAL_RANK", "0")
        return run_multi(args)
    if args.impl == "reference":
        args.steps = min(args.steps, 8)      # every step is ~6-10 s of host work at N = 1
        args.warmup = min(args.warmup, 1)
        run_reference(args)
        return
    if args.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        run_single(args)
    else:
        run_multi(args)


if __name__ == "__main__":
    main()

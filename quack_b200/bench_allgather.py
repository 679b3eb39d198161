"""The multi-GPU leg of bench.py: the all-gather MXFP8 GEMM (total A (32768, 8192) sharded by
rows, weight (28672, 8192) sharded by output features, each rank computing the full-M x
N/world bf16 block with the NCCL ring exchange overlapped with the tiles).

One process per GPU (torch.distributed.run).  One step = gather + GEMM on operands already
quantised and resident; times are CUDA-event times, maximum over ranks.  Strong scaling: the
total work (15.39 TFLOP) is fixed, `value` is total FLOP / time.  Besides the contract's keys the
line carries `overlap`: the same kernel timed on a pre-gathered A on all SMs (the pure-GEMM roof
of this rank's block) and the ratio roof / overlapped.
"""

from __future__ import annotations

import json
import os
import statistics

import torch
import torch.distributed as dist


def run_allgather_bench(args, metric, unit, peaks, ClockSampler):
    from . import _lib, _ops
    from .blockscaled import BlockScaledOperand
    from .distributed import BlockScaledAllGatherRunner
    from .gemm import gemm as kernel_gemm

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    M, N, K = 32768, 28672, 8192
    assert M % world == 0 and N % world == 0
    shard_m, n_loc = M // world, N // world
    fmt = "mxfp8_e4m3"

    def randn_bf16(rows, cols, seed, scale=1.0):
        g = torch.Generator(device=dev).manual_seed(seed)
        x = torch.randn(rows, cols, generator=g, device=dev, dtype=torch.float32) * scale
        return x.to(torch.bfloat16)

    a_shard_hp = randn_bf16(shard_m, K, 1000 + rank)
    idx = torch.randperm(K, generator=torch.Generator().manual_seed(0))[: max(1, round(0.001 * K))].to(dev)
    a_shard_hp[:, idx] *= 20
    w_hp = randn_bf16(n_loc, K, 1234 + rank, 0.02)
    A_shard = BlockScaledOperand.quantize(a_shard_hp, fmt)
    W = BlockScaledOperand.quantize(w_hp, fmt)
    del w_hp
    out = torch.empty(M, n_loc, dtype=torch.bfloat16, device=dev)
    transport = os.environ.get("QK_AG_TRANSPORT", "auto")   # copy engines when the peers' buffers can be mapped, else NCCL
    chunks = int(os.environ.get("QK_AG_CHUNKS", "1"))   # row chunks per shard, one arrival flag each
    runner = BlockScaledAllGatherRunner(shard_m, K, fmt, device=dev, comm_sms=int(os.environ.get("QK_COMM_SMS", "16")),
                                        transport=transport, arrival_chunks=chunks,
                                        push_streams=int(os.environ["QK_AG_PUSH_STREAMS"]) if "QK_AG_PUSH_STREAMS" in os.environ else None,
                                        chunk_streams=os.environ.get("QK_AG_CHUNK_STREAMS", "0") not in ("", "0"),
                                        exclusive_ingress=(os.environ["QK_AG_EXCLUSIVE"] not in ("", "0")) if "QK_AG_EXCLUSIVE" in os.environ else None)
    max_ctas = runner.gemm_max_ctas
    arrival = os.environ.get("QK_AG_ORDER", "arrival") == "arrival"   # shards consumed as they land ("ring": strict ring order)

    def step():
        with runner.gather(A_shard) as (a_full, ag_args):
            kernel_gemm(a_full.qdata, W.qdata, out, None, None, 256, 256, 2, 1, SFA=a_full.scale, SFB=W.scale,
                        bs_format_a=fmt, bs_format_b=fmt, ag_args=ag_args, max_ctas=max_ctas, ag_arrival_order=arrival)

    warm = max(args.warmup, 3)
    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    _ops.check_status(dev)

    # correctness of the overlapped path: bitwise equal to the plain GEMM on the gathered operand
    a_full = BlockScaledOperand.from_parts(runner.gathered_a().clone().view(torch.float8_e4m3fn),
                                           runner.sf_bufs[runner.last_parity].clone().view(-1, runner.rk, 32, 4, 4), fmt)
    ref = torch.empty_like(out)
    kernel_gemm(a_full.qdata, W.qdata, ref, None, None, 256, 256, 2, 1, SFA=a_full.scale, SFB=W.scale, bs_format_a=fmt,
                bs_format_b=fmt)
    torch.cuda.synchronize()
    bitwise_ok = bool(torch.equal(ref, out))

    def time_roof():
        # pure-GEMM roof of this rank's block: pre-gathered A, every SM
        for _ in range(3):
            kernel_gemm(a_full.qdata, W.qdata, ref, None, None, 256, 256, 2, 1, SFA=a_full.scale, SFB=W.scale,
                        bs_format_a=fmt, bs_format_b=fmt)
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for _ in range(args.steps):
            kernel_gemm(a_full.qdata, W.qdata, ref, None, None, 256, 256, 2, 1, SFA=a_full.scale, SFB=W.scale,
                        bs_format_a=fmt, bs_format_b=fmt)
        r1.record()
        torch.cuda.synchronize()
        return r0.elapsed_time(r1) / args.steps

    roof_before = time_roof()
    launches0 = _lib.launch_count()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        launches = _lib.launch_count() - launches0
        # the timed region lasts tens of milliseconds: keep the same load going (untimed, all ranks in
        # step) until the clock sampler has had 0.4 s of it
        import time
        extra = int(max(0.0, 0.4 - e0.elapsed_time(e1) / 1e3) / max(e0.elapsed_time(e1) / 1e3 / args.steps, 1e-4))
        t_extra = torch.tensor([extra], device=dev, dtype=torch.int64)
        dist.all_reduce(t_extra, op=dist.ReduceOp.MAX)
        for i in range(int(t_extra.item())):
            step()
            if i % 16 == 15:
                torch.cuda.synchronize()
                time.sleep(0)
        torch.cuda.synchronize()
    dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    _ops.check_status(dev)

    # the roof is timed before and after the overlapped loop (the GPU's clock drifts with temperature
    # and power over the run); the faster of the two is the denominator of the efficiency
    roof_ms = min(roof_before, time_roof())
    # the same dense block for 0.4 s with the clock sampler running: says whether the overlapped loop and its roof
    # saw the same SM clock (the exchange draws power too, and the part runs at its power cap)
    with ClockSampler(local) as roof_clocks:
        n_sus = max(args.steps, int(0.4 / max(roof_ms * 1e-3, 1e-5)))
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for i in range(n_sus):
            kernel_gemm(a_full.qdata, W.qdata, ref, None, None, 256, 256, 2, 1, SFA=a_full.scale, SFB=W.scale,
                        bs_format_a=fmt, bs_format_b=fmt)
        r1.record()
        torch.cuda.synchronize()
        roof_sustained_ms = r0.elapsed_time(r1) / n_sus
    roof_clk = roof_clocks.summary()

    # end to end: pinned bf16 shard -> device -> quantise -> gather + GEMM -> bf16 block -> pinned host.
    # Copy-in, compute and copy-out of consecutive steps overlap (three streams, two buffers each), as a
    # serving loop would run them; every step still moves its own input and output over PCIe.
    a_host = a_shard_hp.cpu().pin_memory()
    d_hosts = [torch.empty(M, n_loc, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    cur = torch.cuda.current_stream(dev)
    a_bufs = [torch.empty(shard_m, K, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    o_bufs = [out, ref]
    ev_in, ev_used, ev_done, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(4))

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
            shard = BlockScaledOperand.quantize(a_bufs[b], fmt)
            ev_used[b].record(cur)
            with runner.gather(shard) as (af, ag):
                kernel_gemm(af.qdata, W.qdata, o_bufs[b], None, None, 256, 256, 2, 1, SFA=af.scale, SFB=W.scale, bs_format_a=fmt,
                            bs_format_b=fmt, ag_args=ag, max_ctas=max_ctas, ag_arrival_order=arrival)
            ev_done[b].record(cur)
            s_out.wait_event(ev_done[b])
            with torch.cuda.stream(s_out):
                d_hosts[b].copy_(o_bufs[b], non_blocking=True)
                ev_out[b].record(s_out)
        cur.wait_stream(s_out)

    e2e_run(2)
    torch.cuda.synchronize()
    dist.barrier()
    e2e_steps = max(4, min(args.steps, 16))
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    e2e_run(e2e_steps)
    x1.record()
    torch.cuda.synchronize()
    e2e_ms = x0.elapsed_time(x1) / e2e_steps
    _ops.check_status(dev)
    d_host = d_hosts[0]

    # The same workload on ONE GPU (the whole 32768 x 28672 x 8192 problem, operands resident, no exchange), timed on
    # rank 0 while the other ranks wait: the like-for-like denominator of the scaling curve (the single-GPU headline
    # of this benchmark is a different problem in a different format).
    w1_ms = 0.0
    if world > 1:
        if rank == 0:
            try:
                a_all = BlockScaledOperand.quantize(torch.cat([randn_bf16(shard_m, K, 1000 + r) for r in range(world)]), fmt)
                w_all = BlockScaledOperand.quantize(randn_bf16(N, K, 4321, 0.02), fmt)
                d_all = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                for _ in range(2):
                    kernel_gemm(a_all.qdata, w_all.qdata, d_all, None, None, 256, 256, 2, 1, SFA=a_all.scale, SFB=w_all.scale,
                                bs_format_a=fmt, bs_format_b=fmt)
                w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 5
                w0.record()
                for _ in range(reps):
                    kernel_gemm(a_all.qdata, w_all.qdata, d_all, None, None, 256, 256, 2, 1, SFA=a_all.scale, SFB=w_all.scale,
                                bs_format_a=fmt, bs_format_b=fmt)
                w1.record()
                torch.cuda.synchronize()
                w1_ms = w0.elapsed_time(w1) / reps
                del a_all, w_all, d_all
            except torch.OutOfMemoryError:
                w1_ms = 0.0
        dist.barrier()

    t = torch.tensor([ms, roof_ms, e2e_ms, 0.0 if bitwise_ok else 1.0], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, roof_ms, e2e_ms, bad = t.tolist()
    total_flops = 2.0 * M * N * K
    value = total_flops / (ms * 1e-3) / 1e12
    per_gpu = value / world
    peak = 2.0 * peaks["bf16"]   # burst figure: the timed region lasts tens of milliseconds
    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": warm,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp8_e4m3 x ue8m0 block scales, fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"allgather_mxfp8_gemm_32768x28672x8192_tp{world}", "m": M, "n_per_rank": n_loc, "k": K,
                       "tile": "256x256x128, CTA pair", "transport": {"ce": "copy-engine pushes into peers' buffers (CUDA IPC), per-shard flags",
                                     "pull": "in-kernel: one warp per CTA of the GEMM bulk-copies the peers' shards over NVLink "
                                             "(CUDA IPC mappings) into this GPU's buffer, per-shard flags",
                                     "mc": "in-kernel: one warp per CTA of the GEMM stores this rank's shard through an NVSwitch "
                                           "multicast mapping of all ranks' buffers (multimem.st), per-shard flags",
                                     "nccl": "NCCL ring send/recv on a side stream, per-shard flags"}[runner.transport],
                       "gemm_ctas": max_ctas, "shard_order": "arrival" if arrival else "ring", "l2": "operands per rank (A 256 MiB + W) exceed the 126 MB L2",
                       "gated_output_bitwise_equal_to_dense": not bad},
            "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s", "frac": per_gpu / peak,
                         "frac_of_sustained": per_gpu / (2.0 * peaks["bf16_sustained"]),
                         "peak_basis": f"2 x {peaks['bf16']} TFLOP/s burst bf16 ({peaks['source']}; sustained "
                                       f"{peaks['bf16_sustained']}) per GPU; achieved is per GPU", "traffic": None},
            "overlap": {"gemm_only_ms": roof_ms, "overlapped_ms": ms, "efficiency": roof_ms / ms,
                        # the same ratio against the dense block timed for 0.4 s (the overlapped loop runs after
                        # seconds of load, at the clock the power cap leaves; the 50-launch roof above is a burst)
                        "efficiency_vs_sustained": roof_sustained_ms / ms,
                        "gemm_only_sustained_ms": roof_sustained_ms, "gemm_only_sm_mhz": roof_clk.get("sm_mhz"),
                        "gemm_only_power_w_max": roof_clk.get("power_w_max"),
                        "nvlink_bytes_in_per_rank": (world - 1) * shard_m * (K + K // 32), "arrival_chunks": chunks,
                        "push_streams": len(runner.comm_streams), "chunks_spread_over_streams": runner.chunk_streams,
                        "receiver_exclusive_ingress": runner.exclusive_ingress, "turn_early": runner.turn_early,
                        # in-kernel transport, rank 0, last timed call (QK_AG_PULL_TIMES=1): per shard, microseconds from
                        # the kernel's start to the shard's flag and the wait for its owner inside that
                        "pull_publish_us": ([[round(v / 1e3, 1) for v in row] for row in runner.publish_ns.tolist()]
                                            if (runner.transport in ("pull", "mc") and os.environ.get("QK_AG_PULL_TIMES")) else None)},
            "w1_same_workload": None if not w1_ms else {
                "ms_per_step": w1_ms, "value": total_flops / (w1_ms * 1e-3) / 1e12, "unit": unit,
                "what": "the whole 32768 x 28672 x 8192 MXFP8 problem on one GPU (rank 0, operands resident, no exchange)"},
            "per_gpu_vs_w1": None if not w1_ms else per_gpu / (total_flops / (w1_ms * 1e-3) / 1e12),
            "cpu_baseline": None,
            "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": unit, "h2d_bytes_per_step": a_host.numel() * 2,
                    "d2h_bytes_per_step": d_host.numel() * 2, "ms_per_step": e2e_ms,
                    "path": "pinned bf16 shard -> device, qk_quantize_blockscaled, all-gather + gated GEMM, bf16 block -> pinned host; "
                            "copy-in / compute / copy-out of consecutive steps overlap on three streams"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    runner.close()
    dist.barrier()
    dist.destroy_process_group()

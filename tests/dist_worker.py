"""Worker of tests/test_distributed_gpu.py: one process per GPU under torch.distributed.run.
Checks the overlapped all-gather GEMM against NCCL-gathered operands and the dense kernel."""

import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    from quack_b200 import _ops
    from quack_b200.blockscaled import BlockScaledOperand
    from quack_b200.distributed import BlockScaledAllGatherRunner
    from quack_b200.gemm import gemm as kernel_gemm

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    shard_m, K, n_loc = 1024, 2048, 1536
    # (format, transport, arrival-order schedule, arrival chunks per shard, chunks of a shard spread over the push streams)
    variants = [("mxfp8_e4m3", "mc", True, 1, False), ("nvfp4", "mc", False, 1, False), ("mxfp8_e4m3", "mc", True, 2, False)] if os.environ.get("QK_TEST_MULTICAST", "1") != "0" else []
    for fmt, transport, arrival, chunks, spread in variants + list((
            ("mxfp8_e4m3", "nccl", False, 1, False), ("nvfp4", "nccl", True, 1, False), ("mxfp8_e4m3", "ce", True, 1, False),
            ("nvfp4", "ce", False, 1, False), ("mxfp8_e4m3", "ce", False, 4, False), ("mxfp8_e4m3", "nccl", False, 2, False),
            ("mxfp8_e4m3", "ce", False, 2, True), ("mxfp8_e4m3", "pull", True, 1, False), ("nvfp4", "pull", False, 1, False))):
        try:
            runner = BlockScaledAllGatherRunner(shard_m, K, fmt, device=dev, comm_sms=16, transport=transport, arrival_chunks=chunks,
                                                push_streams=2, chunk_streams=spread)
        except RuntimeError as e:
            if transport == "mc" and "multicast" in str(e):      # every rank sees the same: no multicast on this system
                if rank == 0:
                    print(f"multicast transport skipped: {e}", flush=True)
                continue
            raise
        assert runner.transport == transport and runner.arrival_chunks == chunks
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        W = BlockScaledOperand.quantize((torch.randn(n_loc, K, generator=g, device=dev) * 0.02).to(torch.bfloat16), fmt)
        out = torch.empty(shard_m * world, n_loc, dtype=torch.bfloat16, device=dev)
        failure, a_full, ag = None, None, None
        for it in range(4):
            try:
                g = torch.Generator(device=dev).manual_seed(1000 + rank + 100 * it)
                shard = BlockScaledOperand.quantize(torch.randn(shard_m, K, generator=g, device=dev).to(torch.bfloat16), fmt)
                # reference gather through NCCL collectives
                ref_q = torch.empty(world * shard_m, shard.qdata.shape[1], dtype=torch.uint8, device=dev)
                ref_sf = torch.empty(world, *shard.scale.shape, dtype=torch.uint8, device=dev)
                dist.all_gather_into_tensor(ref_q, shard.qdata.view(torch.uint8).contiguous())
                dist.all_gather_into_tensor(ref_sf, shard.scale.view(torch.uint8).contiguous())
                if it == 2 and rank == world - 1:
                    time.sleep(0.2)          # a late sender: its peers wait at the arrival gate
                with runner.gather(shard) as (a_full, ag):
                    kernel_gemm(a_full.qdata, W.qdata, out, None, None, 256, 256, 2, 1, SFA=a_full.scale, SFB=W.scale,
                                bs_format_a=fmt, bs_format_b=fmt, ag_args=ag, max_ctas=runner.gemm_max_ctas, ag_arrival_order=arrival)
                torch.cuda.synchronize()
                _ops.check_status(dev)
                assert torch.equal(runner.gathered_a().view(torch.uint8), ref_q), f"{fmt}/{transport} it{it}: gathered codes differ"
                assert torch.equal(a_full.scale.view(torch.uint8).reshape(-1), ref_sf.reshape(-1)), f"{fmt}/{transport} it{it}: gathered scales differ"
                # shard scale atoms concatenate: quantising is per row block along K, so gather == quantise(cat)
                dense = torch.empty_like(out)
                full_ref = BlockScaledOperand.from_parts(ref_q.view(shard.qdata.dtype), ref_sf.view(-1, *shard.scale.shape[1:]), fmt)
                kernel_gemm(full_ref.qdata, W.qdata, dense, None, None, 256, 256, 2, 1, SFA=full_ref.scale, SFB=W.scale,
                            bs_format_a=fmt, bs_format_b=fmt)
                torch.cuda.synchronize()
                assert torch.equal(out, dense), f"{fmt}/{transport} it{it}: gated GEMM differs from the dense GEMM"
            except Exception as e:      # keep the ranks in step: nobody leaves while the others still use the buffers
                failure = f"rank {rank}: {type(e).__name__}: {e}"
            bad = torch.tensor([1 if failure else 0], device=dev)
            dist.all_reduce(bad, op=dist.ReduceOp.MAX)
            if bad.item():
                break
        a_full = ag = None      # (views of the runner's buffers)
        runner.close()
        dist.barrier()
        if bad.item():
            raise AssertionError(failure or f"{fmt}/{transport}: another rank failed")
    # transport="auto" settles for NCCL (on every rank) when the peers' buffers cannot be mapped
    import warnings
    os.environ["QK_DISABLE_IPC"] = "1"
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        fallback = BlockScaledAllGatherRunner(shard_m, K, "mxfp8_e4m3", device=dev)
    del os.environ["QK_DISABLE_IPC"]
    assert fallback.transport == "nccl" and fallback.gemm_max_ctas > 0
    auto = BlockScaledAllGatherRunner(shard_m, K, "mxfp8_e4m3", device=dev)
    assert auto.transport == "ce" and auto.gemm_max_ctas == 0
    auto.close()
    dist.barrier()
    if rank == 0:
        print("DIST_WORKER_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Host logic of the all-gather runner on CPU ranks (gloo, world_size 2 and 3): ring schedule,
buffer placement, shard-concatenation of blocked scale factors, flag / epoch bookkeeping over
several iterations (buffer rotation), operand checks.  No GPU involved."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import blockscaled_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard(rank, shard_m, k, it=0):
    x = orc.make_activation(shard_m, k, 1000 + rank + 17 * it)
    c, s = orc.to_mx_e4m3(x)
    return x, c, s


def _worker(rank, world, port, shard_m, k, iters, q, chunks=1):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from quack_b200.blockscaled import BlockScaledOperand
        from quack_b200.distributed import BlockScaledAllGatherRunner, ring_schedule

        sched = ring_schedule(rank, world)
        assert [s for s, _, _ in sched] == list(range(1, world))
        assert [r for _, _, r in sched] == [(rank + s) % world for s in range(1, world)]   # arrival == consumption order
        runner = BlockScaledAllGatherRunner(shard_m, k, "mxfp8_e4m3", device="cpu", arrival_chunks=chunks)
        assert runner.gemm_max_ctas == 0 and runner.flags.numel() == world * chunks
        for it in range(iters):
            _, c, s = _shard(rank, shard_m, k, it)
            op = BlockScaledOperand.from_parts(torch.from_numpy(c).view(torch.float8_e4m3fn),
                                               torch.from_numpy(orc.pack_scale_blocked(s)), "mxfp8_e4m3")
            with runner.gather(op) as (full, ag):
                assert ag.num_shards == world and ag.first_shard == rank and ag.num_chunks == chunks
                assert ag.epoch.item() == it + 1 and (ag.flags >= it + 1).all()   # every shard published
                # reference: quantise the concatenation of all shards at once
                xs = [_shard(r, shard_m, k, it) for r in range(world)]
                codes = np.concatenate([t[1] for t in xs])
                sfs = orc.pack_scale_blocked(np.concatenate([t[2] for t in xs]))
                assert np.array_equal(full.qdata.view(torch.uint8).numpy(), codes)
                assert np.array_equal(full.scale.view(torch.uint8).numpy(), sfs)   # shard scale atoms concatenate
                assert full.shape == (shard_m * world, k) and full.quant_dim == -1
            assert runner.gathered_a().data_ptr() == full.qdata.data_ptr()
            assert runner.next_local_slot().data_ptr() != runner.gathered_a()[rank * shard_m:].data_ptr()
        # operand checks
        _, c, s = _shard(rank, shard_m, k)
        good = BlockScaledOperand.from_parts(torch.from_numpy(c).view(torch.float8_e4m3fn),
                                             torch.from_numpy(orc.pack_scale_blocked(s)), "mxfp8_e4m3")
        for bad, exc in ((good.mT, ValueError), ((good.qdata, good.scale), TypeError)):
            try:
                with runner.gather(bad):
                    pass
                raise AssertionError("expected a rejection")
            except exc:
                pass
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, "".join(traceback.format_exception(e))))


@pytest.mark.parametrize("world,shard_m,chunks", [(2, 128, 1), (3, 128, 1), (2, 512, 4)])
def test_runner_on_cpu_ranks(world, shard_m, chunks):
    """``chunks`` > 1: every shard travels in row chunks with one flag each (whole scale atoms per chunk)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shard_m, 256, 3, q, chunks)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(msg == "ok" for _, msg in results), results


def test_nvfp4_tensor_scale_is_rejected_single_rank():
    port = _free_port()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        from quack_b200.blockscaled import BlockScaledOperand
        from quack_b200.distributed import BlockScaledAllGatherRunner

        runner = BlockScaledAllGatherRunner(128, 256, "nvfp4", device="cpu")
        x = orc.make_activation(128, 256, 0)
        c, s = orc.to_nvfp4(x, 0.01)
        op = BlockScaledOperand.from_parts(torch.from_numpy(c).view(torch.float4_e2m1fn_x2),
                                           torch.from_numpy(orc.pack_scale_blocked(s)), "nvfp4",
                                           per_tensor_scale=torch.tensor([0.01]))
        with pytest.raises(ValueError, match="per_tensor_scale"):
            with runner.gather(op):
                pass
        op2 = BlockScaledOperand.from_parts(op.qdata, op.scale, "nvfp4")
        with runner.gather(op2) as (full, ag):        # world_size 1: local copy, no gate
            assert ag is None and torch.equal(full.qdata.view(torch.uint8), op2.qdata.view(torch.uint8))
        with pytest.raises(AssertionError, match="multiple of 128"):
            BlockScaledAllGatherRunner(100, 256, "mxfp8_e4m3", device="cpu")
        with pytest.raises(AssertionError, match="arrival_chunks"):     # a chunk must hold whole 128-row scale atoms
            BlockScaledAllGatherRunner(128, 256, "mxfp8_e4m3", device="cpu", arrival_chunks=2)
        with pytest.raises(NotImplementedError, match="capture"):
            BlockScaledAllGatherRunner(128, 256, "mxfp8_e4m3", device="cpu", capture_lockstep=True)
        # transports: names and the shapes the in-kernel ones take are checked before anything is allocated
        with pytest.raises(ValueError, match="transport must be"):
            BlockScaledAllGatherRunner(128, 256, "mxfp8_e4m3", device="cpu", transport="smoke-signals")
        with pytest.raises(ValueError, match="arrival_chunks == 1"):
            BlockScaledAllGatherRunner(512, 256, "mxfp8_e4m3", device="cpu", transport="pull", arrival_chunks=2)
        with pytest.raises(ValueError, match="whole 256-row tiles"):
            BlockScaledAllGatherRunner(256, 256, "mxfp8_e4m3", device="cpu", transport="mc", arrival_chunks=2)
        # off the GPU (or alone) every transport name ends at the synchronous path
        for name in ("pull", "mc", "ce", "auto"):
            r1 = BlockScaledAllGatherRunner(256, 256, "mxfp8_e4m3", device="cpu", transport=name)
            assert r1.transport == "nccl" and r1.gemm_max_ctas == 0 and r1._arena is None
        runner.quiesce(last_parity=0)
        assert runner.last_parity == 0
    finally:
        dist.destroy_process_group()


def test_host_deadline_helper_names_what_is_stuck():
    """The copy-engine transport polls the completion of the pushes of two calls ago before it enqueues new
    ones; a peer that stopped calling gather() shows up as an event that never completes.  Here the events
    are host-side stand-ins: one completes after a few polls, one never does."""
    from quack_b200.distributed import wait_events_or_report
    calls = {"n": 0}
    def soon():
        calls["n"] += 1
        return calls["n"] > 3
    assert wait_events_or_report([lambda: True, soon], timeout_s=5.0, describe=lambda: "never") is None
    assert calls["n"] == 4
    assert wait_events_or_report([lambda: True, lambda: False], timeout_s=0.05, describe=lambda: [1, 2]) == [1, 2]

"""In-kernel all-gather transport (``qk_ag_pull_args``) on ONE GPU.

The "peers" are other allocations of the same device: every emulated peer owns a full-size gather buffer in which
only its own shard is valid (the rest is poison), a flag array and a drained array.  The GEMM's transport warps
must copy exactly the remote shards into the local gather buffer, publish the flags, report the reads to the
owners and leave the arrival counters at zero; the product is compared bitwise with the plain kernel on the whole
operand (the reference's gated == dense check, tests/test_blockscaled_distributed_gemm.py:106-160).  Nothing in
these launches waits for another launch: every flag a kernel polls is set before it starts."""

import ctypes as C

import pytest
import torch

from tests.helpers import dev, make_operand_pair

pytestmark = pytest.mark.gpu


def _table(t):
    raw = torch.frombuffer(bytearray(C.string_at(C.addressof(t), C.sizeof(t))), dtype=torch.uint8)
    return raw.cuda()


def _setup(fmt, m, n, k, world, rank, seed):
    from quack_b200 import _lib
    ops = make_operand_pair(fmt, m, n, k, seed=seed, use_pts=False)
    codes, sf = dev(ops["ac"]), dev(ops["asf_b"])          # (m, k_storage) bytes, (m/128, rk, 32, 4, 4) bytes
    shard_m = m // world
    rm_shard = shard_m // 128
    code_sz, sf_sz = codes[:shard_m].numel(), sf[:rm_shard].numel()
    poison_c, poison_s = 0x7E, 0x00
    local_c = torch.full_like(codes, poison_c)
    local_s = torch.full_like(sf, poison_s)
    local_c[rank * shard_m:(rank + 1) * shard_m] = codes[rank * shard_m:(rank + 1) * shard_m]
    local_s[rank * rm_shard:(rank + 1) * rm_shard] = sf[rank * rm_shard:(rank + 1) * rm_shard]
    peers = []
    for s in range(world):
        if s == rank:
            peers.append(None)
            continue
        pc = torch.full_like(codes, 0x11 + s)
        ps = torch.full_like(sf, 0x70 + s)
        pc[s * shard_m:(s + 1) * shard_m] = codes[s * shard_m:(s + 1) * shard_m]
        ps[s * rm_shard:(s + 1) * rm_shard] = sf[s * rm_shard:(s + 1) * rm_shard]
        peers.append(dict(c=pc, s=ps, flags=torch.zeros(world, dtype=torch.int32, device="cuda"),
                          drained=torch.zeros(world, dtype=torch.int32, device="cuda")))
    flags = torch.zeros(world, dtype=torch.int32, device="cuda")
    arrive = torch.zeros(world, dtype=torch.int32, device="cuda")
    t = _lib.AgPullArgs()
    t.num_payloads, t.rank = 2, rank
    t.shard_bytes[0], t.shard_bytes[1] = code_sz, sf_sz
    t.local_base[0], t.local_base[1] = local_c.data_ptr(), local_s.data_ptr()
    for s in range(world):
        if s == rank:
            continue
        t.peer_base[s][0], t.peer_base[s][1] = peers[s]["c"].data_ptr(), peers[s]["s"].data_ptr()
        t.peer_flags[s] = peers[s]["flags"].data_ptr()
        t.peer_drained[s] = peers[s]["drained"].data_ptr()
    t.arrive, t.flags_rw = arrive.data_ptr(), flags.data_ptr()
    return dict(ops=ops, codes=codes, sf=sf, local_c=local_c, local_s=local_s, peers=peers, flags=flags, arrive=arrive,
                table=_table(t), keep=t)


@pytest.mark.parametrize("fmt,m,n,k,world,rank", [
    ("mxfp8_e4m3", 2048, 512, 1152, 4, 1),      # scale bytes per shard: 4.5 slots (a short last piece)
    ("mxfp8_e4m3", 4096, 768, 512, 8, 7),       # wrap-around of the shard order
    ("nvfp4", 2048, 512, 1024, 2, 0),
    ("mxfp8_e4m3", 8192, 1024, 2048, 4, 2),     # more pieces per CTA than ring slots
])
def test_pull_transport_gathers_and_matches_dense(fmt, m, n, k, world, rank):
    from quack_b200 import _lib, _ops
    from quack_b200.gemm import AllGatherArguments
    S = _setup(fmt, m, n, k, world, rank, seed=21)
    ops = S["ops"]
    fid = _ops.format_id(fmt)
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    dense = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _ops.gemm_blockscaled(fid, S["codes"], S["sf"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, d=dense, tile_n=256,
                          cta_group=2, status=st)
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call, sched in enumerate((_lib.SCHED_ARRIVAL, _lib.SCHED_STATIC, _lib.SCHED_ARRIVAL), start=1):
        # a new "call": the local buffer is refilled with poison outside the own shard, every owner has staged
        e = 40 + call
        epoch.fill_(e)
        shard_m = m // world
        keep_c = S["local_c"][rank * shard_m:(rank + 1) * shard_m].clone()
        S["local_c"].fill_(0x7E)
        S["local_c"][rank * shard_m:(rank + 1) * shard_m] = keep_c
        rm_shard = shard_m // 128
        keep_s = S["local_s"][rank * rm_shard:(rank + 1) * rm_shard].clone()
        S["local_s"].fill_(0x00)
        S["local_s"][rank * rm_shard:(rank + 1) * rm_shard] = keep_s
        S["flags"][rank] = e
        for s in range(world):
            if s != rank:
                S["peers"][s]["flags"][s] = e
        D = torch.zeros_like(dense)
        _ops.gemm_blockscaled(fid, S["local_c"], S["local_s"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, d=D, status=st,
                              timeout_ns=500_000_000, scheduler=sched,
                              ag=AllGatherArguments(S["flags"], epoch, world, rank, 1, S["table"]))
        torch.cuda.synchronize()
        assert st.tolist()[0] == 0, f"kernel reported status {st.tolist()}"
        assert torch.equal(S["local_c"], S["codes"]), "gathered codes differ from the whole operand"
        assert torch.equal(S["local_s"], S["sf"]), "gathered scale bytes differ from the whole operand"
        assert torch.equal(D, dense), "product on the in-kernel gather differs from the dense kernel"
        assert S["flags"].tolist() == [e] * world
        assert S["arrive"].tolist() == [0] * world
        for s in range(world):
            if s != rank:
                want = [0] * world
                want[rank] = e
                assert S["peers"][s]["drained"].tolist() == want


def test_pull_transport_reports_an_owner_that_never_staged():
    """The owner's flag stays behind the epoch: the transport's bounded wait gives up, the kernel returns with
    status 7 naming the shard, and the context stays usable (the same launch then completes)."""
    from quack_b200 import _ops
    from quack_b200.gemm import AllGatherArguments
    fmt, m, n, k, world, rank = "mxfp8_e4m3", 1024, 256, 256, 2, 0
    S = _setup(fmt, m, n, k, world, rank, seed=3)
    ops = S["ops"]
    fid = _ops.format_id(fmt)
    epoch = torch.full((1,), 5, dtype=torch.int32, device="cuda")
    S["flags"][rank] = 5
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    D = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    args = dict(d=D, status=st, timeout_ns=50_000_000, ag=AllGatherArguments(S["flags"], epoch, world, rank, 1, S["table"]))
    _ops.gemm_blockscaled(fid, S["local_c"], S["local_s"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, **args)
    torch.cuda.synchronize()
    s = st.tolist()
    assert s[0] in (5, 7), s          # whichever bounded wait ran out first: the transport's (7) or the gate's (5)
    if s[0] == 7:
        assert s[1] == 1000 + 1 and s[3] == 5
    st.zero_()
    S["arrive"].zero_()
    S["peers"][1]["flags"][1] = 5
    _ops.gemm_blockscaled(fid, S["local_c"], S["local_s"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, **args)
    torch.cuda.synchronize()
    assert st.tolist()[0] == 0
    dense = torch.empty_like(D)
    _ops.gemm_blockscaled(fid, S["codes"], S["sf"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, d=dense, tile_n=256, cta_group=2,
                          status=st)
    torch.cuda.synchronize()
    assert torch.equal(D, dense)


def test_pull_transport_argument_checks():
    from quack_b200 import _ops
    from quack_b200.gemm import AllGatherArguments
    fmt, m, n, k, world, rank = "mxfp8_e4m3", 1024, 256, 256, 2, 0
    S = _setup(fmt, m, n, k, world, rank, seed=4)
    ops = S["ops"]
    epoch = torch.full((1,), 1, dtype=torch.int32, device="cuda")
    D = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError, match="256-wide CTA-pair"):
        _ops.gemm_blockscaled(_ops.format_id(fmt), S["local_c"], S["local_s"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, d=D,
                              tile_n=128, cta_group=1, ag=AllGatherArguments(S["flags"], epoch, world, rank, 1, S["table"]))
    with pytest.raises(ValueError, match="one chunk per shard"):
        flags2 = torch.zeros(2 * world, dtype=torch.int32, device="cuda")
        _ops.gemm_blockscaled(_ops.format_id(fmt), S["local_c"], S["local_s"], dev(ops["bc"]), dev(ops["bsf_b"]), m, n, k, d=D,
                              ag=AllGatherArguments(flags2, epoch, world, rank, 2, S["table"]))

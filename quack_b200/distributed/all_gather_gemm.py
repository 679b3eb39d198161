"""Overlapped all-gather + block-scaled GEMM: the transport half.

Column-parallel linear with token-sharded activations: every rank holds ``shard_m`` rows of A
(quantised codes + blocked scale factors) and ``N / world`` rows of the weight; each rank
computes the full-M x N/world output block.  The runner fills a local gather buffer shard by
shard while the GEMM (given ``ag_args``) consumes the shards in the same order through its
arrival gate.  API of the reference's ``quack/distributed/all_gather_gemm.py``
(``AllGatherRunner`` :275-815, ``BlockScaledAllGatherRunner`` :818-1048); the transport is
different by design:

* Two transports behind one flag contract.  ``"ce"`` (what ``"auto"`` picks whenever the ranks can map each
  other's buffers): every rank PUSHES its shard into its peers' gather buffers with copy-engine
  ``cudaMemcpyAsync`` copies over NVLink (buffers shared through CUDA IPC), needs no SM, and the GEMM keeps
  the whole GPU; details below.  ``"nccl"``: a ring of ``world - 1`` steps on a side stream; in step ``s`` a
  rank sends its own shard to ``rank - s`` and receives the shard of ``rank + s`` (one ``ncclSend`` /
  ``ncclRecv`` group per step, the scale-factor bytes in the same group), so shards arrive in exactly the
  order the GEMM visits them; NCCL's kernels need SMs while the persistent GEMM is resident, so the GEMM is
  then launched on ``num_sms - comm_sms`` CTAs (``gemm_max_ctas``).
* Every rank's data lands in its OWN HBM before any TMA load reads it: no load ever touches a
  peer's memory, and nothing uses cluster multicast.
* A shard travels in ``arrival_chunks`` row chunks; after each chunk a 4-byte device-to-device copy publishes
  its arrival flag (``flags[shard * chunks + c] = epoch``); the GEMM's producer warp waits on the flag of
  the chunk a tile's rows belong to, with a deadline.
* ``quant_dim`` must be -1 and NVFP4 per-tensor scales are rejected, as in the reference
  (:995-1010): a per-rank tensor scale cannot be folded into one alpha.
* Every rank must call ``gather()`` the same number of times.  The epoch that orders buffer reuse across
  ranks is a host counter, so a ``gather()`` cannot be captured in a CUDA graph (it raises); ``quiesce()`` is
  the fence to use before reading the buffers from another stream.

With CPU tensors and the gloo backend the same schedule runs synchronously; that is how the
host logic is tested without GPUs.

Second transport, ``transport="ce"`` (the reference's measured optimum, all_gather_gemm.py:31-38):
every rank opens its peers' gather buffers and flag arrays through CUDA IPC and PUSHES its shard
into them with ``cudaMemcpyAsync`` device-to-device copies (copy engines over NVLink, no SM), in
reverse ring order so that every receiver gets the shard it needs next first, each followed by a
4-byte copy of the epoch into the receiver's flag.  The GEMM then keeps every SM.  Only copies
write peer memory; no kernel is ever handed a peer pointer.  A peer's buffer is overwritten only
after that peer has signalled (a 4-byte copy into this rank's ``drained`` array, awaited with a
stream-ordered 32-bit wait) that its GEMM of two calls ago, the last reader, has finished.  The
buffers must come from cudaMalloc (the default torch allocator; not expandable segments).
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from typing import Optional

import torch
import torch.distributed as dist

from ..blockscaled.operand import BlockScaledFormat, BlockScaledOperand, _coerce_format
from ..gemm import AllGatherArguments

__all__ = ["AllGatherRunner", "BlockScaledAllGatherRunner", "ring_schedule", "wait_events_or_report"]


def _lib_max_ranks() -> int:
    from .. import _lib
    return _lib.AG_MAX_RANKS


def wait_events_or_report(queries, timeout_s: float, describe, poll_s: float = 0.001):
    """Poll ``queries`` (callables returning True once their event has completed) until all are done or
    ``timeout_s`` has passed; returns None on completion, else ``describe()``.  Completed events cost one
    call each, so the check is free in the steady state."""
    import time
    deadline = None
    for q in queries:
        while not q():
            now = time.monotonic()
            if deadline is None:
                deadline = now + timeout_s
            if now >= deadline:
                return describe()
            time.sleep(poll_s)
    return None


def ring_schedule(rank: int, world: int):
    """[(step, send_to, recv_from)] of the ring exchange: in step s the shard of rank + s
    arrives, which is the s-th shard the rotated tile order visits."""
    return [(s, (rank - s) % world, (rank + s) % world) for s in range(1, world)]


class AllGatherRunner:
    """Rotating gather buffers, arrival flags, the comm stream and the ring exchange for a
    plain byte matrix ``(shard_m, row_bytes)`` per rank.  Knows nothing about the GEMM."""

    def __init__(self, shard_m: int, k: int, dtype: torch.dtype, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None, arrival_chunks: int = 1, capture_lockstep: bool = False,
                 comm_sms: int = 16, transport: str = "auto", push_streams: Optional[int] = None, chunk_streams: bool = False,
                 exclusive_ingress: Optional[bool] = None, _arena_reserve: int = 0, turn_early: Optional[float] = None):
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world_size = dist.get_world_size(self.group)
        self.shard_m, self.k, self.dtype = shard_m, k, dtype
        if arrival_chunks < 1 or shard_m % arrival_chunks:
            raise ValueError(f"arrival_chunks ({arrival_chunks}) must divide the shard rows ({shard_m})")
        if capture_lockstep:
            raise NotImplementedError("capture_lockstep selects how a CUDA-graph capture of gather() joins its side "
                                      "streams; this runner's epoch is a host counter and gather() cannot be captured")
        self.arrival_chunks = arrival_chunks
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        self.on_gpu = self.device.type == "cuda"
        self.comm_sms = comm_sms
        self.chunk_streams = bool(chunk_streams)
        # copy-engine transport: a receiver takes one sender at a time, in the order its GEMM consumes the shards
        # (a turn word handed from sender to sender).  Measured overlap efficiency with / without: 0.72 / 0.47-0.68 at
        # 8 ranks, 0.79-0.81 / 0.82 at 4; with 2 ranks there is only one sender
        self.exclusive_ingress = (dist.get_world_size(self.group) >= 8) if exclusive_ingress is None else bool(exclusive_ingress)
        # `turn_early` > 0 hands the turn on before the sender's copy has finished (the last fraction of the codes
        # travels while the next sender's stream wait fires).  Measured at 8 ranks: 0.25 -> 1.010 ms per step, 0.5 ->
        # 0.996 ms, off -> 0.934-0.939 ms: two senders at one receiver cost more than the idle hand-over, so it is off
        self.turn_early = float(os.environ.get("QK_AG_TURN_EARLY", "0")) if turn_early is None else float(turn_early)
        if push_streams is None:
            # measured (copy-engine transport, MXFP8 32768 x 28672 x 8192): at 8 ranks one push stream delivers
            # the shard the receiver needs next at full rate (0.68 vs 0.64 overlap efficiency with two); at 2-4
            # ranks a second stream hides the per-copy fixed costs
            push_streams = 1 if dist.get_world_size(self.group) >= 8 else 2
        m_total = shard_m * self.world_size
        if transport not in ("nccl", "ce", "pull", "mc", "auto"):
            raise ValueError(f"transport must be 'auto', 'ce', 'pull', 'mc' or 'nccl', got {transport!r}")
        if transport in ("pull", "mc") and self.world_size > _lib_max_ranks():
            raise ValueError(f"transport={transport!r} takes at most {_lib_max_ranks()} ranks")
        if transport == "pull" and arrival_chunks != 1:
            raise ValueError("transport='pull' needs arrival_chunks == 1")
        if transport == "mc" and (self.world_size * arrival_chunks > 32 or shard_m % (256 * arrival_chunks)):
            raise ValueError("transport='mc': ranks x arrival_chunks must not exceed 32 and a chunk must hold whole 256-row tiles")
        # "mc": buffers, flags and drained words live in ONE symmetric allocation that is also bound to an NVSwitch
        # multicast object; the GEMM kernel stores this rank's shard through the multicast mapping
        self._arena = None
        if transport == "mc" and self.on_gpu and self.world_size > 1:
            code_bytes = m_total * k * torch.empty(0, dtype=dtype).element_size()
            self._mc_init(2 * (code_bytes + 256) + _arena_reserve + 4096)
        self.bufs = [self._new_buffer((m_total, k), dtype) for _ in range(2)]
        # flags[shard] >= epoch (modular) means the shard is resident; never reset
        self.flags = self._new_buffer((self.world_size * arrival_chunks,), torch.int32, zero=True)
        self.epoch_dev = torch.zeros(2, dtype=torch.int32, device=self.device)   # one slot per buffer parity
        self.epoch = 0
        self.last_parity = 0
        self._in_gather = False
        # "auto": copy engines when every rank can map its peers' buffers, else NCCL (decided at the first gather)
        # "pull": the GEMM kernel fetches the remote shards itself (one more warp per CTA reads the peers' buffers)
        self._transport_requested = transport
        self._ce_error = ""
        self.transport = ({"ce": "ce", "auto": "ce", "pull": "pull", "mc": "mc"}.get(transport, "nccl")
                          if (self.on_gpu and self.world_size > 1) else "nccl")
        if self.on_gpu:
            # copy-engine pushes rotate over `push_streams` streams so that a sender keeps more than
            # one destination in flight (per-copy latencies and receivers that are busy with another
            # sender would otherwise idle its links); NCCL uses the first stream only
            self.comm_streams = [torch.cuda.Stream(device=self.device) for _ in range(max(1, push_streams))]
            self.comm_stream = self.comm_streams[0]
            self.ev_push_end = [[torch.cuda.Event() for _ in self.comm_streams] for _ in range(2)]   # [parity][stream]
            self._push_recorded = [False, False]
            # the device status word of the GEMMs (written when a bounded wait gives up) is copied to pinned host
            # memory after every call and looked at, without blocking, by the calls after it
            self._status_host = [torch.zeros(4, dtype=torch.int32).pin_memory() for _ in range(2)]
            self._status_ev = [torch.cuda.Event(), torch.cuda.Event()]
            self._status_pending = [False, False]
            self.ev_staged = torch.cuda.Event()
            self.ev_gemm_end = [torch.cuda.Event(), torch.cuda.Event()]
            self.ev_comm_end = torch.cuda.Event()
            self._gemm_recorded = [False, False]
            self.barrier_stream = torch.cuda.Stream(device=self.device)
            # drained[r] = last epoch whose GEMM rank r has finished (written by rank r's copies)
            self.drained = self._new_buffer((self.world_size,), torch.int32, zero=True)
            # turn[d] = last epoch for which this rank may push to receiver d (written by rank - 1, the sender that
            # serves d just before this rank does)
            self.turn = torch.zeros(self.world_size, dtype=torch.int32, device=self.device)
            self.drain_src = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._peer = None   # transport == "ce": per peer rank, the mapped addresses of its buffers
        self._opened = {}
        if self.world_size > 1:
            dist.barrier(self.group)
        if type(self) is AllGatherRunner:
            self._decide_transport([[self.bufs[0]], [self.bufs[1]]])

    # ---- symmetric allocation of the multicast transport ----
    def _mc_init(self, nbytes: int) -> None:
        import torch.distributed._symmetric_memory as symm_mem
        try:
            symm_mem.enable_symm_mem_for_group(self.group.group_name)
        except Exception:
            pass   # newer torch enables groups on demand
        nbytes = (nbytes + 2 * 1024 * 1024 - 1) // (2 * 1024 * 1024) * (2 * 1024 * 1024)
        self._arena = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
        self._arena.zero_()
        torch.cuda.synchronize(self.device)
        self._mc_hdl = symm_mem.rendezvous(self._arena, self.group)
        if not getattr(self._mc_hdl, "multicast_ptr", 0):
            raise RuntimeError("transport='mc': this system offers no NVSwitch multicast mapping for symmetric memory")
        self._arena_off = 0

    def _new_buffer(self, shape, dtype, zero: bool = False) -> torch.Tensor:
        """A device tensor: from the symmetric arena when the multicast transport owns one, else a plain one."""
        if self._arena is None:
            return (torch.zeros if zero else torch.empty)(*shape, dtype=dtype, device=self.device)
        n = 1
        for d in shape:
            n *= d
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        off = (self._arena_off + 255) // 256 * 256
        assert off + nbytes <= self._arena.numel(), "symmetric arena too small"
        self._arena_off = off + nbytes
        return self._arena[off:off + nbytes].view(dtype).view(*shape)      # (the arena was zeroed)

    def _mc_addr(self, t: torch.Tensor) -> int:
        """Multicast address of a tensor that lives in the symmetric arena (the multicast mapping and this rank's
        own mapping cover the same allocation, so offsets carry over)."""
        base = int(self._mc_hdl.buffer_ptrs[self.rank])
        off = t.data_ptr() - base
        assert 0 <= off and off + t.numel() * t.element_size() <= int(self._mc_hdl.buffer_size), "tensor outside the symmetric allocation"
        return int(self._mc_hdl.multicast_ptr) + off

    # ---- geometry shared with the GEMM ----
    @property
    def gemm_max_ctas(self) -> int:
        """Persistent-grid cap that leaves ``comm_sms`` SMs to the NCCL kernels (0 = no cap)."""
        if not self.on_gpu or self.world_size == 1 or self.transport in ("ce", "pull", "mc"):
            return 0
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return max(2, (sms - self.comm_sms) // 2 * 2)

    def gathered_a(self) -> torch.Tensor:
        """The gathered matrix of the last call; valid until the next call (buffers rotate)."""
        return self.bufs[self.last_parity]

    def next_local_slot(self) -> torch.Tensor:
        """The local-shard rows of the buffer the NEXT gather() will fill: a producer may write
        there directly and pass the view as the shard (the staging copy is then skipped)."""
        buf = self.bufs[self.last_parity ^ 1]
        return buf[self.rank * self.shard_m:(self.rank + 1) * self.shard_m]

    def quiesce(self, last_parity: Optional[int] = None, replay_stream=None) -> None:
        """Fence between gather() calls and anything else that touches the runner's buffers (reference
        all_gather_gemm.py:458-521): orders, on the CURRENT stream, everything the runner has in flight - the
        exchange of the last calls on the comm streams, the drain signals on the barrier stream and the GEMMs
        that read the two buffers - and, when ``replay_stream`` is given, whatever was enqueued on that
        stream.  ``last_parity`` re-points ``gathered_a()`` / ``next_local_slot()`` (0 or 1).  Never called
        under stream capture."""
        if self.on_gpu:
            assert not torch.cuda.is_current_stream_capturing(), "quiesce() is an eager-only boundary"
            cur = torch.cuda.current_stream(self.device)
            if replay_stream is not None:
                cur.wait_stream(replay_stream)
            for st in self.comm_streams:
                cur.wait_stream(st)
            cur.wait_stream(self.barrier_stream)
            for parity in (0, 1):
                if self._gemm_recorded[parity]:
                    cur.wait_event(self.ev_gemm_end[parity])
        if last_parity is not None:
            assert last_parity in (0, 1)
            self.last_parity = last_parity

    # ---- pieces of one gather ----
    def _rows(self, buf: torch.Tensor, shard: int) -> torch.Tensor:
        return buf[shard * self.shard_m:(shard + 1) * self.shard_m]

    @staticmethod
    def _chunk(t: torch.Tensor, c: int, chunks: int) -> torch.Tensor:
        """Rows of chunk ``c`` of a shard-sized tensor (its leading dim divides into ``chunks``)."""
        n = t.shape[0] // chunks
        return t[c * n:(c + 1) * n]

    def _publish(self, shard: int, epoch_slot: torch.Tensor, chunk: Optional[int] = None) -> None:
        # 4-byte device-to-device copies: handled by a copy engine, need no SM
        C = self.arrival_chunks
        for c in (range(C) if chunk is None else (chunk,)):
            self.flags[shard * C + c:shard * C + c + 1].copy_(epoch_slot, non_blocking=True)

    def _exchange(self, payloads, parity: int) -> None:
        """Ring steps for a list of (buffer, local shard tensor) payloads that travel together, chunk by chunk."""
        epoch_slot = self.epoch_dev[parity:parity + 1]
        C = self.arrival_chunks
        for _, send_to, recv_from in ring_schedule(self.rank, self.world_size):
            dst, src = dist.get_global_rank(self.group, send_to), dist.get_global_rank(self.group, recv_from)
            for c in range(C):
                ops = []
                for rows_of, shard in payloads:
                    ops.append(dist.P2POp(dist.isend, self._chunk(shard, c, C), dst, self.group))
                    ops.append(dist.P2POp(dist.irecv, self._chunk(rows_of(recv_from), c, C), src, self.group))
                for w in dist.batch_isend_irecv(ops):
                    w.wait()   # NCCL: orders the current (comm) stream after the transfer; the host does not block
                self._publish(recv_from, epoch_slot, c)

    # ---- copy-engine transport ----
    def _ce_setup(self, all_bufs) -> bool:
        """Exchange CUDA IPC handles of the flag array, the drained array and the gather buffers
        of both parities (``all_bufs[parity]`` = list of payload buffers) and map every peer's.
        Collective.  Returns False (on every rank) when some rank could not export or map: the
        caller then uses the NCCL transport (``transport="auto"``) or raises (``"ce"``)."""
        from .. import _lib
        local = [self.flags, self.drained, self.turn] + list(all_bufs[0]) + list(all_bufs[1])
        try:
            if os.environ.get("QK_DISABLE_IPC"):   # lets a test (or an operator) take the fall-back path
                raise RuntimeError("IPC disabled by QK_DISABLE_IPC")
            exported, err = [_lib.ipc_export(t.data_ptr()) for t in local], None
        except Exception as e:   # e.g. memory from a virtual-memory pool (expandable segments)
            exported, err = None, f"rank {self.rank}: {e}"
        gathered = [None] * self.world_size
        dist.all_gather_object(gathered, (exported, err), group=self.group)
        errors = [g[1] for g in gathered if g[1] is not None]
        n = len(all_bufs[0])
        self._opened = {}       # handle bytes -> mapped base (a handle is opened once per process)
        self._peer = []
        if not errors:
            try:
                for r in range(self.world_size):
                    if r == self.rank:
                        self._peer.append(None)
                        continue
                    ptrs = []
                    for handle, offset in gathered[r][0]:
                        if handle not in self._opened:
                            self._opened[handle] = _lib.ipc_open(handle)
                        ptrs.append(self._opened[handle] + offset)
                    self._peer.append({"flags": ptrs[0], "drained": ptrs[1], "turn": ptrs[2],
                                       "bufs": [ptrs[3:3 + n], ptrs[3 + n:3 + 2 * n]]})
                err = None
            except Exception as e:
                err = f"rank {self.rank}: {e}"
            second = [None] * self.world_size
            dist.all_gather_object(second, err, group=self.group)
            errors = [e for e in second if e is not None]
        if errors:
            for base in self._opened.values():
                _lib.lib.qk_ipc_close(base)
            self._opened, self._peer = {}, None
            self._ce_error = "; ".join(errors)
            dist.barrier(self.group)
            return False
        self._ce_build_ops(all_bufs)
        if self.transport == "pull":
            self._pull_build(all_bufs)
        dist.barrier(self.group)
        return True

    def _decide_transport(self, all_bufs) -> None:
        """Collective, once: map the peers' buffers, or settle for NCCL when that is not possible
        and the caller asked for "auto".  Runs in the constructors so that ``gemm_max_ctas`` is
        final before the first GEMM is configured."""
        if self.on_gpu and self.transport == "mc":
            if not getattr(self, "_pull_tables", None):
                self._build_local_ops(all_bufs)
                self._mc_build(all_bufs)
                dist.barrier(self.group)
            return
        if not (self.on_gpu and self.transport in ("ce", "pull") and self._peer is None):
            return
        if self._ce_setup(all_bufs):
            return
        if self._transport_requested in ("ce", "pull"):
            raise RuntimeError(f"{self._transport_requested} transport unavailable (peer buffers cannot be mapped): {self._ce_error}")
        import warnings
        warnings.warn(f"quack_b200: copy-engine all-gather transport unavailable ({self._ce_error}); using NCCL")
        self.transport = "nccl"

    def _ce_build_ops(self, all_bufs) -> None:
        """The per-call operation lists of both parities, built once: one foreign-function call then enqueues
        a whole step (the addresses never change; only the epoch values are patched per call)."""
        from .. import _lib
        S = len(self.comm_streams)
        self._build_local_ops(all_bufs)
        self._push_ops, self._push_waits, self._drain_ops = [], [], []
        self._push_srcs, self._push_turns = [], []
        for parity in (0, 1):
            slots = [self._rows(b, self.rank) if b.shape[0] == self.shard_m * self.world_size else b[self.rank]
                     for b in all_bufs[parity]]
            epoch_ptr = self.epoch_dev.data_ptr() + 4 * parity
            ops, waits, srcs, turns = [], [], [], []     # srcs: (op index, payload index, byte offset inside the shard)
            for step in range(1, self.world_size):
                # to rank-1 first, then rank-2 ...: every receiver gets the shard its GEMM reads next first
                dst = (self.rank - step) % self.world_size
                peer = self._peer[dst]
                C = self.arrival_chunks
                # which push stream carries what: by default a whole shard per stream, destinations rotating over
                # the streams; with chunk_streams the chunks of ONE shard are spread over the streams (several copy
                # engines work on the shard the receiver needs next; every chunk has its own flag, so no
                # cross-stream ordering is needed)
                by_chunk = self.chunk_streams and C > 1
                streams = ([self.comm_streams[c % S].cuda_stream for c in range(C)] if by_chunk
                           else [self.comm_streams[(step - 1) % S].cuda_stream] * C)
                # dst's GEMM of two calls ago (the last reader of this parity) has finished
                for stream in dict.fromkeys(streams):
                    waits.append(len(ops))
                    ops.append((_lib.OP_WAIT_GEQ32, 0, stream, self.drained.data_ptr() + 4 * dst, 0, 0))
                # receiver-exclusive ingress: dst takes its senders one at a time, dst + 1 first (this rank when
                # step == 1), each handing the turn to the next; without it two senders that have drifted apart
                # meet at one receiver and both copies run at half rate
                take_turn = self.exclusive_ingress and step > 1
                pass_turn = self.exclusive_ingress and step < self.world_size - 1
                if take_turn:
                    for stream in dict.fromkeys(streams):
                        turns.append(len(ops))
                        ops.append((_lib.OP_WAIT_GEQ32, 0, stream, self.turn.data_ptr() + 4 * dst, 0, 0))
                early = pass_turn and not by_chunk and 0.0 < self.turn_early < 1.0
                for c in range(C):
                    stream = streams[c]
                    for i, slot in enumerate(slots):
                        nbytes = slot.numel() * slot.element_size()
                        cb = nbytes // C
                        dst0 = peer["bufs"][parity][i] + self.rank * nbytes + c * cb
                        head = cb
                        if early and c == C - 1 and i == 0:
                            head = int(cb * (1.0 - self.turn_early)) // 256 * 256
                        if 0 < head < cb:
                            # codes of the last chunk: head, the turn to the next sender, tail
                            srcs.append((len(ops), i, c * cb))
                            ops.append((_lib.OP_COPY, 0, stream, dst0, slot.data_ptr() + c * cb, head))
                            nxt = self._peer[(self.rank + 1) % self.world_size]
                            ops.append((_lib.OP_COPY, 0, stream, nxt["turn"] + 4 * dst, epoch_ptr, 4))
                            srcs.append((len(ops), i, c * cb + head))
                            ops.append((_lib.OP_COPY, 0, stream, dst0 + head, slot.data_ptr() + c * cb + head, cb - head))
                            pass_turn = False
                        else:
                            srcs.append((len(ops), i, c * cb))
                            ops.append((_lib.OP_COPY, 0, stream, dst0, slot.data_ptr() + c * cb, cb))
                    ops.append((_lib.OP_COPY, 0, stream, peer["flags"] + 4 * (self.rank * C + c), epoch_ptr, 4))
                if pass_turn:
                    # (with the chunks of a shard on several streams the turn follows the stream of the last chunk:
                    # the next sender may then overlap the tail of the other streams' chunks)
                    nxt = self._peer[(self.rank + 1) % self.world_size]
                    ops.append((_lib.OP_COPY, 0, streams[C - 1], nxt["turn"] + 4 * dst, epoch_ptr, 4))
            arr = (_lib.StreamOp * len(ops))(*[_lib.StreamOp(*o) for o in ops])
            self._push_ops.append(arr)
            self._push_waits.append(waits)
            self._push_srcs.append(srcs)
            self._push_turns.append(turns)
            src = self.drain_src.data_ptr() + 4 * parity
            bstream = self.barrier_stream.cuda_stream
            dops = [(_lib.OP_WRITE32, 0, bstream, src, 0, 0)]
            for step in range(1, self.world_size):
                dst = (self.rank + step) % self.world_size
                dops.append((_lib.OP_COPY, 0, bstream, self._peer[dst]["drained"] + 4 * self.rank, src, 4))
            self._drain_ops.append((_lib.StreamOp * len(dops))(*[_lib.StreamOp(*o) for o in dops]))

    def _build_local_ops(self, all_bufs) -> None:
        """Per parity: the epoch write and the staging of the own shard (copies + the own flag) as stream operations."""
        from .. import _lib
        self._epoch_ops, self._local_ops, self._local_bytes = [], [], []
        for parity in (0, 1):
            slots = [self._rows(b, self.rank) if b.shape[0] == self.shard_m * self.world_size else b[self.rank]
                     for b in all_bufs[parity]]
            epoch_ptr = self.epoch_dev.data_ptr() + 4 * parity
            self._epoch_ops.append((_lib.StreamOp * 1)(_lib.StreamOp(_lib.OP_WRITE32, 0, 0, epoch_ptr, 0, 0)))
            lops = [(_lib.OP_COPY, 0, 0, slot.data_ptr(), 0, 0) for slot in slots]
            for c in range(self.arrival_chunks):
                lops.append((_lib.OP_COPY, 0, 0, self.flags.data_ptr() + 4 * (self.rank * self.arrival_chunks + c), epoch_ptr, 4))
            self._local_ops.append((_lib.StreamOp * len(lops))(*[_lib.StreamOp(*o) for o in lops]))
            self._local_bytes.append([slot.numel() * slot.element_size() for slot in slots])

    def _pull_build(self, all_bufs) -> None:
        """In-kernel transport: per buffer parity, the table of peer addresses the GEMM's transport warps read
        (``qk_ag_pull_args``, kept in device memory) and the stream waits that protect this rank's own rows: its
        staging copy of call e overwrites what the peers read during call e - 2, so it waits until every peer's
        ``drained`` word (written by that peer's kernel when its last CTA has read the shard) has reached e - 2."""
        from .. import _lib
        import ctypes as C
        self.arrive = torch.zeros(self.world_size, dtype=torch.int32, device=self.device)
        # per shard: (ns from the publishing CTA's start to the shard's flag, ns that CTA waited for the owner's flag)
        # of the last call; filled only when QK_AG_PULL_TIMES is set
        self.publish_ns = torch.zeros(self.world_size, 2, dtype=torch.int64, device=self.device)
        self._pull_tables, self._pull_waits = [], []
        for parity in (0, 1):
            t = _lib.AgPullArgs()
            t.num_payloads, t.rank = len(all_bufs[parity]), self.rank
            for i, b in enumerate(all_bufs[parity]):
                nbytes = b.numel() * b.element_size() // self.world_size
                assert nbytes % 16 == 0 and b.data_ptr() % 16 == 0 and b.is_contiguous(), "gather buffers: 16-byte granular shards"
                t.shard_bytes[i] = nbytes
                t.local_base[i] = b.data_ptr()
            for r in range(self.world_size):
                if r == self.rank:
                    continue
                for i in range(len(all_bufs[parity])):
                    t.peer_base[r][i] = self._peer[r]["bufs"][parity][i]
                t.peer_flags[r] = self._peer[r]["flags"]
                t.peer_drained[r] = self._peer[r]["drained"]
            t.arrive, t.flags_rw = self.arrive.data_ptr(), self.flags.data_ptr()
            t.publish_ns = self.publish_ns.data_ptr() if os.environ.get("QK_AG_PULL_TIMES") else None
            raw = torch.frombuffer(bytearray(C.string_at(C.addressof(t), C.sizeof(t))), dtype=torch.uint8)
            self._pull_tables.append(raw.to(self.device))
            waits = [(_lib.OP_WAIT_GEQ32, 0, 0, self.drained.data_ptr() + 4 * r, 0, 0)
                     for r in range(self.world_size) if r != self.rank]
            self._pull_waits.append((_lib.StreamOp * len(waits))(*[_lib.StreamOp(*o) for o in waits]))
        torch.cuda.synchronize(self.device)

    def _mc_build(self, all_bufs) -> None:
        """Multicast push: per parity, the table the GEMM's transport warps read (``qk_ag_pull_args`` with mode 1: the
        multicast addresses of the gather buffers, of the flag arrays and of the drained arrays) and the stream
        waits on every peer's ``drained`` word (written through the multicast mapping by the last CTA of that
        peer's GEMM of two calls ago)."""
        from .. import _lib
        import ctypes as C
        self.arrive = torch.zeros(self.world_size * self.arrival_chunks, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.publish_ns = torch.zeros(self.world_size, 2, dtype=torch.int64, device=self.device)
        self._pull_tables, self._pull_waits = [], []
        for parity in (0, 1):
            t = _lib.AgPullArgs()
            t.num_payloads, t.rank, t.mode, t.chunks = len(all_bufs[parity]), self.rank, 1, self.arrival_chunks
            for i, b in enumerate(all_bufs[parity]):
                nbytes = b.numel() * b.element_size() // self.world_size
                assert nbytes % 16 == 0 and b.data_ptr() % 16 == 0 and b.is_contiguous(), "gather buffers: 16-byte granular shards"
                assert nbytes % (16 * self.arrival_chunks) == 0, "chunks of a shard: 16-byte granular"
                t.shard_bytes[i] = nbytes
                t.local_base[i] = b.data_ptr()
                t.mc_base[i] = self._mc_addr(b)
            t.arrive, t.flags_rw, t.done = self.arrive.data_ptr(), self.flags.data_ptr(), self.done.data_ptr()
            t.mc_flags, t.mc_drained = self._mc_addr(self.flags), self._mc_addr(self.drained)
            t.publish_ns = self.publish_ns.data_ptr() if os.environ.get("QK_AG_PULL_TIMES") else None
            raw = torch.frombuffer(bytearray(C.string_at(C.addressof(t), C.sizeof(t))), dtype=torch.uint8)
            self._pull_tables.append(raw.to(self.device))
            waits = [(_lib.OP_WAIT_GEQ32, 0, 0, self.drained.data_ptr() + 4 * r, 0, 0)
                     for r in range(self.world_size) if r != self.rank]
            self._pull_waits.append((_lib.StreamOp * len(waits))(*[_lib.StreamOp(*o) for o in waits]))
        torch.cuda.synchronize(self.device)

    def _pull_wait_readers(self, parity: int, stream: int) -> None:
        """On the caller's stream, before the staging copy: every peer has read this rank's rows of two calls ago."""
        from .. import _lib
        ops = self._pull_waits[parity]
        want = (self.epoch - 2) & 0xFFFFFFFF
        for op in ops:
            op.value = want
            op.stream = stream
        _lib.check(_lib.lib.qk_stream_ops(ops, len(ops)), "qk_stream_ops")

    def _ce_epoch(self, parity: int, stream: int) -> None:
        """On the caller's stream: epoch_dev[parity] = epoch (the value every flag copy of this call reads)."""
        from .. import _lib
        ops = self._epoch_ops[parity]
        ops[0].value = self.epoch & 0xFFFFFFFF
        ops[0].stream = stream
        _lib.check(_lib.lib.qk_stream_ops(ops, 1), "qk_stream_ops")

    def _ce_local(self, payloads_local, parity: int, stream: int) -> None:
        """On the caller's stream: the local shard into its own rows of the gather buffers (skipped when the
        producer wrote it there), flags[rank] = epoch."""
        from .. import _lib
        ops = self._local_ops[parity]
        for op in ops:
            op.stream = stream
        for i, shard in enumerate(payloads_local):
            op = ops[i]
            src = shard.data_ptr()
            op.src = src
            op.bytes = 0 if src == op.dst else self._local_bytes[parity][i]
        _lib.check(_lib.lib.qk_stream_ops(ops, len(ops)), "qk_stream_ops")

    def _ce_push(self, parity: int, payloads_local) -> None:
        """The owner pushes its shard into every peer's buffer and publishes it there; enqueued on the push
        streams.  The copies read the caller's shard tensors directly, so they run alongside the local staging
        copy instead of after it."""
        from .. import _lib
        ops = self._push_ops[parity]
        want = (self.epoch - 2) & 0xFFFFFFFF
        for i in self._push_waits[parity]:
            ops[i].value = want
        for i in self._push_turns[parity]:
            ops[i].value = self.epoch & 0xFFFFFFFF
        bases = [sh.data_ptr() for sh in payloads_local]
        for idx, payload, off in self._push_srcs[parity]:
            ops[idx].src = bases[payload] + off
        _lib.check(_lib.lib.qk_stream_ops(ops, len(ops)), "qk_stream_ops")

    def _ce_check_progress(self, parity: int) -> None:
        """Host-side deadline of the copy-engine transport.  The pushes of the call two calls ago (same parity)
        were gated on stream-ordered waits for the peers' ``drained`` words, which have no timeout: if a peer
        stopped calling gather() (an exception, an uneven step count) those pushes never run and every later
        call queues behind them.  Before enqueueing this call's pushes, give the old ones
        ``QK_AG_HOST_TIMEOUT_S`` seconds (default 60) to finish and raise, naming the peers whose ``drained``
        word lags, instead of blocking forever at the next synchronize."""
        if not self._push_recorded[parity]:
            return
        from .. import _lib
        timeout_s = float(os.environ.get("QK_AG_HOST_TIMEOUT_S", "60"))
        lag = wait_events_or_report(
            [ev.query for ev in self.ev_push_end[parity]], timeout_s,
            lambda: self._lagging_peers(self.epoch - 2 - 2))
        if lag is not None:
            raise _lib.QuackB200Error(
                f"all-gather runner (rank {self.rank}): the pushes of epoch {self.epoch - 2} did not finish within "
                f"{timeout_s:.0f} s; peers whose drain signal lags: {lag} (every rank must call gather() the same number of times)")

    def _lagging_peers(self, want_epoch: int):
        """Ranks whose ``drained`` word is behind ``want_epoch`` (read on a fresh stream: the runner's own
        streams may be the ones that are stuck)."""
        side = torch.cuda.Stream(device=self.device)
        with torch.cuda.stream(side):
            host = self.drained.to("cpu", non_blocking=False)
        return [r for r in range(self.world_size) if r != self.rank and ((int(host[r]) - want_epoch) & 0xFFFFFFFF) >= 0x80000000]

    def _ce_signal_drained(self, parity: int) -> None:
        """After this rank's GEMM of the current call: tell every peer that the buffers of this
        parity may be overwritten.  Stream-ordered 32-bit write + 4-byte copies: no kernel."""
        from .. import _lib
        ops = self._drain_ops[parity]
        ops[0].value = self.epoch & 0xFFFFFFFF
        _lib.check(_lib.lib.qk_stream_ops(ops, len(ops)), "qk_stream_ops")

    def close(self) -> None:
        """Unmap the peers' buffers (copy-engine transport).  Collective: every rank calls it,
        after its last gather; the runner is unusable afterwards."""
        if self._arena is not None:
            # multicast transport: every rank stops using the mapping before anyone releases it
            torch.cuda.synchronize(self.device)
            dist.barrier(self.group)
            self.bufs, self.flags, self.drained = [], None, None
            if hasattr(self, "sf_bufs"):
                self.sf_bufs = []
            self._pull_tables, self._mc_hdl, self._arena = [], None, None
            dist.barrier(self.group)
            return
        if self._peer is None:
            return
        from .. import _lib
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for base in self._opened.values():
            _lib.check(_lib.lib.qk_ipc_close(base), "qk_ipc_close")
        self._opened, self._peer = {}, None
        dist.barrier(self.group)

    @contextmanager
    def _gather_payloads(self, payloads_local, bufs_for):
        """Common skeleton of gather(): ``payloads_local`` are the local shard tensors,
        ``bufs_for(parity)`` the matching gather buffers.  Yields (parity, ag_args)."""
        assert not self._in_gather, "gather() calls cannot nest or overlap"
        if self.on_gpu and torch.cuda.is_current_stream_capturing():
            raise NotImplementedError("gather() cannot be captured in a CUDA graph: the epoch that orders buffer reuse "
                                      "across ranks is a host counter (capture the GEMMs around it, or run it eagerly)")
        self._in_gather = True
        try:
            self._raise_on_reported_status()
            self.last_parity ^= 1
            parity = self.last_parity
            bufs = bufs_for(parity)
            self.epoch += 1
            epoch_slot = self.epoch_dev[parity:parity + 1]
            cur = torch.cuda.current_stream(self.device) if self.on_gpu else None
            if self.on_gpu and self._gemm_recorded[parity]:
                # the GEMM that last read this buffer (two calls ago) must be done before it is refilled
                cur.wait_event(self.ev_gemm_end[parity])
            if self.on_gpu and self.transport in ("ce", "pull") and self._peer is None:
                self._decide_transport([bufs_for(0), bufs_for(1)])   # (subclasses that did not decide in their constructor)
            ce = self.on_gpu and self.transport == "ce"
            pull = self.on_gpu and self.transport in ("pull", "mc")
            ce_fast = (ce or pull) and all(sh.is_contiguous() for sh in payloads_local)
            if pull:
                # (host-side deadline: the staging of two calls ago sat behind stream waits that have no timeout)
                self._ce_check_progress(parity)
                self._pull_wait_readers(parity, cur.cuda_stream)
            if ce_fast:
                # epoch write, staging copies and the local flag as lists of stream operations (no kernel); the
                # pushes only need the epoch and the caller's shard, so they are released before the staging copy
                self._ce_epoch(parity, cur.cuda_stream)
                self.ev_staged.record(cur)
                self._ce_local(payloads_local, parity, cur.cuda_stream)
            else:
                epoch_slot.fill_(self.epoch)
                # local shard: resident at once
                for buf, shard in zip(bufs, payloads_local):
                    slot = self._rows(buf, self.rank) if buf.shape[0] == self.shard_m * self.world_size else None
                    dst = slot if slot is not None else buf[self.rank]
                    if dst.data_ptr() != shard.data_ptr():
                        dst.copy_(shard, non_blocking=True)
                self._publish(self.rank, epoch_slot)
            if self.world_size == 1:
                yield parity, None
                return
            if pull:
                self.ev_push_end[parity][0].record(cur)
                self._push_recorded[parity] = True
            elif ce:
                self._ce_check_progress(parity)
                if not ce_fast:
                    self.ev_staged.record(cur)
                for st in self.comm_streams:
                    st.wait_event(self.ev_staged)
                # (shards that are not contiguous were staged above: push the staged copy)
                self._ce_push(parity, payloads_local if ce_fast else [
                    self._rows(b, self.rank) if b.shape[0] == self.shard_m * self.world_size else b[self.rank] for b in bufs])
                for st, ev in zip(self.comm_streams, self.ev_push_end[parity]):
                    ev.record(st)
                self._push_recorded[parity] = True
            elif self.on_gpu:
                self.ev_staged.record(cur)
                self.comm_stream.wait_event(self.ev_staged)
                with torch.cuda.stream(self.comm_stream):
                    self._run_exchange(bufs, payloads_local, parity)
                    self.ev_comm_end.record(self.comm_stream)
            else:
                self._run_exchange(bufs, payloads_local, parity)
            if self.on_gpu and self.transport == "mc":
                # every (rank, chunk) pair is a shard of its own to the GEMM: it takes them as their flags flip
                C = self.arrival_chunks
                yield parity, AllGatherArguments(self.flags, epoch_slot, self.world_size * C, self.rank * C, 1,
                                                 self._pull_tables[parity])
            else:
                yield parity, AllGatherArguments(self.flags, epoch_slot, self.world_size, self.rank, self.arrival_chunks,
                                                 self._pull_tables[parity] if pull else None)
            if self.on_gpu:
                self.ev_gemm_end[parity].record(cur)
                self._gemm_recorded[parity] = True
                # the next call's staging (on the current stream) must not overtake this exchange
                if self.transport == "ce":
                    for ev in self.ev_push_end[parity]:
                        cur.wait_event(ev)
                elif self.transport == "nccl":
                    cur.wait_event(self.ev_comm_end)
                if self.transport == "ce":
                    self.barrier_stream.wait_event(self.ev_gemm_end[parity])
                    self._ce_signal_drained(parity)
                self._snapshot_status(parity)
        finally:
            self._in_gather = False

    def _snapshot_status(self, parity: int) -> None:
        """After a call's GEMM: copy the device status word to pinned host memory (16 bytes, on the caller's stream)."""
        from .. import _ops
        st = _ops._status_bufs.get((self.device.type, self.device.index))
        if st is None:      # no GEMM has run on this device through the package yet
            return
        self._status_host[parity].copy_(st, non_blocking=True)
        self._status_ev[parity].record(torch.cuda.current_stream(self.device))
        self._status_pending[parity] = True

    def _raise_on_reported_status(self) -> None:
        """Looks at the snapshots of earlier calls that have landed (never blocks): a gate that timed out two calls
        ago surfaces here as an exception instead of silently wrong rows."""
        if not self.on_gpu:
            return
        from .. import _lib, _ops
        for parity in (0, 1):
            if self._status_pending[parity] and self._status_ev[parity].query():
                self._status_pending[parity] = False
                st = self._status_host[parity].tolist()
                if st[0] != 0:
                    if getattr(self, "arrive", None) is not None:
                        self.arrive.zero_()     # a transport warp that gave up leaves its shard's counter short
                    if getattr(self, "done", None) is not None:
                        self.done.zero_()
                    _ops.check_status(self.device)      # clears the device word and the split-K scratch, raises
                    raise _lib.QuackB200Error(f"all-gather GEMM reported status {st}")

    def _run_exchange(self, bufs, payloads_local, parity):
        payloads = []
        for buf, shard in zip(bufs, payloads_local):
            if buf.shape[0] == self.shard_m * self.world_size:
                payloads.append(((lambda s, b=buf: self._rows(b, s)), shard))
            else:
                payloads.append(((lambda s, b=buf: b[s]), shard))
        self._exchange(payloads, parity)

    @contextmanager
    def gather(self, a_shard: torch.Tensor):
        """``with runner.gather(a_shard) as (a_full, ag_args): gemm(..., ag_args=ag_args)``.
        a_full is not complete on entry: the GEMM consumes shards as their flags flip."""
        assert a_shard.shape == (self.shard_m, self.k) and a_shard.dtype == self.dtype
        assert a_shard.stride(-1) == 1, "A shard must be K-major (row-contiguous)"
        with self._gather_payloads([a_shard], lambda p: [self.bufs[p]]) as (parity, ag_args):
            yield self.bufs[parity], ag_args


class BlockScaledAllGatherRunner(AllGatherRunner):
    """Gathers ``BlockScaledOperand`` shards: codes plus the blocked scale factors, which
    concatenate byte-wise across ranks because scale blocks run along K and ``shard_m`` is a
    multiple of 128 (reference :853-864).  One flag publishes both payloads."""

    def __init__(self, shard_m: int, k: int, a_format="mxfp8_e4m3", group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None, arrival_chunks: int = 1, capture_lockstep: bool = False,
                 comm_sms: int = 16, transport: str = "auto", push_streams: Optional[int] = None, chunk_streams: bool = False,
                 exclusive_ingress: Optional[bool] = None, turn_early: Optional[float] = None):
        fmt = _coerce_format(a_format)
        assert shard_m % (128 * arrival_chunks) == 0, (
            f"shard_m ({shard_m}) must be a multiple of 128 x arrival_chunks ({arrival_chunks}): whole scale atoms per chunk")
        assert k % (4 * fmt.sf_vec_size) == 0, f"K ({k}) must be a multiple of {4 * fmt.sf_vec_size} for {fmt.name}"
        self.a_format = fmt
        self.logical_k = k
        world = dist.get_world_size(group if group is not None else dist.group.WORLD)
        sf_bytes = world * (shard_m // 128) * (k // (4 * fmt.sf_vec_size)) * 512
        super().__init__(shard_m, fmt.storage_k(k), fmt.qdata_dtype if fmt.qdata_dtype != torch.float4_e2m1fn_x2 else torch.uint8,
                         group, device, arrival_chunks, capture_lockstep, comm_sms, transport, push_streams, chunk_streams,
                         exclusive_ingress, _arena_reserve=2 * (sf_bytes + 256), turn_early=turn_early)
        self.rm_shard = shard_m // 128
        self.rk = k // (4 * fmt.sf_vec_size)
        self.sf_bufs = [self._new_buffer((self.world_size, self.rm_shard, self.rk, 32, 4, 4), torch.uint8) for _ in range(2)]
        self._decide_transport([[self.bufs[p], self.sf_bufs[p]] for p in (0, 1)])

    @contextmanager
    def gather(self, shard: BlockScaledOperand):
        if not isinstance(shard, BlockScaledOperand):
            raise TypeError("BlockScaledAllGatherRunner.gather takes a BlockScaledOperand shard")
        if shard.format != self.a_format:
            raise ValueError(f"shard format {shard.format.name} != runner format {self.a_format.name}")
        if shard.quant_dim != -1:
            raise ValueError("the gathered A must be quantized along its last dim (quant_dim=-1)")
        if shard.per_tensor_scale is not None:
            raise ValueError("per_tensor_scale operands cannot be all-gathered: every rank would carry its own "
                             "tensor scale and the GEMM folds a single alpha")
        q = shard.qdata.view(self.dtype)
        assert q.shape == (self.shard_m, self.k), f"shard codes {tuple(q.shape)} != {(self.shard_m, self.k)}"
        assert q.stride(-1) == 1
        sf = shard.scale.view(torch.uint8)
        assert tuple(sf.shape) == (self.rm_shard, self.rk, 32, 4, 4) and sf.is_contiguous(), (
            f"shard scales {tuple(sf.shape)} != {(self.rm_shard, self.rk, 32, 4, 4)} contiguous")
        with self._gather_payloads([q, sf], lambda p: [self.bufs[p], self.sf_bufs[p]]) as (parity, ag_args):
            full = BlockScaledOperand.from_parts(
                self.bufs[parity].view(self.a_format.qdata_dtype),
                self.sf_bufs[parity].view(self.world_size * self.rm_shard, self.rk, 32, 4, 4).view(self.a_format.scale_dtype),
                self.a_format, orig_dtype=shard.orig_dtype)
            yield full, ag_args

"""Single-GPU checks of the transport helpers of the C ABI (the multi-GPU behaviour is covered by
tests/test_distributed_gpu.py): stream-ordered copies, 32-bit writes and satisfied waits, and the
IPC export of tensors that share an allocation."""

import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_stream_ops_copy_write_wait():
    from quack_b200 import _lib
    dev = torch.device("cuda")
    src = torch.arange(4096, dtype=torch.int32, device=dev)
    dst = torch.zeros_like(src)
    word = torch.zeros(2, dtype=torch.int32, device=dev)
    side = torch.cuda.Stream()
    s = side.cuda_stream
    ops = (_lib.StreamOp * 4)(
        _lib.StreamOp(_lib.OP_WRITE32, 41, s, word.data_ptr(), None, 0),
        _lib.StreamOp(_lib.OP_WAIT_GEQ32, 40, s, word.data_ptr(), None, 0),          # 41 >= 40: passes
        _lib.StreamOp(_lib.OP_COPY, 0, s, dst.data_ptr(), src.data_ptr(), src.numel() * 4),
        _lib.StreamOp(_lib.OP_COPY, 0, s, word.data_ptr() + 4, word.data_ptr(), 4))  # "flag" published after the data
    side.wait_stream(torch.cuda.current_stream())
    _lib.check(_lib.lib.qk_stream_ops(ops, 4), "qk_stream_ops")
    side.synchronize()
    assert torch.equal(dst, src) and word.tolist() == [41, 41]
    # modular comparison: a value "behind" by wrap-around still counts as reached
    _lib.check(_lib.lib.qk_stream_write32(s, word.data_ptr(), 5), "write32")
    _lib.check(_lib.lib.qk_stream_wait_geq32(s, word.data_ptr(), 0xFFFFFFF0), "wait")   # 5 - (-16) = 21 >= 0
    side.synchronize()
    assert word[0].item() == 5


def test_ipc_export_of_tensors_in_one_allocation():
    from quack_b200 import _lib
    big = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    a, b = big[1024:], big[65536:]
    ha, oa = _lib.ipc_export(a.data_ptr())
    hb, ob = _lib.ipc_export(b.data_ptr())
    assert ha == hb and len(ha) == _lib.IPC_HANDLE_BYTES      # same allocation, same handle
    assert ob - oa == 65536 - 1024
    with pytest.raises(_lib.QuackB200Error):
        _lib.ipc_export(ctypes.addressof(ctypes.c_int(0)))   # a host address is not a device allocation


def test_runner_surfaces_a_reported_status_without_blocking():
    """The runner copies the GEMMs' device status word to pinned memory after every call and the next calls
    look at it (a query, never a wait): a status left by a kernel that gave up a bounded wait becomes an
    exception, and the device word is cleared.  The status is written by hand here (no kernel is made to wait)."""
    import socket
    import torch.distributed as dist
    from quack_b200 import _lib, _ops
    from quack_b200.distributed import BlockScaledAllGatherRunner
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        dev = torch.device("cuda", 0)
        runner = BlockScaledAllGatherRunner(128, 256, "mxfp8_e4m3", device=dev)
        st = _ops.status_buffer(dev)
        runner._snapshot_status(0)
        torch.cuda.synchronize()
        runner._raise_on_reported_status()                 # clean status: nothing happens
        st.copy_(torch.tensor([5, 3, 0, 7], dtype=torch.int32))
        runner._snapshot_status(1)
        torch.cuda.synchronize()
        with pytest.raises(_lib.QuackB200Error, match="all-gather arrival gate"):
            runner._raise_on_reported_status()
        assert st.tolist() == [0, 0, 0, 0]
        runner._raise_on_reported_status()                 # reported once
    finally:
        dist.destroy_process_group()

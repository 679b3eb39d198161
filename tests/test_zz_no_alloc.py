"""qk_gemm_blockscaled_noalloc, the GEMM entry point for callers that cannot allocate device
memory (a serving process whose device-memory plan is frozen, a language binding without a CUDA
allocator): its scratch - status block and cycle counters - is a static device array inside the
library instead of buffers the caller hands over.

Called through the C ABI twice in a row (the array keeps the previous call's contents, so the
second call proves the clearing works) and compared with the regular entry point on the same
operands.  Collected last, so a failure here cannot hide the other tests' results."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import blockscaled_oracle as orc
from tests.helpers import dev, make_operand_pair, rel_err

pytestmark = pytest.mark.gpu


def _args(fmt_id, ops, m, n, k, D, bias, alpha):
    from quack_b200 import _lib
    A, B, SFA, SFB = dev(ops["ac"]), dev(ops["bc"]), dev(ops["asf_b"]), dev(ops["bsf_b"])
    a = _lib.GemmArgs()
    a.format, a.m, a.n, a.k = fmt_id, m, n, k
    a.a, a.lda, a.b, a.ldb = A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0)
    a.sfa, a.sfa_stride_rm, a.sfa_stride_rk = SFA.data_ptr(), SFA.stride(0), SFA.stride(1)
    a.sfb, a.sfb_stride_rm, a.sfb_stride_rk = SFB.data_ptr(), SFB.stride(0), SFB.stride(1)
    a.d, a.ldd, a.d_dtype = D.data_ptr(), D.stride(0), _lib.DT_BF16
    a.bias, a.bias_dtype = bias.data_ptr(), _lib.DT_F32
    a.alpha = alpha
    a.stream = torch.cuda.current_stream().cuda_stream
    return a, (A, B, SFA, SFB)   # keep the operands alive


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
def test_noalloc_entry_matches_regular_entry(fmt):
    from quack_b200 import _lib, _ops
    m, n, k = 640, 768, 1024
    ops = make_operand_pair(fmt, m, n, k, seed=31)
    bias = orc.make_bias(n).cuda()
    alpha = 1.0 if ops["pa"] is None else ops["pa"] * ops["pb"]
    fmt_id = _ops.format_id(fmt)

    # regular entry point: the caller brings the status buffer
    D_ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    a, keep = _args(fmt_id, ops, m, n, k, D_ref, bias, alpha)
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    a.status = st.data_ptr()
    _lib.check(_lib.lib.qk_gemm_blockscaled(C.byref(a)), "qk_gemm_blockscaled")
    torch.cuda.synchronize()
    assert st.tolist()[0] == 0
    oracle = orc.gemm_blockscaled_ref(ops["adq"], ops["bdq"], alpha=alpha, bias=bias.cpu())
    assert rel_err(D_ref.float().cpu().numpy(), oracle) < 5e-3

    # no-alloc entry point, two calls in a row; outputs and copies are the caller's own buffers
    status_out = torch.full((4,), 7, dtype=torch.int32, device="cuda")
    prof_out = torch.full((16 * _lib.NOALLOC_MAX_CTAS,), -1, dtype=torch.int64, device="cuda")
    for call in range(2):
        D = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        b, keep2 = _args(fmt_id, ops, m, n, k, D, bias, alpha)
        rc = _lib.lib.qk_gemm_blockscaled_noalloc(C.byref(b), C.c_void_p(status_out.data_ptr()),
                                                  C.c_void_p(prof_out.data_ptr()) if call == 1 else None)
        _lib.check(rc, "qk_gemm_blockscaled_noalloc")
        torch.cuda.synchronize()
        assert status_out.tolist() == [0, 0, 0, 0], f"call {call}: status {status_out.tolist()}"
        # same kernel, same operands: identical bits; and within the GEMM tolerance of the oracle
        assert torch.equal(D, D_ref), f"call {call}: output differs from qk_gemm_blockscaled"
        assert rel_err(D.float().cpu().numpy(), oracle) < 5e-3
    counters = prof_out.view(_lib.NOALLOC_MAX_CTAS, 16).cpu().numpy()
    assert (counters >= 0).all() and counters[:, 0].max() > 0       # cleared, then filled by the CTAs that ran


def test_noalloc_entry_rejects_what_it_cannot_serve():
    from quack_b200 import _lib, _ops
    m, n, k = 128, 128, 128
    ops = make_operand_pair("mxfp8_e4m3", m, n, k, seed=32)
    bias = orc.make_bias(n).cuda()
    D = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    a, keep = _args(_ops.format_id("mxfp8_e4m3"), ops, m, n, k, D, bias, 1.0)
    a.max_ctas = _lib.NOALLOC_MAX_CTAS + 1                 # beyond the static scratch
    assert _lib.lib.qk_gemm_blockscaled_noalloc(C.byref(a), None, None) == -4
    assert b"static scratch covers" in _lib.lib.qk_last_error()
    a.max_ctas = 0
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    a.status = st.data_ptr()                               # the library owns the status block here
    assert _lib.lib.qk_gemm_blockscaled_noalloc(C.byref(a), None, None) == -1
    assert b"NULL" in _lib.lib.qk_last_error()
    assert _lib.lib.qk_gemm_blockscaled_noalloc(None, None, None) == -1

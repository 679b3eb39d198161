"""torch.library custom ops, torch.compile and CUDA-graph capture of the block-scaled GEMMs (the reference's
quack::gemm_out / gemm_quant_out / gemm_add_out / gemm_act_out ops, quack/gemm_interface.py:1311-1449, :3052-3068):
compiled results are bit-equal to eager ones, and a captured loop of launches replays to the same bytes."""

import pytest
import torch

from oracle import blockscaled_oracle as orc

pytestmark = pytest.mark.gpu


def _operands(fmt, m, n, k):
    from quack_b200.blockscaled import BlockScaledOperand, nvfp4_per_tensor_scale
    a, w = orc.make_activation(m, k, 0).cuda(), orc.make_weight(n, k, 1).cuda()
    kw_a = dict(per_tensor_scale=nvfp4_per_tensor_scale(a.abs().amax())) if fmt == "nvfp4" else {}
    kw_w = dict(per_tensor_scale=nvfp4_per_tensor_scale(w.abs().amax())) if fmt == "nvfp4" else {}
    return BlockScaledOperand.quantize(a, fmt, **kw_a), BlockScaledOperand.quantize(w, fmt, **kw_w)


@pytest.mark.parametrize("fmt", ["mxfp8_e4m3", "nvfp4"])
def test_compiled_gemm_equals_eager(fmt):
    """Configuration 0 (M = 2048, N = K = 4096) through torch.compile(fullgraph=True): the container is taken
    apart before the op boundary, the op fills a tensor allocated in the graph."""
    from quack_b200 import _torch_ops
    from quack_b200.gemm_interface import gemm, gemm_act, gemm_add
    A, W = _operands(fmt, 2048, 4096, 4096)
    bias = orc.make_bias(4096).cuda()
    assert hasattr(getattr(torch.ops, _torch_ops.NAMESPACE), "gemm_out")

    def f(A, W, bias):
        return gemm(A, W.mT, bias=bias) * 1.0

    eager = f(A, W, bias)
    compiled = torch.compile(f, fullgraph=True)(A, W, bias)
    assert torch.equal(eager, compiled)

    C = torch.randn(2048, 4096, device="cuda", dtype=torch.bfloat16)

    def g(A, W, C, bias):
        y = gemm_add(A, W.mT, C, bias=bias, beta=0.5)
        pre, post = gemm_act(A, W.mT, bias=bias, activation="swiglu", store_preact=False)
        return y, post

    e1, e2 = g(A, W, C, bias)
    c1, c2 = torch.compile(g, fullgraph=True)(A, W, C, bias)
    assert torch.equal(e1, c1) and torch.equal(e2, c2)


def test_compiled_quantised_outputs_equal_eager():
    from quack_b200.gemm_interface import gemm, gemm_act_quant
    A, W = _operands("nvfp4", 512, 1024, 1024)
    pts = torch.tensor([2e-3], device="cuda")

    def f(A, W):
        d = gemm(A, W.mT, out_dtype="mxfp8_e4m3")
        h = gemm_act_quant(A, W.mT, activation="swiglu", postact_format="nvfp4", postact_per_tensor_scale=pts)
        return d.qdata.view(torch.uint8), d.scale.view(torch.uint8), h.qdata.view(torch.uint8), h.scale.view(torch.uint8)

    eager = f(A, W)
    compiled = torch.compile(f)(A, W)
    for e, c in zip(eager, compiled):
        assert torch.equal(e, c)


def test_cuda_graph_capture_and_replay():
    """A loop of GEMM launches (large and few-row shapes, fused epilogue) captured once and replayed: same bytes
    as the eager launches, also after the inputs change in place."""
    from quack_b200 import _ops
    from quack_b200.blockscaled import BlockScaledOperand
    from quack_b200.gemm_interface import gemm, gemm_act
    A, W = _operands("mxfp8_e4m3", 1024, 2048, 4096)
    A16 = BlockScaledOperand.quantize(orc.make_activation(16, 4096, 5).cuda(), "mxfp8_e4m3")
    bias = orc.make_bias(2048).cuda()
    out = torch.empty(1024, 2048, dtype=torch.bfloat16, device="cuda")
    out16 = torch.empty(16, 2048, dtype=torch.bfloat16, device="cuda")
    post = torch.empty(1024, 1024, dtype=torch.bfloat16, device="cuda")

    def step():
        gemm(A, W.mT, out=out, bias=bias)
        gemm(A16, W.mT, out=out16)
        gemm_act(A, W.mT, bias=bias, activation="swiglu", store_preact=False, postact_out=post)

    step()
    torch.cuda.synchronize()
    want = (out.clone(), out16.clone(), post.clone())
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        step()                       # first use of this stream: its scratch is allocated outside the capture
        side.synchronize()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(3):
                step()
        for t in (out, out16, post):
            t.zero_()
        graph.replay()
        side.synchronize()
    for got, ref in zip((out, out16, post), want):
        assert torch.equal(got, ref)
    # new activation bytes in the same storage: the replay computes with them
    A2 = BlockScaledOperand.quantize(orc.make_activation(1024, 4096, 9).cuda(), "mxfp8_e4m3")
    ref2 = gemm(A2, W.mT, bias=bias)
    A.qdata.copy_(A2.qdata)
    A.scale.view(torch.uint8).copy_(A2.scale.view(torch.uint8))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref2)
    _ops.check_status(torch.device("cuda", 0))

"""GPU tests of ``torch.ops.fav4.bshd_forward``: bit-identical to the C ABI
call it wraps, torch.library.opcheck, use inside a torch.compile graph and in
a captured CUDA graph, and no silent gradient."""
import math

import pytest
import torch

from grad_checks import dq_close

import fav4_bshd as F
from fav4_bshd import ops

pytestmark = pytest.mark.gpu


def _inputs(b, h, sq, sk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(s, generator=gen, device="cuda", dtype=torch.bfloat16)
            for s in ((b, sq, h, 128), (b, sk, h, 128), (b, sk, h, 128))]


@pytest.mark.parametrize("b,h,sq,sk", [(2, 4, 300, 517), (1, 8, 1024, 1024), (3, 2, 77, 77)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("config", [0, 1, 3])
def test_op_matches_c_abi(runner, b, h, sq, sk, causal, config):
    q, k, v = _inputs(b, h, sq, sk, seed=b + sq)
    o, lse = torch.ops.fav4.bshd_forward(q, k, v, causal, config, -1.0, True)
    want_o = torch.empty_like(q)
    want_l = torch.empty((b, h, sq), device="cuda")
    runner.call(q, k, v, want_o, want_l, causal, config, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert torch.equal(o, want_o) and torch.equal(lse, want_l)
    o2 = ops.attention(q, k, v, causal=causal, config=config, scale=0.07)
    runner.call(q, k, v, want_o, None, causal, config, 0.07)
    torch.cuda.synchronize()
    assert torch.equal(o2, want_o)


def test_opcheck():
    q, k, v = _inputs(2, 3, 200, 300, seed=5)
    for causal, lse in ((False, True), (True, False)):
        torch.library.opcheck(torch.ops.fav4.bshd_forward.default, (q, k, v, causal, 0, -1.0, lse))


def test_inside_torch_compile_graph():
    q, k, v = _inputs(2, 4, 256, 256, seed=6)

    # elementwise work around the operator only: a reduction's order may
    # differ between Inductor and eager, which says nothing about the operator
    def block(q, k, v):
        o = ops.attention(q * 0.5, k, v, causal=True)
        return o.float() * 2.0 + 1.0

    want = block(q, k, v)
    got = torch.compile(block, fullgraph=True)(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_cuda_graph_capture_replays():
    q, k, v = _inputs(2, 4, 384, 384, seed=7)
    ops.attention(q, k, v)  # first call on the device happens outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ops.attention(q, k, v, causal=True)
    want = ops.attention(q, k, v, causal=True)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)


def test_gradients_through_the_operator(runner):
    q, k, v = _inputs(2, 4, 300, 300, seed=8)
    do = torch.randn_like(q)
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    o = ops.attention(qg, kg, vg, causal=True)
    o.backward(do)
    # the same C ABI calls by hand
    lse = torch.empty((2, 4, 300), device="cuda")
    o2 = torch.empty_like(q)
    runner.call(q, k, v, o2, lse, True, 0, 1 / math.sqrt(128))
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    runner.backward(q, k, v, o2, do, lse, dq, dk, dv, True, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert torch.equal(o.detach(), o2)
    assert torch.equal(kg.grad, dk) and torch.equal(vg.grad, dv)
    # dQ is summed by FP32 atomic reductions: the order, and so the last bit, may differ between runs
    assert dq_close(qg.grad, dq)


def test_gqa_gradients_through_the_operator(runner):
    gen = torch.Generator(device="cuda").manual_seed(17)
    q = torch.randn((2, 300, 8, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn((2, 400, 2, 128), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    do = torch.randn_like(q)
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    o = ops.attention(qg, kg, vg, causal=True)
    o.backward(do)
    lse = torch.empty((2, 8, 300), device="cuda")
    o2 = torch.empty_like(q)
    runner.call_gqa(q, k, v, o2, lse, True, 0, 1 / math.sqrt(128))
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    runner.backward(q, k, v, o2, do, lse, dq, dk, dv, True, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert torch.equal(o.detach(), o2)
    assert torch.equal(kg.grad, dk) and torch.equal(vg.grad, dv)
    assert dq_close(qg.grad, dq)


def test_gradient_limits_raise():
    q, k, v = _inputs(1, 2, 128, 128, seed=10)
    qg = q.clone().requires_grad_(True)
    o, lse = torch.ops.fav4.bshd_forward(qg, k, v, False, 0, -1.0, False)  # no LSE kept
    with pytest.raises(RuntimeError):
        o.float().sum().backward()
    qg = q.clone().requires_grad_(True)
    o, lse = ops.attention(qg, k, v, return_lse=True)
    with pytest.raises(NotImplementedError):
        (o.float().sum() + lse.sum()).backward()


def test_varlen_op_and_gradients_match_c_abi(runner):
    lens_q, lens_k, h, hk = (129, 0, 700, 64), (200, 50, 900, 1), 8, 2
    gen = torch.Generator(device="cuda").manual_seed(31)
    q = torch.randn((sum(lens_q), h, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn((sum(lens_k), hk, 128), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    do = torch.randn_like(q)
    cu = lambda lens: torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int32)  # noqa
    cu_q, cu_k = cu(lens_q), cu(lens_k)
    for causal in (False, True):
        qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
        o, lse = ops.varlen_attention(qg, kg, vg, cu_q, cu_k, max(lens_q), max(lens_k), causal, return_lse=True)
        o.backward(do)
        want_o, want_l = torch.empty_like(q), torch.empty((h, q.shape[0]), device="cuda")
        runner.call_varlen(q, k, v, want_o, want_l, cu_q, cu_k, max(lens_q), causal)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        runner.backward_varlen(q, k, v, want_o, do, want_l, dq, dk, dv, cu_q, cu_k, max(lens_q), max(lens_k), causal)
        torch.cuda.synchronize()
        assert torch.equal(o.detach(), want_o) and torch.equal(lse.detach(), want_l)
        assert torch.equal(kg.grad, dk) and torch.equal(vg.grad, dv)
        assert dq_close(qg.grad, dq)


def test_varlen_opcheck():
    gen = torch.Generator(device="cuda").manual_seed(32)
    q = torch.randn((300, 4, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn((260, 4, 128), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    cu_q = torch.tensor([0, 100, 300], device="cuda", dtype=torch.int32)
    cu_k = torch.tensor([0, 60, 260], device="cuda", dtype=torch.int32)
    torch.library.opcheck(torch.ops.fav4.varlen_forward.default, (q, k, v, cu_q, cu_k, 200, 200, True, -1.0),
                          test_utils=("test_schema", "test_faketensor", "test_autograd_registration"))

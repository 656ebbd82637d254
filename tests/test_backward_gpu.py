"""GPU tests of the backward pass (fav4_bshd_backward, the fused kernel with
FP32 dQ reductions, and fav4_bshd_backward_deterministic): dQ, dK, dV against
torch autograd in FP32 on the GPU (same BF16 inputs) and against the FP64
oracle on small cases, dense and top-left causal, ragged shapes, Sq != Sk;
run-to-run reproducibility of the deterministic path; dK and dV of both paths
bit-identical; keys no query row sees get zero gradients; grouped-query
gradients (fav4_bshd_backward_gqa) against torch autograd on repeated K/V."""
import math

import numpy as np
import pytest
import torch

from oracle import ref_attention as R

pytestmark = pytest.mark.gpu


def _inputs(b, h, sq, sk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(s, generator=gen, device="cuda", dtype=torch.bfloat16)
               for s in ((b, sq, h, 128), (b, sk, h, 128), (b, sk, h, 128)))
    do = torch.randn((b, sq, h, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    return q, k, v, do


def _run(runner, q, k, v, do, causal, scale, deterministic=False):
    b, sq, h, _ = q.shape
    o = torch.empty_like(q)
    lse = torch.empty((b, h, sq), device="cuda")
    if k.shape[2] == h:
        runner.call(q, k, v, o, lse, causal, 0, scale)
    else:
        runner.call_gqa(q, k, v, o, lse, causal, 0, scale)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    runner.backward(q, k, v, o, do, lse, dq, dk, dv, causal, scale, deterministic=deterministic)
    torch.cuda.synchronize()
    return dq, dk, dv


def _torch_grads(q, k, v, do, causal, scale):
    tq, tk, tv = (x.float().transpose(1, 2).detach().requires_grad_(True) for x in (q, k, v))
    s = tq @ tk.transpose(-1, -2) * scale
    if causal:
        s = s.masked_fill(torch.ones(q.shape[1], k.shape[1], dtype=torch.bool, device="cuda").triu(1), float("-inf"))
    o = torch.softmax(s, -1) @ tv
    o.backward(do.float().transpose(1, 2))
    return [x.grad.transpose(1, 2) for x in (tq, tk, tv)]


def _check(got, want, name):
    err = (got.float() - want).abs()
    scale = want.abs()
    assert torch.isfinite(got.float()).all(), name
    # BF16 outputs: relative to the gradient's own magnitude
    assert err.max().item() <= 0.02 * scale.max().item() + 1e-3, (name, err.max().item(), scale.max().item())
    assert err.mean().item() <= 0.01 * scale.mean().item() + 1e-5, (name, err.mean().item(), scale.mean().item())


@pytest.mark.parametrize("b,h,sq,sk", [(1, 2, 128, 128), (2, 3, 300, 517), (1, 2, 1000, 1537), (2, 2, 1537, 1000),
                                       (1, 4, 64, 2000), (2, 2, 257, 1), (1, 8, 2048, 2048)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("deterministic", [False, True])
def test_backward_matches_torch_autograd(runner, b, h, sq, sk, causal, deterministic):
    q, k, v, do = _inputs(b, h, sq, sk, seed=sq + sk)
    scale = 1 / math.sqrt(128)
    got = _run(runner, q, k, v, do, causal, scale, deterministic)
    want = _torch_grads(q, k, v, do, causal, scale)
    for g, w, n in zip(got, want, ("dq", "dk", "dv")):
        _check(g, w, n)
    if causal and sq < sk:
        # keys at or past sq are seen by no query row
        assert torch.count_nonzero(got[1][:, sq:]) == 0 and torch.count_nonzero(got[2][:, sq:]) == 0
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("deterministic", [False, True])
def test_backward_against_fp64_oracle(runner, causal, deterministic):
    q, k, v, do = _inputs(1, 2, 200, 333, seed=5)
    scale = 0.09
    got = _run(runner, q, k, v, do, causal, scale, deterministic)
    dq, dk, dv, _, _ = R.reference_backward(*(x.float().cpu().numpy() for x in (q, k, v, do)), causal, scale)
    for g, w, n in zip(got, (dq, dk, dv), ("dq", "dk", "dv")):
        _check(g, torch.tensor(w, device="cuda", dtype=torch.float32), n)


def test_backward_deterministic_is_reproducible(runner):
    q, k, v, do = _inputs(2, 4, 700, 700, seed=9)
    a = _run(runner, q, k, v, do, True, 0.08, deterministic=True)
    b = _run(runner, q, k, v, do, True, 0.08, deterministic=True)
    assert all(torch.equal(x, y) for x, y in zip(a, b))


@pytest.mark.parametrize("causal", [False, True])
def test_fused_dk_dv_match_deterministic_bitwise(runner, causal):
    # same elementwise arithmetic and MMA order for dK, dV; only dQ's summation order differs
    q, k, v, do = _inputs(2, 3, 700, 900, seed=11)
    fused = _run(runner, q, k, v, do, causal, 0.08)
    det = _run(runner, q, k, v, do, causal, 0.08, deterministic=True)
    assert torch.equal(fused[1], det[1]) and torch.equal(fused[2], det[2])
    err = (fused[0].float() - det[0].float()).abs().max().item()
    assert err <= 0.01 * det[0].float().abs().max().item() + 1e-3, err
    assert runner.pipeline_status() == 0


def _gqa_inputs(b, h, hk, sq, sk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((b, sq, h, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn((b, sk, hk, 128), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    do = torch.randn((b, sq, h, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    return q, k, v, do


def _torch_gqa_grads(q, k, v, do, causal, scale):
    # repeat K/V over each group, differentiate, sum the repeated heads' gradients back
    g = q.shape[2] // k.shape[2]
    kr, vr = (x.float().detach().requires_grad_(True) for x in (k, v))
    tq = q.float().transpose(1, 2).detach().requires_grad_(True)
    tk = kr.repeat_interleave(g, dim=2).transpose(1, 2)
    tv = vr.repeat_interleave(g, dim=2).transpose(1, 2)
    s = tq @ tk.transpose(-1, -2) * scale
    if causal:
        s = s.masked_fill(torch.ones(q.shape[1], k.shape[1], dtype=torch.bool, device="cuda").triu(1), float("-inf"))
    o = torch.softmax(s, -1) @ tv
    o.backward(do.float().transpose(1, 2))
    return tq.grad.transpose(1, 2), kr.grad, vr.grad


@pytest.mark.parametrize("b,h,hk,sq,sk", [(2, 8, 2, 300, 517), (1, 4, 1, 1000, 700), (1, 6, 3, 129, 1)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("deterministic", [False, True])
def test_gqa_backward_matches_torch_autograd(runner, b, h, hk, sq, sk, causal, deterministic):
    q, k, v, do = _gqa_inputs(b, h, hk, sq, sk, seed=h * 7 + sq)
    scale = 1 / math.sqrt(128)
    got = _run(runner, q, k, v, do, causal, scale, deterministic)
    want = _torch_gqa_grads(q, k, v, do, causal, scale)
    for g, w, n in zip(got, want, ("dq", "dk", "dv")):
        _check(g, w, n)
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("causal", [False, True])
def test_gqa_fused_dk_dv_match_deterministic_bitwise(runner, causal):
    q, k, v, do = _gqa_inputs(2, 8, 2, 700, 900, seed=13)
    fused = _run(runner, q, k, v, do, causal, 0.08)
    det = _run(runner, q, k, v, do, causal, 0.08, deterministic=True)
    assert torch.equal(fused[1], det[1]) and torch.equal(fused[2], det[2])
    assert runner.pipeline_status() == 0


def test_gqa_with_group_one_equals_mha(runner):
    # kv_heads == heads through fav4_bshd_backward_gqa is fav4_bshd_backward
    import ctypes as C
    import fav4_bshd as F
    q, k, v, do = _inputs(1, 4, 333, 444, seed=21)
    mha = _run(runner, q, k, v, do, True, 0.08, deterministic=True)
    o = torch.empty_like(q)
    lse = torch.empty((1, 4, 333), device="cuda")
    runner.call(q, k, v, o, lse, True, 0, 0.08)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = F.BwdArgs(*(x.data_ptr() for x in (q, k, v, o, do, lse, dq, dk, dv)), 1, 4, 333, 444, 0.08)
    ws = torch.empty(runner.lib.fav4_bshd_backward_workspace_bytes(C.byref(a)), dtype=torch.uint8, device="cuda")
    st = runner.lib.fav4_bshd_backward_gqa(C.byref(a), 4, 1, 1, ws.data_ptr(), ws.numel(),
                                          torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert st == 0
    assert torch.equal(dq, mha[0]) and torch.equal(dk, mha[1]) and torch.equal(dv, mha[2])


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("deterministic", [False, True])
def test_backward_peaky_softmax(runner, causal, deterministic):
    # scale 0.5 and Q x 4: logits of several hundred, rows dominated by a few keys (the regime of
    # the edge configuration's large-logit pattern); both paths against torch autograd in FP32
    q, k, v, do = _inputs(2, 3, 333, 517, seed=41)
    q = (q.float() * 4).to(torch.bfloat16)
    got = _run(runner, q, k, v, do, causal, 0.5, deterministic)
    want = _torch_grads(q, k, v, do, causal, 0.5)
    for g, w, n in zip(got, want, ("dq", "dk", "dv")):
        _check(g, w, n)
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("b,h,hk,s", [(4, 8, 8, 4096), (2, 8, 2, 4096), (1, 8, 8, 16384)])
def test_causal_head_pair_schedule(runner, b, h, hk, s):
    """Causal shapes large enough for the host to run the fused backward with
    head-pair work items (a head's longest and shortest key tile on one CTA):
    dK and dV equal the deterministic path's bit for bit (which walks its key
    tiles with the plain schedule), and dQ agrees with it within the FP32
    reduction-order tolerance of test_fused_dk_dv_match_deterministic_bitwise."""
    q, k, v, do = _inputs(b, h, s, s, 41)
    if hk != h:
        k, v = k[:, :, :hk].contiguous(), v[:, :, :hk].contiguous()
    scale = 1 / math.sqrt(128)
    fused = _run(runner, q, k, v, do, True, scale)
    det = _run(runner, q, k, v, do, True, scale, deterministic=True)
    assert torch.equal(fused[1], det[1]) and torch.equal(fused[2], det[2])
    err = (fused[0].float() - det[0].float()).abs().max().item()
    assert err <= 0.01 * det[0].float().abs().max().item() + 1e-3, err
    assert runner.pipeline_status() == 0

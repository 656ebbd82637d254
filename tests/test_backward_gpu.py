"""GPU tests of the backward pass (fav4_bshd_backward, the fused kernel with
FP32 dQ reductions, and fav4_bshd_backward_deterministic): dQ, dK, dV against
torch autograd in FP32 on the GPU (same BF16 inputs) and against the FP64
oracle on small cases, dense and top-left causal, ragged shapes, Sq != Sk;
run-to-run reproducibility of the deterministic path; dK and dV of both paths
bit-identical; keys no query row sees get zero gradients."""
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
    runner.call(q, k, v, o, lse, causal, 0, scale)
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

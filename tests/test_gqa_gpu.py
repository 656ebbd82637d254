"""GPU tests of grouped-query attention (fav4_bshd_forward_gqa): with K/V
heads shared by groups of query heads, the output is bit-identical to
fav4_bshd_forward on K/V repeated to every query head, and matches the FP64
oracle; the PyTorch operator takes the same path."""
import math

import numpy as np
import pytest
import torch

import fav4_bshd as F
from fav4_bshd import ops  # noqa: F401
from oracle import ref_attention as R

pytestmark = pytest.mark.gpu


def _inputs(b, h, hk, sq, sk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(s, generator=gen, device="cuda", dtype=torch.bfloat16)
            for s in ((b, sq, h, 128), (b, sk, hk, 128), (b, sk, hk, 128))]


@pytest.mark.parametrize("h,hk", [(8, 2), (8, 1), (6, 3), (4, 4)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("config", [0, 1, 3])
def test_gqa_equals_repeated_kv(runner, h, hk, causal, config):
    b, sq, sk = 2, 300, 517
    q, k, v = _inputs(b, h, hk, sq, sk, seed=h * 10 + hk)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, sq), float("nan"), device="cuda")
    runner.call_gqa(q, k, v, o, lse, causal, config)
    kr = k.repeat_interleave(h // hk, dim=2).contiguous()
    vr = v.repeat_interleave(h // hk, dim=2).contiguous()
    want_o = torch.empty_like(q)
    want_l = torch.empty((b, h, sq), device="cuda")
    runner.call(q, kr, vr, want_o, want_l, causal, config)
    torch.cuda.synchronize()
    assert torch.equal(o, want_o) and torch.equal(lse, want_l)
    assert runner.pipeline_status() == 0


def test_gqa_against_oracle(runner):
    b, h, hk, sq, sk = 1, 8, 2, 1000, 1537
    q, k, v = _inputs(b, h, hk, sq, sk, seed=3)
    for causal in (False, True):
        o = torch.empty_like(q)
        lse = torch.empty((b, h, sq), device="cuda")
        runner.call_gqa(q, k, v, o, lse, causal, 0)
        torch.cuda.synchronize()
        rows = R.sample_rows(sq)
        qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
        ref, ref_lse = R.reference_chunked(qn, kn, vn, causal, rows)
        R.errors(o.float().cpu().numpy()[:, rows].transpose(0, 2, 1, 3), lse.cpu().numpy()[:, :, rows], ref, ref_lse)


def test_gqa_operator_path():
    q, k, v = _inputs(2, 8, 2, 256, 384, seed=4)
    o, lse = torch.ops.fav4.bshd_forward(q, k, v, True, 0, -1.0, True)
    want = torch.empty_like(q)
    want_l = torch.empty_like(lse)
    F.Runner().call_gqa(q, k, v, want, want_l, True, 0, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert torch.equal(o, want) and torch.equal(lse, want_l)

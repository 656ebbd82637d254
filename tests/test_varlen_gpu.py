"""GPU tests of packed variable-length sequences (fav4_bshd_forward_varlen):
every sequence's output and LSE are bit-identical to fav4_bshd_forward on
that sequence alone (ragged lengths, empty sequences, Sq != Sk, GQA, dense
and top-left causal, every config), and malformed offsets stay inside the
tensors (clamped on the device). The packed backward
(fav4_bshd_backward_varlen) against the backward of each sequence alone."""
import math

import pytest
import torch

from grad_checks import dq_close

pytestmark = pytest.mark.gpu


def _packed(lens_q, lens_k, h, hk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    tq, tk = sum(lens_q), sum(lens_k)
    q = torch.randn((max(tq, 1), h, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    k = torch.randn((max(tk, 1), hk, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    v = torch.randn((max(tk, 1), hk, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    cu = lambda lens: torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int32)  # noqa
    return q, k, v, cu(lens_q), cu(lens_k)


CASES = [((1, 129, 1000, 300), (5, 200, 1537, 128), 4, 4), ((256, 0, 77, 640), (256, 300, 77, 0), 2, 2),
         ((513, 2048), (513, 2048), 8, 2), ((64,) * 7, (4000, 1, 2, 3, 4, 5, 6), 2, 1)]


@pytest.mark.parametrize("lens_q,lens_k,h,hk", CASES)
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("config", [0, 1, 3])
def test_varlen_equals_per_sequence_forward(runner, lens_q, lens_k, h, hk, causal, config):
    q, k, v, cu_q, cu_k = _packed(lens_q, lens_k, h, hk, seed=len(lens_q) * 10 + h)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((h, q.shape[0]), float("nan"), device="cuda")
    runner.call_varlen(q, k, v, o, lse, cu_q, cu_k, max(lens_q), causal, config)
    torch.cuda.synchronize()
    for b, (nq, nk) in enumerate(zip(lens_q, lens_k)):
        if nq == 0:
            continue
        q0, k0 = int(cu_q[b]), int(cu_k[b])
        got_o, got_l = o[q0:q0 + nq], lse[:, q0:q0 + nq]
        if nk == 0:
            assert torch.count_nonzero(got_o) == 0 and torch.isneginf(got_l).all()
            continue
        qs = q[q0:q0 + nq].unsqueeze(0).contiguous()
        ks, vs = (x[k0:k0 + nk].unsqueeze(0).contiguous() for x in (k, v))
        want_o = torch.empty_like(qs)
        want_l = torch.empty((1, h, nq), device="cuda")
        cfg = config if config else (1 if max(lens_q) < 128 else 2)
        if hk == h:
            runner.call(qs, ks, vs, want_o, want_l, causal, cfg)
        else:
            runner.call_gqa(qs, ks, vs, want_o, want_l, causal, cfg)
        torch.cuda.synchronize()
        assert torch.equal(got_o, want_o[0]), (b, nq, nk)
        assert torch.equal(got_l, want_l[0]), (b, nq, nk)
    assert runner.pipeline_status() == 0


def test_varlen_malformed_offsets_stay_inside(runner):
    # offsets beyond the totals and decreasing offsets are clamped on the device
    h = 2
    q = torch.randn((300, h, 128), device="cuda", dtype=torch.bfloat16)
    k = torch.randn((200, h, 128), device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    canary = torch.full((300 + 64, h, 128), 7.0, device="cuda", dtype=torch.bfloat16)
    o = canary[:300]
    cu_q = torch.tensor([0, 250, 100, 10_000], device="cuda", dtype=torch.int32)
    cu_k = torch.tensor([0, 999, 50, 200], device="cuda", dtype=torch.int32)
    runner.call_varlen(q, k, v, o, None, cu_q, cu_k, 300, False, 0)
    torch.cuda.synchronize()
    assert torch.all(canary[300:] == 7.0)
    assert runner.pipeline_status() == 0


BWD_CASES = [((1, 129, 1000, 300), (5, 200, 1537, 128), 4, 4), ((256, 0, 77, 640), (256, 300, 77, 0), 2, 2),
             ((513, 700), (513, 900), 8, 2), ((64,) * 5, (400, 1, 2, 3, 130), 2, 1)]


@pytest.mark.parametrize("lens_q,lens_k,h,hk", BWD_CASES)
@pytest.mark.parametrize("causal", [False, True])
def test_varlen_backward_equals_per_sequence_backward(runner, lens_q, lens_k, h, hk, causal):
    # fav4_bshd_backward_varlen against fav4_bshd_backward / _gqa on each sequence alone: dK, dV
    # bit-identical (same tiles, same arithmetic), dQ within one BF16 ulp (FP32 reduction order)
    q, k, v, cu_q, cu_k = _packed(lens_q, lens_k, h, hk, seed=len(lens_q) * 10 + h + 1)
    gen = torch.Generator(device="cuda").manual_seed(99)
    do = torch.randn(q.shape, generator=gen, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    o = torch.empty_like(q)
    lse = torch.empty((h, q.shape[0]), device="cuda")
    runner.call_varlen(q, k, v, o, lse, cu_q, cu_k, max(lens_q), causal, 0, scale)
    dq = torch.full_like(q, float("nan"))
    dk, dv = torch.full_like(k, float("nan")), torch.full_like(v, float("nan"))
    runner.backward_varlen(q, k, v, o, do, lse, dq, dk, dv, cu_q, cu_k, max(lens_q), max(max(lens_k), 1), causal,
                           scale)
    torch.cuda.synchronize()
    assert runner.pipeline_status() == 0
    for b, (nq, nk) in enumerate(zip(lens_q, lens_k)):
        q0, k0 = int(cu_q[b]), int(cu_k[b])
        if nq == 0 or nk == 0:
            # no query row sees these keys / no keys: zero gradients
            assert torch.count_nonzero(dk[k0:k0 + nk]) == 0 and torch.count_nonzero(dv[k0:k0 + nk]) == 0
            assert torch.count_nonzero(dq[q0:q0 + nq]) == 0
            continue
        qs, os_, dos = (x[q0:q0 + nq].unsqueeze(0).contiguous() for x in (q, o, do))
        ks, vs = (x[k0:k0 + nk].unsqueeze(0).contiguous() for x in (k, v))
        ls = lse[:, q0:q0 + nq].unsqueeze(0).contiguous()
        wq, wk, wv = torch.empty_like(qs), torch.empty_like(ks), torch.empty_like(vs)
        runner.backward(qs, ks, vs, os_, dos, ls, wq, wk, wv, causal, scale)
        torch.cuda.synchronize()
        assert torch.equal(dk[k0:k0 + nk], wk[0]) and torch.equal(dv[k0:k0 + nk], wv[0]), (b, nq, nk)
        assert dq_close(dq[q0:q0 + nq], wq[0]), (b, nq, nk)
    assert runner.pipeline_status() == 0


def test_varlen_backward_malformed_offsets_stay_inside(runner):
    # offsets beyond the totals, decreasing offsets and sequences longer than max_sq / max_sk are clamped
    # on the device: nothing past the gradient tensors is written and the pipeline reports no error
    h = 2
    q = torch.randn((300, h, 128), device="cuda", dtype=torch.bfloat16)
    k = torch.randn((200, h, 128), device="cuda", dtype=torch.bfloat16)
    v, do, o = torch.randn_like(k), torch.randn_like(q), torch.randn_like(q)
    lse = torch.randn((h, 300), device="cuda")
    qcan = torch.full((300 + 64, h, 128), 7.0, device="cuda", dtype=torch.bfloat16)
    kcan = torch.full((2, 200 + 64, h, 128), 7.0, device="cuda", dtype=torch.bfloat16)
    dq, dk, dv = qcan[:300], kcan[0, :200], kcan[1, :200]
    cu_q = torch.tensor([0, 250, 100, 10_000], device="cuda", dtype=torch.int32)
    cu_k = torch.tensor([0, 999, 50, 200], device="cuda", dtype=torch.int32)
    for causal in (False, True):
        runner.backward_varlen(q, k, v, o, do, lse, dq, dk, dv, cu_q, cu_k, 130, 120, causal)
        torch.cuda.synchronize()
        assert torch.all(qcan[300:] == 7.0) and torch.all(kcan[:, 200:] == 7.0)
        assert runner.pipeline_status() == 0

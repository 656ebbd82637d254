"""GPU tests of fav4_bshd_forward_host (forward from page-locked host
buffers, pipelined over batch chunks): every output is bit-identical to
fav4_bshd_forward on device copies of the same inputs, for ragged chunkings,
one or two staging slots, with and without LSE, on a side stream."""
import math

import pytest
import torch

import fav4_bshd as F

pytestmark = pytest.mark.gpu


def _host(shape, gen, dtype=torch.bfloat16):
    return torch.randn(shape, generator=gen, dtype=torch.float32).to(dtype).pin_memory()


@pytest.mark.parametrize("b,h,sq,sk,chunks", [(5, 4, 300, 517, 3), (5, 4, 300, 517, 1), (3, 2, 128, 128, 8),
                                              (4, 8, 1000, 1000, 4), (1, 3, 77, 2049, 2),
                                              (4, 8, 4096, 4096, 4)])  # dense Auto: the wide-step kernel
def test_host_forward_matches_device_forward(runner, b, h, sq, sk, chunks):
    gen = torch.Generator().manual_seed(b * 1000 + sq + chunks)
    q, k, v = _host((b, sq, h, 128), gen), _host((b, sk, h, 128), gen), _host((b, sk, h, 128), gen)
    specs = [(False, 0, True), (True, 0, False), (True, 3, True)]
    outs = []
    for causal, config, with_lse in specs:
        o = torch.full((b, sq, h, 128), float("nan"), dtype=torch.bfloat16).pin_memory()
        lse = torch.full((b, h, sq), float("nan")).pin_memory() if with_lse else None
        outs.append((o, lse, causal, config))
    side = torch.cuda.Stream()
    runner.forward_host(q, k, v, outs, chunks=chunks, stream=side)
    side.synchronize()
    dq, dk, dv = (x.cuda() for x in (q, k, v))
    for (o, lse, causal, config) in outs:
        want_o = torch.empty_like(dq)
        want_l = torch.empty((b, h, sq), device="cuda") if lse is not None else None
        runner.call(dq, dk, dv, want_o, want_l, causal, config)
        torch.cuda.synchronize()
        assert torch.equal(o, want_o.cpu()), (causal, config)
        if lse is not None:
            assert torch.equal(lse, want_l.cpu()), (causal, config)
    assert runner.pipeline_status() == 0


def test_host_forward_is_ordered_after_prior_stream_work(runner):
    # the inputs are written by a copy queued on the same stream just before
    gen = torch.Generator().manual_seed(7)
    b, sq, h = 6, 256, 2
    src = [_host((b, sq, h, 128), gen) for _ in range(3)]
    q, k, v = (torch.empty_like(x).pin_memory() for x in src)
    o = torch.empty((b, sq, h, 128), dtype=torch.bfloat16).pin_memory()
    side = torch.cuda.Stream()
    dev = [x.cuda() for x in src]
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        torch.cuda._sleep(20_000_000)  # ~10 ms of GPU time before the host copies below
        for dst, d in zip((q, k, v), dev):
            dst.copy_(d, non_blocking=True)
    runner.forward_host(q, k, v, [(o, None, True, 0)], chunks=3, stream=side)
    side.synchronize()
    want = torch.empty_like(dev[0])
    runner.call(*dev, want, None, True, 0)
    torch.cuda.synchronize()
    assert torch.equal(o, want.cpu())


def test_host_forward_reuses_workspace(runner):
    gen = torch.Generator().manual_seed(11)
    q, k, v = (_host((4, 200, 2, 128), gen) for _ in range(3))
    o1 = torch.empty((4, 200, 2, 128), dtype=torch.bfloat16).pin_memory()
    o2 = torch.empty_like(o1).pin_memory()
    runner.forward_host(q, k, v, [(o1, None, False, 0)], chunks=2)
    torch.cuda.synchronize()
    ws = runner._host_ws
    runner.forward_host(q, k, v, [(o2, None, False, 0)], chunks=2, scale=1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert runner._host_ws is ws and torch.equal(o1, o2)

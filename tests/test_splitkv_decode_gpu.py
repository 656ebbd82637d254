"""GPU tests of the one-launch split-KV forward (fav4_bshd_forward_splitkv):
on decode-like shapes (few query rows, many keys) and ordinary ones, for
every config, both masks and several split counts, it agrees with
fav4_bshd_forward within the split-KV tolerance and with the FP64 oracle;
one split is bit-identical to the plain forward; the automatic split count
fills the GPU for decode shapes and stays 1 for large ones."""
import ctypes as C
import math

import pytest
import torch

import fav4_bshd as F
from oracle import ref_attention as R

pytestmark = pytest.mark.gpu


def _inputs(b, h, sq, sk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(s, generator=gen, device="cuda", dtype=torch.bfloat16)
            for s in ((b, sq, h, 128), (b, sk, h, 128), (b, sk, h, 128))]


def _plain(runner, q, k, v, causal, config):
    b, sq, h, _ = q.shape
    o = torch.empty_like(q)
    lse = torch.empty((b, h, sq), device="cuda")
    runner.call(q, k, v, o, lse, causal, config)
    return o, lse


def _close(o, lse, o_ref, l_ref):
    assert torch.isfinite(o.float()).all()
    d = (o.float() - o_ref.float()).abs()
    assert d.max().item() < 2e-2 and d.mean().item() < 2e-3
    fin = torch.isfinite(l_ref)
    assert torch.equal(torch.isneginf(lse), torch.isneginf(l_ref))
    if fin.any():
        assert (lse[fin] - l_ref[fin]).abs().max().item() < 1e-3


SHAPES = [(1, 8, 1, 32768), (1, 8, 16, 20000), (2, 4, 64, 8192), (1, 8, 128, 65536), (2, 4, 300, 5000),
          (1, 2, 1000, 1537)]


@pytest.mark.parametrize("b,h,sq,sk", SHAPES)
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("splits", [0, 2, 7, 16, 32])
def test_splitkv_matches_forward(runner, b, h, sq, sk, causal, splits):
    q, k, v = _inputs(b, h, sq, sk, seed=sq + sk)
    o_ref, l_ref = _plain(runner, q, k, v, causal, 0)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, sq), float("nan"), device="cuda")
    runner.call_splitkv(q, k, v, o, lse, causal, 0, splits)
    torch.cuda.synchronize()
    _close(o, lse, o_ref, l_ref)
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("config", [1, 2, 3])
def test_splitkv_every_config(runner, config):
    q, k, v = _inputs(2, 4, 200, 9000, seed=config)
    for causal in (False, True):
        o_ref, l_ref = _plain(runner, q, k, v, causal, config)
        o = torch.empty_like(q)
        lse = torch.empty_like(l_ref)
        runner.call_splitkv(q, k, v, o, lse, causal, config, 5)
        torch.cuda.synchronize()
        _close(o, lse, o_ref, l_ref)


def test_one_split_is_the_plain_forward(runner):
    q, k, v = _inputs(1, 8, 64, 4096, seed=2)
    o_ref, l_ref = _plain(runner, q, k, v, False, 0)
    o = torch.empty_like(q)
    lse = torch.empty_like(l_ref)
    assert runner.call_splitkv(q, k, v, o, lse, False, 0, 1) == 1
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(lse, l_ref)


def test_splitkv_against_oracle(runner):
    q, k, v = _inputs(1, 4, 16, 30000, seed=7)
    for causal in (False, True):
        o = torch.empty_like(q)
        lse = torch.empty((1, 4, 16), device="cuda")
        used = runner.call_splitkv(q, k, v, o, lse, causal, 0, 0)
        torch.cuda.synchronize()
        qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
        rows = list(range(16))
        ref, ref_lse = R.reference_chunked(qn, kn, vn, causal, rows)
        R.errors(o.float().cpu().numpy().transpose(0, 2, 1, 3), lse.cpu().numpy(), ref, ref_lse,
                 R.NORTH_STAR_TOL["lse"])
        if not causal:
            assert used > 1


def test_automatic_split_count(runner):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    lib = runner.lib

    def splits(b, h, sq, sk, causal=0, config=0):
        a = F.Args(16, 32, 48, 64, None, b, h, sq, sk, 1 / math.sqrt(128))
        return lib.fav4_bshd_splitkv_splits(C.byref(a), causal, config)

    assert splits(1, 8, 1, 131072) == min(32, sms // 8)
    assert splits(32, 8, 4096, 4096) == 1
    assert splits(1, 8, 1, 1024) == 2          # at least 4 key tiles per split
    assert splits(1, 8, 1, 131072, causal=1) == 1  # top-left causal: one visible key tile

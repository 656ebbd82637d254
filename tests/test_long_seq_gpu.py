"""GPU parity at the long sequence lengths of the benchmark configurations,
against the FP64 oracle on the rows the reference's benchmark checks at every
length before timing it (benchmarks/bshd.py:147-156, R.sample_rows):

* the sequence sweep's lengths past the headline, S = 8192, 16384, 32768,
  dense and top-left causal, through fav4_bshd_forward (Auto config), torch
  RNG seed 2 as in the sweep (batch reduced to bound the test's time; the
  kernel's work decomposition per (batch, head) is the same);
* the long-context case B1 H8 S131072 causal (seed 4, LSE on) through
  fav4_bshd_forward, and through the path the multi-GPU split-KV driver takes
  (fav4_bshd.splitkv): zigzag key chunks per "rank", each rank's two chunk
  partials merged, then the ranks' partials combined -- all on one device;
* packed variable-length sequences (fav4_bshd_forward_varlen) checked directly
  against the oracle, sequence by sequence, grouped-query heads included;
* the causal work-tile schedules: a batch the host runs with head-pair work
  items against the same rows as packed sequences (plain schedule), bit for
  bit.
"""
import functools
import math

import numpy as np
import pytest
import torch

from fav4_bshd.splitkv import zigzag_chunks
from oracle import ref_attention as R

pytestmark = pytest.mark.gpu


def _check(o, lse, ref, ref_lse, rows):
    o = o.float().cpu().numpy()[:, rows].transpose(0, 2, 1, 3)
    lse_np = None if lse is None else lse.cpu().numpy()[:, :, rows]
    return R.errors(o, lse_np, ref, ref_lse)


def _inputs(shape, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(shape, generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(3)]


@pytest.mark.parametrize("seq,batch", [(8192, 2), (16384, 1), (32768, 1)])
@pytest.mark.parametrize("causal", [False, True])
def test_sweep_lengths_sampled_rows(runner, cuda, seq, batch, causal):
    q, k, v = _inputs((batch, seq, 8, 128), 2)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((batch, 8, seq), float("nan"), device="cuda")
    runner.call(q, k, v, o, lse, causal, 0)
    torch.cuda.synchronize()
    rows = R.sample_rows(seq)
    qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
    ref, ref_lse = R.reference_chunked(qn, kn, vn, causal, rows)
    _check(o, lse, ref, ref_lse, rows)
    assert runner.pipeline_status() == 0


@functools.lru_cache(maxsize=1)
def _long_context():
    """BASELINE configs[4] inputs and the FP64 oracle on the sampled rows."""
    n = 131072
    q, k, v = _inputs((1, n, 8, 128), 4)
    rows = R.sample_rows(n)
    qn = q[:, rows].float().cpu().numpy()
    kn, vn = (x.float().cpu().numpy() for x in (k, v))
    # the oracle takes every query row and a row index; only the sampled rows are read
    qfull = np.zeros((1, n, 8, 128), dtype=np.float32)
    qfull[:, rows] = qn
    ref, ref_lse = R.reference_chunked(qfull, kn, vn, True, rows)
    return (q, k, v), rows, ref, ref_lse


def test_long_context_forward_sampled_rows(runner, cuda):
    (q, k, v), rows, ref, ref_lse = _long_context()
    o = torch.full_like(q, float("nan"))
    lse = torch.full((1, 8, q.shape[1]), float("nan"), device="cuda")
    runner.call(q, k, v, o, lse, True, 0)
    torch.cuda.synchronize()
    _check(o, lse, ref, ref_lse, rows)
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("world", [2, 8])
def test_long_context_zigzag_split_kv_on_one_device(runner, cuda, world):
    """The multi-GPU long-context path with every rank's work on one device:
    rank g's zigzag chunks g and 2G-1-g, its local merge, the combine over
    ranks, against FP64 and against the single forward."""
    (q, k, v), rows, ref, ref_lse = _long_context()
    n = q.shape[1]
    rank_o, rank_l = [], []
    for g in range(world):
        chunk_o, chunk_l = [], []
        for b, e in zigzag_chunks(n, world, g):
            o = torch.empty_like(q)
            lse = torch.empty((1, 8, n), device="cuda")
            runner.call_partial(q, k, v, o, lse, True, b, e)
            chunk_o.append(o)
            chunk_l.append(lse)
        merged_o, merged_l = torch.empty_like(q), torch.empty((1, 8, n), device="cuda")
        runner.combine(chunk_o, chunk_l, merged_o, merged_l)
        rank_o.append(merged_o)
        rank_l.append(merged_l)
        del chunk_o, chunk_l
    out = torch.full_like(q, float("nan"))
    lse = torch.full((1, 8, n), float("nan"), device="cuda")
    runner.combine(rank_o, rank_l, out, lse)
    torch.cuda.synchronize()
    _check(out, lse, ref, ref_lse, rows)
    full_o = torch.empty_like(q)
    full_l = torch.empty((1, 8, n), device="cuda")
    runner.call(q, k, v, full_o, full_l, True, 0)
    torch.cuda.synchronize()
    assert (out.float() - full_o.float()).abs().max().item() < 2e-2
    assert (lse - full_l).abs().max().item() < 1e-3
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("h,hk", [(4, 4), (8, 2)])
def test_varlen_against_oracle(runner, cuda, causal, h, hk):
    lens_q, lens_k = (1, 129, 1000, 300, 0), (5, 200, 1537, 128, 40)
    gen = torch.Generator(device="cuda").manual_seed(77 + h)
    tq, tk = sum(lens_q), sum(lens_k)
    q = torch.randn((tq, h, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    k = torch.randn((tk, hk, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    v = torch.randn((tk, hk, 128), generator=gen, device="cuda", dtype=torch.bfloat16)
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(lens_q)]), device="cuda", dtype=torch.int32)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(lens_k)]), device="cuda", dtype=torch.int32)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((h, tq), float("nan"), device="cuda")
    runner.call_varlen(q, k, v, o, lse, cu_q, cu_k, max(lens_q), causal, 0)
    torch.cuda.synchronize()
    qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
    on, ln = o.float().cpu().numpy(), lse.cpu().numpy()
    for b, (nq, nk) in enumerate(zip(lens_q, lens_k)):
        if nq == 0:
            continue
        q0, k0 = int(cu_q[b]), int(cu_k[b])
        ref, ref_lse = R.reference(qn[None, q0:q0 + nq], kn[None, k0:k0 + nk], vn[None, k0:k0 + nk], causal)
        got_o = on[None, q0:q0 + nq].transpose(0, 2, 1, 3)
        got_l = ln[None, :, q0:q0 + nq]
        R.errors(got_o, got_l, ref, ref_lse)
    assert math.isfinite(float(o.float().sum()))
    assert runner.pipeline_status() == 0


@pytest.mark.parametrize("b,s,h", [(4, 4096, 8), (2, 4096, 8), (16, 4096, 8), (3, 2944, 5), (1, 16384, 8)])
def test_causal_schedules_agree(runner, cuda, b, s, h):
    """Causal launches of one batch of equal sequences pick the head-pair
    schedule when it balances better (the host simulates both); packed
    sequences always take the plain one. Every tile computes the same numbers
    either way, so the two outputs agree bit for bit, and both cover every row
    (NaN pre-fill)."""
    q, k, v = _inputs((b, s, h, 128), 11)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, s), float("nan"), device="cuda")
    runner.call(q, k, v, o, lse, True, 0)
    cu = torch.arange(0, (b + 1) * s, s, device="cuda", dtype=torch.int32)
    ov = torch.full((b * s, h, 128), float("nan"), device="cuda", dtype=torch.bfloat16)
    lv = torch.full((h, b * s), float("nan"), device="cuda")
    runner.call_varlen(q.view(b * s, h, 128), k.view(b * s, h, 128), v.view(b * s, h, 128), ov, lv, cu, cu, s,
                       True, 0)
    torch.cuda.synchronize()
    assert torch.equal(o.view(b * s, h, 128), ov)
    assert torch.equal(lse.permute(1, 0, 2).reshape(h, b * s), lv)
    assert runner.pipeline_status() == 0

"""CPU tests of the oracle: pinned against the reference's own FP64 outputs.

The golden fixtures were produced by the reference's benchmarks/bshd.py
`reference()` (benchmarks/bshd.py:90-100) and `errors()` (:22-32); these tests
check the oracle's restatement against them and check the kernel-faithful
emulation (lazy rescale, BF16 P, polynomial exp2) against the same outputs
with the reference's tolerances.
"""
import hashlib
import math
import re
from pathlib import Path

import numpy as np
import pytest

import golden_cases as G
from oracle import ref_attention as R

ROOT = Path(__file__).resolve().parents[1]
NAMES = G.names()


def test_bf16_rounding_known_answers():
    x = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -2.5, 3.0e38, 1e-40, 0.0], np.float32)
    got = R.bf16_round(x)
    # 1+2^-8 is a tie -> even (1.0); 1+1.5*2^-8 rounds up to 1+2^-7
    assert got[0] == 1.0 and got[1] == 1.0 and got[2] == np.float32(1.0078125) and got[3] == np.float32(1.0078125)
    assert got[4] == -2.5 and got[7] == 0.0
    assert R.bf16_bits(np.array([np.nan], np.float32))[0] == 0x7FC0


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_fixture(name):
    meta, rows, o_gold, lse_gold = G.load(name)
    q, k, v = G.inputs_for(meta)
    h = hashlib.sha256()
    for x in (q, k, v):
        h.update(R.bf16_bits(x).tobytes())
    assert h.hexdigest() == meta["input_sha256"], "input generator no longer reproduces the fixture inputs"
    o, lse = R.reference(q, k, v, meta["causal"], rows, meta["scale"])
    # fixtures store O as float32: compare at float32 resolution
    np.testing.assert_allclose(o, o_gold, rtol=2e-6, atol=2e-7)
    np.testing.assert_allclose(lse, lse_gold, rtol=1e-12, atol=1e-9)


@pytest.mark.parametrize("name", NAMES)
def test_tolerance_restatement_matches_reference_verdicts(name):
    meta, rows, o_gold, lse_gold = G.load(name)
    for eps, lse_eps, verdict in zip(meta["planted"], meta["planted_lse"], meta["reference_verdicts"]):
        o_try = o_gold + eps * np.sign(np.cos(np.arange(o_gold.size))).reshape(o_gold.shape)
        assert R.reference_criteria_pass(o_try, lse_gold + lse_eps, o_gold, lse_gold) == verdict


@pytest.mark.parametrize("name", [n for n in NAMES if not n.startswith("edge")] + [
    "edge_b3h5_1000x1537_isqrt_dense", "edge_b3h5_1000x1537_half_causal"])
@pytest.mark.parametrize("poly_per8", [0, 2, 4])
def test_emulation_within_tolerance(name, poly_per8):
    meta, rows, o_gold, lse_gold = G.load(name)
    q, k, v = G.inputs_for(meta)
    o, lse = R.emulate(q, k, v, meta["causal"], meta["scale"], poly_per8=poly_per8)
    lse_limit = R.NORTH_STAR_TOL["lse"] if meta["kind"] == "edge" else R.REF_TOL["lse"]
    R.errors(o[:, rows].transpose(0, 2, 1, 3), lse[:, :, rows], o_gold, lse_gold, lse_limit)


def test_emulated_split_kv_combine_matches_full():
    """Split-KV slices + LSE combine (the multi-GPU long-context path) equal
    the full computation in exact arithmetic; checked on the emulation."""
    q, k, v = R.inputs(1, 2, 300, 300, "normal", seed=5)
    for causal in (False, True):
        ref, ref_lse = R.reference(q, k, v, causal)
        bounds = [0, 77, 150, 300]
        parts = [R.emulate(q, k, v, causal, kv_begin=a, kv_end=b) for a, b in zip(bounds[:-1], bounds[1:])]
        lses = np.stack([p[1] for p in parts])  # [G,B,H,Sq]
        mx = lses.max(0)
        w = np.where(np.isneginf(lses), 0.0, np.exp(lses - np.where(np.isneginf(mx), 0, mx)))
        wsum = w.sum(0)
        o = sum(w[g].transpose(0, 2, 1)[..., None] * parts[g][0] for g in range(len(parts))) / \
            wsum.transpose(0, 2, 1)[..., None]
        lse = mx + np.log(wsum)
        R.errors(o.transpose(0, 2, 1, 3), lse, ref, ref_lse)


@pytest.mark.parametrize("scale", [1 / math.sqrt(128), 0.5])
def test_edge_inputs_force_the_rescale_path(scale):
    q, k, v, jumps = R.edge_inputs()
    for head, pos in jumps.items():
        jump = R.realised_jump_base2(q, k, head, pos, scale)
        assert np.median(jump) > 8.0 and (jump > 8.0).mean() > 0.9, (head, np.median(jump))
    # heads 0-1 have large logits
    s = np.einsum("bqd,bkd->bqk", q[:, :, 0].astype(np.float64), k[:, :, 0].astype(np.float64)) * scale
    assert np.abs(s).max() > 100


def test_exp2_polynomial_fit_and_kernel_constants():
    from fav4_bshd import exp2_poly as P
    coeffs, err = P.fit()
    assert err < 1.02e-4
    np.testing.assert_allclose(coeffs, P.KERNEL_COEFFS, rtol=0, atol=2e-6)
    assert P.max_rel_error_f32(P.KERNEL_COEFFS) < 1.02e-4
    src = (ROOT / "flash-attention-v4-rocm_b200" / "csrc" / "attn_fwd_sm100.cuh").read_text()
    consts = [float(re.search(rf"kPolyC{i} = ([0-9.e-]+)f;", src).group(1)) for i in (1, 2, 3)]
    assert consts == list(P.KERNEL_COEFFS)
    assert R.POLY == (1.0, *P.KERNEL_COEFFS)
    # the oracle's FP32 evaluation of the split: exact at integers, bounded elsewhere
    x = np.linspace(-30, 8, 200001).astype(np.float32)
    rel = np.abs(R.ex2_poly(x).astype(np.float64) / np.exp2(x.astype(np.float64)) - 1)
    assert rel.max() < 1.1e-4
    ints = np.arange(-125, 9, dtype=np.float32)
    assert np.array_equal(R.ex2_poly(ints), np.exp2(ints))


def test_grouped_query_reference_is_repeated_kv():
    """Grouped-query attention in the oracle: query head h reads K/V head
    h // (H / H_kv), which equals ordinary attention on repeated K/V."""
    q, _, _ = R.inputs(2, 6, 40, 40, "normal", seed=9)
    _, k, v = R.inputs(2, 2, 40, 56, "normal", seed=10)
    assert R.expand_kv(k, 6).shape == (2, 56, 6, 128)
    assert np.array_equal(R.expand_kv(k, 6)[:, :, 2], k[:, :, 0]) and np.array_equal(R.expand_kv(k, 6)[:, :, 3], k[:, :, 1])
    for causal in (False, True):
        o, lse = R.reference(q, k, v, causal)
        o2, lse2 = R.reference(q, np.repeat(k, 3, axis=2), np.repeat(v, 3, axis=2), causal)
        assert np.array_equal(o, o2) and np.array_equal(lse, lse2)
        oc, lc = R.reference_chunked(q, k, v, causal, np.arange(40), max_elems=512)
        np.testing.assert_allclose(oc, o, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("causal", [False, True])
def test_reference_backward_matches_torch_autograd(causal):
    """The oracle's FP64 gradients equal torch autograd of the same FP64 math."""
    import torch
    q, k, v = R.inputs(2, 3, 70, 90, "normal", seed=12)
    do = R.inputs(2, 3, 70, 70, "normal", seed=13)[0]
    scale = 0.1
    dq, dk, dv, o, lse = R.reference_backward(q, k, v, do, causal, scale)
    tq, tk, tv = (torch.tensor(x.transpose(0, 2, 1, 3), dtype=torch.float64, requires_grad=True) for x in (q, k, v))
    s = tq @ tk.transpose(-1, -2) * scale
    if causal:
        s = s.masked_fill(torch.ones(70, 90, dtype=torch.bool).triu(1), float("-inf"))
    to = torch.softmax(s, -1) @ tv
    to.backward(torch.tensor(do.transpose(0, 2, 1, 3), dtype=torch.float64))
    for mine, theirs in ((dq, tq.grad), (dk, tk.grad), (dv, tv.grad), (o, to.detach())):
        np.testing.assert_allclose(mine.transpose(0, 2, 1, 3), theirs.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, torch.logsumexp(s, -1).detach().numpy(), rtol=1e-12, atol=1e-12)
    ref_o, ref_lse = R.reference(q, k, v, causal, scale=scale)
    np.testing.assert_allclose(o.transpose(0, 2, 1, 3), ref_o, rtol=1e-12, atol=1e-12)

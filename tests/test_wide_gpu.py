"""GPU parity of the wide-step forward kernel (fav4_bshd_forward_wide, and the
dense launches that Auto routes to it) against the FP64 oracle.

The wide kernel computes S for 256 keys per step and splits each row's softmax
over two warpgroups that exchange their row maxima, so its rounding differs
from config 2 within the same tolerances (benchmarks/bshd.py:22-32 and the
north-star bounds), checked here on the reference's validation shapes, ragged
key counts that are not multiples of 256, peaky inputs, and headline-size
sampled rows.
"""
import math

import numpy as np
import pytest
import torch

from oracle import ref_attention as R

pytestmark = pytest.mark.gpu


def to_dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda").to(torch.bfloat16)


def check(o, lse, ref, ref_lse, rows=None):
    o = o.float().cpu().numpy()
    lse = lse.cpu().numpy()
    if rows is not None:
        o, lse = o[:, rows], lse[:, :, rows]
    return R.errors(o.transpose(0, 2, 1, 3), lse, ref, ref_lse)


CASES = [(1, 1, 1, 1, "normal"), (2, 3, 17, 31, "normal"), (2, 3, 63, 65, "normal"), (1, 8, 127, 129, "normal"),
         (3, 8, 193, 257, "normal"), (1, 8, 256, 512, "zero"), (1, 8, 256, 512, "large"),
         (1, 8, 256, 512, "late_max"), (1, 8, 129, 65, "negative"), (2, 8, 512, 512, "normal"),
         (2, 4, 1000, 1537, "normal"), (1, 2, 300, 2000, "late_max"), (2, 2, 700, 2305, "large")]


@pytest.mark.parametrize("i", range(len(CASES)), ids=[f"b{c[0]}h{c[1]}_{c[2]}x{c[3]}_{c[4]}" for c in CASES])
def test_wide_against_oracle(runner, cuda, i):
    # the first ten are the reference's validation shapes with the seeds of
    # test_parity_gpu.py; the output's BF16 rounding alone can take a "large"
    # input past the 2e-2 bound for other seeds, whatever the kernel
    b, h, sq, sk, pat = CASES[i]
    q, k, v = R.inputs(b, h, sq, sk, pat, seed=100 + i)
    ref, ref_lse = R.reference(q, k, v, False)
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    o = torch.full_like(qd, float("nan"))
    lse = torch.full((b, h, sq), float("nan"), device="cuda")
    runner.call_wide(qd, kd, vd, o, lse)
    torch.cuda.synchronize()
    check(o, lse, ref, ref_lse)
    assert runner.pipeline_status(clear=False) == 0


@pytest.mark.parametrize("scale", [1 / math.sqrt(128), 0.5], ids=["isqrt", "half"])
def test_wide_edge_config(runner, cuda, scale):
    """Q x 30, late maximum jumps and a constant-K head (the rescale edge case)."""
    q, k, v, _ = R.edge_inputs()
    ref, ref_lse = R.reference(q, k, v, False, scale=scale)
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    o = torch.full_like(qd, float("nan"))
    lse = torch.full((q.shape[0], q.shape[2], q.shape[1]), float("nan"), device="cuda")
    runner.call_wide(qd, kd, vd, o, lse, scale=scale)
    torch.cuda.synchronize()
    o_np = o.float().cpu().numpy().transpose(0, 2, 1, 3)
    R.errors(o_np, lse.cpu().numpy(), ref, ref_lse, lse_limit=R.NORTH_STAR_TOL["lse"])


def test_auto_routes_wave_quantised_dense_to_wide(runner, cuda):
    """B4 H8 S4096 dense: 256-row tiles need 4 waves of the SMs, 128-row tiles
    7 (< 1.84 x 4), so Auto runs the wide kernel (bit-identical to the explicit
    entry), checked against FP64 on sampled rows; B32 stays on config 2."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    gen = torch.Generator(device="cuda").manual_seed(21)
    for b, want_wide in ((4, True), (32, False)):
        q, k, v = (torch.randn(b, 4096, 8, 128, generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        t2, tw = b * 8 * 16, b * 8 * 32
        waves2, wavesw = -(-t2 // sms), -(-tw // sms)
        expect = wavesw * 25 < waves2 * 46 and 2 * t2 > sms
        assert expect == want_wide or sms != 148
        outs = {}
        for name in ("auto", "wide", "c2"):
            o = torch.full_like(q, float("nan"))
            lse = torch.full((b, 8, 4096), float("nan"), device="cuda")
            if name == "auto":
                runner.call(q, k, v, o, lse, False, 0)
            elif name == "wide":
                runner.call_wide(q, k, v, o, lse)
            else:
                runner.call(q, k, v, o, lse, False, 2)
            outs[name] = (o, lse)
        torch.cuda.synchronize()
        same = outs["wide"] if expect else outs["c2"]
        assert torch.equal(outs["auto"][0], same[0]) and torch.equal(outs["auto"][1], same[1]), b
        if b == 4:
            rows = np.arange(0, 4096, 97)
            qn, kn, vn = (x[:1].float().cpu().numpy() for x in (q, k, v))
            ref, ref_lse = R.reference_chunked(qn, kn, vn, False, rows)
            check(outs["wide"][0][:1], outs["wide"][1][:1], ref, ref_lse, rows)
        del q, k, v, outs
    assert runner.pipeline_status(clear=False) == 0


def test_gqa_auto_wide_matches_expanded_heads(runner, cuda):
    """Grouped-query Auto on a shape that takes the wide kernel equals the wide
    kernel on K/V heads repeated per group, bit for bit."""
    gen = torch.Generator(device="cuda").manual_seed(22)
    q = torch.randn(4, 4096, 8, 128, generator=gen, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn(4, 4096, 2, 128, generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    o = torch.full_like(q, float("nan"))
    lse = torch.full((4, 8, 4096), float("nan"), device="cuda")
    runner.call_gqa(q, k, v, o, lse, False, 0)
    ke, ve = (x.repeat_interleave(4, dim=2).contiguous() for x in (k, v))
    o2 = torch.full_like(q, float("nan"))
    lse2 = torch.full_like(lse, float("nan"))
    runner.call_wide(q, ke, ve, o2, lse2)
    torch.cuda.synchronize()
    assert torch.equal(o, o2) and torch.equal(lse, lse2)


def test_wide_without_lse_ragged_rows(runner, cuda):
    """LSE off, Sq not a multiple of 128 and Sk not a multiple of 256: every
    row is written (NaN pre-fill) and within the bounds."""
    q, k, v = R.inputs(2, 3, 333, 700, "normal", seed=33)
    ref, ref_lse = R.reference(q, k, v, False)
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    out = torch.full_like(qd, float("nan"))
    runner.call_wide(qd, kd, vd, out, None)
    torch.cuda.synchronize()
    r = R.error_stats(out.float().cpu().numpy().transpose(0, 2, 1, 3), None, ref, ref_lse)
    assert r["finite"] and r["max_abs"] <= R.NORTH_STAR_TOL["max_abs"], r
    assert r["mean_abs"] <= R.NORTH_STAR_TOL["mean_abs"], r

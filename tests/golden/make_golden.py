"""Generate the golden fixtures in this folder from the reference's own code.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference /path/to/flash-attention-v4-rocm

It imports the reference's benchmark harness (benchmarks/bshd.py) and calls
its FP64 `reference()` (benchmarks/bshd.py:90-100) on CPU tensors built by
oracle.ref_attention.inputs / edge_inputs. The harness hard-codes
device='cuda' in the causal mask's torch.arange; a module-local stand-in for
`torch` drops that device argument so the unmodified function runs on the CPU.
The reference's own `errors()` (benchmarks/bshd.py:22-32) is evaluated on a
planted perturbation for every case and stored too, so the CPU tests can check
the oracle's restatement of the tolerance test against the reference's.

Each fixture stores: the case description, the sha256 of the BF16 inputs (so
the tests can confirm they regenerate the same inputs), the sampled query
rows, and O (float32) / LSE (float64) on those rows in the reference's
[B, H, rows, 128] / [B, H, rows] layout.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
from oracle import ref_attention as R  # noqa: E402

# The reference's validation cases (benchmarks/bshd.py:112-115), the CPU check
# config (B1 H2 S256, seed 0) and the structured edge config (B3 H5 1000x1537).
VALIDATE_CASES = [(1, 1, 1, 1, "normal"), (2, 3, 17, 31, "normal"), (2, 3, 63, 65, "normal"),
                  (1, 8, 127, 129, "normal"), (3, 8, 193, 257, "normal"), (1, 8, 256, 512, "zero"),
                  (1, 8, 256, 512, "large"), (1, 8, 256, 512, "late_max"), (1, 8, 129, 65, "negative"),
                  (2, 8, 512, 512, "normal")]
SEED_VALIDATE = 11939  # the reference harness's seed (benchmarks/bshd.py:201), used here for numpy


def case_list():
    out = []
    for i, (b, h, sq, sk, pat) in enumerate(VALIDATE_CASES):
        out.append(dict(name=f"v{i}_b{b}h{h}_{sq}x{sk}_{pat}", kind="pattern", b=b, h=h, sq=sq, sk=sk,
                        pattern=pat, seed=SEED_VALIDATE + i, scale=1.0 / math.sqrt(128)))
    out.append(dict(name="cpu_b1h2_256", kind="pattern", b=1, h=2, sq=256, sk=256, pattern="normal", seed=0,
                    scale=1.0 / math.sqrt(128)))
    for sname, scale in (("isqrt", 1.0 / math.sqrt(128)), ("half", 0.5)):
        out.append(dict(name=f"edge_b3h5_1000x1537_{sname}", kind="edge", b=3, h=5, sq=1000, sk=1537,
                        pattern="edge", seed=3, scale=scale))
    return out


def case_inputs(c):
    if c["kind"] == "edge":
        q, k, v, _ = R.edge_inputs(seed=c["seed"], b=c["b"], h=c["h"], sq=c["sq"], sk=c["sk"])
    else:
        q, k, v = R.inputs(c["b"], c["h"], c["sq"], c["sk"], c["pattern"], seed=c["seed"])
    return q, k, v


def case_rows(c):
    sq = c["sq"]
    if sq <= 24:
        return np.arange(sq)
    rows = {0, 1, sq // 2, sq - 1, sq - 2} | {r for r in (63, 64, 127, 128, 599, 600, 601, 999) if r < sq}
    rows |= set(range(0, sq, max(1, sq // 6)))
    return np.array(sorted(rows), dtype=np.int64)


def input_digest(q, k, v) -> str:
    h = hashlib.sha256()
    for x in (q, k, v):
        h.update(R.bf16_bits(x).tobytes())
    return h.hexdigest()


def load_reference_harness(ref_root: Path):
    spec = importlib.util.spec_from_file_location("ref_bshd", ref_root / "benchmarks" / "bshd.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    class _CpuTorch:
        """`torch` as seen by the harness, with arange's device argument dropped."""

        def __getattr__(self, name):
            return getattr(torch, name)

        @staticmethod
        def arange(*args, **kwargs):
            kwargs.pop("device", None)
            return torch.arange(*args, **kwargs)

    mod.torch = _CpuTorch()
    return mod


def to_torch_bf16(x):
    return torch.from_numpy(R.bf16_bits(x).view(np.int16).copy()).view(torch.bfloat16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="reference checkout root")
    args = ap.parse_args()
    mod = load_reference_harness(args.reference)
    index = []
    for c in case_list():
        q, k, v = case_inputs(c)
        rows = case_rows(c)
        qt, kt, vt = to_torch_bf16(q), to_torch_bf16(k), to_torch_bf16(v)
        rows_t = torch.from_numpy(rows)
        for causal in (False, True):
            if c["scale"] != 1.0 / math.sqrt(128):
                # the harness bakes in 1/sqrt(128): rescale Q in FP64 so its
                # scores equal q.k*scale exactly (sqrt(128)*scale is applied to Q)
                qd = qt.double() * (c["scale"] * math.sqrt(128))
                o_ref, lse_ref = mod.reference(qd, kt, vt, causal, rows_t)
            else:
                o_ref, lse_ref = mod.reference(qt, kt, vt, causal, rows_t)
            o_ref = o_ref.numpy()
            lse_ref = lse_ref.numpy()
            # the reference's own tolerance verdicts on three planted outputs
            verdicts = []
            for eps, lse_eps in ((0.0, 0.0), (0.004, 1e-4), (0.05, 5e-4)):
                o_try = torch.from_numpy(o_ref + eps * np.sign(np.cos(np.arange(o_ref.size))).reshape(o_ref.shape))
                l_try = torch.from_numpy(lse_ref + lse_eps)
                try:
                    mod.errors(o_try, l_try, torch.from_numpy(o_ref),
                               torch.from_numpy(lse_ref), torch.bfloat16)
                    verdicts.append(True)
                except AssertionError:
                    verdicts.append(False)
            name = f"{c['name']}_{'causal' if causal else 'dense'}"
            meta = dict(c, causal=causal, input_sha256=input_digest(q, k, v), planted=[0.0, 0.004, 0.05],
                        planted_lse=[0.0, 1e-4, 5e-4], reference_verdicts=verdicts)
            np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), rows=rows,
                                o=o_ref.astype(np.float32), lse=lse_ref)
            index.append(name)
            print(name, o_ref.shape, verdicts, flush=True)
    (HERE / "index.json").write_text(json.dumps(index, indent=1) + "\n")


if __name__ == "__main__":
    main()

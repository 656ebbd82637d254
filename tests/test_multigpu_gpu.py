"""Multi-GPU tests, run only when the box has at least two GPUs.

* The long-context split-KV path (fav4_bshd.splitkv) across 2 ranks under
  torchrun: each rank's output rows must match a single-GPU forward of the
  whole causal problem within the north-star tolerance.
* bench.py's batch-sharded headline run under torchrun prints one JSON line
  with n_gpus = 2, the global batch split in two, no pipeline timeouts, and
  its sweep and long-context keys (the latter within tolerance of FP64).
* The decode split-KV path (fav4_bshd.splitkv.DecodeSplitKV) across 2 ranks:
  every rank's full output matches one GPU's split-KV forward.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _torchrun(n, *args, timeout=600):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29533", str(ROOT / "bench.py"), *args]
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "0"))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


@needs2
def test_long_context_split_kv_two_gpus():
    out = _torchrun(2, "--long-context", "--lc-seq", "16384", "--steps", "2", "--warmup", "1", "--gpus", "2")
    assert out["n_gpus"] == 2 and out["vs_single_gpu"]["within_tolerance"], out


@needs2
def test_batch_sharded_bench_two_gpus():
    out = _torchrun(2, "--gpus", "2", "--steps", "3", "--warmup", "3", "--seqs", "512,4096", "--lc-seq", "16384")
    assert out["n_gpus"] == 2 and out["value"] > 0 and out["scaling"] == "strong", out
    assert out["config"]["batch_per_gpu"] == 16 and out["config"]["global_batch"] == 32, out
    assert out["pipeline_status"] == {"headline_and_e2e": 0, "after_sweep_and_long_context": 0}, out
    assert out["e2e"]["outputs_match"] and len(out["e2e"]["h2d_gbs_per_rank"]) == 2, out
    assert len(out["sweep"]["points"]) == 4, out
    assert out["long_context"]["vs_fp64_sampled_rows"]["within_tolerance"], out


@needs2
def test_decode_split_kv_two_gpus():
    out = _torchrun(2, "--decode", "--decode-sq", "16", "--decode-sk", "65536", "--steps", "3", "--warmup", "1",
                    "--gpus", "2")
    assert out["n_gpus"] == 2 and out["vs_single_gpu"]["within_tolerance"], out

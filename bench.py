#!/usr/bin/env python3
"""Benchmark of the B200 BF16 attention forward (one JSON line on stdout).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Workload: global B=32, H=8, Sq=Sk=4096, D=128, BSHD
contiguous, Q/K/V BF16 N(0,1) (torch RNG, seed 1), scale 1/sqrt(128), LSE
off, O buffers reused. One step = one dense and one top-left causal forward
through the C ABI (fav4_bshd_forward), i.e. the reference's two headline
cases. FLOPs use the reference's convention (benchmarks/bshd.py:168-170):
dense 4*B*H*D*S^2, causal 4*B*H*D*S(S+1)/2.

Multi-GPU: one process per GPU. The global batch of 32 is sharded: rank r
runs the unchanged C ABI on its contiguous batch slice of 32/N entries
(batch sharding needs no collective), so scaling is strong and N=1 is the
single-GPU headline. Timing: W warm-up steps, then exactly K steps between a
barrier + synchronize on both sides; an L2 flush (a 256 MiB memset) runs
before every step, outside the step's CUDA events, and a step's time is its
first-to-last event interval on the launching stream; the max over ranks of
the summed step times gives `value`.

Extra keys of the same line:
* `e2e`: the metric with Q/K/V copied from pinned host memory and both
  outputs copied back inside the timed region, through fav4_bshd_forward_host,
  plus each rank's standalone host<->device copy bandwidth.
* `roofline`: the dense kernel's launches against the measured BF16 peak.
* `sweep`: BASELINE configs[2] (S = 512..32768, dense and causal, the global
  B=32 sharded over the ranks) timed with the reference's graph protocol
  (benchmarks/bshd.py:34-51,157-166): a 5-call warm-up graph, then a 20-call
  graph replayed per observation; input sets rotate so that the bytes between
  two reads of one set exceed the L2.
* `long_context`: BASELINE configs[4] (B1 H8 S131072 causal): one GPU's
  forward at N=1, the key sequence split over the ranks at N>1
  (fav4_bshd.splitkv.SplitKV), checked against the FP64 oracle on the
  reference's sampled rows.
* `cpu_baseline` (rank 0, N=1): the FP64 CPU oracle -- the reference's
  benchmarks/bshd.py:90-100 math -- on a bounded sample, on every host core.

--impl reference times that same CPU oracle as the reference arm: the
reference implementation is HIP for AMD gfx1250 and cannot run here, so the
reference's own CPU math (numpy FP64 port) is what is timed.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "flash-attention-v4-rocm_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

B, H, S, D = 32, 8, 4096, 128
METRIC = "fwd TFLOPS (B32 H8 D128 S4096, dense+causal step; aggregate over GPUs)"


def set_shape(b, s):
    """Non-default shapes are for profiling small cases only (never the bench line's metric)."""
    global B, S, METRIC, STEP_FLOPS
    B, S = b, s
    METRIC = f"fwd TFLOPS (B{B} H8 D128 S{S}, dense+causal step; aggregate over GPUs)"
    STEP_FLOPS = flops(B, H, S, False) + flops(B, H, S, True)
UNIT = "TFLOP/s"


def flops(b, h, s, causal):
    area = s * (s + 1) // 2 if causal else s * s
    return 4 * b * h * D * area


STEP_FLOPS = flops(B, H, S, False) + flops(B, H, S, True)


def dense_kernel_label(nb, config):
    """The forward kernel a dense launch of B=nb, H, S runs: the library's Auto
    rule (include/fav4_bshd.h, config 0), restated here only to name it."""
    if config != 0:
        return f"attn_fwd_sm100_kernel (dense, config {config})"
    if S < 128:
        return "attn_fwd_sm100_kernel (dense, config Auto=1)"
    import torch
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    t2, tw = nb * H * (-(-S // 256)), nb * H * (-(-S // 128))
    if 2 * t2 <= sms:
        return "attn_fwd_sm100_kernel (dense, config Auto=1)"
    if S >= 2048 and (-(-tw // sms)) * 25 < (-(-t2 // sms)) * 46:
        return "attn_fwd_wide_kernel (dense, Auto: wide-step kernel)"
    return "attn_fwd_sm100_kernel (dense, config Auto=2)"


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def committed_traffic():
    """DRAM bytes per dense launch from the committed ncu summary, if any."""
    try:
        return json.loads((ROOT / "profiles" / "traffic.json").read_text())
    except (OSError, ValueError):
        return None


# ------------------------------------------------------------ clocks ----
class ClockSampler:
    """Polls NVML (read-only) for SM clock and throttle reasons."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000002: "applications_clocks_setting",
        0x0000000000000001: "gpu_idle",
    }

    def __init__(self, index, period=0.01):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001 - NVML is optional telemetry
            self.error = str(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.thread.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "error", "")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ------------------------------------------------------- CPU baseline ----
def host_cores() -> int:
    """Cores this process may run on (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_threads_limit():
    """Context that lets numpy's BLAS/OpenMP pools use every host core, whatever
    OMP_NUM_THREADS the launcher set (torchrun sets 1). Yields the count."""
    import contextlib

    @contextlib.contextmanager
    def ctx():
        import numpy  # noqa: F401 - loads the BLAS the pools belong to
        n = host_cores()
        try:
            from threadpoolctl import threadpool_limits
            with threadpool_limits(limits=n):
                yield n
        except ImportError:
            yield 1
    return ctx()


def cpu_sample(budget_s: float, seed: int = 1, rows_per_slice: int | None = None):
    """Time the FP64 CPU oracle on (batch, head) slices of the workload, dense
    and causal alternately, until `budget_s` elapses (at least one of each).
    Returns (TFLOP/s, description)."""
    import numpy as np

    from oracle import ref_attention as R
    rng = np.random.default_rng(seed)
    q = R.bf16_round(rng.standard_normal((1, S, 1, D), dtype=np.float32))
    k = R.bf16_round(rng.standard_normal((1, S, 1, D), dtype=np.float32))
    v = R.bf16_round(rng.standard_normal((1, S, 1, D), dtype=np.float32))
    if rows_per_slice is None or rows_per_slice >= S:
        rows = np.arange(S)
    else:
        rows = np.linspace(0, S - 1, rows_per_slice).astype(np.int64)
    f_dense = 4 * D * len(rows) * S
    f_causal = 4 * D * int((rows + 1).sum())
    done = {False: 0, True: 0}
    t0 = time.perf_counter()
    spent = 0.0
    total_flops = 0
    while spent < budget_s or not (done[False] and done[True]):
        causal = done[False] > done[True]
        R.reference(q, k, v, causal, rows)
        done[causal] += 1
        total_flops += f_causal if causal else f_dense
        spent = time.perf_counter() - t0
    desc = (f"FP64 numpy oracle (benchmarks/bshd.py:90-100 math) on {done[False]} dense + {done[True]} causal "
            f"(b,h) slices of B32 H8 S4096 ({len(rows)} of {S} query rows each), {spent:.1f} s")
    return total_flops / spent / 1e12, desc


# ------------------------------------------------------------ helpers ----
def emit(obj):
    print(json.dumps(obj), flush=True)


def run_reference_arm(args, rank, world):
    """The reference arm: the CPU oracle, rank 0 only, on every host core."""
    if rank != 0:
        return
    with cpu_threads_limit() as cores:
        _reference_arm(args, world, cores)


def _reference_arm(args, world, cores):
    # size each step so (W + K) steps take about two minutes in total
    per_step = max(0.2, min(10.0, 120.0 / max(1, args.steps + args.warmup)))
    rows = S
    # calibrate: one dense + one causal slice of 256 query rows
    tf, _ = cpu_sample(0.0, rows_per_slice=256)
    est_slice_s = 2 * flops(1, 1, S, False) / (tf * 1e12) * 0.75  # dense + causal
    if est_slice_s > per_step:
        rows = max(64, int(S * per_step / est_slice_s))
    for _ in range(args.warmup):
        cpu_sample(0.0, rows_per_slice=rows)
    vals, descs = [], []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, d = cpu_sample(0.0, rows_per_slice=rows)
        vals.append(v)
        descs.append(d)
    wall = time.perf_counter() - t0
    value = statistics.mean(vals)
    sample = (f"per step: one dense + one causal (b,h) slice of B32 H8 S4096 with {rows} of {S} query rows, "
              f"FP64 numpy oracle of benchmarks/bshd.py:90-100; the reference's kernel is HIP for gfx1250")
    emit({"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
          "warmup": args.warmup, "ms_per_step": wall / args.steps * 1e3, "higher_is_better": True,
          "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
          "config": {"workload": "B32 H8 Sq=Sk=4096 D128 BSHD dense+causal (BASELINE configs[1]); CPU sample",
                     "global_batch": B, "heads": H, "seq_len": S, "head_dim": D, "lse": False,
                     "cpu_threads": cores},
          "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
          "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def run_sweep(args):
    """B32 H8 D128, S in {512..32768}, dense and causal,
    one GPU. For each point: W untimed calls, then K calls timed with CUDA
    events; prints one JSON line per point (the driver's bench line is the
    default mode, not this one)."""
    import torch

    import fav4_bshd
    runner = fav4_bshd.Runner()
    pk, pk_kind = peaks()
    gen = torch.Generator(device="cuda").manual_seed(2)
    for n in [int(x) for x in args.seqs.split(",")]:
        q, k, v = (torch.randn((B, n, H, D), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        o = torch.empty_like(q)
        for causal in (False, True):
            for _ in range(max(3, args.warmup)):
                runner.call(q, k, v, o, None, causal, args.config)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                runner.call(q, k, v, o, None, causal, args.config)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / args.steps
            f = flops(B, H, n, causal)
            tf = f / us / 1e6
            byts = 4 * B * n * H * D * 2
            emit({"seq": n, "causal": causal, "us": us, "tflops": tf, "frac_of_measured_bf16": tf / pk["bf16_tflops"],
                  "frac_of_nominal_2250": tf / 2250.0, "gbs": byts / us / 1e3,
                  "frac_of_measured_hbm": byts / us / 1e3 / pk["hbm_gbs"], "peak_source": pk_kind,
                  "batch": B, "heads": H, "config": args.config})
        del q, k, v, o
        torch.cuda.empty_cache()


def _library_impls(torch):
    """Same-box attention libraries on identical BSHD tensors (the analogue of
    the reference's CK comparator, benchmarks/ck_bshd.hip:62-66): each entry
    maps (q, k, v, causal, scale) -> O in BSHD, or is the reason it cannot run."""
    import torch.nn.functional as Fn
    from torch.nn.attention import SDPBackend, sdpa_kernel

    def sdpa(backend):
        def run(q, k, v, causal, scale):
            with sdpa_kernel(backend):
                o = Fn.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                    is_causal=causal, scale=scale)
            return o.transpose(1, 2)
        return run

    impls = {"torch-sdpa-cudnn": sdpa(SDPBackend.CUDNN_ATTENTION),
             "torch-sdpa-flash": sdpa(SDPBackend.FLASH_ATTENTION)}
    try:
        from flash_attn import __version__ as fa_version
        from flash_attn import flash_attn_func

        impls[f"flash_attn-{fa_version}"] = lambda q, k, v, causal, scale: flash_attn_func(
            q, k, v, causal=causal, softmax_scale=scale)
    except Exception as e:  # noqa: BLE001
        impls["flash_attn"] = f"import failed: {type(e).__name__}: {e}"
    return impls


def run_compare(args):
    """Same-box comparison (one GPU): this library and the installed attention
    libraries on the same Q/K/V (B32 H8 D128 BF16, seed 2), dense and causal,
    for each sequence length of --seqs. Calls of all implementations are
    interleaved over --steps rounds; one JSON line per (seq, mask,
    implementation) with the median time and the max |dO| against this
    library's output."""
    import torch

    import fav4_bshd
    runner = fav4_bshd.Runner()
    impls = _library_impls(torch)
    scale = 1 / math.sqrt(D)
    gen = torch.Generator(device="cuda").manual_seed(2)
    for n in [int(x) for x in args.seqs.split(",")]:
        q, k, v = (torch.randn((B, n, H, D), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        o = torch.empty_like(q)
        for causal in (False, True):
            def ours():
                runner.call(q, k, v, o, None, causal, args.config)
                return o
            runs = {"fav4_bshd (this library)": ours}
            notes = {}
            for name, fn in impls.items():
                if isinstance(fn, str):
                    notes[name] = fn
                    continue
                try:
                    fn(q, k, v, causal, scale)
                    torch.cuda.synchronize()
                    runs[name] = (lambda fn=fn: fn(q, k, v, causal, scale))
                except Exception as e:  # noqa: BLE001
                    notes[name] = f"{type(e).__name__}: {str(e).splitlines()[0][:160]}"
                    torch.cuda.synchronize()
            ref = ours().clone()
            diffs = {name: float((fn().float() - ref.float()).abs().max()) for name, fn in runs.items()}
            times = {name: [] for name in runs}
            for _ in range(max(3, args.warmup)):
                for fn in runs.values():
                    fn()
            torch.cuda.synchronize()
            for _ in range(args.steps):
                for name, fn in runs.items():
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn()
                    e1.record()
                    e1.synchronize()
                    times[name].append(e0.elapsed_time(e1) * 1e3)
            f = flops(B, H, n, causal)
            for name in runs:
                us = statistics.median(times[name])
                emit({"mode": "compare", "impl": name, "seq": n, "causal": causal, "us": us, "tflops": f / us / 1e6,
                      "max_abs_diff_vs_fav4": diffs[name], "batch": B, "heads": H, "head_dim": D,
                      "timing": f"median of {args.steps} single calls, CUDA events, calls interleaved"})
            for name, why in notes.items():
                emit({"mode": "compare", "impl": name, "seq": n, "causal": causal, "unavailable": why})
        del q, k, v, o
        torch.cuda.empty_cache()


def run_backward(args):
    """Backward pass, one GPU: B H S of the headline (or --batch/--seq), dense
    and causal. FLOPs by the usual convention, 2.5x the forward's (five
    matmuls: dV, dP, dQ, dK and the recomputed S). fav4_bshd_backward (the
    fused kernel, five matmuls) is the timed path; the deterministic two-kernel
    path (seven matmuls) and torch SDPA's cuDNN backward on the same tensors
    are timed beside it. One JSON line per mask."""
    import torch
    import torch.nn.functional as Fn
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import fav4_bshd
    runner = fav4_bshd.Runner()
    pk, pk_kind = peaks()
    gen = torch.Generator(device="cuda").manual_seed(5)
    q, k, v, do = (torch.randn((B, S, H, D), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o = torch.empty_like(q)
    lse = torch.empty((B, H, S), device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    scale = 1 / math.sqrt(D)

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    for causal in (False, True):
        runner.call(q, k, v, o, lse, causal, 0, scale)
        ms = timed(lambda: runner.backward(q, k, v, o, do, lse, dq, dk, dv, causal, scale))
        f = 2.5 * flops(B, H, S, causal)
        line = {"mode": "backward", "batch": B, "heads": H, "seq": S, "causal": causal, "ms": ms,
                "tflops": f / (ms * 1e-3) / 1e12, "frac_of_measured_bf16": f / (ms * 1e-3) / 1e12 / pk["bf16_tflops"],
                "peak_source": pk_kind, "flop_convention": "2.5 x forward (5 matmuls)",
                "pipeline_status": runner.pipeline_status(clear=True)}
        dms = timed(lambda: runner.backward(q, k, v, o, do, lse, dq, dk, dv, causal, scale, deterministic=True))
        line["deterministic_ms"] = dms
        line["deterministic_tflops"] = f / (dms * 1e-3) / 1e12
        try:
            tq, tk, tv = (x.transpose(1, 2).detach().requires_grad_(True) for x in (q, k, v))
            tdo = do.transpose(1, 2)
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                out = Fn.scaled_dot_product_attention(tq, tk, tv, is_causal=causal, scale=scale)
                cms = timed(lambda: torch.autograd.grad(out, (tq, tk, tv), tdo, retain_graph=True))
            line["torch_sdpa_cudnn_ms"] = cms
            line["torch_sdpa_cudnn_tflops"] = f / (cms * 1e-3) / 1e12
        except Exception as e:  # noqa: BLE001
            line["torch_sdpa_cudnn"] = f"unavailable: {type(e).__name__}: {str(e).splitlines()[0][:120]}"
        emit(line)


def run_decode(args):
    """Decode-like shapes on one GPU (few query rows against a long key cache):
    fav4_bshd_forward against the one-launch split-KV forward with the
    automatic split count, on the same tensors. Both are timed as K calls
    replayed from a CUDA graph (device time: at tens of microseconds per call
    the host's per-call work would otherwise be measured); the split path is
    also timed launched call by call. One JSON line per shape with the times,
    the split count, and the K/V bytes read per microsecond (the path is
    HBM-bound: every key and value is read once)."""
    import torch

    import fav4_bshd
    runner = fav4_bshd.Runner()
    pk, pk_kind = peaks()
    gen = torch.Generator(device="cuda").manual_seed(4)
    for sk in [int(x) for x in args.decode_sk.split(",")]:
        for sq in [int(x) for x in args.decode_sq.split(",")]:
            b, h = 1, H
            q = torch.randn((b, sq, h, D), generator=gen, device="cuda", dtype=torch.bfloat16)
            k, v = (torch.randn((b, sk, h, D), generator=gen, device="cuda", dtype=torch.bfloat16) for _ in range(2))
            o = torch.empty_like(q)
            o_split = torch.empty_like(q)
            used = runner.call_splitkv(q, k, v, o_split, None, False, args.config, 0)
            runner.call(q, k, v, o, None, False, args.config)
            torch.cuda.synchronize()
            diff = float((o.float() - o_split.float()).abs().max())

            def timed(fn, graph):
                for _ in range(max(3, args.warmup)):
                    fn()
                torch.cuda.synchronize()
                if graph:  # device time: the calls replayed from a CUDA graph (no host work per call)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        for _ in range(args.steps):
                            fn()
                    g.replay()
                    torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                if graph:
                    g.replay()
                else:
                    for _ in range(args.steps):
                        fn()
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) * 1e3 / args.steps

            plain = lambda: runner.call(q, k, v, o, None, False, args.config)  # noqa: E731
            split = lambda: runner.call_splitkv(q, k, v, o_split, None, False, args.config, used)  # noqa: E731
            us_plain, us_split = timed(plain, True), timed(split, True)
            us_split_eager = timed(split, False)
            kv_bytes = 2 * b * sk * h * D * 2
            emit({"mode": "decode", "batch": b, "heads": h, "sq": sq, "sk": sk, "splits": used,
                  "us_forward": us_plain, "us_splitkv": us_split, "speedup": us_plain / us_split,
                  "us_splitkv_eager_calls": us_split_eager,
                  "timing": f"{args.steps} calls replayed from one CUDA graph (device time); eager: the same "
                            "calls launched one by one from Python",
                  "kv_gbs_splitkv": kv_bytes / us_split / 1e3,
                  "frac_of_measured_hbm": kv_bytes / us_split / 1e3 / pk["hbm_gbs"], "peak_source": pk_kind,
                  "max_abs_diff": diff, "config": args.config,
                  "note": "each call re-reads K/V from HBM (K/V are larger than L2 from sk=32768)"})
            del q, k, v, o, o_split
            torch.cuda.empty_cache()


def run_decode_multi(args, rank, world, local):
    """Decode step across the N ranks of this torchrun job (fav4_bshd.splitkv.
    DecodeSplitKV): B1 H8, the first --decode-sq query rows against the last
    --decode-sk keys, one contiguous key chunk per GPU, combine over NVLink
    peer reads. Times K steps (device events, max over ranks), checks every
    rank's full output against one GPU's split-KV forward. One JSON line."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import fav4_bshd
    from fav4_bshd.splitkv import DecodeSplitKV
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        b, h = 1, H
        sq = int(args.decode_sq.split(",")[0])
        sk = int(args.decode_sk.split(",")[-1])
        gen = torch.Generator(device=dev).manual_seed(4)  # same inputs on every rank
        q = torch.randn((b, sq, h, D), generator=gen, device=dev, dtype=torch.bfloat16)
        k, v = (torch.randn((b, sk, h, D), generator=gen, device=dev, dtype=torch.bfloat16) for _ in range(2))
        dec = DecodeSplitKV(dist.group.WORLD, b, h, sq, sk, dev, causal=False, config=args.config)
        for _ in range(max(1, args.warmup)):
            dec.forward(q, k, v)
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            o, lse = dec.forward(q, k, v)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / args.steps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
        one_o = torch.empty_like(q)
        one_l = torch.empty((b, h, sq), device=dev, dtype=torch.float32)
        runner = fav4_bshd.Runner()
        one_splits = runner.call_splitkv(q, k, v, one_o, one_l, False, args.config, 0)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            runner.call_splitkv(q, k, v, one_o, one_l, False, args.config, one_splits)
        e1.record()
        torch.cuda.synchronize()
        us_one = e0.elapsed_time(e1) * 1e3 / args.steps
        err = torch.tensor([(o.float() - one_o.float()).abs().max().item(), (o.float() - one_o.float()).abs().mean().item(),
                            (lse - one_l).abs().max().item()], device=dev, dtype=torch.float64)
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
        if rank == 0:
            kv_bytes = 2 * b * sk * h * D * 2
            emit({"mode": "decode_split_kv", "metric": "decode step time (B1 H8 D128), key cache split over GPUs",
                  "us_per_step": us, "n_gpus": world, "steps": args.steps, "sq": sq, "sk": sk,
                  "splits_per_gpu": dec.splits, "kv_gbs_aggregate": kv_bytes / us / 1e3,
                  "single_gpu_us": us_one, "speedup_vs_single_gpu": us_one / us, "config": args.config,
                  "vs_single_gpu": {"max_abs_o": err[0].item(), "mean_abs_o": err[1].item(),
                                    "max_abs_lse": err[2].item(),
                                    "within_tolerance": bool(err[0] <= 2e-2 and err[1] <= 2e-3 and err[2] <= 1e-3)}})
        del dec
    finally:
        dist.destroy_process_group()


def run_long_context(args, rank, world, local):
    """B1 H8 S131072 causal, KV split over the N ranks of
    this torchrun job (fav4_bshd.splitkv: zigzag chunks, combine over NVLink
    peer reads). Times K forward steps (device events, max over ranks), then
    checks every rank's output rows against a single-GPU forward of the whole
    problem on that rank. One JSON line from rank 0."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import fav4_bshd
    from fav4_bshd.splitkv import SplitKV
    for key, val in (("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29531"), ("RANK", "0"), ("WORLD_SIZE", "1")):
        os.environ.setdefault(key, val)  # single process without torchrun
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        b, h, n = 1, 8, args.lc_seq
        gen = torch.Generator(device=dev).manual_seed(4)  # same inputs on every rank
        q, k, v = (torch.randn((b, n, h, D), generator=gen, device=dev, dtype=torch.bfloat16) for _ in range(3))
        sk = SplitKV(dist.group.WORLD, b, h, n, n, dev)
        for _ in range(max(1, args.warmup)):
            sk.forward(q, k, v, True, args.config)
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            o, lse = sk.forward(q, k, v, True, args.config)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        # agreement with one GPU computing the whole problem
        full_o = torch.empty_like(q)
        full_l = torch.empty((b, h, n), device=dev, dtype=torch.float32)
        fav4_bshd.Runner().call(q, k, v, full_o, full_l, True, args.config)
        torch.cuda.synchronize()
        err = torch.tensor([(o.float() - full_o[:, sk.r0:sk.r1].float()).abs().max().item(),
                            (o.float() - full_o[:, sk.r0:sk.r1].float()).abs().mean().item(),
                            (lse - full_l[:, :, sk.r0:sk.r1]).abs().max().item()], device=dev, dtype=torch.float64)
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
        f = flops(b, h, n, True)
        if rank == 0:
            emit({"mode": "long_context_split_kv", "metric": "causal fwd TFLOPS, B1 H8 D128, KV split over GPUs",
                  "value": f / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                  "ms_per_step": ms, "seq_len": n, "heads": h, "config": args.config,
                  "vs_single_gpu": {"max_abs_o": err[0].item(), "mean_abs_o": err[1].item(),
                                    "max_abs_lse": err[2].item(),
                                    "within_tolerance": bool(err[0] <= 2e-2 and err[1] <= 2e-3 and err[2] <= 1e-3)}})
        del sk
    finally:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=0, help="fav4 config id (0 = Auto)")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU oracle timing (N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=B, help="profiling only: per-GPU batch")
    ap.add_argument("--seq", type=int, default=S, help="profiling only: sequence length")
    ap.add_argument("--sweep", action="store_true", help="BASELINE configs[2] sequence sweep, one GPU")
    ap.add_argument("--backward", action="store_true", help="backward pass timing (B/S of the headline or --batch/--seq)")
    ap.add_argument("--decode", action="store_true",
                    help="decode-like shapes (B1 H8, few query rows, long key cache): forward vs one-launch split-KV")
    ap.add_argument("--decode-sq", default="1,16,64,128")
    ap.add_argument("--decode-sk", default="8192,32768,131072")
    ap.add_argument("--compare", action="store_true",
                    help="same-box comparison with torch SDPA (cuDNN, flash) and flash_attn, one GPU")
    ap.add_argument("--seqs", default="512,1024,2048,4096,8192,16384,32768")
    ap.add_argument("--long-context", action="store_true",
                    help="BASELINE configs[4]: B1 H8 causal split-KV across the torchrun ranks")
    ap.add_argument("--lc-seq", type=int, default=131072)
    ap.add_argument("--e2e-chunks", type=int, default=32, help="batch chunks of the host-buffer pipeline (clamped to B)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the configs[2] sweep key")
    ap.add_argument("--no-long-context", action="store_true", help="skip the configs[4] long-context key")
    args = ap.parse_args()
    if args.sweep:
        run_sweep(args)
        return
    if args.compare:
        run_compare(args)
        return
    if args.backward:
        if (args.batch, args.seq) != (B, S):
            set_shape(args.batch, args.seq)
        run_backward(args)
        return
    if args.decode:
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            run_decode_multi(args, int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]),
                             int(os.environ.get("LOCAL_RANK", "0")))
        else:
            run_decode(args)
        return
    if (args.batch, args.seq) != (B, S):
        set_shape(args.batch, args.seq)
    args.warmup = max(3, args.warmup)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.long_context:
        run_long_context(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    run_bench(args, rank, world, local)


# ------------------------------------------------------------ the bench ----
L2_FLUSH_BYTES = 256 << 20  # twice the 126 MB L2


def shard(world, rank, total=None):
    """Batch entries [b0, b1) of the global batch owned by `rank`."""
    total = B if total is None else total
    if total % world:
        raise SystemExit(f"global batch {total} is not divisible by {world} GPUs")
    per = total // world
    return rank * per, (rank + 1) * per


def global_inputs(dev, b0, b1, b, s, seed):
    """The global problem's Q/K/V drawn with one seed on every rank (so the
    shards of all ranks form the same global batch N=1 computes), sliced to
    this rank's batch entries."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for _ in range(3):
        full = torch.randn((b, s, H, D), generator=gen, device=dev, dtype=torch.bfloat16)
        out.append(full[b0:b1].clone())
        del full
    return out


def timed_steps(step, steps, stream, flush):
    """Run `steps` steps, each after an L2 flush; returns the per-step
    first-to-last event intervals (ms) and the per-launch intervals."""
    import torch
    evs = []
    for _ in range(steps):
        flush()
        ev = step(True)
        evs.append(ev)
    torch.cuda.synchronize()
    per_step = [ev[0].elapsed_time(ev[-1]) for ev in evs]
    per_launch = [[ev[i].elapsed_time(ev[i + 1]) for i in range(len(ev) - 1)] for ev in evs]
    return per_step, per_launch


def max_over_ranks(vals, world, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_ranks(vals, world, dev):
    """[world][len(vals)] from every rank's list (same length on every rank)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if world == 1:
        return [t.tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [x.tolist() for x in out]


def sweep_key(args, runner, world, rank, dev, barrier):
    """BASELINE configs[2] with the reference's graph protocol
    (benchmarks/bshd.py:34-51,157-166): per (S, mask) a CUDA graph of 5 calls
    (warm-up) and one of 20 calls; an observation replays the warm-up graph,
    synchronises, and times one replay of the 20-call graph with CUDA events.
    Observations: 6 up to S=4096, 3 at 8192, 2 above (bounded bench time).
    The global B=32 is sharded over the ranks; input sets (Q, K, V, O) rotate
    through the graph's calls so that more than 256 MiB is touched between two
    reads of one set (inputs larger than L2). Per point: the max over ranks of
    the median per-call time, the aggregate TFLOP/s it gives, and the per-GPU
    fraction of the measured peak."""
    import torch
    pk, pk_kind = peaks()
    b0, b1 = shard(world, rank)
    nb = b1 - b0
    stream = torch.cuda.current_stream()
    points = []
    for n in [int(x) for x in args.seqs.split(",")]:
        set_bytes = 4 * nb * n * H * D * 2
        sets = max(1, -(-L2_FLUSH_BYTES // set_bytes))
        data = []
        for i in range(sets):
            q, k, v = global_inputs(dev, b0, b1, B, n, 2 + 1000 * i)
            data.append((q, k, v, torch.empty_like(q)))
        obs = 6 if n <= 4096 else (3 if n <= 8192 else 2)
        for causal in (False, True):
            def calls(count, causal=causal):
                for c in range(count):
                    q, k, v, o = data[c % sets]
                    runner.call(q, k, v, o, None, causal, args.config)
            calls(2)  # one-time attribute set-up outside capture
            torch.cuda.synchronize()
            warm, timed = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(warm):
                calls(5)
            with torch.cuda.graph(timed):
                calls(20)
            us = []
            barrier()
            for _ in range(obs):
                warm.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                timed.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                us.append(e0.elapsed_time(e1) * 1e3 / 20)
            del warm, timed
            med = statistics.median(us)
            worst = max_over_ranks([med], world, dev)[0]
            f = flops(B, H, n, causal)
            tf = f / worst / 1e6
            points.append({"seq": n, "causal": causal, "us_per_call": worst, "tflops": tf,
                           "tflops_per_gpu": tf / world, "frac_of_measured_bf16_per_gpu": tf / world / pk["bf16_tflops"],
                           "gbs_per_gpu": set_bytes / worst / 1e3,
                           "frac_of_measured_hbm_per_gpu": set_bytes / worst / 1e3 / pk["hbm_gbs"],
                           "observations": obs, "input_sets": sets})
        del data
        torch.cuda.empty_cache()
    work_tiles = {p["seq"]: nb * H * -(-p["seq"] // 256) for p in points if not p["causal"]}
    return {"points": points, "global_batch": B, "batch_per_gpu": nb, "heads": H, "head_dim": D,
            "protocol": "reference graph protocol: 5-call warm-up graph, 20-call timed graph, median of "
                        "observations, max over ranks", "peak_source": pk_kind,
            "work_tiles_per_gpu_of_256_rows": work_tiles,
            "limiter_note": "per GPU the kernel walks batch_per_gpu*8*ceil(S/256) work tiles over 148 SMs; at "
                            "short S and small per-GPU batches the last wave and the per-tile pipeline fill "
                            "and drain bound the rate"}


def long_context_key(args, world, rank, local, dev, barrier):
    """B1 H8 S131072 causal, LSE on, seed 4. N=1: one
    forward of the whole problem; N>1: the key sequence split over the ranks
    (zigzag chunks, NVLink combine). Timed over K steps after W warm-up steps
    (device events, max over ranks); the output rows the reference's benchmark
    samples (benchmarks/bshd.py:147-148) are gathered to rank 0 and checked
    against the FP64 oracle."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import fav4_bshd
    from oracle import ref_attention as R
    b, h, n = 1, H, args.lc_seq
    gen = torch.Generator(device=dev).manual_seed(4)  # same inputs on every rank
    q, k, v = (torch.randn((b, n, h, D), generator=gen, device=dev, dtype=torch.bfloat16) for _ in range(3))
    if world > 1:
        from fav4_bshd.splitkv import SplitKV
        skv = SplitKV(dist.group.WORLD, b, h, n, n, dev)
        r0, r1 = skv.r0, skv.r1

        def fwd():
            return skv.forward(q, k, v, True, args.config)
    else:
        runner = fav4_bshd.Runner()
        o_full = torch.empty_like(q)
        l_full = torch.empty((b, h, n), device=dev, dtype=torch.float32)
        r0, r1 = 0, n

        def fwd():
            runner.call(q, k, v, o_full, l_full, True, args.config)
            return o_full, l_full
    lc_steps, lc_warm = max(2, min(5, args.steps)), 2
    for _ in range(lc_warm):
        fwd()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(lc_steps):
        o, lse = fwd()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks([e0.elapsed_time(e1) / lc_steps], world, dev)[0]
    # sampled rows: each rank contributes the rows it owns, rank 0 checks them
    rows = R.sample_rows(n)
    got_o = torch.zeros((len(rows), h, D), device=dev, dtype=torch.float32)
    got_l = torch.zeros((h, len(rows)), device=dev, dtype=torch.float32)
    for i, r in enumerate(rows.tolist()):
        if r0 <= r < r1:
            got_o[i] = o[0, r - r0].float()
            got_l[:, i] = lse[0, :, r - r0]
    if world > 1:
        dist.all_reduce(got_o)
        dist.all_reduce(got_l)
    f = flops(b, h, n, True)
    out = {"workload": f"B1 H8 Sq=Sk={n} D128 causal, LSE on, seed 4 (BASELINE configs[4])",
           "mode": "one GPU forward" if world == 1 else f"key sequence split over {world} GPUs (zigzag, NVLink combine)",
           "ms_per_step": ms, "tflops": f / (ms * 1e-3) / 1e12, "tflops_per_gpu": f / (ms * 1e-3) / 1e12 / world,
           "steps": lc_steps, "warmup": lc_warm}
    if rank == 0:
        with cpu_threads_limit():
            qn = np.zeros((1, n, h, D), dtype=np.float32)
            qn[0, rows] = q[0, torch.as_tensor(rows, device=dev)].float().cpu().numpy()
            kn, vn = (x.float().cpu().numpy() for x in (k, v))
            ref, ref_lse = R.reference_chunked(qn, kn, vn, True, rows)
        go = got_o.cpu().numpy().transpose(1, 0, 2)[None].astype(np.float64)  # [1, H, rows, D]
        gl = got_l.cpu().numpy()[None].astype(np.float64)
        st = R.error_stats(go, gl, ref, ref_lse)
        out["vs_fp64_sampled_rows"] = {
            "rows": len(rows), "max_abs_o": st["max_abs"], "mean_abs_o": st["mean_abs"],
            "max_abs_lse": st["lse_max_abs"], "reference_criteria": R.reference_criteria_pass(go, gl, ref, ref_lse),
            "within_tolerance": bool(st["finite"] and st["max_abs"] <= 2e-2 and st["mean_abs"] <= 2e-3
                                     and st["lse_max_abs"] <= 1e-3)}
    if world > 1:
        del skv
    del q, k, v
    torch.cuda.empty_cache()
    return out


def copy_bandwidth(hq, hk, hv, dev, world, stream):
    """Each rank's standalone copy rates, all ranks at the same time: Q/K/V
    host -> device, then two outputs device -> host (page-locked buffers)."""
    import torch
    dq, dk, dv = (torch.empty(x.shape, dtype=x.dtype, device=dev) for x in (hq, hk, hv))
    ho = torch.empty(hq.shape, dtype=hq.dtype).pin_memory()
    torch.cuda.synchronize()
    res = []
    for direction in ("h2d", "d2h"):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(3):
            if direction == "h2d":
                for d, hsrc in ((dq, hq), (dk, hk), (dv, hv)):
                    d.copy_(hsrc, non_blocking=True)
            else:
                ho.copy_(dq, non_blocking=True)
                ho.copy_(dk, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        nbytes = 3 * (3 if direction == "h2d" else 2) * hq.numel() * hq.element_size()
        res.append(nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    return gather_ranks(res, world, dev)


def run_bench(args, rank, world, local):
    import torch
    import torch.distributed as dist

    import fav4_bshd

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    lib = fav4_bshd.load_library()
    runner = fav4_bshd.Runner(lib)
    b0, b1 = shard(world, rank)
    nb = b1 - b0
    q, k, v = global_inputs(dev, b0, b1, B, S, 1)
    o_dense, o_causal = torch.empty_like(q), torch.empty_like(q)
    stream = torch.cuda.current_stream()
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def flush():
        flush_buf.zero_()

    def step(timed=False):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if timed else None
        if timed:
            ev[0].record(stream)
        runner.call(q, k, v, o_dense, None, False, args.config)
        if timed:
            ev[1].record(stream)
        runner.call(q, k, v, o_causal, None, True, args.config)
        if timed:
            ev[2].record(stream)
        return ev

    for _ in range(args.warmup):
        flush()
        step()
    torch.cuda.synchronize()

    try:
        nvml_index = torch.cuda._get_nvml_device_index(dev)
    except Exception:  # noqa: BLE001
        nvml_index = local
    sampler = ClockSampler(nvml_index)
    barrier()
    torch.cuda.synchronize()
    region0, region1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        region0.record(stream)
        per_step, per_launch = timed_steps(step, args.steps, stream, flush)
        region1.record(stream)
        torch.cuda.synchronize()
    barrier()
    region_ms = region0.elapsed_time(region1)
    dense_ms = [x[0] for x in per_launch]
    causal_ms = [x[1] for x in per_launch]
    ms_sum, region_max = max_over_ranks([sum(per_step), region_ms], world, dev)
    value = STEP_FLOPS * args.steps / (ms_sum * 1e-3) / 1e12

    # ---- end to end through the C ABI with host buffers ----
    # fav4_bshd_forward_host: one upload of Q/K/V from page-locked memory,
    # the dense and the causal forward, both outputs copied back; batch
    # chunks overlap the two copy directions and the kernels.
    e2e_steps = max(3, min(10, args.steps // 10))
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    ho_d = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    ho_c = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    outs = [(ho_d, None, False, args.config), (ho_c, None, True, args.config)]
    chunks = min(args.e2e_chunks, nb)

    def e2e_step():
        runner.forward_host(hq, hk, hv, outs, chunks=chunks, stream=stream)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    te = max_over_ranks([e0.elapsed_time(e1)], world, dev)[0]
    e2e_value = STEP_FLOPS * e2e_steps / (te * 1e-3) / 1e12
    h2d = 3 * q.numel() * q.element_size()
    d2h = 2 * q.numel() * q.element_size()
    ok_e2e = torch.equal(ho_d, o_dense.cpu()) and torch.equal(ho_c, o_causal.cpu())
    barrier()
    copy_rates = copy_bandwidth(hq, hk, hv, dev, world, stream)
    del hq, hk, hv, ho_d, ho_c
    status_main = runner.pipeline_status(clear=False)
    del q, k, v, o_dense, o_causal
    torch.cuda.empty_cache()

    # ---- BASELINE configs[2] sweep and configs[4] long context (extra keys) ----
    sweep = None if args.no_sweep else sweep_key(args, runner, world, rank, dev, barrier)
    lc = None if args.no_long_context else long_context_key(args, world, rank, local, dev, barrier)
    status = runner.pipeline_status(clear=False)
    statuses = gather_ranks([float(status_main), float(status)], world, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    pk, pk_kind = peaks()
    dense_avg = statistics.mean(dense_ms)
    achieved = flops(nb, H, S, False) / (dense_avg * 1e-3) / 1e12
    long_region = region_max > 2000.0
    peak = pk.get("bf16_tflops_sustained" if long_region else "bf16_tflops", 1590.0)
    traffic = committed_traffic()
    roofline = {"bound": "tensor", "kernel": f"{dense_kernel_label(nb, args.config)}, B{nb} per GPU",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": f"{pk_kind} {'sustained' if long_region else 'burst'} bf16",
                "traffic": (traffic.get("dense_dram_bytes_per_launch") if traffic and nb == 32 else None),
                "algorithmic_flops_per_launch": flops(nb, H, S, False),
                "algorithmic_bytes_per_launch": 4 * nb * S * H * D * 2,
                "dense_ms_median": statistics.median(dense_ms), "causal_ms_median": statistics.median(causal_ms),
                "dense_tflops": achieved,
                "causal_tflops": flops(nb, H, S, True) / (statistics.mean(causal_ms) * 1e-3) / 1e12,
                "frac_of_nominal_2250": achieved / 2250.0}
    h2d_rates = [r[0] for r in copy_rates]
    d2h_rates = [r[1] for r in copy_rates]
    out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms_sum / args.steps, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": f"B{B} H{H} Sq=Sk={S} D128 BSHD, one dense + one causal forward per step"
                                  + (" (BASELINE configs[1])" if (B, S) == (32, 4096) else " (profiling shape)"),
                      "global_batch": B, "batch_per_gpu": nb, "heads": H, "seq_len": S, "head_dim": D,
                      "lse": False, "fav4_config": args.config,
                      "parallelism": f"global batch sharded over {world} GPU(s) ({nb} per GPU), no collective",
                      "l2": "flushed before every step (256 MiB memset, outside the step's events)",
                      "timing": "sum over steps of each step's first-to-last CUDA event interval, max over ranks",
                      "region_ms_max_over_ranks": region_max},
           "gpu_launches": 2 * args.steps,
           "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world,
                   "d2h_bytes_per_step": d2h * world, "h2d_bytes_per_step_per_gpu": h2d,
                   "d2h_bytes_per_step_per_gpu": d2h, "steps": e2e_steps, "outputs_match": ok_e2e,
                   "api": f"fav4_bshd_forward_host, {chunks} batch chunks per GPU, page-locked host buffers",
                   "h2d_gbs_per_rank": h2d_rates, "d2h_gbs_per_rank": d2h_rates,
                   "copy_bound_ms_per_step": max(h2d / (r * 1e9) * 1e3 for r in h2d_rates),
                   "note": "h2d/d2h_gbs_per_rank: standalone copies of one step's inputs / outputs, all ranks "
                           "at once; the e2e step cannot beat its upload time (copy_bound_ms_per_step)"},
           "roofline": roofline, "clocks": sampler.summary(),
           "pipeline_status": {"headline_and_e2e": int(max(r[0] for r in statuses)),
                               "after_sweep_and_long_context": int(max(r[1] for r in statuses))}}
    if sweep is not None:
        out["sweep"] = sweep
    if lc is not None:
        out["long_context"] = lc
    if world == 1 and not args.no_cpu_baseline:
        with cpu_threads_limit() as cores:
            v_cpu, desc = cpu_sample(args.cpu_budget)
        out["cpu_baseline"] = {"value": v_cpu, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc}
    emit(out)


if __name__ == "__main__":
    main()

"""GPU test of fav4_bshd_forward_splitkv_static, the entry point that
allocates no device memory.

Some callers cannot call cudaMalloc: plugins whose host application owns all
device memory through its own pool (a cudaMalloc there fails or takes memory
the host has promised elsewhere), and latency-critical paths that cannot
afford cudaMalloc's implicit device synchronisation. For them the library
keeps the split-KV partials in a fixed 64 MiB device array of its own. This
test calls that entry point through the C ABI twice in a row, on different
problems, and checks each result against the existing entry point
(fav4_bshd_forward) with the same tolerance the split-KV tests use. It also
checks that a problem too large for the array is refused before anything
runs, and that a repeated call leaves the device's free memory unchanged.

The file name sorts last so a run that stops at its first failure has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

import fav4_bshd as F
from oracle import ref_attention as R

pytestmark = pytest.mark.gpu

CUDA_ERROR_MEMORY_ALLOCATION = 2


def _args(q, k, v, o, lse):
    b, sq, h, _ = q.shape
    return F.Args(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                  None if lse is None else lse.data_ptr(), b, h, sq, k.shape[1], 1 / math.sqrt(128))


def _inputs(b, h, sq, sk, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(s, generator=gen, device="cuda", dtype=torch.bfloat16)
            for s in ((b, sq, h, 128), (b, sk, h, 128), (b, sk, h, 128))]


def _run_both(lib, q, k, v, causal, splits):
    stream = torch.cuda.current_stream().cuda_stream
    b, sq, h, _ = q.shape
    o_ref = torch.full_like(q, float("nan"))
    l_ref = torch.full((b, h, sq), float("nan"), device="cuda")
    assert lib.fav4_bshd_forward(C.byref(_args(q, k, v, o_ref, l_ref)), int(causal), 0, stream) == 0
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, sq), float("nan"), device="cuda")
    status = lib.fav4_bshd_forward_splitkv_static(C.byref(_args(q, k, v, o, lse)), int(causal), 0, splits, stream)
    assert status == 0
    torch.cuda.synchronize()
    return o, lse, o_ref, l_ref


def _check_against_forward(o, lse, o_ref, l_ref):
    # the split-KV tolerance of tests/test_parity_gpu.py
    diff = (o.float() - o_ref.float()).abs()
    assert torch.isfinite(o.float()).all()
    assert diff.max().item() < 2e-2 and diff.mean().item() < 2e-3
    assert (lse - l_ref).abs().max().item() < 1e-3


@pytest.fixture(scope="module")
def lib(cuda):
    return F.load_library()


def test_static_splitkv_matches_forward_on_two_calls(lib):
    # call 1: long causal keys, 8 slices; call 2 reuses the same array for a
    # different (dense, ragged) problem with 3 slices
    cases = [(1, 8, 512, 8192, True, 8, 31), (2, 4, 300, 1537, False, 3, 32)]
    for b, h, sq, sk, causal, splits, seed in cases:
        q, k, v = _inputs(b, h, sq, sk, seed)
        o, lse, o_ref, l_ref = _run_both(lib, q, k, v, causal, splits)
        _check_against_forward(o, lse, o_ref, l_ref)
        # and against the FP64 oracle on sampled rows
        rows = R.sample_rows(sq)
        qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
        ref, ref_lse = R.reference_chunked(qn, kn, vn, causal, rows)
        R.errors(o.float().cpu().numpy()[:, rows].transpose(0, 2, 1, 3), lse.cpu().numpy()[:, :, rows], ref,
                 ref_lse)


def test_repeat_call_allocates_nothing(lib):
    q, k, v = _inputs(2, 4, 300, 1537, 33)
    o, lse, _, _ = _run_both(lib, q, k, v, False, 3)  # warm: same kernels as the measured call
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    assert lib.fav4_bshd_forward_splitkv_static(C.byref(_args(q, k, v, o, lse)), 0, 0, 3, stream) == 0
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_too_large_for_the_array_is_refused(lib):
    # 16 slices of a B8 H16 S4096 problem need 16 * 8*4096*16*260 bytes >> 64 MiB
    q = torch.zeros(8, 4096, 16, 128, device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)
    a = _args(q, q, q, o, None)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.fav4_bshd_forward_splitkv_static(C.byref(a), 1, 0, 16, stream) == CUDA_ERROR_MEMORY_ALLOCATION
    assert lib.fav4_bshd_forward_splitkv_static(C.byref(a), 1, 0, 0, stream) == F.CUDA_ERROR_INVALID_VALUE
    assert lib.fav4_bshd_forward_splitkv_static(C.byref(a), 1, 0, 17, stream) == F.CUDA_ERROR_INVALID_VALUE
    assert np.isfinite(float(q.sum()))  # the context is still fine
